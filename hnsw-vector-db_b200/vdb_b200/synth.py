"""Seeded synthetic workloads with the shapes and distributions of the benchmark configs
(lib/libvdbsynth.so). Harness code: used by tests and bench.py, not by the search path."""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import LIB_DIR, padded_dim

_lib = None


def _l():
    global _lib
    if _lib is None:
        path = os.path.join(LIB_DIR, "libvdbsynth.so")
        if not os.path.exists(path):
            raise ImportError(f"{path} is missing: build it with make")
        l = ctypes.CDLL(path)
        l.synth_mixture.restype = None
        l.synth_mixture.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                    ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                    ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p,
                                    ctypes.c_int]
        l.synth_metadata.restype = None
        l.synth_metadata.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64, ctypes.c_uint32,
                                     ctypes.c_uint32, ctypes.c_double, ctypes.c_uint64, ctypes.c_void_p,
                                     ctypes.c_void_p, ctypes.c_int]
        l.synth_meta_payload.restype = ctypes.c_uint64
        l.synth_meta_payload.argtypes = [ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
                                         ctypes.c_void_p, ctypes.c_uint64]
        l.synth_zipf.restype = None
        l.synth_zipf.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_double, ctypes.c_uint64,
                                 ctypes.c_void_p]
        _lib = l
    return _lib


def mixture(n, dim, ncentres, centres="uniform", lo=0.0, hi=100.0, sigma=10.0, integer=False,
            normalize=False, seed=0, stream=0, threads=0) -> np.ndarray:
    """n rows of padded_dim(dim) float32 from a Gaussian mixture (zero padding)."""
    pd = padded_dim(dim)
    out = np.empty((n, pd), dtype=np.float32)
    flags = (1 if integer else 0) | (2 if normalize else 0)
    _l().synth_mixture(n, dim, pd, ncentres, 0 if centres == "uniform" else 1, lo, hi, sigma, flags,
                       seed, stream, out.ctypes.data, threads)
    return out


# The benchmark configs (seeded; base rows use stream 0, queries stream 1).
def flat_int(n, nq, dim=128, seed=0):
    """Config 0 / 3: centres U[0,100]^d, sigma 10, clipped to [0,255], rounded."""
    kw = dict(centres="uniform", lo=0.0, hi=100.0, sigma=10.0, integer=True, seed=seed)
    return mixture(n, dim, 100, stream=0, **kw), mixture(nq, dim, 100, stream=1, **kw)


def sq8_cosine(n, nq, dim=128, seed=1):
    """Config 1: centres N(0,1)^d, sigma 0.3, then L2-normalised."""
    kw = dict(centres="normal", sigma=0.3, normalize=True, seed=seed)
    return mixture(n, dim, 1000, stream=0, **kw), mixture(nq, dim, 1000, stream=1, **kw)


def ivfpq_l2(n, nq, dim=96, seed=2):
    """Config 2: centres U[-1,1]^d, sigma 0.15."""
    kw = dict(centres="uniform", lo=-1.0, hi=1.0, sigma=0.15, seed=seed)
    return mixture(n, dim, 1000, stream=0, **kw), mixture(nq, dim, 1000, stream=1, **kw)


def sharded_cosine(n, nq, dim=128, seed=4, stream_base=0):
    """Config 4: centres U[0,100]^d, sigma 10 (not rounded), then L2-normalised."""
    kw = dict(centres="uniform", lo=0.0, hi=100.0, sigma=10.0, normalize=True, seed=seed)
    return (mixture(n, dim, 100, stream=stream_base, **kw),
            mixture(nq, dim, 100, stream=stream_base + 1, **kw))


def metadata(n, seed=4, year_lo=1990, year_hi=2024, max_tags=5, vocab=1000, zipf_s=1.1, threads=0):
    years = np.empty(n, dtype=np.int64)
    tags = np.empty((n, max_tags), dtype=np.uint32)
    _l().synth_metadata(n, year_lo, year_hi, max_tags, vocab, zipf_s, seed, years.ctypes.data,
                        tags.ctypes.data, threads)
    return years, tags


def meta_payload(years, tags) -> bytes:
    """meta.bin's payload for the schema [year int64, tags keyword_list] (tags as "w<id>")."""
    years = np.ascontiguousarray(years, dtype=np.int64)
    tags = np.ascontiguousarray(tags, dtype=np.uint32)
    n, mt = tags.shape
    size = _l().synth_meta_payload(n, years.ctypes.data, tags.ctypes.data, mt, None, 0)
    out = np.empty(size, dtype=np.uint8)
    _l().synth_meta_payload(n, years.ctypes.data, tags.ctypes.data, mt, out.ctypes.data, size)
    return out.tobytes()


def zipf_tags(n, vocab=1000, zipf_s=1.1, seed=5):
    out = np.empty(n, dtype=np.uint32)
    _l().synth_zipf(n, vocab, zipf_s, seed, out.ctypes.data)
    return out


# Config 4: 64 segments of 1,562,500 rows (normalised C0-style mixture, not rounded) with int64
# "year" U[1990, 2024] and keyword_list "tags" (1-5 Zipf(1.1) words of 1,000), and queries with one
# filter per distinct Zipf-drawn tag: year >= 2020 AND tags contains the tag.
C4_DIM = 128


def c4_segment(s, seg_rows):
    """Segment s of config 4: rows (normalised mixture), external ids, year / tags metadata."""
    rows = mixture(seg_rows, C4_DIM, 100, centres="uniform", lo=0.0, hi=100.0, sigma=10.0, normalize=True,
                   seed=4, stream=10 + s)
    ids = np.arange(s * seg_rows, (s + 1) * seg_rows, dtype=np.uint64)
    years, tags = metadata(seg_rows, seed=1000 + s)
    return rows, ids, years, tags


def c4_queries(nq):
    """Queries of config 4, their filters (JSON, one per distinct Zipf-drawn tag) and each query's
    filter index."""
    import json
    qs = mixture(nq, C4_DIM, 100, centres="uniform", lo=0.0, hi=100.0, sigma=10.0, normalize=True, seed=4,
                 stream=9)
    qtags = zipf_tags(nq, seed=5)
    distinct = sorted(set(qtags.tolist()))
    pos = {t: i for i, t in enumerate(distinct)}
    filters = [json.dumps({"and": [{"field": "year", "gte": 2020}, {"field": "tags", "eq": f"w{t}"}]})
               for t in distinct]
    qf = np.array([pos[t] for t in qtags.tolist()], dtype=np.int32)
    return qs, filters, qf
