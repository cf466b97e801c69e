"""Test infrastructure, not product code: the CPU checkers of the GPU search path.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use this package, and only
as the checker (never as the thing measured or shipped).

  Ref     the reference's own index layer (vdb, KoduruChandrasekhar/HNSW-Vector-DB) compiled in
          place by oracle/Makefile into oracle/_ref/libvdbref.so, behind ref_shim.cc's C ABI.
  Oracle  our plain-C restatement of the same algorithms (oracle.c -> liboracle.so), pinned
          against Ref's outputs by the golden fixtures in tests/golden/.
Index files written by the reference are parsed here in numpy (independently of the GPU
library's C++ reader) so the oracle can search the same graphs and codebooks.
"""
from __future__ import annotations

import ctypes
import os
import struct
import subprocess
from dataclasses import dataclass
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(HERE, "_ref", "libvdbref.so")
REF_ENGINE_LIB = os.path.join(HERE, "_ref", "libvdbref_engine.so")
REF_GPUINDEX_LIB = os.path.join(HERE, "_ref", "libvdbref_gpuindex.so")
ORACLE_LIB = os.path.join(HERE, "liboracle.so")
# The reference checkout sits beside this repository unless VDB_REFERENCE_SRC names it.
REFERENCE_SRC = os.environ.get("VDB_REFERENCE_SRC",
                               os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))

ORDER_SCALAR, ORDER_AVX512, ORDER_AVX2 = 0, 1, 2
L2, IP, COSINE = 0, 1, 2
_P = ctypes.c_void_p


def build(ref: bool = True) -> None:
    """Builds liboracle.so, and the reference's own libraries under _ref/ when the reference
    sources are present (the vdb::GpuIndex harness too once lib/libvdbgpu.so exists)."""
    targets = ["oracle"]
    if ref and os.path.isdir(os.path.join(REFERENCE_SRC, "src")):
        targets += ["ref", "engine"]
        if os.path.exists(os.path.join(os.path.dirname(HERE), "hnsw-vector-db_b200", "lib", "libvdbgpu.so")):
            targets += ["gpuindex"]
    subprocess.run(["make", "-s", "-C", HERE, f"REF={REFERENCE_SRC}", "-j8"] + targets, check=True)


def _ptr(a) -> Optional[int]:
    return None if a is None else a.ctypes.data


def host_kernel_order() -> int:
    """The summation order of the reference kernel set this CPU selects (cpu_features.cc:36-42)."""
    flags = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags = line
                    break
    except OSError:
        pass
    fl = set(flags.split())
    env = os.environ.get("VDB_KERNELS", "")
    avx2 = "avx2" in fl and "fma" in fl
    avx512 = avx2 and "avx512f" in fl
    if env == "scalar":
        return ORDER_SCALAR
    if env == "avx2" and avx2:
        return ORDER_AVX2
    if env == "avx512" and avx512:
        return ORDER_AVX512
    return ORDER_AVX512 if avx512 else (ORDER_AVX2 if avx2 else ORDER_SCALAR)


# ---------------------------------------------------------------------------------------- Ref

class Ref:
    """The reference's index layer (oracle/_ref/libvdbref.so)."""

    def __init__(self, path: str = REF_LIB):
        if not os.path.exists(path):
            raise ImportError(f"{path} is missing (build with `make -C oracle ref`)")
        l = ctypes.CDLL(path)
        sig = {
            "ref_last_error": (ctypes.c_char_p, []),
            "ref_kernel_set": (ctypes.c_char_p, []),
            "ref_distance": (ctypes.c_float, [ctypes.c_int, _P, _P, ctypes.c_size_t]),
            "ref_sq8_distance": (ctypes.c_float, [ctypes.c_int, _P, _P, _P, _P, ctypes.c_size_t]),
            "ref_normalize_rows": (ctypes.c_uint64, [_P, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32]),
            "ref_index_build": (_P, [ctypes.c_int, ctypes.c_int, _P, ctypes.c_uint64, ctypes.c_uint32,
                                     ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                     ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int]),
            "ref_index_load": (_P, [_P, ctypes.c_size_t, ctypes.c_int, _P, ctypes.c_uint64, ctypes.c_uint32,
                                    ctypes.c_uint32, ctypes.c_uint32]),
            "ref_index_free": (None, [_P]),
            "ref_index_extend": (_P, [_P, _P, ctypes.c_uint64, ctypes.c_int]),
            "ref_index_type": (ctypes.c_int, [_P]),
            "ref_index_save": (ctypes.c_size_t, [_P, ctypes.POINTER(_P)]),
            "ref_free": (None, [_P]),
            "ref_index_search": (None, [_P, _P, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64,
                                        ctypes.c_uint64, ctypes.c_int, _P, ctypes.c_int, _P, _P, _P, _P]),
            "ref_flat_search_batch": (None, [ctypes.c_int, _P, ctypes.c_uint64, ctypes.c_uint32,
                                             ctypes.c_uint32, _P, ctypes.c_uint64, ctypes.c_uint32,
                                             ctypes.c_int, _P, _P]),
            "ref_sq8_train_encode": (None, [_P, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, _P, _P,
                                            _P, ctypes.c_int]),
            "ref_sq8_scan_search": (None, [ctypes.c_int, _P, ctypes.c_uint64, ctypes.c_uint32,
                                           ctypes.c_uint32, _P, _P, _P, _P, ctypes.c_uint64,
                                           ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int, _P, _P, _P, _P]),
            "ref_topk": (ctypes.c_uint32, [_P, _P, ctypes.c_uint64, ctypes.c_uint32, _P, _P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        self.l = l

    def kernel_set(self) -> str:
        return self.l.ref_kernel_set().decode()

    def distance(self, which: int, a: np.ndarray, b: np.ndarray) -> float:
        return self.l.ref_distance(which, _ptr(a), _ptr(b), a.size)

    def sq8_distance(self, metric, q, code, vmin, scale) -> float:
        return self.l.ref_sq8_distance(metric, _ptr(q), _ptr(code), _ptr(vmin), _ptr(scale), q.size)

    def normalize_rows(self, rows: np.ndarray, dim: int) -> int:
        return self.l.ref_normalize_rows(_ptr(rows), rows.shape[0], dim, rows.shape[1])

    def build_index(self, type: int, metric: int, rows: np.ndarray, dim: int, M=16, efc=200,
                    pq_m=16, nlist=1024, max_train_ppc=256, seed=42, threads=1) -> "RefIndex":
        h = self.l.ref_index_build(type, metric, _ptr(rows), rows.shape[0], dim, rows.shape[1], M, efc,
                                   pq_m, nlist, max_train_ppc, seed, threads)
        if not h:
            raise RuntimeError(self.l.ref_last_error().decode())
        return RefIndex(self, h, rows.shape[0], rows.shape[1])

    def load_index(self, data: bytes, metric: int, rows: np.ndarray, dim: int, pq_m=16) -> "RefIndex":
        buf = np.frombuffer(data, dtype=np.uint8)
        h = self.l.ref_index_load(_ptr(buf), buf.size, metric, _ptr(rows), rows.shape[0], dim,
                                  rows.shape[1], pq_m)
        if not h:
            raise RuntimeError(self.l.ref_last_error().decode())
        return RefIndex(self, h, rows.shape[0], rows.shape[1])

    def flat_search_batch(self, metric, rows, dim, q, k, threads=0):
        nq = q.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.uint32)
        self.l.ref_flat_search_batch(metric, _ptr(rows), rows.shape[0], dim, rows.shape[1], _ptr(q), nq,
                                     k, threads, _ptr(d), _ptr(i))
        return i, d

    def sq8_train_encode(self, rows, dim, threads=0):
        n, pd = rows.shape
        vmin = np.empty(pd, np.float32)
        scale = np.empty(pd, np.float32)
        codes = np.empty((n, pd), np.uint8)
        self.l.ref_sq8_train_encode(_ptr(rows), n, dim, pd, _ptr(vmin), _ptr(scale), _ptr(codes), threads)
        return vmin, scale, codes

    def sq8_scan_search(self, metric, rows, codes, vmin, scale, q, k=10, depth=100, threads=0,
                        pre=False):
        nq = q.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.uint32)
        pd_ = np.empty((nq, depth), np.float32) if pre else None
        pi = np.empty((nq, depth), np.uint32) if pre else None
        self.l.ref_sq8_scan_search(metric, _ptr(rows), rows.shape[0], rows.shape[1], rows.shape[1],
                                   _ptr(codes), _ptr(vmin), _ptr(scale), _ptr(q), nq, k, depth, threads,
                                   _ptr(d), _ptr(i), _ptr(pd_), _ptr(pi))
        return (i, d, pi, pd_) if pre else (i, d)

    def topk(self, dist: np.ndarray, ids: np.ndarray, k: int):
        od = np.empty(k, np.float32)
        oi = np.empty(k, np.uint32)
        n = self.l.ref_topk(_ptr(dist), _ptr(ids), dist.size, k, _ptr(od), _ptr(oi))
        return oi[:n], od[:n]


class RefIndex:
    def __init__(self, ref: Ref, h, n, pd):
        self.ref, self.h, self.n, self.pd = ref, h, n, pd

    def save(self) -> bytes:
        p = _P()
        size = self.ref.l.ref_index_save(self.h, ctypes.byref(p))
        if size == 0:
            raise RuntimeError(self.ref.l.ref_last_error().decode())
        data = ctypes.string_at(p, size)
        self.ref.l.ref_free(p)
        return data

    def extend(self, rows: np.ndarray, threads=0) -> "RefIndex":
        """Index::extend over `rows` (the index's rows first): a new index."""
        h = self.ref.l.ref_index_extend(self.h, _ptr(rows), rows.shape[0], threads)
        if not h:
            raise RuntimeError(self.ref.l.ref_last_error().decode())
        return RefIndex(self.ref, h, rows.shape[0], rows.shape[1])

    def search(self, q, k=10, ef=64, nprobe=16, rerank=-1, allow=None, threads=0):
        nq = q.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.uint32)
        c = np.empty(nq, np.uint32)
        dc = np.empty(nq, np.uint64)
        self.ref.l.ref_index_search(self.h, _ptr(q), nq, k, ef, nprobe, rerank, _ptr(allow), threads,
                                    _ptr(d), _ptr(i), _ptr(c), _ptr(dc))
        return i, d, dc

    def __del__(self):
        try:
            self.ref.l.ref_index_free(self.h)
        except Exception:
            pass


STRATEGIES = {"auto": 0, "prefilter": 1, "exact": 1, "graph": 2, "postfilter": 3}


def _engine_lib(lib_path: str = REF_ENGINE_LIB):
    if not os.path.exists(lib_path):
        raise ImportError(f"{lib_path} is missing (build with `make -C oracle engine`)")
    l = ctypes.CDLL(lib_path)
    c64, c32, ci = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int
    sig = {
        "ref_coll_last_error": (ctypes.c_char_p, []),
        "ref_coll_create": (_P, [ctypes.c_char_p, ctypes.c_char_p, ci]),
        "ref_coll_open": (_P, [ctypes.c_char_p, ci]),
        "ref_coll_free": (None, [_P]),
        "ref_coll_bulk_load": (ci, [_P, _P, _P, c64, _P, _P, c32]),
        "ref_coll_bulk_load_json": (ci, [_P, _P, _P, c64, ctypes.c_char_p]),
        "ref_coll_remove_flush": (ci, [_P, _P, c64, _P, _P, c64, _P]),
        "ref_coll_upsert_json": (ci, [_P, _P, _P, c64, ctypes.c_char_p]),
        "ref_coll_remove": (ci, [_P, _P, c64, _P]),
        "ref_coll_flush": (ci, [_P]),
        "ref_coll_stats": (ci, [_P, ctypes.c_char_p, ctypes.c_size_t]),
        "ref_coll_search_batch": (ci, [_P, _P, c64, c32, c64, c64, ci, ci, c64, c64, ctypes.c_char_p, _P, _P]),
        "ref_coll_explain": (ci, [_P, _P, c32, c64, c64, ci, ci, c64, c64, ctypes.c_char_p, ctypes.c_char_p,
                                  ctypes.c_size_t]),
        "ref_segment_filter_bitmap": (ci, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, _P, c64]),
        "ref_filter_parse": (ci, [ctypes.c_char_p, ctypes.c_char_p]),
    }
    for name, (res, args) in sig.items():
        f = getattr(l, name)
        f.restype = res
        f.argtypes = args
    return l


class GpuIndexHarness:
    """The reference's SearchDiskSegment over a collection directory's disk segments, opened by
    Segment::Open with their CPU indexes (use_gpu False) or with vdb::GpuIndex as each segment's
    prebuilt index (use_gpu True): oracle/_ref/libvdbref_gpuindex.so (ref_gpuindex_shim.cc)."""

    def __init__(self, path: str, use_gpu: bool, device: int = 0, lib_path: str = REF_GPUINDEX_LIB):
        if not os.path.exists(lib_path):
            raise ImportError(f"{lib_path} is missing (build with `make -C oracle gpuindex`)")
        l = ctypes.CDLL(lib_path)
        c64, c32, ci = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int
        for name, res, args in (("gi_last_error", ctypes.c_char_p, []),
                                ("gi_open", _P, [ctypes.c_char_p, ci, ci]),
                                ("gi_close", None, [_P]),
                                ("gi_segments", c32, [_P]),
                                ("gi_search", ci, [_P, _P, c32, c64, c64, ci, ci, c64, c64, ctypes.c_char_p, _P, _P,
                                                   _P, ctypes.c_char_p, ctypes.c_size_t])):
            f = getattr(l, name)
            f.restype, f.argtypes = res, args
        self.l = l
        self.h = l.gi_open(path.encode(), int(use_gpu), device)
        if not self.h:
            raise RuntimeError(l.gi_last_error().decode())
        self.nseg = l.gi_segments(self.h)

    def search(self, q: np.ndarray, k=10, ef=64, nprobe=16, rerank=-1, strategy="auto", filter=None,
               prefilter_threshold=10000, post_filter_alpha=10):
        """Per segment (segment-local rows, dists, hit counts) and the explain list of one query."""
        import json
        q = np.ascontiguousarray(q, dtype=np.float32)
        d = np.empty((self.nseg, k), np.float32)
        r = np.empty((self.nseg, k), np.uint32)
        c = np.empty(self.nseg, np.uint32)
        buf = ctypes.create_string_buffer(1 << 16)
        rc = self.l.gi_search(self.h, _ptr(q), k, ef, nprobe, rerank, STRATEGIES[strategy], prefilter_threshold,
                              post_filter_alpha, _fj(filter), _ptr(d), _ptr(r), _ptr(c), buf, len(buf))
        if rc != 0:
            raise RuntimeError(self.l.gi_last_error().decode())
        return r, d, c, json.loads(buf.value.decode())

    def close(self):
        if getattr(self, "h", None):
            self.l.gi_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ref_filter_parse(schema: list, filter_json: str, lib_path: str = REF_ENGINE_LIB):
    """FilterExpr::Parse of the reference: (0, canonical text) or (status code, message)."""
    import json
    l = _engine_lib(lib_path)
    rc = l.ref_filter_parse(json.dumps(schema).encode(), filter_json.encode())
    return rc, l.ref_coll_last_error().decode()


def ref_segment_bitmap(segment_dir: str, schema: list, filter_json: str, rows: int,
                       lib_path: str = REF_ENGINE_LIB) -> np.ndarray:
    """The reference's filter bitmap over one segment's meta.bin (32 rows per uint32 word)."""
    import json
    l = _engine_lib(lib_path)
    out = np.zeros((rows + 31) // 32, np.uint32)
    rc = l.ref_segment_filter_bitmap(segment_dir.encode(), json.dumps(schema).encode(),
                                     filter_json.encode(), _ptr(out), rows)
    if rc != 0:
        raise RuntimeError(l.ref_coll_last_error().decode())
    return out


class RefCollection:
    """The reference's Collection (oracle/_ref/libvdbref_engine.so): bulk-loaded on-disk segments
    with metadata, filtered batched search through its planner and merge."""

    def __init__(self, path: str, dim: int, metric: str = "cosine", index: Optional[dict] = None,
                 schema: Optional[list] = None, threads: int = 0, lib_path: str = REF_ENGINE_LIB):
        import json
        self.l = _engine_lib(lib_path)
        self.dim = dim
        self.path = path
        self.schema = schema if schema is not None else [{"name": "year", "type": "int64"},
                                                          {"name": "tags", "type": "keyword_list"}]
        opts = {"dim": dim, "metric": metric, "sync": "none",
                "index": index or {"type": "hnsw", "M": 16, "ef_construction": 200},
                "schema": self.schema}
        self.h = self.l.ref_coll_create(path.encode(), json.dumps(opts).encode(), threads)
        if not self.h:
            raise RuntimeError(self.l.ref_coll_last_error().decode())

    @classmethod
    def open(cls, path: str, threads: int = 0, lib_path: str = REF_ENGINE_LIB) -> "RefCollection":
        """Collection::Open of an existing directory (recovery replays its logs)."""
        self = cls.__new__(cls)
        self.l = _engine_lib(lib_path)
        self.path = path
        self.h = self.l.ref_coll_open(path.encode(), threads)
        if not self.h:
            raise RuntimeError(self.l.ref_coll_last_error().decode())
        import json
        with open(os.path.join(path, "CURRENT")) as f:
            cur = f.read().strip()
        with open(os.path.join(path, cur), "rb") as f:
            opts = json.loads(f.read()[24:])["options"]
        self.dim, self.schema = opts["dim"], opts["schema"]
        return self

    def bulk_load(self, ids: np.ndarray, vectors: np.ndarray, years=None, tags=None, metadata=None):
        """One on-disk segment. Metadata either as (years int64, tags uint32 word ids with
        UINT32_MAX = unused, stored as keywords "w<id>") or as a list of dicts."""
        import json
        v = np.ascontiguousarray(vectors[:, :self.dim], dtype=np.float32)
        ids = np.ascontiguousarray(ids, dtype=np.uint64)
        if metadata is not None:
            rc = self.l.ref_coll_bulk_load_json(self.h, _ptr(ids), _ptr(v), ids.size,
                                                json.dumps(metadata).encode())
        else:
            mt = 0 if tags is None else tags.shape[1]
            rc = self.l.ref_coll_bulk_load(self.h, _ptr(ids), _ptr(v), ids.size,
                                           _ptr(None if years is None else np.ascontiguousarray(years, np.int64)),
                                           _ptr(None if tags is None else np.ascontiguousarray(tags, np.uint32)), mt)
        if rc != 0:
            raise RuntimeError(self.l.ref_coll_last_error().decode())

    def upsert(self, ids: np.ndarray, vectors: np.ndarray, metadata=None):
        """Collection::UpsertBatch (one log record per row); metadata a list of dicts or None."""
        import json
        v = np.ascontiguousarray(vectors[:, :self.dim], dtype=np.float32)
        ids = np.ascontiguousarray(ids, dtype=np.uint64)
        rc = self.l.ref_coll_upsert_json(self.h, _ptr(ids), _ptr(v), ids.size,
                                         None if metadata is None else json.dumps(metadata).encode())
        if rc != 0:
            raise RuntimeError(self.l.ref_coll_last_error().decode())

    def remove(self, ids: np.ndarray) -> int:
        """Collection::RemoveBatch; returns how many of ids were live."""
        ids = np.ascontiguousarray(ids, dtype=np.uint64)
        removed = np.zeros(1, dtype=np.uint64)
        if self.l.ref_coll_remove(self.h, _ptr(ids), ids.size, _ptr(removed)) != 0:
            raise RuntimeError(self.l.ref_coll_last_error().decode())
        return int(removed[0])

    def stats(self) -> dict:
        """Collection::Stats (rows, deletes, LSNs, per-segment id / kind / index / rows / deleted / lsn)."""
        import json
        buf = ctypes.create_string_buffer(1 << 20)
        if self.l.ref_coll_stats(self.h, buf, len(buf)) != 0:
            raise RuntimeError(self.l.ref_coll_last_error().decode())
        return json.loads(buf.value.decode())

    def flush(self):
        if self.l.ref_coll_flush(self.h) != 0:
            raise RuntimeError(self.l.ref_coll_last_error().decode())

    def remove_flush(self, ids: np.ndarray, up_ids: np.ndarray, up_vectors: np.ndarray) -> int:
        """Collection::RemoveBatch, UpsertBatch (up_ids / up_vectors, no metadata), then Flush: the
        upserts become a new segment and the removed or superseded rows of disk segments are
        written as delete files (deletes-<n>.roar) named in the new manifest. Returns how many of
        ids were live."""
        ids = np.ascontiguousarray(ids, dtype=np.uint64)
        up_ids = np.ascontiguousarray(up_ids, dtype=np.uint64)
        v = np.ascontiguousarray(up_vectors[:, :self.dim], dtype=np.float32)
        removed = np.zeros(1, dtype=np.uint64)
        rc = self.l.ref_coll_remove_flush(self.h, _ptr(ids), ids.size, _ptr(up_ids), _ptr(v), up_ids.size,
                                          _ptr(removed))
        if rc != 0:
            raise RuntimeError(self.l.ref_coll_last_error().decode())
        return int(removed[0])

    def search(self, q: np.ndarray, k=10, ef=64, nprobe=16, rerank=-1, strategy="auto", filter=None,
               prefilter_threshold=10000, post_filter_alpha=10):
        """Collection::SearchBatch: (ids uint64, distances float32), misses UINT64_MAX / +inf."""
        q = np.ascontiguousarray(q[:, :self.dim], dtype=np.float32)
        nq = q.shape[0]
        ids = np.empty((nq, k), np.uint64)
        d = np.empty((nq, k), np.float32)
        rc = self.l.ref_coll_search_batch(self.h, _ptr(q), nq, k, ef, nprobe, rerank, STRATEGIES[strategy],
                                          prefilter_threshold, post_filter_alpha, _fj(filter),
                                          _ptr(ids), _ptr(d))
        if rc != 0:
            raise RuntimeError(self.l.ref_coll_last_error().decode())
        return ids, d

    def explain(self, q: np.ndarray, k=10, ef=64, nprobe=16, rerank=-1, strategy="auto", filter=None,
                prefilter_threshold=10000, post_filter_alpha=10):
        """Per-part explain of Collection::Search for one query (mutable part first)."""
        import json
        q = np.ascontiguousarray(q[:self.dim], dtype=np.float32)
        buf = ctypes.create_string_buffer(1 << 20)
        rc = self.l.ref_coll_explain(self.h, _ptr(q), k, ef, nprobe, rerank, STRATEGIES[strategy],
                                     prefilter_threshold, post_filter_alpha, _fj(filter), buf, len(buf))
        if rc != 0:
            raise RuntimeError(self.l.ref_coll_last_error().decode())
        return json.loads(buf.value.decode())

    def segment_dirs(self):
        d = os.path.join(self.path, "segments")
        return sorted(os.path.join(d, x) for x in os.listdir(d) if x.startswith("seg-") and not x.endswith(".tmp"))

    def close(self):
        if getattr(self, "h", None):
            self.l.ref_coll_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _fj(filter) -> Optional[bytes]:
    import json
    if filter is None:
        return None
    return (filter if isinstance(filter, str) else json.dumps(filter)).encode()


def merge_hits_py(cands, k):
    """The merge of CollectionImpl::Search (src/engine/collection_impl.cc:1079-1108) for one
    query: cands = iterable of (dist, part, row, id); sorted by (dist, part, row), the first hit
    of every id, first k. Returns a list of (dist, part, row, id)."""
    out, seen = [], set()
    for c in sorted(cands, key=lambda t: (t[0], t[1], t[2])):
        if c[3] in seen:
            continue
        seen.add(c[3])
        out.append(c)
        if len(out) >= k:
            break
    return out


# ---------------------------------------------------------------------------------------- files

def split_index_file(data: bytes):
    """CheckIndexFile (src/index/index.cc:46-56) without the CRC check: (magic, body)."""
    return data[:8], data[8:-4]


class _R:
    def __init__(self, b: bytes):
        self.b, self.o = b, 0

    def u32(self):
        v = struct.unpack_from("<I", self.b, self.o)[0]
        self.o += 4
        return v

    def u64(self):
        v = struct.unpack_from("<Q", self.b, self.o)[0]
        self.o += 8
        return v

    def arr(self, dtype, count):
        a = np.frombuffer(self.b, dtype=dtype, count=count, offset=self.o).copy()
        self.o += a.nbytes
        return a


@dataclass
class HnswFile:
    cap: int
    size: int
    M: int
    efc: int
    seed: int
    max_level: int
    entry: int
    level: np.ndarray
    links0: np.ndarray
    upper: np.ndarray
    upper_off: np.ndarray

    def links(self, node: int, layer: int) -> list:
        """The link list of node on layer (hnsw_graph.h links_at)."""
        if layer == 0:
            b = node * (1 + 2 * self.M)
            return self.links0[b + 1:b + 1 + int(self.links0[b])].tolist()
        b = int(self.upper_off[node]) + (layer - 1) * (1 + self.M)
        return self.upper[b + 1:b + 1 + int(self.upper[b])].tolist()


def _parse_graph(r: _R) -> HnswFile:
    """HnswGraph::serialize layout (src/index/hnsw/hnsw_graph.h:387-401)."""
    cap, size = r.u64(), r.u64()
    M, efc = r.u32(), r.u32()
    seed = r.u64()
    maxl = struct.unpack("<i", struct.pack("<I", r.u32()))[0]
    ep = r.u32()
    level = r.arr(np.uint8, cap)
    links0 = r.arr(np.uint32, cap * (1 + 2 * M))
    blocks, offs, at = [], np.zeros(cap, np.uint64), 0
    for i in np.nonzero(level)[0]:
        n = int(level[i]) * (1 + M)
        blocks.append(r.arr(np.uint32, n))
        offs[i] = at
        at += n
    upper = np.concatenate(blocks) if blocks else np.zeros(1, np.uint32)
    return HnswFile(cap, size, M, efc, seed, maxl, ep, level, links0, upper, offs)


def parse_hnsw(data: bytes):
    """index.hnsw (HnswIndex::save, src/index/hnsw/hnsw_index.cc:36-41): (padded_dim, graph)."""
    magic, body = split_index_file(data)
    assert magic == b"VDBHNSW1", magic
    r = _R(body)
    pd = r.u32()
    return pd, _parse_graph(r)


def parse_hnsw_sq8(data: bytes):
    """index.hnsw_sq8 (HnswSq8Index::save, hnsw_index.cc:108-115): rows, (dim, pd, vmin, scale),
    codes, graph."""
    magic, body = split_index_file(data)
    assert magic == b"VDBHSQ81", magic
    r = _R(body)
    n = r.u64()
    dim, pd = r.u32(), r.u32()
    vmin = r.arr(np.float32, pd)
    scale = r.arr(np.float32, pd)
    codes = r.arr(np.uint8, n * pd).reshape(n, pd)
    return n, dim, pd, vmin, scale, codes, _parse_graph(r)


@dataclass
class IvfPqFile:
    rows: int
    pd: int
    nlist: int
    coarse: np.ndarray
    dim: int
    m: int
    centroids: np.ndarray
    list_off: np.ndarray
    ids: np.ndarray
    codes: np.ndarray


def parse_ivfpq(data: bytes) -> IvfPqFile:
    """index.ivf_pq (IvfPqIndex::save, src/index/quant/ivf_pq.cc:236-249)."""
    magic, body = split_index_file(data)
    assert magic == b"VDBIVFP1", magic
    r = _R(body)
    n, pd, nl = r.u64(), r.u32(), r.u32()
    coarse = r.arr(np.float32, nl * pd)
    dim, m = r.u32(), r.u32()
    cents = r.arr(np.float32, m * 256 * (dim // m))
    offs, ids, codes = [0], [], []
    for _ in range(nl):
        sz = r.u64()
        ids.append(r.arr(np.uint32, sz))
        codes.append(r.arr(np.uint8, sz * m))
        offs.append(offs[-1] + sz)
    return IvfPqFile(n, pd, nl, coarse, dim, m, cents, np.array(offs, np.uint64),
                     np.concatenate(ids) if ids else np.zeros(0, np.uint32),
                     np.concatenate(codes) if codes else np.zeros(0, np.uint8))


# ---------------------------------------------------------------------------------------- Oracle

class _OrcHnsw(ctypes.Structure):
    _fields_ = [("cap", ctypes.c_uint64), ("size", ctypes.c_uint64), ("M", ctypes.c_uint32),
                ("M0", ctypes.c_uint32), ("max_level", ctypes.c_int32), ("entry", ctypes.c_uint32),
                ("level", _P), ("links0", _P), ("upper", _P), ("upper_off", _P)]


class _OrcIvfPq(ctypes.Structure):
    _fields_ = [("nlist", ctypes.c_uint32), ("pd", ctypes.c_uint32), ("dim", ctypes.c_uint32),
                ("m", ctypes.c_uint32), ("dsub", ctypes.c_uint32), ("coarse", _P), ("centroids", _P),
                ("list_off", _P), ("ids", _P), ("codes", _P), ("term2", _P)]


class Oracle:
    """The plain-C restatement (oracle/liboracle.so)."""

    def __init__(self, path: str = ORACLE_LIB, order: Optional[int] = None):
        if not os.path.exists(path):
            raise ImportError(f"{path} is missing (build with `make -C oracle oracle`)")
        l = ctypes.CDLL(path)
        F, U32, U64, I = ctypes.c_float, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
        sig = {
            "orc_l2": (F, [_P, _P, ctypes.c_size_t, I]),
            "orc_dot": (F, [_P, _P, ctypes.c_size_t, I]),
            "orc_metric_dist": (F, [I, _P, _P, ctypes.c_size_t, I]),
            "orc_sq8_dist": (F, [I, _P, _P, _P, _P, ctypes.c_size_t, I]),
            "orc_l2_any": (F, [_P, _P, ctypes.c_size_t]),
            "orc_dot_any": (F, [_P, _P, ctypes.c_size_t]),
            "orc_normalize": (I, [_P, ctypes.c_size_t]),
            "orc_topk": (U32, [_P, _P, U64, U32, _P, _P]),
            "orc_flat_search": (U32, [I, _P, U64, U32, _P, U32, _P, I, _P, _P]),
            "orc_sq8_train": (None, [_P, U64, U32, U32, _P, _P]),
            "orc_sq8_encode": (None, [_P, U32, U32, _P, _P, _P]),
            "orc_sq8_scan_search": (U32, [I, _P, U64, U32, _P, _P, _P, _P, U32, U32, I, _P, _P]),
            "orc_pq_compute_table": (None, [_P, I, _P, U32, U32, _P]),
            "orc_pq_adc": (F, [_P, _P, U32]),
            "orc_ivfpq_term2": (None, [_P, U32, U32, _P, U32, U32, _P]),
            "orc_ivfpq_search": (U32, [ctypes.POINTER(_OrcIvfPq), I, _P, _P, U32, U32, I, _P, I, _P, _P, _P]),
            "orc_hnsw_search": (U32, [ctypes.POINTER(_OrcHnsw), I, _P, _P, _P, _P, U32, _P, U32, U32, _P, I,
                                      _P, _P, _P]),
            "orc_hnsw_sq8_search": (U32, [ctypes.POINTER(_OrcHnsw), I, _P, _P, _P, _P, U32, _P, U32, U32, I,
                                          _P, I, _P, _P, _P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        self.l = l
        self.order = host_kernel_order() if order is None else order

    # distances
    def l2(self, a, b, order=None):
        return self.l.orc_l2(_ptr(a), _ptr(b), a.size, self.order if order is None else order)

    def dot(self, a, b, order=None):
        return self.l.orc_dot(_ptr(a), _ptr(b), a.size, self.order if order is None else order)

    def sq8_dist(self, metric, q, code, vmin, scale, order=None):
        return self.l.orc_sq8_dist(metric, _ptr(q), _ptr(code), _ptr(vmin), _ptr(scale), q.size,
                                   self.order if order is None else order)

    def topk(self, dist, ids, k):
        od = np.empty(max(k, 1), np.float32)
        oi = np.empty(max(k, 1), np.uint32)
        n = self.l.orc_topk(_ptr(dist), _ptr(ids), dist.size, k, _ptr(od), _ptr(oi))
        return oi[:n], od[:n]

    def flat_search(self, metric, rows, q, k, allow=None):
        nq = q.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.uint32)
        for j in range(nq):
            self.l.orc_flat_search(metric, _ptr(rows), rows.shape[0], rows.shape[1], _ptr(q[j]), k,
                                   _ptr(allow), self.order, _ptr(d[j]), _ptr(i[j]))
        return i, d

    def sq8_train_encode(self, rows, dim):
        n, pd = rows.shape
        vmin = np.empty(pd, np.float32)
        scale = np.empty(pd, np.float32)
        self.l.orc_sq8_train(_ptr(rows), n, dim, pd, _ptr(vmin), _ptr(scale))
        codes = np.empty((n, pd), np.uint8)
        for r in range(n):
            self.l.orc_sq8_encode(_ptr(rows[r]), dim, pd, _ptr(vmin), _ptr(scale), _ptr(codes[r]))
        return vmin, scale, codes

    def sq8_scan_search(self, metric, rows, codes, vmin, scale, q, k=10, depth=100):
        nq = q.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.uint32)
        for j in range(nq):
            self.l.orc_sq8_scan_search(metric, _ptr(rows), rows.shape[0], rows.shape[1], _ptr(codes),
                                       _ptr(vmin), _ptr(scale), _ptr(q[j]), k, depth, self.order,
                                       _ptr(d[j]), _ptr(i[j]))
        return i, d

    def ivfpq_term2(self, f: IvfPqFile) -> np.ndarray:
        t = np.empty(f.nlist * f.m * 256, np.float32)
        self.l.orc_ivfpq_term2(_ptr(f.coarse), f.nlist, f.pd, _ptr(f.centroids), f.m, f.dim // f.m, _ptr(t))
        return t

    def ivfpq_search(self, f: IvfPqFile, metric, rows, q, k=10, nprobe=16, rerank=-1, allow=None,
                     precomputed=True):
        term2 = self.ivfpq_term2(f) if (precomputed and metric == L2) else None
        s = _OrcIvfPq(f.nlist, f.pd, f.dim, f.m, f.dim // f.m, _ptr(f.coarse), _ptr(f.centroids),
                      _ptr(f.list_off), _ptr(f.ids), _ptr(f.codes), _ptr(term2))
        nq = q.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.uint32)
        dc = np.empty(nq, np.uint64)
        for j in range(nq):
            self.l.orc_ivfpq_search(ctypes.byref(s), metric, _ptr(rows), _ptr(q[j]), k, nprobe, rerank,
                                    _ptr(allow), self.order, _ptr(d[j]), _ptr(i[j]), _ptr(dc[j:j + 1]))
        return i, d, dc

    @staticmethod
    def _graph(g: HnswFile) -> _OrcHnsw:
        return _OrcHnsw(g.cap, g.size, g.M, 2 * g.M, g.max_level, g.entry, _ptr(g.level), _ptr(g.links0),
                        _ptr(g.upper), _ptr(g.upper_off))

    def hnsw_search(self, g: HnswFile, metric, rows, q, k=10, ef=64, allow=None):
        s = self._graph(g)
        nq = q.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.uint32)
        dc = np.empty(nq, np.uint64)
        for j in range(nq):
            self.l.orc_hnsw_search(ctypes.byref(s), metric, _ptr(rows), None, None, None, rows.shape[1],
                                   _ptr(q[j]), k, ef, _ptr(allow), self.order, _ptr(d[j]), _ptr(i[j]),
                                   _ptr(dc[j:j + 1]))
        return i, d, dc

    def hnsw_sq8_search(self, g: HnswFile, metric, rows, codes, vmin, scale, q, k=10, ef=64, rerank=-1,
                        allow=None):
        s = self._graph(g)
        nq = q.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.uint32)
        dc = np.empty(nq, np.uint64)
        for j in range(nq):
            self.l.orc_hnsw_sq8_search(ctypes.byref(s), metric, _ptr(rows), _ptr(codes), _ptr(vmin),
                                       _ptr(scale), rows.shape[1], _ptr(q[j]), k, ef, rerank, _ptr(allow),
                                       self.order, _ptr(d[j]), _ptr(i[j]), _ptr(dc[j:j + 1]))
        return i, d, dc


def recall_at_k(found: np.ndarray, truth: np.ndarray, k: int) -> float:
    """Recall (tests/test_util.h:65-71): |found[:k] & truth[:k]| / k, averaged over queries."""
    hits = 0
    for f, t in zip(found, truth):
        hits += len(set(f[:k].tolist()) & set(t[:k].tolist()))
    return hits / (k * len(found))


def ids_match_up_to_ties(ids_a, d_a, ids_b, d_b, rel=1e-4) -> bool:
    """True when two closest-first lists hold the same ids, except where a swapped position sits in
    a tie (distances within `rel` relative)."""
    for ia, da, ib, db in zip(ids_a, d_a, ids_b, d_b):
        if np.array_equal(ia, ib):
            continue
        sa, sb = set(ia.tolist()), set(ib.tolist())
        diff = sa ^ sb
        if not diff:
            continue
        # Every id outside the common set must sit at the boundary distance (a tie).
        bound = max(float(da[-1]), float(db[-1]))
        tol = rel * max(1.0, abs(bound))
        for j, x in enumerate(ia):
            if x in diff and abs(float(da[j]) - bound) > tol:
                return False
        for j, x in enumerate(ib):
            if x in diff and abs(float(db[j]) - bound) > tol:
                return False
    return True
