"""vdb_b200: batched nearest-neighbour search on B200 GPUs, behind vdb's Index interface.

A thin Python host over the C ABI of include/vdbgpu.h (lib/libvdbgpu.so, built in place by the
package Makefile). It mirrors the reference's Python surface: `Index.search(queries, k, ef,
nprobe, rerank, filter)` returns `(ids, dists)` arrays of shape (nq, k), closest first, with
missing slots as (UINT32_MAX, +inf) like `_vdb._Collection.search` (python/bindings.cc:107-142).
Errors map as the reference binding does (bindings.cc:27-34): invalid argument -> ValueError,
not found -> KeyError, anything else -> RuntimeError.

There is no CPU fallback: importing works without a GPU, but opening a Context raises.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(os.path.dirname(_HERE), "lib")
LIB_PATH = os.environ.get("VDBGPU_LIB") or os.path.join(LIB_DIR, "libvdbgpu.so")

OK, INVALID_ARGUMENT, NOT_FOUND, IO_ERROR, CORRUPTION = 0, 1, 2, 4, 5
RESOURCE_EXHAUSTED, UNAVAILABLE, NOT_SUPPORTED = 7, 8, 9
STATUS_NAMES = {
    0: "OK", 1: "InvalidArgument", 2: "NotFound", 3: "AlreadyExists", 4: "IOError",
    5: "Corruption", 6: "FailedPrecondition", 7: "ResourceExhausted", 8: "Unavailable",
    9: "NotSupported", 10: "Internal",
}

METRICS = {"l2": 0, "ip": 1, "inner_product": 1, "cosine": 2}
INDEX_TYPES = {"flat": 0, "hnsw": 1, "hnsw_sq8": 2, "pq_flat": 3, "ivf_pq": 4, "sq8_flat": 16}
# ParseFilterStrategy (src/util/status.cc:115-128).
STRATEGIES = {"auto": 0, "prefilter": 1, "exact": 1, "graph": 2, "postfilter": 3}

# vdbgpu_hit: one merged collection hit (24 bytes).
HIT_DTYPE = np.dtype([("dist", "<f4"), ("part", "<u4"), ("row", "<u4"), ("pad", "<u4"), ("id", "<u8")])


class VdbError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class SearchParams(ctypes.Structure):
    """vdb::SearchParams (include/vdb/options.h:59-67)."""
    _fields_ = [("ef", ctypes.c_uint64), ("nprobe", ctypes.c_uint64), ("rerank", ctypes.c_int32),
                ("strategy", ctypes.c_int32), ("prefilter_threshold", ctypes.c_uint64),
                ("post_filter_alpha", ctypes.c_uint64)]


class IndexInfo(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int32), ("metric", ctypes.c_int32), ("rows", ctypes.c_uint64),
                ("dim", ctypes.c_uint32), ("padded_dim", ctypes.c_uint32),
                ("device_bytes", ctypes.c_uint64)]


class CollectionInfo(ctypes.Structure):
    _fields_ = [("dim", ctypes.c_uint32), ("padded_dim", ctypes.c_uint32), ("metric", ctypes.c_int32),
                ("index_type", ctypes.c_int32), ("segments_total", ctypes.c_uint32),
                ("segments_local", ctypes.c_uint32), ("rows_local", ctypes.c_uint64),
                ("device_bytes", ctypes.c_uint64)]


# Every symbol declared in include/vdbgpu.h, with its ctypes signature.
_P = ctypes.c_void_p
_SIGNATURES = {
    "vdbgpu_abi_version": (ctypes.c_int, []),
    "vdbgpu_launch_count": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint64)]),
    "vdbgpu_device_count": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "vdbgpu_open": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(_P)]),
    "vdbgpu_close": (None, [_P]),
    "vdbgpu_last_error": (ctypes.c_size_t, [_P, ctypes.c_char_p, ctypes.c_size_t]),
    "vdbgpu_synchronize": (ctypes.c_int, [_P]),
    "vdbgpu_set_stream": (ctypes.c_int, [_P, _P]),
    "vdbgpu_set_timing": (ctypes.c_int, [_P, ctypes.c_int]),
    "vdbgpu_stage_times": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_float), ctypes.c_int]),
    "vdbgpu_stage_counters": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int]),
    "vdbgpu_search_params_default": (None, [ctypes.POINTER(SearchParams)]),
    "vdbgpu_index_load": (ctypes.c_int, [_P, _P, ctypes.c_size_t, ctypes.c_int, _P, ctypes.c_uint64,
                                         ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(_P)]),
    "vdbgpu_index_create": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_uint64,
                                           ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(_P)]),
    "vdbgpu_index_free": (None, [_P]),
    "vdbgpu_index_get_info": (ctypes.c_int, [_P, ctypes.POINTER(IndexInfo)]),
    "vdbgpu_index_search": (ctypes.c_int, [_P, _P, ctypes.c_uint64, ctypes.c_uint32,
                                           ctypes.POINTER(SearchParams), _P, _P, _P, _P]),
    "vdbgpu_index_search_noalloc": (ctypes.c_int, [_P, _P, ctypes.c_uint64, ctypes.c_uint32,
                                                   ctypes.POINTER(SearchParams), _P, _P, _P]),
    "vdbgpu_index_file_inspect": (ctypes.c_int, [_P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int)]),
    "vdbgpu_index_sq8_export": (ctypes.c_int, [_P, _P, _P, _P]),
    "vdbgpu_collection_open": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_uint32, ctypes.c_uint32,
                                              ctypes.POINTER(_P)]),
    "vdbgpu_collection_create": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.POINTER(_P)]),
    "vdbgpu_collection_add_segment": (ctypes.c_int, [_P, ctypes.c_uint32, ctypes.c_uint32, _P, ctypes.c_uint64,
                                                     _P, _P, ctypes.c_size_t, _P, ctypes.c_size_t]),
    "vdbgpu_collection_set_deleted": (ctypes.c_int, [_P, ctypes.c_uint32, _P]),
    "vdbgpu_collection_free": (None, [_P]),
    "vdbgpu_collection_get_info": (ctypes.c_int, [_P, ctypes.POINTER(CollectionInfo)]),
    "vdbgpu_collection_search": (ctypes.c_int, [_P, _P, ctypes.c_uint64, ctypes.c_uint32,
                                                ctypes.POINTER(SearchParams), ctypes.c_char_p, _P, _P]),
    "vdbgpu_collection_search_grouped": (ctypes.c_int, [_P, _P, ctypes.c_uint64, ctypes.c_uint32,
                                                        ctypes.POINTER(SearchParams),
                                                        ctypes.POINTER(ctypes.c_char_p), ctypes.c_uint32,
                                                        _P, _P, _P, _P]),
    "vdbgpu_collection_stats": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_int]),
    "vdbgpu_collection_explain": (ctypes.c_int, [_P, _P, ctypes.c_uint32, ctypes.POINTER(SearchParams),
                                                 ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]),
    "vdbgpu_collection_filter_bitmap": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_uint32, _P,
                                                       ctypes.POINTER(ctypes.c_uint64)]),
    "vdbgpu_merge_hits": (ctypes.c_int, [_P, _P, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32,
                                         _P, _P, _P]),
    "vdbgpu_shard_id": (ctypes.c_int, [_P]),
    "vdbgpu_shard_group_open": (ctypes.c_int, [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_P)]),
    "vdbgpu_shard_group_close": (None, [_P]),
    "vdbgpu_shard_merge": (ctypes.c_int, [_P, _P, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int, _P, _P, _P]),
    "vdbgpu_hnsw_build": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
                                         ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64, ctypes.POINTER(_P),
                                         ctypes.POINTER(ctypes.c_size_t)]),
    "vdbgpu_hnsw_extend": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_size_t, _P, ctypes.c_uint64, ctypes.c_uint32,
                                          ctypes.c_uint32, ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_size_t)]),
    "vdbgpu_ivfpq_build": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
                                          ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64,
                                          ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_size_t)]),
    "vdbgpu_buffer_free": (None, [_P]),
    "vdbgpu_filter_describe": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                                              ctypes.c_size_t]),
    "vdbgpu_collection_inspect": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]),
    "vdbgpu_collection_apply_log": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t,
                                                   ctypes.c_void_p]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded C library; raises if it was not built (no silent fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {os.path.dirname(_HERE)}`")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def _raise(code: int, msg: str):
    if code == INVALID_ARGUMENT:
        raise ValueError(f"InvalidArgument: {msg}")
    if code == NOT_FOUND:
        raise KeyError(f"NotFound: {msg}")
    raise VdbError(code, msg)


def device_count() -> int:
    n = ctypes.c_int(0)
    lib().vdbgpu_device_count(ctypes.byref(n))
    return n.value


def padded_dim(dim: int) -> int:
    """vdb::PaddedDim (include/vdb/types.h:30-32): rows are zero-padded to 16 floats."""
    return (dim + 15) // 16 * 16


def _ptr(a) -> int:
    """Address of a numpy array or a torch tensor (device or host)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    raise TypeError(f"unsupported buffer type {type(a)}")


class Context:
    """One GPU, one stream (vdbgpu_open)."""

    def __init__(self, device: int = 0):
        h = _P()
        code = lib().vdbgpu_open(int(device), ctypes.byref(h))
        if code != OK:
            _raise(code, f"cannot open device {device}")
        self._h = h
        self.device = device

    def last_error(self) -> str:
        buf = ctypes.create_string_buffer(4096)
        lib().vdbgpu_last_error(self._h, buf, len(buf))
        return buf.value.decode(errors="replace")

    def check(self, code: int):
        if code != OK:
            _raise(code, self.last_error())

    def synchronize(self):
        self.check(lib().vdbgpu_synchronize(self._h))

    def set_stream(self, stream_handle: int = 0):
        """Launch on a caller's CUDA stream (e.g. torch.cuda.current_stream().cuda_stream). A handle
        of 0 (which is also torch's default stream) selects the context's own non-blocking stream:
        every call still returns only when its work is done, but it is not ordered after other
        work on the default stream, so finish such work (synchronize) before passing its output."""
        self.check(lib().vdbgpu_set_stream(self._h, stream_handle or None))

    def set_timing(self, on: bool = True):
        self.check(lib().vdbgpu_set_timing(self._h, 1 if on else 0))

    def stage_times(self):
        """Device ms of the last search: [prep (+ a seeded scan's sample pass), scan/walk,
        select+re-rank]."""
        buf = (ctypes.c_float * 8)()
        n = lib().vdbgpu_stage_times(self._h, buf, 8)
        return [buf[i] for i in range(n)]

    def stage_counters(self):
        """Work counters of the last search's dominant kernel (timing must be on)."""
        buf = (ctypes.c_uint64 * 8)()
        n = lib().vdbgpu_stage_counters(self._h, buf, 8)
        return [int(buf[i]) for i in range(n)]

    def close(self):
        if getattr(self, "_h", None):
            lib().vdbgpu_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _rows_f32(rows) -> Tuple[object, int, int]:
    if isinstance(rows, np.ndarray):
        if rows.dtype != np.float32 or not rows.flags.c_contiguous or rows.ndim != 2:
            raise ValueError("rows must be a C-contiguous float32 matrix (n x padded_dim)")
        return rows, rows.shape[0], rows.shape[1]
    return rows, rows.shape[0], rows.shape[1]


class Index:
    """A GPU index: the counterpart of vdb::Index (src/index/index.h:36-55)."""

    def __init__(self, ctx: Context, handle: _P, keep=None):
        self.ctx = ctx
        self._h = handle
        self._keep = keep
        info = IndexInfo()
        ctx.check(lib().vdbgpu_index_get_info(self._h, ctypes.byref(info)))
        self.type, self.metric = info.type, info.metric
        self.rows, self.dim, self.padded_dim = info.rows, info.dim, info.padded_dim
        self.device_bytes = info.device_bytes

    @classmethod
    def load(cls, ctx: Context, file_bytes: bytes, metric, rows, dim: int) -> "Index":
        """LoadIndex (src/index/index.h:61-62) over the segment's rows (n x padded_dim)."""
        m = METRICS[metric] if isinstance(metric, str) else int(metric)
        rows, n, pd = _rows_f32(rows)
        buf = np.frombuffer(file_bytes, dtype=np.uint8)
        h = _P()
        code = lib().vdbgpu_index_load(ctx._h, buf.ctypes.data, buf.size, m, _ptr(rows), n, dim, pd,
                                       ctypes.byref(h))
        ctx.check(code)
        return cls(ctx, h)

    @classmethod
    def create(cls, ctx: Context, type, metric, rows, dim: int) -> "Index":
        """CreateIndex + build for GPU-built types ("flat", "sq8_flat")."""
        t = INDEX_TYPES[type] if isinstance(type, str) else int(type)
        m = METRICS[metric] if isinstance(metric, str) else int(metric)
        rows, n, pd = _rows_f32(rows)
        h = _P()
        ctx.check(lib().vdbgpu_index_create(ctx._h, t, m, _ptr(rows), n, dim, pd, ctypes.byref(h)))
        return cls(ctx, h)

    def search(self, queries, k: int = 10, ef: int = 64, nprobe: int = 16, rerank: int = -1,
               filter=None, strategy: str = "auto", out=None, stats: bool = False):
        """Batched Index::search. `queries` is (nq, padded_dim) float32 (numpy, or a CUDA tensor),
        `filter` an optional allowed-row bitset (uint64 words, bit r of word r//64). Returns
        (ids uint32[nq,k], dists float32[nq,k]) [, distance_computations uint64[nq]]."""
        if isinstance(queries, np.ndarray):
            q = np.ascontiguousarray(queries, dtype=np.float32)
            if q.ndim == 1:
                q = q[None, :]
            if q.shape[1] != self.padded_dim:
                raise ValueError("query dimension does not match the index")
            nq = q.shape[0]
        else:
            q = queries
            nq = int(q.shape[0])
        p = SearchParams()
        lib().vdbgpu_search_params_default(ctypes.byref(p))
        p.ef, p.nprobe, p.rerank, p.strategy = int(ef), int(nprobe), int(rerank), STRATEGIES[strategy]
        if out is None:
            ids = np.empty((nq, k), dtype=np.uint32)
            dists = np.empty((nq, k), dtype=np.float32)
        else:
            ids, dists = out
        dc = np.empty(nq, dtype=np.uint64) if stats else None
        fb = None
        if filter is not None:
            fb = np.ascontiguousarray(filter, dtype=np.uint64)
            if fb.size < (self.rows + 63) // 64:
                raise ValueError("filter bitset is shorter than the index")
        code = lib().vdbgpu_index_search(self._h, _ptr(q), nq, int(k), ctypes.byref(p), _ptr(fb),
                                         _ptr(dists), _ptr(ids), _ptr(dc))
        self.ctx.check(code)
        return (ids, dists, dc) if stats else (ids, dists)

    def search_noalloc(self, queries, out_ids, out_dists, k: int = 10, rerank: int = -1, stream: int = 0):
        """The allocation-free search (vdbgpu_index_search_noalloc): `queries` (nq <= 128, padded
        dim) and the outputs are CUDA tensors on the index's device; nothing is allocated."""
        p = SearchParams()
        lib().vdbgpu_search_params_default(ctypes.byref(p))
        p.rerank = int(rerank)
        nq = int(queries.shape[0])
        code = lib().vdbgpu_index_search_noalloc(self._h, _ptr(queries), nq, int(k), ctypes.byref(p),
                                                 _ptr(out_dists), _ptr(out_ids), stream or None)
        self.ctx.check(code)

    def sq8_export(self, with_codes: bool = True):
        """(vmin, scale, codes) of an SQ8 index (Sq8Quantizer, src/index/quant/sq8.h)."""
        vmin = np.empty(self.padded_dim, dtype=np.float32)
        scale = np.empty(self.padded_dim, dtype=np.float32)
        codes = np.empty((self.rows, self.padded_dim), dtype=np.uint8) if with_codes else None
        self.ctx.check(lib().vdbgpu_index_sq8_export(self._h, _ptr(vmin), _ptr(scale), _ptr(codes)))
        return vmin, scale, codes

    def free(self):
        if getattr(self, "_h", None):
            # A context closed first (garbage collection can finalise a cycle in any order) took
            # its device memory with it; the handle is then dropped, not freed.
            if getattr(self.ctx, "_h", None):
                lib().vdbgpu_index_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def inspect_index_file(file_bytes: bytes) -> int:
    """CheckIndexFile + magic dispatch without a GPU: the index type, or raises."""
    buf = np.frombuffer(file_bytes, dtype=np.uint8)
    t = ctypes.c_int(-1)
    code = lib().vdbgpu_index_file_inspect(buf.ctypes.data, buf.size, ctypes.byref(t))
    if code != OK:
        _raise(code, "bad index file")
    return t.value


def unpack_bitset(words: np.ndarray, n: int) -> np.ndarray:
    return np.unpackbits(words.view(np.uint8), bitorder="little")[:n].astype(bool)


def pack_bitset(allowed: np.ndarray) -> np.ndarray:
    """Dense allowed-row bitset (bit r of word r//64) from a boolean mask."""
    n = allowed.size
    b = np.packbits(allowed.astype(np.uint8), bitorder="little")
    out = np.zeros((n + 63) // 64 * 8, dtype=np.uint8)
    out[: b.size] = b
    return out.view(np.uint64)


# ------------------------------------------------------------------------------ collections

def _params(ef, nprobe, rerank, strategy, prefilter_threshold, post_filter_alpha) -> SearchParams:
    if strategy not in STRATEGIES:
        raise ValueError("bad strategy")
    p = SearchParams()
    lib().vdbgpu_search_params_default(ctypes.byref(p))
    p.ef, p.nprobe, p.rerank, p.strategy = int(ef), int(nprobe), int(rerank), STRATEGIES[strategy]
    p.prefilter_threshold, p.post_filter_alpha = int(prefilter_threshold), int(post_filter_alpha)
    return p


def _filter_text(f) -> Optional[bytes]:
    import json
    if f is None:
        return None
    return (f if isinstance(f, str) else json.dumps(f)).encode()


class Collection:
    """A collection's on-disk segments on one GPU (or one shard of them): the read path of
    vdb::Collection (include/vdb/collection.h). `search` mirrors `_vdb._Collection.search`
    (python/bindings.cc:107-142): raw queries (nq, dim) float32, returns (ids uint64[nq,k],
    dists float32[nq,k]) with misses as (UINT64_MAX, +inf)."""

    def __init__(self, ctx: Context, handle: _P):
        self.ctx = ctx
        self._h = handle
        self._refresh()

    def _refresh(self):
        info = CollectionInfo()
        self.ctx.check(lib().vdbgpu_collection_get_info(self._h, ctypes.byref(info)))
        self.dim, self.padded_dim, self.metric = info.dim, info.padded_dim, info.metric
        self.index_type = info.index_type
        self.segments_total, self.segments_local = info.segments_total, info.segments_local
        self.rows_local, self.device_bytes = info.rows_local, info.device_bytes

    @classmethod
    def open(cls, ctx: Context, path: str, shard: int = 0, nshards: int = 1) -> "Collection":
        """Loads a collection directory written by the reference (this shard's segments)."""
        h = _P()
        ctx.check(lib().vdbgpu_collection_open(ctx._h, path.encode(), int(shard), int(nshards), ctypes.byref(h)))
        return cls(ctx, h)

    @classmethod
    def create(cls, ctx: Context, options) -> "Collection":
        """An empty collection with the reference's options (dict or JSON text)."""
        import json
        text = options if isinstance(options, str) else json.dumps(options)
        h = _P()
        ctx.check(lib().vdbgpu_collection_create(ctx._h, text.encode(), ctypes.byref(h)))
        return cls(ctx, h)

    def add_segment(self, segment_id: int, ordinal: int, rows, ids: np.ndarray, meta: bytes,
                    index_file: bytes):
        """One segment from its files' contents: rows (n, padded_dim) float32 (numpy or a CUDA
        tensor), external ids, the meta.bin payload and the index file."""
        ids = np.ascontiguousarray(ids, dtype=np.uint64)
        mb = np.frombuffer(meta, dtype=np.uint8) if meta else None
        ib = np.frombuffer(index_file, dtype=np.uint8)
        n = int(rows.shape[0])
        self.ctx.check(lib().vdbgpu_collection_add_segment(self._h, int(segment_id), int(ordinal), _ptr(rows), n,
                                                           _ptr(ids), _ptr(mb), 0 if mb is None else mb.size,
                                                           _ptr(ib), ib.size))
        self._refresh()

    def set_deleted(self, segment_id: int, deleted: Optional[np.ndarray]):
        """Deleted rows of a segment as a boolean mask (None clears them)."""
        words = None
        if deleted is not None:
            d = np.asarray(deleted, dtype=bool)
            b = np.packbits(d.astype(np.uint8), bitorder="little")
            pad = np.zeros((d.size + 31) // 32 * 4, np.uint8)
            pad[: b.size] = b
            words = pad.view(np.uint32)
        self.ctx.check(lib().vdbgpu_collection_set_deleted(self._h, int(segment_id), _ptr(words)))

    def _queries(self, queries):
        if isinstance(queries, np.ndarray):
            q = np.ascontiguousarray(queries, dtype=np.float32)
            if q.ndim == 1:
                q = q[None, :]
            if q.shape[1] != self.dim:
                raise ValueError("query dimension does not match the collection")
            return q, q.shape[0]
        return queries, int(queries.shape[0])

    def search(self, queries, k: int = 10, ef: int = 64, nprobe: int = 16, rerank: int = -1,
               filter=None, strategy: str = "auto", prefilter_threshold: int = 10000,
               post_filter_alpha: int = 10, out=None):
        """Collection::SearchBatch with one filter (JSON text or dict) for every query."""
        q, nq = self._queries(queries)
        p = _params(ef, nprobe, rerank, strategy, prefilter_threshold, post_filter_alpha)
        ids, dists = out if out is not None else (np.empty((nq, k), np.uint64), np.empty((nq, k), np.float32))
        self.ctx.check(lib().vdbgpu_collection_search(self._h, _ptr(q), nq, int(k), ctypes.byref(p),
                                                      _filter_text(filter), _ptr(ids), _ptr(dists)))
        return ids, dists

    def search_grouped(self, queries, filters, query_filter=None, k: int = 10, ef: int = 64,
                       nprobe: int = 16, rerank: int = -1, strategy: str = "auto",
                       prefilter_threshold: int = 10000, post_filter_alpha: int = 10, out=None,
                       hits=None):
        """Several filters in one batch: query i uses filters[query_filter[i]] (-1: none).
        `hits` (optional, (nq, k) HIT_DTYPE numpy array or a CUDA uint8 tensor of nq*k*24 bytes)
        receives the merged hit records for a cross-GPU merge. out=False skips the ids / dists."""
        q, nq = self._queries(queries)
        p = _params(ef, nprobe, rerank, strategy, prefilter_threshold, post_filter_alpha)
        texts = [_filter_text(f) for f in filters]
        arr = (ctypes.c_char_p * max(1, len(texts)))(*texts)
        qf = None if query_filter is None else np.ascontiguousarray(query_filter, dtype=np.int32)
        if qf is not None and qf.size != nq:
            raise ValueError("query_filter needs one entry per query")
        if out is None:
            ids, dists = np.empty((nq, k), np.uint64), np.empty((nq, k), np.float32)
        elif out is False:
            ids = dists = None
        else:
            ids, dists = out
        self.ctx.check(lib().vdbgpu_collection_search_grouped(self._h, _ptr(q), nq, int(k), ctypes.byref(p), arr,
                                                              len(texts), _ptr(qf), _ptr(ids), _ptr(dists),
                                                              _ptr(hits)))
        return ids, dists

    def apply_log(self, records: bytes) -> int:
        """Applies write-ahead log records (the reference's log bytes for a write batch, without the
        file header) as recovery replays them; returns how many were applied."""
        n = ctypes.c_uint64(0)
        self.ctx.check(lib().vdbgpu_collection_apply_log(self._h, bytes(records), len(records), ctypes.byref(n)))
        return int(n.value)

    def explain(self, query, k: int = 10, ef: int = 64, nprobe: int = 16, rerank: int = -1, filter=None,
                strategy: str = "auto", prefilter_threshold: int = 10000, post_filter_alpha: int = 10):
        """Per-segment plan of one query (SegmentExplain): strategy, matches, distance
        computations, results."""
        import json
        q, _ = self._queries(np.asarray(query, dtype=np.float32).reshape(1, -1))
        p = _params(ef, nprobe, rerank, strategy, prefilter_threshold, post_filter_alpha)
        buf = ctypes.create_string_buffer(1 << 20)
        self.ctx.check(lib().vdbgpu_collection_explain(self._h, _ptr(q), int(k), ctypes.byref(p),
                                                       _filter_text(filter), buf, len(buf)))
        return json.loads(buf.value.decode())

    STAT_NAMES = ("queries", "exact_rows", "index_distance_computations", "prefilter_pairs",
                  "graph_pairs", "postfilter_pairs", "empty_pairs", "bitmap_words", "index_searches",
                  "us_bitmaps_plan", "us_exact", "us_index", "us_other")

    def stats(self, enable: Optional[bool] = None) -> dict:
        """Work counters of the last search (index distance computations only while enabled)."""
        out = np.zeros(len(self.STAT_NAMES), np.uint64)
        n = lib().vdbgpu_collection_stats(self._h, -1 if enable is None else int(bool(enable)), _ptr(out), out.size)
        return {k: int(v) for k, v in zip(self.STAT_NAMES[:n], out[:n])}

    def filter_bitmap(self, filter, segment_id: int, rows: int) -> Tuple[np.ndarray, int]:
        """The rows of one segment a filter selects: (uint32 words, bit r of word r//32; count)."""
        words = np.zeros((rows + 31) // 32, np.uint32)
        m = ctypes.c_uint64(0)
        self.ctx.check(lib().vdbgpu_collection_filter_bitmap(self._h, _filter_text(filter), int(segment_id),
                                                             _ptr(words), ctypes.byref(m)))
        return words, int(m.value)

    def free(self):
        if getattr(self, "_h", None):
            if getattr(self.ctx, "_h", None):
                lib().vdbgpu_collection_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def merge_hits(ctx: Context, lists, k: int, out=None, hits=None):
    """The collection merge over already-merged hit lists: `lists` is (nlists, nq, k) HIT_DTYPE
    (numpy) or a CUDA uint8 tensor of nlists*nq*k*24 bytes (give nlists, nq via its shape
    (nlists, nq, k*24)). Returns (ids uint64[nq,k], dists float32[nq,k])."""
    if isinstance(lists, np.ndarray):
        if lists.dtype != HIT_DTYPE or lists.ndim != 3:
            raise ValueError("lists must be (nlists, nq, k) of HIT_DTYPE")
        nl, nq = lists.shape[0], lists.shape[1]
        lists = np.ascontiguousarray(lists)
    else:
        nl, nq = int(lists.shape[0]), int(lists.shape[1])
    if out is None:
        ids, dists = np.empty((nq, k), np.uint64), np.empty((nq, k), np.float32)
    else:
        ids, dists = out
    ctx.check(lib().vdbgpu_merge_hits(ctx._h, _ptr(lists), nl, nq, int(k), _ptr(ids), _ptr(dists), _ptr(hits)))
    return ids, dists


def launch_count() -> int:
    """Kernel launches of the library in this process so far (vdbgpu_launch_count)."""
    v = ctypes.c_uint64(0)
    lib().vdbgpu_launch_count(ctypes.byref(v))
    return int(v.value)


SHARD_ID_BYTES = 128


def _same_nccl_as_torch():
    """Points the library at the NCCL that torch links against (the nvidia-nccl wheel), unless the
    caller chose one (VDBGPU_NCCL_LIB). A process holds one libnccl.so.2: whichever loads first
    serves every later user, so the library must not load an older system copy that a later
    `import torch` would then be handed."""
    if os.environ.get("VDBGPU_NCCL_LIB"):
        return
    try:
        import nvidia.nccl
    except ImportError:
        return
    for d in getattr(nvidia.nccl, "__path__", []):
        p = os.path.join(d, "lib", "libnccl.so.2")
        if os.path.exists(p):
            os.environ["VDBGPU_NCCL_LIB"] = p
            return


def shard_id() -> bytes:
    """A rendezvous token for one ShardGroup (ncclGetUniqueId), made on one rank and handed to
    every rank by the caller's own channel."""
    _same_nccl_as_torch()
    buf = ctypes.create_string_buffer(SHARD_ID_BYTES)
    code = lib().vdbgpu_shard_id(buf)
    if code != OK:
        _raise(code, "could not make a shard token (is libnccl.so.2 available?)")
    return buf.raw


class ShardGroup:
    """This rank's membership in the NCCL group of a collection sharded over the GPUs of one node
    (vdbgpu_shard_group_open): merge() exchanges every rank's merged hit records and merges them
    on the receiving GPU(s). Every wait is bounded by timeout_ms; a failure aborts the group."""

    def __init__(self, ctx: Context, token: bytes, rank: int, nranks: int, timeout_ms: int = 60000):
        if len(token) != SHARD_ID_BYTES:
            raise ValueError("the token must be SHARD_ID_BYTES bytes")
        _same_nccl_as_torch()
        self.ctx, self.rank, self.nranks = ctx, int(rank), int(nranks)
        self._token = ctypes.create_string_buffer(token, SHARD_ID_BYTES)
        h = _P()
        ctx.check(lib().vdbgpu_shard_group_open(ctx._h, self._token, self.rank, self.nranks, int(timeout_ms),
                                                ctypes.byref(h)))
        self._h = h

    def merge(self, local, nq: int, k: int, root: int = -1, out=None, hits=None):
        """local: this rank's nq x k merged records (HIT_DTYPE numpy (nq, k), or a CUDA uint8 tensor
        of nq*k*24 bytes). Returns (ids, dists) on receiving ranks (out, or new numpy arrays),
        None elsewhere."""
        receives = root < 0 or root == self.rank
        if out is None and receives:
            out = (np.empty((nq, k), np.uint64), np.empty((nq, k), np.float32))
        ids, dists = out if (out is not None and receives) else (None, None)
        self.ctx.check(lib().vdbgpu_shard_merge(self._h, _ptr(local), int(nq), int(k), int(root), _ptr(ids),
                                                _ptr(dists), _ptr(hits) if receives else None))
        return (ids, dists) if receives else None

    def close(self):
        if getattr(self, "_h", None):
            lib().vdbgpu_shard_group_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def build_hnsw(ctx: Context, metric, rows, dim: int, M: int = 16, candidates: int = 0, seed: int = 42) -> bytes:
    """An HNSW index file (the reference's index.hnsw format) built on the GPU over rows
    (n, padded_dim) float32, numpy or a CUDA tensor."""
    m = METRICS[metric] if isinstance(metric, str) else int(metric)
    n, pd = int(rows.shape[0]), int(rows.shape[1])
    p = _P()
    nb = ctypes.c_size_t(0)
    ctx.check(lib().vdbgpu_hnsw_build(ctx._h, m, _ptr(rows), n, int(dim), pd, int(M), int(candidates), int(seed),
                                      ctypes.byref(p), ctypes.byref(nb)))
    try:
        return ctypes.string_at(p, nb.value)
    finally:
        lib().vdbgpu_buffer_free(p)


def extend_hnsw(ctx: Context, metric, file_bytes: bytes, rows, dim: int) -> bytes:
    """HnswIndex::extend on the GPU: the index.hnsw `file_bytes` (a graph over the first rows of
    `rows`) with the remaining rows inserted, as a new index file in the same format. rows is
    (n, padded_dim) float32, numpy or a CUDA tensor."""
    m = METRICS[metric] if isinstance(metric, str) else int(metric)
    n, pd = int(rows.shape[0]), int(rows.shape[1])
    buf = np.frombuffer(file_bytes, dtype=np.uint8)
    p = _P()
    nb = ctypes.c_size_t(0)
    ctx.check(lib().vdbgpu_hnsw_extend(ctx._h, m, buf.ctypes.data, buf.size, _ptr(rows), n, int(dim), pd,
                                       ctypes.byref(p), ctypes.byref(nb)))
    try:
        return ctypes.string_at(p, nb.value)
    finally:
        lib().vdbgpu_buffer_free(p)


def build_ivfpq(ctx: Context, rows, dim: int, type="ivf_pq", nlist: int = 1024, pq_m: int = 16,
                max_train_points_per_centroid: int = 256, seed: int = 42) -> bytes:
    """The reference's IVF-PQ (or PQ-flat, type "pq_flat") index file for rows (n, padded_dim)
    float32, numpy or a CUDA tensor, built on the GPU with the reference's seeded k-means replayed
    exactly (IndexOptions nlist, pq_m, max_train_points_per_centroid, seed)."""
    t = INDEX_TYPES[type] if isinstance(type, str) else int(type)
    n, pd = int(rows.shape[0]), int(rows.shape[1])
    p = _P()
    nb = ctypes.c_size_t(0)
    ctx.check(lib().vdbgpu_ivfpq_build(ctx._h, t, _ptr(rows), n, int(dim), pd, int(nlist), int(pq_m),
                                       int(max_train_points_per_centroid), int(seed), ctypes.byref(p),
                                       ctypes.byref(nb)))
    try:
        return ctypes.string_at(p, nb.value)
    finally:
        lib().vdbgpu_buffer_free(p)


def filter_describe(schema, filter) -> Tuple[int, str]:
    """FilterExpr::Parse against a schema without a GPU: (0, description) or (code, message)."""
    import json
    st = schema if isinstance(schema, str) else json.dumps(schema)
    buf = ctypes.create_string_buffer(1 << 16)
    code = lib().vdbgpu_filter_describe(st.encode(), _filter_text(filter), buf, len(buf))
    return code, buf.value.decode(errors="replace")


def inspect_collection(path: str) -> dict:
    """The recovery of Collection.open on the host, without a GPU (vdbgpu_collection_inspect):
    Collection::Stats fields of the directory, the mutable segment first. Raises VdbError."""
    import json
    buf = ctypes.create_string_buffer(1 << 20)
    code = lib().vdbgpu_collection_inspect(os.fspath(path).encode(), buf, len(buf))
    if code != OK:
        raise VdbError(code, buf.value.decode(errors="replace"))
    return json.loads(buf.value.decode())
