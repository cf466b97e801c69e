"""Shared test helpers: regenerate the seeded inputs behind each golden fixture and check them."""
import hashlib
import os

import numpy as np

from conftest import golden  # noqa: F401  (re-exported)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def inputs(name, g):
    """(base, queries) of golden fixture `name`, regenerated and checked against its SHA-256."""
    from vdb_b200 import synth
    seed = int(g["seed"])
    n, nq = int(g["n"]), int(g["nq"])
    if name in ("flat_int", "hnsw", "hnsw_sq8"):
        b, q = synth.flat_int(n, nq, dim=128, seed=seed)
    elif name == "flat_float":
        b, q = synth.sharded_cosine(n, nq, dim=int(g["dim"]), seed=seed)
    elif name == "sq8_scan":
        b, q = synth.sq8_cosine(n, nq, dim=128, seed=seed)
    elif name in ("ivfpq", "pqflat"):
        b, q = synth.ivfpq_l2(n, nq, dim=96, seed=seed)
    else:
        raise KeyError(name)
    assert sha(b) == str(g["base_sha"]), f"{name}: regenerated base rows differ from the fixture's"
    assert sha(q) == str(g["query_sha"]), f"{name}: regenerated queries differ from the fixture's"
    return b, q


def assert_same_neighbors(ids_a, d_a, ids_b, d_b, rel=1e-4, exact_dist=True):
    """Ids identical except swaps inside distance ties (within rel); distances bit-equal where
    the ids agree when exact_dist."""
    import oracle
    assert ids_a.shape == ids_b.shape
    assert oracle.ids_match_up_to_ties(ids_a, d_a, ids_b, d_b, rel=rel)
    if exact_dist:
        same = ids_a == ids_b
        np.testing.assert_array_equal(d_a[same], d_b[same])


def extract_collection(g, dest):
    """Writes the collection directory stored in a coll_* fixture (keys "file:<relpath>") under
    dest and returns its path."""
    import os
    path = os.path.join(str(dest), "coll")
    for key in g:
        if not key.startswith("file:"):
            continue
        full = os.path.join(path, key[5:])
        os.makedirs(os.path.dirname(full), exist_ok=True)
        with open(full, "wb") as f:
            f.write(np.asarray(g[key]).tobytes())
    return path


def crc32c(data: bytes) -> int:
    """CRC-32C (Castagnoli, reflected polynomial 0x82F63B78), bitwise; small inputs only."""
    crc = 0xFFFFFFFF
    for b in data:
        crc ^= b
        for _ in range(8):
            crc = (crc >> 1) ^ (0x82F63B78 & -(crc & 1))
    return crc ^ 0xFFFFFFFF


def blob(magic: bytes, payload: bytes) -> bytes:
    """A reference blob file (src/storage/file_format.cc): magic 8, u32 version 1, u32 crc32c of
    the payload, u64 payload length, the payload."""
    return magic + np.array([1, crc32c(payload)], "<u4").tobytes() + np.array([len(payload)], "<u8").tobytes() + payload


def decode_portable_roaring(p: bytes):
    """CRoaring's portable serialization (RoaringFormatSpec) to (sorted values, per-container
    kinds "array" / "bitmap" / "run", cookie, container count). Test-side reader for fixtures."""
    at = 0

    def take(fmt, n):
        nonlocal at
        v = np.frombuffer(p, fmt, n, at)
        at += v.nbytes
        return v

    cookie = int(take("<u4", 1)[0])
    if cookie & 0xFFFF == 12347:
        count = (cookie >> 16) + 1
        runbits = take("u1", (count + 7) // 8)
        isrun = [bool(runbits[i // 8] >> (i % 8) & 1) for i in range(count)]
    else:
        assert cookie == 12346
        count = int(take("<u4", 1)[0])
        isrun = [False] * count
    hdr = take("<u2", 2 * count).reshape(count, 2)
    if not any(isrun) or count >= 4:
        take("<u4", count)
    vals, kinds = [], []
    for i in range(count):
        hi = int(hdr[i, 0]) << 16
        card = int(hdr[i, 1]) + 1
        if isrun[i]:
            n = int(take("<u2", 1)[0])
            r = take("<u2", 2 * n).reshape(n, 2).astype(np.int64)
            for s, l in r:
                vals.append(hi + np.arange(s, s + l + 1))
            kinds.append("run")
        elif card > 4096:
            bits = np.unpackbits(take("u1", 8192), bitorder="little")
            vals.append(hi + np.nonzero(bits)[0])
            kinds.append("bitmap")
        else:
            vals.append(hi + take("<u2", card).astype(np.int64))
            kinds.append("array")
    assert at == len(p)
    v = np.concatenate(vals) if vals else np.zeros(0, np.int64)
    return v, kinds, cookie & 0xFFFF, count


def encode_portable_roaring(values, runs=True) -> bytes:
    """Sorted distinct uint32 values in CRoaring's portable serialization (RoaringFormatSpec):
    per 16-bit key an array (<= 4096 values) or bitmap container, or with runs=True a run
    container where that is smaller. Test-side writer for fixtures."""
    v = np.unique(np.asarray(values, dtype=np.int64))
    keys = np.unique(v >> 16)
    conts = []
    for key in keys:
        lo = (v[(v >> 16) == key] & 0xFFFF).astype(np.int64)
        starts = np.concatenate([[0], np.nonzero(np.diff(lo) != 1)[0] + 1])
        ends = np.concatenate([starts[1:], [lo.size]]) - 1
        kind = "bitmap" if lo.size > 4096 else "array"
        base = 8192 if kind == "bitmap" else 2 + 2 * lo.size
        if runs and 2 + 4 * starts.size < base:
            kind = "run"
        if kind == "run":
            body = np.array([starts.size], "<u2").tobytes() + np.stack(
                [lo[starts], lo[ends] - lo[starts]], 1).astype("<u2").tobytes()
        elif kind == "bitmap":
            bits = np.zeros(65536, np.uint8)
            bits[lo] = 1
            body = np.packbits(bits, bitorder="little").tobytes()
        else:
            body = lo.astype("<u2").tobytes()
        conts.append((int(key), lo.size, kind, body))
    n = len(conts)
    has_runs = any(c[2] == "run" for c in conts)
    if has_runs:
        bits = np.zeros((n + 7) // 8, np.uint8)
        for i, c in enumerate(conts):
            if c[2] == "run":
                bits[i // 8] |= 1 << (i % 8)
        head = np.array([12347 | ((n - 1) << 16)], "<u4").tobytes() + bits.tobytes()
    else:
        head = np.array([12346, n], "<u4").tobytes()
    head += np.array([[c[0], c[1] - 1] for c in conts], "<u2").reshape(-1).tobytes()
    if not has_runs or n >= 4:
        off = len(head) + 4 * n
        offs = []
        for c in conts:
            offs.append(off)
            off += len(c[3])
        head += np.array(offs, "<u4").tobytes()
    return head + b"".join(c[3] for c in conts)
