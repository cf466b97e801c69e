"""The recovery of a collection directory on the host, without a GPU (vdbgpu_collection_inspect:
the manifest, persisted delete sets and the log replay that vdbgpu_collection_open runs before it
uploads anything), against the reference's own Collection::Stats after Collection::Open of the
same directory (fixtures tests/golden/coll_mutable.npz and coll_deletes.npz). Damaged logs and
delete sets give the reference recovery's errors."""
import json
import os

import numpy as np
import pytest

from helpers import blob, extract_collection, golden


def _inspect(path):
    import vdb_b200
    return vdb_b200.inspect_collection(path)


@pytest.mark.parametrize("name", ["coll_mutable", "coll_deletes"])
def test_recovery_matches_reference_stats(tmp_path, name):
    g = golden(name)
    path = extract_collection(g, tmp_path)
    got, want = _inspect(path), json.loads(str(g["stats"]))
    assert got == want


def _log(path):
    d = os.path.join(path, "wal")
    (name,) = os.listdir(d)
    p = os.path.join(d, name)
    data = open(p, "rb").read()
    recs, pos = [], 16
    while pos < len(data):
        plen = int(np.frombuffer(data, "<u4", 1, pos + 4)[0])
        recs.append((pos, 17 + plen, int(np.frombuffer(data, "<u8", 1, pos + 9)[0])))
        pos += 17 + plen
    return p, data, recs


def test_torn_tail_of_the_newest_log_is_ignored(tmp_path):
    g = golden("coll_mutable")
    path = extract_collection(g, tmp_path)
    p, data, recs = _log(path)
    off, ln, _ = recs[-1]
    open(p, "wb").write(data[:off + ln - 3])  # the last upsert (a new id) cut short
    got, want = _inspect(path), json.loads(str(g["stats"]))
    assert got["recovery_records"] == want["recovery_records"] - 1
    assert got["segments"][0]["rows"] == want["segments"][0]["rows"] - 1
    assert got["live_rows"] == want["live_rows"] - 1
    assert got["segments"][1:] == want["segments"][1:]


@pytest.mark.parametrize("case", ["corrupt_middle", "lsn_gap", "bad_header", "bad_upsert"])
def test_damaged_logs_are_corruption(tmp_path, case):
    import vdb_b200
    from helpers import crc32c
    g = golden("coll_mutable")
    path = extract_collection(g, tmp_path)
    p, data, recs = _log(path)
    off, ln, lsn = recs[len(recs) // 2]
    if case == "corrupt_middle":
        b = bytearray(data)
        b[off + 20] ^= 0xFF
        data, want = bytes(b), f"corrupt log record at offset {off} followed by valid records"
    elif case == "lsn_gap":
        data, want = data[:off] + data[off + ln:], f"log sequence gap: expected LSN {lsn}, found {lsn + 1}"
    elif case == "bad_header":
        data, want = b"VDBWAL02" + data[8:], "bad log file header"
    else:
        # A well-framed upsert whose vector has the wrong dimension (checksum recomputed).
        rec = bytearray(data[off:off + ln])
        assert rec[8] == 1
        rec[17 + 8:17 + 12] = np.array([3], "<u4").tobytes()
        rec[0:4] = np.array([crc32c(bytes(rec[4:]))], "<u4").tobytes()
        data, want = data[:off] + bytes(rec) + data[off + ln:], f"bad upsert record at LSN {lsn}"
    open(p, "wb").write(data)
    with pytest.raises(vdb_b200.VdbError) as e:
        _inspect(path)
    assert e.value.code == vdb_b200.CORRUPTION and want in str(e.value), str(e.value)


def test_damaged_delete_set_is_corruption(tmp_path):
    import vdb_b200
    g = golden("coll_deletes")
    path = extract_collection(g, tmp_path)
    seg = json.loads(g[[k for k in g if k.startswith("file:MANIFEST-")][0]].tobytes()[24:])["segments"][2]
    payload = np.array([12347], "<u4").tobytes() + b"\x01" + np.array([0, 19, 1, 2990, 19], "<u2").tobytes()
    with open(os.path.join(path, "segments", f"seg-{seg['id']:06d}", seg["deletes_file"]), "wb") as f:
        f.write(blob(b"VDBDEL01", payload))
    with pytest.raises(vdb_b200.VdbError) as e:
        _inspect(path)
    assert e.value.code == vdb_b200.CORRUPTION and "delete set out of range" in str(e.value)



def _fuzz(tmp_path, name, pick, mutate, n, seed):
    """Mutations of one file of a fixture directory, checksums recomputed so that the decoders
    behind them see the damage: recovery returns a status for each (OK or one of the reference's
    codes) and never fails otherwise (no crash, no unbounded allocation)."""
    import vdb_b200
    g = golden(name)
    base = extract_collection(g, tmp_path / "base")
    target = pick(base, g)
    orig = open(target, "rb").read()
    rng = np.random.default_rng(seed)
    codes = {}
    for _ in range(n):
        open(target, "wb").write(mutate(orig, rng))
        try:
            vdb_b200.inspect_collection(base)
            codes[0] = codes.get(0, 0) + 1
        except vdb_b200.VdbError as e:
            assert e.code in (vdb_b200.CORRUPTION, vdb_b200.INVALID_ARGUMENT, vdb_b200.NOT_FOUND,
                              vdb_b200.IO_ERROR, vdb_b200.RESOURCE_EXHAUSTED), str(e)
            codes[e.code] = codes.get(e.code, 0) + 1
    return codes


def _damage(p: bytes, rng) -> bytes:
    b = bytearray(p)
    kind = int(rng.integers(0, 3))
    if kind == 0:
        for _ in range(int(rng.integers(1, 6))):
            b[int(rng.integers(0, len(b)))] ^= 1 << int(rng.integers(0, 8))
    elif kind == 1:
        b = b[:int(rng.integers(0, len(b)))]
    else:
        i = int(rng.integers(0, len(b) + 1))
        b[i:i] = bytes(rng.integers(0, 256, int(rng.integers(1, 9)), dtype=np.uint8))
    return bytes(b)


def _reblob(orig, rng):
    """A blob file (delete set, manifest) with a damaged payload and a valid checksum."""
    return blob(orig[:8], _damage(orig[24:], rng))


def _relog(orig, rng):
    """A log with one record damaged after its checksum field (type, LSN, payload), checksum
    recomputed; or the raw bytes damaged, framing included."""
    from helpers import crc32c
    if rng.random() < 0.25:
        return orig[:16] + _damage(orig[16:], rng)
    recs, pos = [], 16
    while pos < len(orig):
        plen = int(np.frombuffer(orig, "<u4", 1, pos + 4)[0])
        recs.append((pos, 17 + plen))
        pos += 17 + plen
    off, ln = recs[int(rng.integers(0, len(recs)))]
    r = bytearray(orig[off:off + ln])
    for _ in range(int(rng.integers(1, 4))):
        r[int(rng.integers(8, len(r)))] ^= 1 << int(rng.integers(0, 8))
    r[0:4] = np.array([crc32c(bytes(r[4:]))], "<u4").tobytes()
    return orig[:off] + bytes(r) + orig[off + ln:]


def _revectors(orig, rng):
    """A segment's vectors.f32 with bytes flipped in its rows (a data checksum mismatch), or in its
    4 KiB header with the header checksum recomputed half the time (reaching the field checks)."""
    from helpers import crc32c
    b = bytearray(orig)
    if rng.random() < 0.5:
        for _ in range(int(rng.integers(1, 4))):
            b[4096 + int(rng.integers(0, len(b) - 4096))] ^= 1 << int(rng.integers(0, 8))
    else:
        b[int(rng.integers(0, 64))] ^= 1 << int(rng.integers(0, 8))
        if rng.random() < 0.5:
            b[4092:4096] = np.array([crc32c(bytes(b[:4092]))], "<u4").tobytes()
    return bytes(b)


def _vectors_path(p, g):
    seg = json.loads(g[[k for k in g if k.startswith("file:MANIFEST-")][0]].tobytes()[24:])["segments"][1]
    return os.path.join(p, "segments", f"seg-{seg['id']:06d}", "vectors.f32")


def _reindex(orig, rng):
    """An index file with bytes flipped (its checksum then fails), or with its magic changed and the
    checksum recomputed (an unknown magic). Damage to the body behind a valid checksum is found
    when the index is loaded onto a GPU, so it is not made here."""
    from helpers import crc32c
    b = bytearray(orig)
    if rng.random() < 0.6:
        b[int(rng.integers(0, len(b)))] ^= 1 << int(rng.integers(0, 8))
    else:
        b[int(rng.integers(0, 8))] ^= 1 << int(rng.integers(0, 8))
        b[-4:] = np.array([crc32c(bytes(b[:-4]))], "<u4").tobytes()
    return bytes(b)


def _segment_file(name):
    def pick(p, g):
        seg = json.loads(g[[k for k in g if k.startswith("file:MANIFEST-")][0]].tobytes()[24:])["segments"][1]
        d = os.path.join(p, "segments", f"seg-{seg['id']:06d}")
        return os.path.join(d, name if name != "index" else [f for f in os.listdir(d) if f.startswith("index.")][0])
    return pick


def _manifest_path(p, g):
    return os.path.join(p, [k for k in g if k.startswith("file:MANIFEST-")][0][5:])


def test_fuzzed_logs_never_crash(tmp_path):
    import vdb_b200
    codes = _fuzz(tmp_path, "coll_mutable", lambda p, g: _log(p)[0], _relog, 250, 1)
    assert codes.get(vdb_b200.CORRUPTION, 0) > 0 and codes.get(0, 0) > 0


def test_fuzzed_delete_sets_never_crash(tmp_path):
    import vdb_b200

    def pick(p, g):
        seg = json.loads(g[[k for k in g if k.startswith("file:MANIFEST-")][0]].tobytes()[24:])["segments"][0]
        return os.path.join(p, "segments", f"seg-{seg['id']:06d}", seg["deletes_file"])
    codes = _fuzz(tmp_path, "coll_deletes", pick, _reblob, 150, 2)
    assert codes.get(vdb_b200.CORRUPTION, 0) > 0 and codes.get(0, 0) > 0


def test_fuzzed_manifests_never_crash(tmp_path):
    import vdb_b200
    codes = _fuzz(tmp_path, "coll_mutable", _manifest_path, _reblob, 200, 3)
    assert codes.get(vdb_b200.CORRUPTION, 0) > 0


@pytest.mark.parametrize("which", ["manifest", "log", "vectors", "ids", "meta", "index"])
def test_recovery_matches_live_reference_on_damaged_directories(tmp_path, which):
    """Damaged copies of the mutable fixture (manifest payloads, log records, a segment's vectors
    file; checksums recomputed where they would stop the damage early) recovered by the reference's own Collection::Open and by inspect: the same status
    code class, the same message, and when both open, the same Stats. Needs the reference engine
    (oracle/_ref), built from the reference sources where they are present."""
    import shutil

    import oracle
    import vdb_b200
    if not os.path.exists(oracle.REF_ENGINE_LIB):
        pytest.skip("the reference engine is not built here")
    g = golden("coll_mutable")
    base = extract_collection(g, tmp_path / "base")
    target = {"manifest": _manifest_path, "log": lambda p, g: _log(p)[0], "vectors": _vectors_path,
              "ids": _segment_file("ids.u64"), "meta": _segment_file("meta.bin"),
              "index": _segment_file("index")}[which](base, g)
    mutate = {"manifest": _reblob, "log": _relog, "vectors": _revectors, "ids": _reblob, "meta": _reblob,
              "index": _reindex}[which]
    orig = open(target, "rb").read()
    rng = np.random.default_rng(21)
    bad = []
    for it in range(80):
        open(target, "wb").write(mutate(orig, rng))
        try:
            ours = (0, vdb_b200.inspect_collection(base))
        except vdb_b200.VdbError as e:
            ours = (e.code, str(e).split(": ", 1)[1])
        copy = str(tmp_path / f"copy{it}")
        shutil.copytree(base, copy)  # the reference's recovery writes into the directory
        try:
            c = oracle.RefCollection.open(copy, threads=1)
            ref = (0, c.stats())
            c.close()
        except RuntimeError as e:
            ref = (-1, str(e))
        shutil.rmtree(copy)
        if (ours[0] == 0) != (ref[0] == 0) or (ours[0] == 0 and ours[1] != ref[1]) or \
                (ours[0] != 0 and ours[1].replace(base, copy) not in ref[1]):
            bad.append((it, str(ours)[:160], str(ref)[:160]))
    assert not bad, bad[:4]


def test_recovery_matches_live_reference_on_random_histories(tmp_path):
    """100 random write histories run by the reference's own Collection (bulk loads, upserts of
    new and existing ids with and without metadata, removals of live and absent ids, flushes, on
    collections of every index type, L2 and cosine), closed, then recovered by the reference's
    Collection::Open and by inspect: Stats identical. Needs the reference engine (oracle/_ref)."""
    import shutil

    import oracle
    import vdb_b200
    if not os.path.exists(oracle.REF_ENGINE_LIB):
        pytest.skip("the reference engine is not built here")
    bad = []
    for sc in range(100):
        rng = np.random.default_rng(4000 + sc)
        path, copy = str(tmp_path / f"c{sc}"), str(tmp_path / f"r{sc}")
        dim = 8
        index = {"type": str(rng.choice(["flat", "hnsw", "hnsw_sq8", "pq", "ivf_pq"])), "M": 8,
                 "ef_construction": 32, "pq_m": 4, "nlist": 4}
        c = oracle.RefCollection(path, dim, metric=str(rng.choice(["l2", "cosine"])), index=index,
                                 schema=[{"name": "year", "type": "int64"}], threads=1)
        live, next_id = [], 1
        for _ in range(int(rng.integers(3, 12))):
            op = rng.random()
            if op < 0.25:
                m = int(rng.integers(1, 300))
                ids = np.arange(next_id, next_id + m, dtype=np.uint64)
                next_id += m
                c.bulk_load(ids, rng.standard_normal((m, dim)).astype(np.float32))
                live += ids.tolist()
            elif op < 0.6:
                m = int(rng.integers(1, 60))
                if live and rng.random() < 0.5:
                    ids = np.array([live[int(i)] for i in rng.integers(0, len(live), m)], np.uint64)
                else:
                    ids = np.arange(next_id, next_id + m, dtype=np.uint64)
                    next_id += m
                meta = [None if rng.random() < 0.5 else {"year": int(rng.integers(1990, 2030))} for _ in range(m)]
                c.upsert(ids, rng.standard_normal((m, dim)).astype(np.float32), meta)
                live = sorted(set(live) | set(ids.tolist()))
            elif op < 0.85:
                m = int(rng.integers(1, 40))
                ids = np.array([live[int(i)] for i in rng.integers(0, len(live), m)] if live else [1], np.uint64)
                c.remove(np.concatenate([ids, np.array([10**9], np.uint64)]))
                live = sorted(set(live) - set(ids.tolist()))
            else:
                c.flush()
        c.close()
        shutil.copytree(path, copy)  # the reference's recovery writes into the directory
        ours = vdb_b200.inspect_collection(path)
        r = oracle.RefCollection.open(copy, threads=1)
        want = r.stats()
        r.close()
        if ours != want:
            bad.append((sc, ours, want))
        shutil.rmtree(path)
        shutil.rmtree(copy)
    assert not bad, bad[:2]


def test_inspect_errors_through_the_c_abi(tmp_path):
    """A missing directory is the reference's IOError text for CURRENT; a buffer too small for the
    JSON is VDBGPU_RESOURCE_EXHAUSTED with a truncated, terminated prefix; a null path is
    VDBGPU_INVALID_ARGUMENT."""
    import ctypes

    import vdb_b200
    lib = vdb_b200.lib()
    buf = ctypes.create_string_buffer(256)
    missing = str(tmp_path / "nope")
    assert lib.vdbgpu_collection_inspect(missing.encode(), buf, len(buf)) == vdb_b200.IO_ERROR
    assert buf.value.decode() == f"open {missing}/CURRENT: No such file or directory"
    path = extract_collection(golden("coll_mutable"), tmp_path)
    small = ctypes.create_string_buffer(16)
    assert lib.vdbgpu_collection_inspect(path.encode(), small, len(small)) == vdb_b200.RESOURCE_EXHAUSTED
    assert small.value.decode() == json.dumps(_inspect(path), separators=(",", ":"))[:15]
    assert lib.vdbgpu_collection_inspect(None, buf, len(buf)) == vdb_b200.INVALID_ARGUMENT


def test_random_delete_sets_decode_as_the_reference(tmp_path):
    """Random delete sets over the 200,000-row fixture segment (sparse rows, dense ranges, every
    other row of a key, whole keys; serialized with and without run containers, so every cookie,
    container kind and offset layout occurs) recovered by inspect: the deleted count is the set's
    size, and where the reference engine is built, equal to its Collection::Open."""
    import shutil

    import oracle
    import vdb_b200
    from helpers import decode_portable_roaring, encode_portable_roaring
    live_ref = os.path.exists(oracle.REF_ENGINE_LIB)
    g = golden("coll_deletes")
    path = extract_collection(g, tmp_path / "base")
    seg = json.loads(g[[k for k in g if k.startswith("file:MANIFEST-")][0]].tobytes()[24:])["segments"][0]
    target = os.path.join(path, "segments", f"seg-{seg['id']:06d}", seg["deletes_file"])
    rows = seg["rows"]
    rng = np.random.default_rng(31)
    kinds_seen = set()
    for it in range(40):
        parts = []
        for _ in range(int(rng.integers(1, 6))):
            kind = int(rng.integers(0, 4))
            if kind == 0:
                parts.append(rng.choice(rows, int(rng.integers(1, 3000)), replace=False))
            elif kind == 1:
                a = int(rng.integers(0, rows - 1))
                parts.append(np.arange(a, min(rows, a + int(rng.integers(1, 20000)))))
            elif kind == 2:
                key = int(rng.integers(0, rows >> 16))
                parts.append(np.arange(key << 16, min(rows, (key + 1) << 16), int(rng.integers(2, 4))))
            else:
                key = int(rng.integers(0, (rows >> 16) + 1))
                parts.append(np.arange(key << 16, min(rows, (key + 1) << 16)))
        want = np.unique(np.concatenate(parts))
        payload = encode_portable_roaring(want, runs=bool(it % 2))
        got_vals, kinds, _, _ = decode_portable_roaring(payload)
        assert np.array_equal(got_vals, want)
        kinds_seen |= set(kinds)
        open(target, "wb").write(blob(b"VDBDEL01", payload))
        st = vdb_b200.inspect_collection(path)
        assert st["segments"][1]["deleted"] == want.size
        if live_ref:
            copy = str(tmp_path / f"r{it}")
            shutil.copytree(path, copy)
            r = oracle.RefCollection.open(copy, threads=1)
            assert r.stats() == st
            r.close()
            shutil.rmtree(copy)
    assert kinds_seen == {"array", "bitmap", "run"}


@pytest.mark.parametrize("name", ["coll_hnsw", "coll_ivfpq", "coll_flat"])
def test_every_collection_fixture_passes_recovery(tmp_path, name):
    """The read-path fixtures pass every recovery check that Collection.open runs before its
    uploads (segment headers and data checksums, ids, metadata rows, index framing)."""
    import vdb_b200
    g = golden(name)
    st = vdb_b200.inspect_collection(extract_collection(g, tmp_path))
    assert [s["rows"] for s in st["segments"][1:]] == [int(x) for x in g["sizes"]]
    assert st["live_rows"] == int(np.sum(g["sizes"]))
