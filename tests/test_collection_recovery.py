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
