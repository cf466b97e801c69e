"""GPU parity for batched HNSW search over the reference's own index.hnsw / index.hnsw_sq8 files:
the same graph and inputs give the same neighbours, distances and distance computations as the
reference (golden fixtures made by running it)."""
import numpy as np
import pytest

import oracle
from helpers import golden, inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["pooled", "shared_memory"], autouse=True)
def walk_mode(request, monkeypatch):
    """Every test runs with both walk state layouts: pooled (the default: visited bits and
    candidates beyond a sorted front in global memory) and the shared-memory arrays kept for
    unfiltered walks when VDB_HNSW_POOLED_EF is large."""
    if request.param == "shared_memory":
        monkeypatch.setenv("VDB_HNSW_POOLED_EF", "1000000")
    else:
        monkeypatch.delenv("VDB_HNSW_POOLED_EF", raising=False)
    return request.param


def test_hnsw_matches_reference_exactly(ctx):
    import vdb_b200
    g = golden("hnsw")
    base, qs = inputs("hnsw", g)
    idx = vdb_b200.Index.load(ctx, bytes(g["index_file"]), "l2", base, 128)
    assert idx.type == 1 and idx.rows == base.shape[0]
    for ef in (16, 64, 128):
        ids, d, dc = idx.search(qs, k=10, ef=ef, stats=True)
        np.testing.assert_array_equal(ids, g[f"ids_ef{ef}"])
        np.testing.assert_array_equal(d, g[f"dists_ef{ef}"])
        np.testing.assert_array_equal(dc, g[f"dc_ef{ef}"])


def test_hnsw_filtered_matches_reference(ctx):
    import vdb_b200
    g = golden("hnsw")
    base, qs = inputs("hnsw", g)
    idx = vdb_b200.Index.load(ctx, bytes(g["index_file"]), "l2", base, 128)
    even = (np.arange(base.shape[0]) % 2) == 0
    ids, d, dc = idx.search(qs, k=10, ef=64, filter=vdb_b200.pack_bitset(even), stats=True)
    np.testing.assert_array_equal(ids, g["filt_ids"])
    np.testing.assert_array_equal(d, g["filt_dists"])
    np.testing.assert_array_equal(dc, g["filt_dc"])
    assert np.all(ids % 2 == 0)


def test_hnsw_sq8_matches_reference_exactly(ctx):
    import vdb_b200
    g = golden("hnsw_sq8")
    base, qs = inputs("hnsw_sq8", g)
    idx = vdb_b200.Index.load(ctx, bytes(g["index_file"]), "l2", base, 128)
    assert idx.type == 2
    for ef, rr in ((32, -1), (64, -1), (64, 0), (64, 20)):
        tag = f"ef{ef}_r{'auto' if rr < 0 else rr}"
        ids, d, dc = idx.search(qs, k=10, ef=ef, rerank=rr, stats=True)
        np.testing.assert_array_equal(ids, g[f"ids_{tag}"])
        np.testing.assert_array_equal(d, g[f"dists_{tag}"])
        np.testing.assert_array_equal(dc, g[f"dc_{tag}"])


def test_hnsw_rejects_corrupt_files(ctx):
    import vdb_b200
    g = golden("hnsw")
    base, _ = inputs("hnsw", g)
    data = bytearray(bytes(g["index_file"]))
    data[len(data) // 3] ^= 0x5A
    with pytest.raises(vdb_b200.VdbError) as e:
        vdb_b200.Index.load(ctx, bytes(data), "l2", base, 128)
    assert e.value.code == 5
    with pytest.raises(vdb_b200.VdbError):
        vdb_b200.Index.load(ctx, bytes(g["index_file"]), "l2", base[:100], 128)
