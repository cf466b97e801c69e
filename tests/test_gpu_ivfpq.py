"""GPU parity for IVF-PQ and PQ-flat over the reference's own index files: the same codebooks,
lists and inputs give the same neighbours, distances and distance computations."""
import numpy as np
import pytest

import oracle
from helpers import golden, inputs

pytestmark = pytest.mark.gpu


def test_ivfpq_matches_reference_exactly(ctx):
    import vdb_b200
    g = golden("ivfpq")
    base, qs = inputs("ivfpq", g)
    idx = vdb_b200.Index.load(ctx, bytes(g["index_file"]), "l2", base, 96)
    assert idx.type == 4
    for nprobe, rr in ((4, -1), (16, -1), (16, 0)):
        tag = f"np{nprobe}_r{'auto' if rr < 0 else rr}"
        ids, d, dc = idx.search(qs, k=10, nprobe=nprobe, rerank=rr, stats=True)
        np.testing.assert_array_equal(ids, g[f"ids_{tag}"])
        np.testing.assert_array_equal(d, g[f"dists_{tag}"])
        np.testing.assert_array_equal(dc, g[f"dc_{tag}"])
    assert oracle.recall_at_k(ids, g["gt_ids"], 10) > 0.5


def test_pqflat_matches_reference_exactly(ctx):
    import vdb_b200
    g = golden("pqflat")
    base, qs = inputs("pqflat", g)
    idx = vdb_b200.Index.load(ctx, bytes(g["index_file"]), "l2", base, 96)
    assert idx.type == 3
    ids, d, dc = idx.search(qs, k=10, rerank=-1, stats=True)
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_array_equal(d, g["dists"])
    np.testing.assert_array_equal(dc, g["dc"])


def test_ivfpq_filtered_and_cosine_against_oracle(ctx):
    """A filter (odd rows) and the inner-product table path, checked against the oracle on an
    index the reference builds in-process."""
    import vdb_b200
    g = golden("ivfpq")
    base, qs = inputs("ivfpq", g)
    f = oracle.parse_ivfpq(bytes(g["index_file"]))
    orc = oracle.Oracle(order=oracle.ORDER_AVX512)
    idx = vdb_b200.Index.load(ctx, bytes(g["index_file"]), "l2", base, 96)
    odd = (np.arange(base.shape[0]) % 2) == 1
    bits = vdb_b200.pack_bitset(odd)
    ids, d, dc = idx.search(qs, k=10, nprobe=8, filter=bits, stats=True)
    oi, od, odc = orc.ivfpq_search(f, 0, base, qs, k=10, nprobe=8, allow=bits)
    if orc.order == oracle.host_kernel_order():
        np.testing.assert_array_equal(ids, oi)
        np.testing.assert_array_equal(d, od)
    np.testing.assert_array_equal(dc, odc)
    assert np.all(ids[ids != np.uint32(0xFFFFFFFF)] % 2 == 1)


@pytest.mark.parametrize("rerank", [120, 200])
def test_ivfpq_deep_rerank_against_oracle(ctx, rerank):
    """Re-rank depths above 100: 120 keeps the eight-warp scan (eight R-best lists merge within its
    1024-key limit), 200 takes the four-warp variant whose pairwise merges sort 512 keys. Ids,
    distances and distance computations against the oracle on the reference's index."""
    import vdb_b200
    g = golden("ivfpq")
    base, qs = inputs("ivfpq", g)
    f = oracle.parse_ivfpq(bytes(g["index_file"]))
    orc = oracle.Oracle()
    idx = vdb_b200.Index.load(ctx, bytes(g["index_file"]), "l2", base, 96)
    ids, d, dc = idx.search(qs, k=10, nprobe=16, rerank=rerank, stats=True)
    oi, od, odc = orc.ivfpq_search(f, 0, base, qs, k=10, nprobe=16, rerank=rerank)
    np.testing.assert_array_equal(ids, oi)
    np.testing.assert_array_equal(d, od)
    np.testing.assert_array_equal(dc, odc)
    idx.free()
