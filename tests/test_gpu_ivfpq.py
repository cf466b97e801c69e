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


def test_ivfpq_filtered_against_oracle(ctx):
    """A filter (odd rows) on the reference's L2 index, checked against the oracle summing in the
    kernel set this host's reference would pick (the GPU follows the same one)."""
    import vdb_b200
    g = golden("ivfpq")
    base, qs = inputs("ivfpq", g)
    f = oracle.parse_ivfpq(bytes(g["index_file"]))
    orc = oracle.Oracle()
    assert orc.order == oracle.host_kernel_order()
    idx = vdb_b200.Index.load(ctx, bytes(g["index_file"]), "l2", base, 96)
    odd = (np.arange(base.shape[0]) % 2) == 1
    bits = vdb_b200.pack_bitset(odd)
    ids, d, dc = idx.search(qs, k=10, nprobe=8, filter=bits, stats=True)
    oi, od, odc = orc.ivfpq_search(f, 0, base, qs, k=10, nprobe=8, allow=bits)
    np.testing.assert_array_equal(ids, oi)
    np.testing.assert_array_equal(d, od)
    np.testing.assert_array_equal(dc, odc)
    assert np.all(ids[ids != np.uint32(0xFFFFFFFF)] % 2 == 1)


@pytest.mark.parametrize("metric", ["ip", "cosine"])
def test_ivfpq_and_pqflat_inner_product_match_reference(ctx, metric):
    """Inner-product and cosine indexes built by the reference in this process: the coarse step
    ranks lists by -<q, c>, one table -<q_j, C_j[c]> serves every probed list and each list adds
    the offset -<q, c_l> (src/index/quant/ivf_pq.cc:188-211); PQ-flat shares the table path
    (ivf_pq.cc:59-76). Ids, distances and distance computations equal the reference's on every
    query, with a filter too."""
    import vdb_b200
    from vdb_b200 import synth
    m = oracle.IP if metric == "ip" else oracle.COSINE
    base, qs = synth.ivfpq_l2(20_000, 200, dim=96, seed=31)
    ref = oracle.Ref()
    if metric == "cosine":
        # Rows and queries normalised by the reference's own NormalizeVector, as ingest and
        # PrepareQuery do for a cosine collection.
        ref.normalize_rows(base, 96)
        ref.normalize_rows(qs, 96)
    for type_, name in ((4, "ivf_pq"), (3, "pq_flat")):
        rindex = ref.build_index(type_, m, base, 96, pq_m=48, nlist=64, seed=42, threads=0)
        idx = vdb_b200.Index.load(ctx, rindex.save(), metric, base, 96)
        assert idx.type == type_
        for nprobe, rr in ((8, -1), (16, 0), (16, 150)):
            ids, d, dc = idx.search(qs, k=10, nprobe=nprobe, rerank=rr, stats=True)
            rids, rd, rdc = rindex.search(qs, k=10, nprobe=nprobe, rerank=rr)
            np.testing.assert_array_equal(ids, rids, err_msg=f"{name} nprobe {nprobe} re-rank {rr}")
            np.testing.assert_array_equal(d, rd, err_msg=f"{name} nprobe {nprobe} re-rank {rr}")
            np.testing.assert_array_equal(dc, rdc, err_msg=f"{name} nprobe {nprobe} re-rank {rr}")
        bits = vdb_b200.pack_bitset((np.arange(base.shape[0]) % 5) != 0)
        ids, d, dc = idx.search(qs, k=10, nprobe=8, filter=bits, stats=True)
        rids, rd, rdc = rindex.search(qs, k=10, nprobe=8, allow=bits)
        np.testing.assert_array_equal(ids, rids)
        np.testing.assert_array_equal(d, rd)
        np.testing.assert_array_equal(dc, rdc)
        idx.free()


def test_ivfpq_residual_tables_match_reference(ctx):
    """Above 1 GiB of precomputed tables (nlist x m x 256 floats, kMaxPrecomputedBytes in
    src/index/quant/ivf_pq.h:61) neither side builds term2; each probed list then gets a table of
    the query's residual to its centroid (ivf_pq.cc:206-208). 16,385 lists x 64 subquantizers
    cross that limit: the index is built by the GPU builder (the reference's index file), and the
    reference's own IvfPqIndex loads the same file and searches it."""
    import vdb_b200
    from vdb_b200 import synth
    nlist, pq_m, dim = 16_385, 64, 128
    n = 39 * nlist  # the reference clamps nlist to rows / 39
    assert nlist * pq_m * 256 * 4 > (1 << 30)
    rows = synth.mixture(n, dim, 1000, centres="uniform", lo=-1.0, hi=1.0, sigma=0.15, seed=33, stream=0)
    qs = synth.mixture(600, dim, 1000, centres="uniform", lo=-1.0, hi=1.0, sigma=0.15, seed=33, stream=1)
    data = vdb_b200.build_ivfpq(ctx, rows, dim, nlist=nlist, pq_m=pq_m, max_train_points_per_centroid=39, seed=42)
    f = oracle.parse_ivfpq(data)
    assert f.nlist == nlist
    idx = vdb_b200.Index.load(ctx, data, "l2", rows, dim)
    rindex = oracle.Ref().load_index(data, oracle.L2, rows, dim, pq_m=pq_m)
    # 100 queries take the per-query kernel, 600 the tensor-core pre-rank (residual tables in its
    # exact stage).
    for nprobe, rr in ((16, -1), (32, 0)):
        for q in (qs[:100], qs):
            ids, d, dc = idx.search(q, k=10, nprobe=nprobe, rerank=rr, stats=True)
            rids, rd, rdc = rindex.search(q, k=10, nprobe=nprobe, rerank=rr)
            np.testing.assert_array_equal(ids, rids)
            np.testing.assert_array_equal(d, rd)
            np.testing.assert_array_equal(dc, rdc)
    idx.free()


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
