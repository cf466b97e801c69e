"""IVF-PQ search of large batches with the tensor-core pre-rank (the list mode of the scan,
hnsw-vector-db_b200/csrc/ivf_mma.cu): batches of at least 512 unfiltered L2 queries are cut into
query tiles per probed list, the rows of each list are keyed on fp16 decoded residuals, and the
cpre best keys per query go to the exact stage, which computes the reference's ADC (four partial
sums of term2 + 2 * (-<q_j, C_j[c]>), or the residual tables) and re-ranks on fp32 rows
(IvfPqIndex::search, src/index/quant/ivf_pq.cc:169-222). Ids, distances and distance computations
equal the reference's own IvfPqIndex search of the same file, and the per-query kernel's
(VDB_IVF_TENSOR=0)."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

DIM, PQ_M = 96, 48


def _data(n, nq, seed):
    from vdb_b200 import synth
    rows = synth.mixture(n, DIM, 1000, centres="uniform", lo=-1.0, hi=1.0, sigma=0.15, seed=seed, stream=0)
    qs = synth.mixture(nq, DIM, 1000, centres="uniform", lo=-1.0, hi=1.0, sigma=0.15, seed=seed, stream=1)
    return rows, qs


# (rows, nlist, queries, nprobe, rerank). 1,024 lists of about 98 rows: a query's nearest list
# holds fewer rows than the exact stage takes (128 for re-rank depth 100), so no bound is published
# before the full scan, every row of the probed lists stays a candidate, and the exact stage cuts
# them to its 128 by a radix select over the lists.
CASES = [(200_000, 256, 1500, 16, -1), (200_000, 256, 1500, 32, 0), (100_000, 1024, 600, 16, -1)]


@pytest.mark.parametrize("case", CASES, ids=["np16_r100", "np32_r0", "small_lists"])
def test_tensor_prerank_matches_reference(ctx, monkeypatch, case):
    import vdb_b200
    n, nlist, nq, nprobe, rr = case
    rows, qs = _data(n, nq, seed=41 + nlist)
    data = vdb_b200.build_ivfpq(ctx, rows, DIM, nlist=nlist, pq_m=PQ_M, max_train_points_per_centroid=64, seed=42)
    idx = vdb_b200.Index.load(ctx, data, "l2", rows, DIM)
    ids, d, dc = idx.search(qs, k=10, nprobe=nprobe, rerank=rr, stats=True)
    rindex = oracle.Ref().load_index(data, oracle.L2, rows, DIM, pq_m=PQ_M)
    rids, rd, rdc = rindex.search(qs, k=10, nprobe=nprobe, rerank=rr)
    bad = np.nonzero(~np.all(ids == rids, axis=1))[0]
    assert bad.size == 0, (bad.size, bad[:5].tolist())
    np.testing.assert_array_equal(d, rd)
    np.testing.assert_array_equal(dc, rdc)
    monkeypatch.setenv("VDB_IVF_TENSOR", "0")
    pids, pdist, pdc = idx.search(qs, k=10, nprobe=nprobe, rerank=rr, stats=True)
    np.testing.assert_array_equal(ids, pids)
    np.testing.assert_array_equal(d, pdist)
    np.testing.assert_array_equal(dc, pdc)
    idx.free()


def test_tensor_prerank_device_buffers_and_k(ctx):
    """Device-resident queries and outputs, k = 1 and k = 12 (re-rank depths 100 and 120)."""
    import torch
    import vdb_b200
    rows, qs = _data(150_000, 800, seed=7)
    data = vdb_b200.build_ivfpq(ctx, rows, DIM, nlist=128, pq_m=PQ_M, max_train_points_per_centroid=64, seed=42)
    idx = vdb_b200.Index.load(ctx, data, "l2", rows, DIM)
    rindex = oracle.Ref().load_index(data, oracle.L2, rows, DIM, pq_m=PQ_M)
    q_dev = torch.from_numpy(qs).cuda()
    for k in (1, 12):
        ids_dev = torch.empty((len(qs), k), dtype=torch.int32, device="cuda")
        d_dev = torch.empty((len(qs), k), dtype=torch.float32, device="cuda")
        idx.search(q_dev, k=k, nprobe=8, out=(ids_dev, d_dev))
        rids, rd, _ = rindex.search(qs, k=k, nprobe=8)
        np.testing.assert_array_equal(ids_dev.cpu().numpy().view(np.uint32), rids)
        np.testing.assert_array_equal(d_dev.cpu().numpy(), rd)
    idx.free()


def test_config2_full_size_matches_reference(ctx):
    """Config 2 at full size: 10,000,000 x 96 rows (the benchmark's mixture), nlist 4096, M = 48,
    nprobe 32, re-rank depth 100, the 10,000-query batch. The index is the GPU builder's (the
    reference's own file); ids, distances and distance computations equal the reference's
    IvfPqIndex on every query."""
    import vdb_b200
    from vdb_b200 import synth
    rows = synth.mixture(10_000_000, DIM, 1000, centres="uniform", lo=-1.0, hi=1.0, sigma=0.15, seed=2, stream=0)
    qs = synth.mixture(10_000, DIM, 1000, centres="uniform", lo=-1.0, hi=1.0, sigma=0.15, seed=2, stream=1)
    data = vdb_b200.build_ivfpq(ctx, rows, DIM, nlist=4096, pq_m=PQ_M, max_train_points_per_centroid=122, seed=42)
    idx = vdb_b200.Index.load(ctx, data, "l2", rows, DIM)
    ids, d, dc = idx.search(qs, k=10, nprobe=32, stats=True)
    rindex = oracle.Ref().load_index(data, oracle.L2, rows, DIM, pq_m=PQ_M)
    rids, rd, rdc = rindex.search(qs, k=10, nprobe=32)
    bad = np.nonzero(~np.all(ids == rids, axis=1))[0]
    assert bad.size == 0, (bad.size, bad[:5].tolist())
    np.testing.assert_array_equal(d, rd)
    np.testing.assert_array_equal(dc, rdc)
    idx.free()
