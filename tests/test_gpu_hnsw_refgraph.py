"""GPU parity for batched HNSW search on graphs the reference builds itself at a size where the walk
is long: 100,000 integer rows of config 3's mixture, HnswIndex / HnswSq8Index {M=16,
ef_construction=200, seed=42} built on the host cores by the reference's own code
(src/index/hnsw/hnsw_index.cc:22-34, 63-129) and saved in its index.hnsw / index.hnsw_sq8 format.
The GPU loads the same file and, for every one of 1,000 queries, must return the reference's
neighbours, distances and distance computations (src/index/hnsw/hnsw_graph.h:286-309).

A parallel build is not deterministic, so both sides load the one file the reference wrote in
this process; the graph is never compared, only searches over it."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

N_ROWS, N_QUERIES, DIM = 100_000, 1_000, 128
HNSW, HNSW_SQ8 = 1, 2


@pytest.fixture(scope="module")
def data():
    from vdb_b200 import synth
    return synth.flat_int(N_ROWS, N_QUERIES, dim=DIM, seed=3)


@pytest.fixture(scope="module")
def ref():
    return oracle.Ref()


def _same(ids, d, dc, rids, rd, rdc, what):
    bad = np.nonzero(~np.all(ids == rids, axis=1))[0]
    assert bad.size == 0, f"{what}: {bad.size} queries differ in ids (first {bad[:5].tolist()})"
    np.testing.assert_array_equal(d, rd, err_msg=f"{what}: distances")
    np.testing.assert_array_equal(dc, rdc, err_msg=f"{what}: distance computations")


def test_hnsw_reference_graph_all_queries(ctx, data, ref):
    import vdb_b200
    base, qs = data
    rindex = ref.build_index(HNSW, oracle.L2, base, DIM, M=16, efc=200, seed=42, threads=0)
    file = rindex.save()
    idx = vdb_b200.Index.load(ctx, file, "l2", base, DIM)
    assert idx.type == HNSW and idx.rows == N_ROWS
    for ef in (64, 128, 256):
        ids, d, dc = idx.search(qs, k=10, ef=ef, stats=True)
        rids, rd, rdc = rindex.search(qs, k=10, ef=ef)
        _same(ids, d, dc, rids, rd, rdc, f"ef {ef}")
    # A filtered walk (every third row allowed) on the same graph.
    allow = (np.arange(N_ROWS) % 3) == 0
    bits = vdb_b200.pack_bitset(allow)
    ids, d, dc = idx.search(qs, k=10, ef=64, filter=bits, stats=True)
    rids, rd, rdc = rindex.search(qs, k=10, ef=64, allow=bits)
    _same(ids, d, dc, rids, rd, rdc, "filtered ef 64")
    idx.free()


def test_hnsw_sq8_reference_graph_all_queries(ctx, data, ref):
    import vdb_b200
    base, qs = data
    rindex = ref.build_index(HNSW_SQ8, oracle.L2, base, DIM, M=16, efc=200, seed=42, threads=0)
    file = rindex.save()
    idx = vdb_b200.Index.load(ctx, file, "l2", base, DIM)
    assert idx.type == HNSW_SQ8 and idx.rows == N_ROWS
    for ef, rr in ((64, -1), (128, -1), (256, -1), (64, 0), (128, 40)):
        ids, d, dc = idx.search(qs, k=10, ef=ef, rerank=rr, stats=True)
        rids, rd, rdc = rindex.search(qs, k=10, ef=ef, rerank=rr)
        _same(ids, d, dc, rids, rd, rdc, f"ef {ef} re-rank {rr}")
    idx.free()
