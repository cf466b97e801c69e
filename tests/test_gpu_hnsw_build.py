"""The GPU HNSW builder (vdbgpu_hnsw_build): its files carry the reference's index.hnsw framing
and pass the structural checks HnswGraph::Deserialize makes (src/index/hnsw/hnsw_graph.h:403-449);
its graphs reach the reference's own recall bar (tests/hnsw_test.cc:53-71: recall@10 >= 0.95 at
ef 100); and the GPU's search of a GPU-built graph equals the reference's search of the same file
(fixture hnsw_gpu_built.npz, made by tests/golden/make_gpu_graph_golden.py)."""
import numpy as np
import pytest

from helpers import golden

pytestmark = pytest.mark.gpu


def _recall(ids, gt):
    return np.mean([len(set(a.tolist()) & set(b.tolist())) / gt.shape[1] for a, b in zip(ids, gt)])


@pytest.mark.parametrize("metric", ["l2", "cosine"])
def test_built_graph_recall(ctx, metric):
    import vdb_b200
    from vdb_b200 import synth
    if metric == "l2":
        base, qs = synth.flat_int(20000, 300, seed=3)
    else:
        base, qs = synth.sharded_cosine(20000, 300, seed=3)
    f = vdb_b200.build_hnsw(ctx, metric, base, 128, M=16)
    assert vdb_b200.inspect_index_file(f) == vdb_b200.INDEX_TYPES["hnsw"]
    idx = vdb_b200.Index.load(ctx, f, metric, base, 128)
    ids, _ = idx.search(qs, k=10, ef=100)
    flat = vdb_b200.Index.create(ctx, "flat", metric, base, 128)
    gt, _ = flat.search(qs, k=10)
    assert _recall(ids, gt) >= 0.95


def test_built_graph_structure(ctx):
    import oracle
    import vdb_b200
    from vdb_b200 import synth
    base, _ = synth.sharded_cosine(6000, 1, seed=5)
    M = 8
    f = vdb_b200.build_hnsw(ctx, "cosine", base, 128, M=M, seed=7)
    _, g = oracle.parse_hnsw(f)
    n = base.shape[0]
    assert g.cap == n and g.M == M and g.level[g.entry] == g.max_level
    assert g.max_level == int(g.level.max())
    for i in range(n):
        for l in range(int(g.level[i]) + 1):
            lst = g.links(i, l)
            assert len(lst) <= (2 * M if l == 0 else M)
            assert len(set(lst)) == len(lst) and i not in lst
            assert all(g.level[j] >= l for j in lst)
    # Every node is reachable from the entry point on layer 0.
    seen = np.zeros(n, bool)
    stack = [g.entry]
    seen[g.entry] = True
    while stack:
        u = stack.pop()
        for v in g.links(u, 0):
            if not seen[v]:
                seen[v] = True
                stack.append(v)
    assert seen.mean() >= 0.995


def test_gpu_built_graph_search_matches_reference(ctx):
    import vdb_b200
    from vdb_b200 import synth
    g = golden("hnsw_gpu_built")
    base, qs = synth.sharded_cosine(int(g["n"]), int(g["nq"]), seed=int(g["seed"]))
    idx = vdb_b200.Index.load(ctx, bytes(g["index_file"]), "cosine", base, 128)
    for ef in (16, 64):
        ids, d, dc = idx.search(qs, k=10, ef=ef, stats=True)
        assert np.array_equal(ids, g[f"ids_{ef}"])
        assert np.array_equal(d, g[f"dist_{ef}"])
        assert np.array_equal(dc, g[f"dc_{ef}"])
