"""Index::extend for HNSW on the GPU (vdbgpu_hnsw_extend; HnswIndex::extend,
src/index/hnsw/hnsw_index.cc:50-58): a graph the reference built over the first rows gets the
remaining rows inserted.
* The extended file is a valid index.hnsw: the reference's own LoadIndex accepts it (its
  Deserialize checks every link and level), the old nodes keep their levels, new levels follow
  level_for with the graph's seed, degree bounds hold and layer 0 stays connected.
* The reference and the GPU search the extended file identically (ids, distances, counts).
* Its recall matches the reference's own extend of the same graph (same rows, same queries).
* Flat extends by rebuilding over the superset (FlatIndex::extend); other types are refused as
  the reference refuses them."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _recall(ids, gt):
    return float(np.mean([len(set(a.tolist()) & set(b.tolist())) / gt.shape[1] for a, b in zip(ids, gt)]))


@pytest.fixture(scope="module")
def data():
    from vdb_b200 import synth
    return synth.flat_int(26_000, 500, dim=128, seed=13)


def test_hnsw_extend_is_a_valid_graph_searched_like_the_reference(ctx, data):
    import vdb_b200
    base, qs = data
    n0 = 20_000
    ref = oracle.Ref()
    r0 = ref.build_index(1, oracle.L2, base[:n0], 128, M=16, efc=200, seed=42, threads=0)
    f0 = r0.save()
    f1 = vdb_b200.extend_hnsw(ctx, "l2", f0, base, 128)
    assert vdb_b200.inspect_index_file(f1) == vdb_b200.INDEX_TYPES["hnsw"]
    _, g0 = oracle.parse_hnsw(f0)
    _, g1 = oracle.parse_hnsw(f1)
    n = base.shape[0]
    assert g1.cap == n and g1.M == g0.M and g1.seed == g0.seed
    assert np.array_equal(g1.level[:n0], g0.level[:n0])
    M = g1.M
    for i in range(n):
        for l in range(int(g1.level[i]) + 1):
            lst = g1.links(i, l)
            assert len(lst) <= (2 * M if l == 0 else M)
            assert len(set(lst)) == len(lst) and i not in lst
            assert all(g1.level[j] >= l for j in lst)
    assert g1.level[g1.entry] == g1.max_level == int(g1.level.max())
    seen = np.zeros(n, bool)
    stack = [g1.entry]
    seen[g1.entry] = True
    while stack:
        u = stack.pop()
        for v in g1.links(u, 0):
            if not seen[v]:
                seen[v] = True
                stack.append(v)
    assert seen.mean() >= 0.995
    # The reference's LoadIndex accepts the file, and both search it identically.
    rr = ref.load_index(f1, oracle.L2, base, 128)
    idx = vdb_b200.Index.load(ctx, f1, "l2", base, 128)
    for ef in (32, 64):
        ids, d, dc = idx.search(qs, k=10, ef=ef, stats=True)
        rids, rd, rdc = rr.search(qs, k=10, ef=ef)
        np.testing.assert_array_equal(ids, rids)
        np.testing.assert_array_equal(d, rd)
        np.testing.assert_array_equal(dc, rdc)
    # Recall of the extended graph against the reference's own extend of the same graph.
    flat = vdb_b200.Index.create(ctx, "flat", "l2", base, 128)
    gt, _ = flat.search(qs, k=10)
    re = r0.extend(base)
    ids, _, _ = idx.search(qs, k=10, ef=64, stats=True)
    rids, _, _ = re.search(qs, k=10, ef=64)
    ours, theirs = _recall(ids, gt), _recall(rids, gt)
    assert ours >= theirs - 0.02, (ours, theirs)
    # New rows as queries find themselves (they are reachable).
    own, _ = idx.search(base[n0:n0 + 300], k=1, ef=64)
    assert np.mean(own[:, 0] == np.arange(n0, n0 + 300)) >= 0.98
    idx.free()
    flat.free()


def test_extend_refusals(ctx, data):
    import vdb_b200
    base, _ = data
    ref = oracle.Ref()
    f0 = ref.build_index(1, oracle.L2, base[:2000], 128, M=8, efc=64, seed=3, threads=0).save()
    with pytest.raises(ValueError):  # fewer rows than the graph holds
        vdb_b200.extend_hnsw(ctx, "l2", f0, base[:1000], 128)
    fivf = ref.build_index(4, oracle.L2, base[:4000], 128, pq_m=16, nlist=16, seed=3, threads=0).save()
    with pytest.raises(vdb_b200.VdbError) as e:
        vdb_b200.extend_hnsw(ctx, "l2", fivf, base[:5000], 128)
    assert e.value.code == vdb_b200.NOT_SUPPORTED
    # A graph built on the GPU extends the same way.
    g = vdb_b200.build_hnsw(ctx, "l2", base[:3000], 128, M=8, seed=9)
    g2 = vdb_b200.extend_hnsw(ctx, "l2", g, base[:3500], 128)
    _, gg = oracle.parse_hnsw(g2)
    assert gg.cap == 3500
    ref.load_index(g2, oracle.L2, base[:3500], 128)
