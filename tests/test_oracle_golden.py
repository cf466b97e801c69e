"""The oracle (our C restatement) against the reference's own outputs (tests/golden, made by
running the reference with tests/golden/make_golden.py). Everything here is bit-exact: the
oracle follows the reference's summation order for the kernel set the fixtures were made with."""
import numpy as np
import pytest

import oracle
from helpers import golden, inputs


@pytest.fixture(scope="module")
def orc():
    g = golden("kernels")
    order = {"avx512": oracle.ORDER_AVX512, "avx2": oracle.ORDER_AVX2, "scalar": oracle.ORDER_SCALAR}
    return oracle.Oracle(order=order[str(g["kernel_set"])])


def test_distance_kernels_bit_exact(orc):
    g = golden("kernels")
    for j, d in enumerate(g["dims"]):
        pd = (int(d) + 15) // 16 * 16
        a, b = g["pair_a"][j][:pd].copy(), g["pair_b"][j][:pd].copy()
        assert orc.l2(a, b) == g["l2"][j], d
        assert orc.dot(a, b) == g["dot"][j], d
        assert -orc.dot(a, b) == g["ip"][j], d
    for j, d in enumerate(g["sq8_dims"]):
        pd = (int(d) + 15) // 16 * 16
        q, c = g["sq8_q"][j][:pd].copy(), g["sq8_c"][j][:pd].copy()
        vmin, scale = g["sq8_vmin"][j][:pd].copy(), g["sq8_scale"][j][:pd].copy()
        assert orc.sq8_dist(0, q, c, vmin, scale) == g["sq8_l2"][j]
        assert orc.sq8_dist(1, q, c, vmin, scale) == g["sq8_ip"][j]


def test_metric_convention(orc):
    # tests/distance_test.cc:86-91: L2(a,b) = 0.5, IP(a,b) = -0.5 for a=(1,0), b=(0.5,0.5).
    g = golden("kernels")
    a = np.zeros(16, np.float32); a[0] = 1
    b = np.zeros(16, np.float32); b[:2] = 0.5
    assert orc.l2(a, b) == g["convention"][0] == 0.5
    assert -orc.dot(a, b) == g["convention"][1] == -0.5


def test_topk_with_ties(orc):
    g = golden("kernels")
    for t in range(len(g["topk_n"])):
        n, k = int(g["topk_n"][t]), int(g["topk_k"][t])
        d = g["topk_d"][t][:n].copy()
        ids, dists = orc.topk(d, np.arange(n, dtype=np.uint32), k)
        m = min(n, k)
        np.testing.assert_array_equal(ids, g["topk_ids"][t][:m])
        np.testing.assert_array_equal(dists, g["topk_dists"][t][:m])


def test_flat_integer_rows(orc):
    g = golden("flat_int")
    base, qs = inputs("flat_int", g)
    ids, d = orc.flat_search(0, base, qs, 10)
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_array_equal(d, g["dists"])
    odd = (np.arange(base.shape[0]) % 2) == 1
    import vdb_b200
    fi, fd = orc.flat_search(0, base, qs, 50, allow=vdb_b200.pack_bitset(odd))
    np.testing.assert_array_equal(fi, g["filt_ids"])
    np.testing.assert_array_equal(fd, g["filt_dists"])
    assert np.all(fi % 2 == 1)


def test_flat_every_metric_odd_dim(orc):
    g = golden("flat_float")
    base, qs = inputs("flat_float", g)
    for m in (0, 1, 2):
        ids, d = orc.flat_search(m, base, qs, 20)
        np.testing.assert_array_equal(ids, g[f"ids_m{m}"])
        np.testing.assert_array_equal(d, g[f"dists_m{m}"])


def test_sq8_quantizer_and_scan(orc):
    g = golden("sq8_scan")
    base, qs = inputs("sq8_scan", g)
    vmin, scale, codes = orc.sq8_train_encode(base, 128)
    np.testing.assert_array_equal(vmin, g["vmin"])
    np.testing.assert_array_equal(scale, g["scale"])
    np.testing.assert_array_equal(codes, g["codes"])
    ids, d = orc.sq8_scan_search(2, base, codes, vmin, scale, qs, k=10, depth=100)
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_array_equal(d, g["dists"])


def test_sq8_half_step_bound(orc):
    # tests/distance_test.cc:106-126: decoded values lie within half a step of the input.
    rng = np.random.default_rng(5)
    n, dim, pd = 2000, 100, 112
    rows = np.zeros((n, pd), np.float32)
    rows[:, :dim] = rng.normal(0, 3, (n, dim)).astype(np.float32)
    vmin, scale, codes = orc.sq8_train_encode(rows, dim)
    back = vmin[None, :] + codes.astype(np.float32) * scale[None, :]
    err = np.abs(back[:, :dim] - rows[:, :dim])
    assert np.all(err <= scale[None, :dim] * 0.5 * 1.0001 + 1e-6)
    assert np.all(back[:, dim:] == 0)


def test_hnsw_search_bit_exact(orc):
    g = golden("hnsw")
    base, qs = inputs("hnsw", g)
    pd, graph = oracle.parse_hnsw(bytes(g["index_file"]))
    assert pd == 128 and graph.cap == base.shape[0]
    for ef in (16, 64, 128):
        ids, d, dc = orc.hnsw_search(graph, 0, base, qs, k=10, ef=ef)
        np.testing.assert_array_equal(ids, g[f"ids_ef{ef}"])
        np.testing.assert_array_equal(d, g[f"dists_ef{ef}"])
        np.testing.assert_array_equal(dc, g[f"dc_ef{ef}"])
    import vdb_b200
    even = (np.arange(base.shape[0]) % 2) == 0
    ids, d, dc = orc.hnsw_search(graph, 0, base, qs, k=10, ef=64, allow=vdb_b200.pack_bitset(even))
    np.testing.assert_array_equal(ids, g["filt_ids"])
    np.testing.assert_array_equal(dc, g["filt_dc"])


def test_hnsw_sq8_search_bit_exact(orc):
    g = golden("hnsw_sq8")
    base, qs = inputs("hnsw_sq8", g)
    n, dim, pd, vmin, scale, codes, graph = oracle.parse_hnsw_sq8(bytes(g["index_file"]))
    v2, s2, c2 = orc.sq8_train_encode(base, dim)
    np.testing.assert_array_equal(c2, codes)
    for ef, rr in ((32, -1), (64, -1), (64, 0), (64, 20)):
        tag = f"ef{ef}_r{'auto' if rr < 0 else rr}"
        ids, d, dc = orc.hnsw_sq8_search(graph, 0, base, codes, vmin, scale, qs, k=10, ef=ef, rerank=rr)
        np.testing.assert_array_equal(ids, g[f"ids_{tag}"])
        np.testing.assert_array_equal(d, g[f"dists_{tag}"])
        np.testing.assert_array_equal(dc, g[f"dc_{tag}"])


def test_ivfpq_search_bit_exact(orc):
    g = golden("ivfpq")
    base, qs = inputs("ivfpq", g)
    f = oracle.parse_ivfpq(bytes(g["index_file"]))
    assert f.nlist == 64 and f.m == 48 and f.rows == base.shape[0]
    for nprobe, rr in ((4, -1), (16, -1), (16, 0)):
        tag = f"np{nprobe}_r{'auto' if rr < 0 else rr}"
        ids, d, dc = orc.ivfpq_search(f, 0, base, qs, k=10, nprobe=nprobe, rerank=rr)
        np.testing.assert_array_equal(ids, g[f"ids_{tag}"])
        np.testing.assert_array_equal(d, g[f"dists_{tag}"])
        np.testing.assert_array_equal(dc, g[f"dc_{tag}"])
    # IVF-PQ with re-rank finds most of the exact neighbours (tests/pq_test.cc:108-117).
    assert oracle.recall_at_k(g["ids_np16_rauto"], g["gt_ids"], 10) >= 0.9
