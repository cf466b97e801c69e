"""GPU parity for exact flat search and the exhaustive SQ8 scan (tensor-core pre-rank + exact
fp32 re-rank) against the reference's outputs (golden fixtures) and the oracle."""
import numpy as np
import pytest

import oracle
from helpers import assert_same_neighbors, golden, inputs

pytestmark = pytest.mark.gpu


def test_flat_integer_rows_bit_exact(ctx):
    import vdb_b200
    g = golden("flat_int")
    base, qs = inputs("flat_int", g)
    idx = vdb_b200.Index.load(ctx, bytes(g["flat_file"]), "l2", base, 128)
    ids, d, dc = idx.search(qs, k=10, stats=True)
    # Integer rows: tensor-core keys are exact, so ids (tie order included) and distances match.
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_array_equal(d, g["dists"])
    assert np.all(dc == base.shape[0])  # FlatIndex::search counts every row (flat_index.cc:76)
    odd = (np.arange(base.shape[0]) % 2) == 1
    fi, fd = idx.search(qs, k=50, filter=vdb_b200.pack_bitset(odd))
    np.testing.assert_array_equal(fi, g["filt_ids"])
    np.testing.assert_array_equal(fd, g["filt_dists"])


def test_flat_every_metric_odd_dim(ctx):
    import vdb_b200
    g = golden("flat_float")
    base, qs = inputs("flat_float", g)
    for m in (0, 1, 2):
        idx = vdb_b200.Index.create(ctx, "flat", m, base, 100)
        ids, d = idx.search(qs, k=20)
        assert_same_neighbors(ids, d, g[f"ids_m{m}"], g[f"dists_m{m}"])
        idx.free()


def test_flat_edge_cases(ctx):
    import vdb_b200
    orc = oracle.Oracle()
    from vdb_b200 import synth
    # k larger than the rows, a batch that is not a multiple of 128, rows not a multiple of 256.
    for n, nq, k in ((5, 3, 100), (300, 130, 7), (1, 1, 1), (513, 257, 32)):
        base, qs = synth.flat_int(n, nq, dim=48, seed=n)
        idx = vdb_b200.Index.create(ctx, "flat", "l2", base, 48)
        ids, d = idx.search(qs, k=k)
        oi, od = orc.flat_search(0, base, qs, k)
        np.testing.assert_array_equal(ids, oi)
        np.testing.assert_array_equal(d, od)
        assert np.all(ids[:, n:] == np.uint32(0xFFFFFFFF)) and np.all(np.isinf(d[:, n:]))
        idx.free()
    # A filter that allows nothing returns only misses.
    base, qs = synth.flat_int(1000, 10, dim=128, seed=3)
    idx = vdb_b200.Index.create(ctx, "flat", "l2", base, 128)
    ids, d = idx.search(qs, k=5, filter=vdb_b200.pack_bitset(np.zeros(1000, bool)))
    assert np.all(ids == np.uint32(0xFFFFFFFF)) and np.all(np.isinf(d))
    with pytest.raises(ValueError):
        idx.search(qs[:, :64], k=5)


def test_flat_full_size_config0(ctx):
    """Config 0 at full size (100k x 128 integer rows, 1000 queries): ids (tie order included) and
    distances identical to the reference's own FlatSearchBatch on every query."""
    import vdb_b200
    from vdb_b200 import synth
    base, qs = synth.flat_int(100_000, 1000, dim=128, seed=0)
    idx = vdb_b200.Index.create(ctx, "flat", "l2", base, 128)
    ids, d = idx.search(qs, k=10)
    ri, rd = oracle.Ref().flat_search_batch(oracle.L2, base, 128, qs, 10, threads=0)
    bad = np.nonzero(~np.all(ids == ri, axis=1))[0]
    assert bad.size == 0, f"{bad.size} queries differ (first {bad[:5].tolist()})"
    np.testing.assert_array_equal(d, rd)


def test_sq8_train_encode_bit_exact(ctx):
    import vdb_b200
    g = golden("sq8_scan")
    base, qs = inputs("sq8_scan", g)
    idx = vdb_b200.Index.create(ctx, "sq8_flat", "cosine", base, 128)
    vmin, scale, codes = idx.sq8_export()
    np.testing.assert_array_equal(vmin, g["vmin"])
    np.testing.assert_array_equal(scale, g["scale"])
    np.testing.assert_array_equal(codes, g["codes"])


def test_sq8_scan_matches_reference(ctx):
    import vdb_b200
    g = golden("sq8_scan")
    base, qs = inputs("sq8_scan", g)
    idx = vdb_b200.Index.create(ctx, "sq8_flat", "cosine", base, 128)
    ids, d = idx.search(qs, k=10, rerank=100)
    # Final ids identical; distances are the reference's fp32 re-rank, bit for bit.
    assert_same_neighbors(ids, d, g["ids"], g["dists"])
    assert oracle.recall_at_k(ids, g["ids"], 10) == 1.0


def test_sq8_scan_full_size_config1(ctx):
    """Config 1 at full size (1M x 128, cosine): the reference's own SQ8 codes, and 1,000 of the
    10k-query batch (every tenth) with the same neighbours as the reference's composed path
    (Sq8Quantizer + sq8_ip + TopK(100) + Rerank), distances bit-equal where ids agree."""
    import vdb_b200
    from vdb_b200 import synth
    base, qs = synth.sq8_cosine(1_000_000, 10_000, dim=128, seed=1)
    idx = vdb_b200.Index.create(ctx, "sq8_flat", "cosine", base, 128)
    ids, d = idx.search(qs, k=10, rerank=100)
    ref = oracle.Ref()
    vmin, scale, codes = idx.sq8_export()
    rv, rs, rc = ref.sq8_train_encode(base, 128, threads=0)
    np.testing.assert_array_equal(vmin, rv)
    np.testing.assert_array_equal(scale, rs)
    np.testing.assert_array_equal(codes, rc)
    sample = np.arange(0, 10_000, 10)
    oi, od = ref.sq8_scan_search(2, base, rc, rv, rs, qs[sample], k=10, depth=100, threads=0)
    assert_same_neighbors(ids[sample], d[sample], oi, od)
    assert np.all(np.diff(d, axis=1) >= 0)


@pytest.mark.parametrize("metric", [0, 1])
def test_grouped_scan_is_the_ungrouped_scan(ctx, monkeypatch, metric):
    """Batches of at least 2048 queries over operands of 64k rows and more are scanned in the
    order of each query's nearest pivot (up to 1024 rows picked from a row sample), and the
    results written back in the caller's order. Ids (tie order included) and distances equal those of the same
    index built without grouping (VDB_SCAN_GROUP=0), for the batch and for a shuffled copy of it,
    and the oracle's on a sample (integer rows: tensor-core keys are exact). On clustered rows the
    grouped scan finds candidates in fewer 32-query x 32-row chunks."""
    import vdb_b200
    from vdb_b200 import synth
    base, qs = synth.flat_int(100_000, 4000, dim=128, seed=21)
    idx = vdb_b200.Index.create(ctx, "flat", metric, base, 128)
    ctx.set_timing(True)
    ids, d = idx.search(qs, k=10)
    grouped_chunks = ctx.stage_counters()[1]
    ctx.set_timing(False)
    perm = np.random.default_rng(5).permutation(len(qs))
    ids2, d2 = idx.search(np.ascontiguousarray(qs[perm]), k=10)
    np.testing.assert_array_equal(ids2, ids[perm])
    np.testing.assert_array_equal(d2, d[perm])
    monkeypatch.setenv("VDB_SCAN_GROUP", "0")
    plain = vdb_b200.Index.create(ctx, "flat", metric, base, 128)
    ctx.set_timing(True)
    pi, pdist = plain.search(qs, k=10)
    plain_chunks = ctx.stage_counters()[1]
    ctx.set_timing(False)
    np.testing.assert_array_equal(ids, pi)
    np.testing.assert_array_equal(d, pdist)
    if metric == 0:
        assert grouped_chunks < 0.8 * plain_chunks, (grouped_chunks, plain_chunks)
    sample = np.arange(0, len(qs), 200)
    oi, od = oracle.Oracle().flat_search(metric, base, qs[sample], 10)
    np.testing.assert_array_equal(ids[sample], oi)
    np.testing.assert_array_equal(d[sample], od)
    plain.free()
    idx.free()


@pytest.mark.parametrize("keep", [None, 1, 6])
def test_seeded_scan_is_exact(ctx, monkeypatch, keep):
    """Batches of at least 5e7 (query, row) pairs over operands of 64k rows and more start every
    query's bound from a strided row sample. The
    seed is an estimate: queries left with fewer than C keys below it are rescanned unseeded.
    keep = 1 makes most queries fall back (about s - 1 rows of the operand lie below the minimum of
    a sample of every s-th row), keep = 6 some of them; results stay identical to the unseeded scan and to the
    oracle, ties included (integer rows)."""
    import vdb_b200
    from vdb_b200 import synth
    base, qs = synth.flat_int(120_000, 8400, dim=128, seed=11)
    idx = vdb_b200.Index.create(ctx, "flat", "l2", base, 128)
    if keep is not None:
        monkeypatch.setenv("VDB_SCAN_SEED_KEEP", str(keep))
    ctx.set_timing(True)
    ids, d = idx.search(qs, k=10)
    c = ctx.stage_counters()
    ctx.set_timing(False)
    assert c[5] == 1, "the scan was not seeded"
    if keep == 1:
        assert 0.5 * len(qs) < c[4] <= len(qs)
    elif keep == 6:
        assert 0 < c[4] < len(qs)
    orc = oracle.Oracle()
    sample = np.arange(0, len(qs), 280)
    oi, od = orc.flat_search(0, base, qs[sample], 10)
    np.testing.assert_array_equal(ids[sample], oi)
    np.testing.assert_array_equal(d[sample], od)
    monkeypatch.setenv("VDB_SCAN_SAMPLE", "0")
    plain = vdb_b200.Index.create(ctx, "flat", "l2", base, 128)
    pi, pd_ = plain.search(qs, k=10)
    np.testing.assert_array_equal(ids, pi)
    np.testing.assert_array_equal(d, pd_)
    plain.free()
    idx.free()


@pytest.mark.parametrize("levels", ["1", "2"])
def test_seeded_sq8_scan_with_fallbacks(ctx, monkeypatch, levels):
    """The seeded SQ8 scan (cosine, C = 128; 300k rows, one or two sample levels) with part of
    the batch rescanned: same ids and distances as the unseeded scan."""
    import vdb_b200
    from vdb_b200 import synth
    monkeypatch.setenv("VDB_SCAN_SAMPLE_LEVELS", levels)
    base, qs = synth.sq8_cosine(300_000, 3400, dim=128, seed=12)
    idx = vdb_b200.Index.create(ctx, "sq8_flat", "cosine", base, 128)
    monkeypatch.setenv("VDB_SCAN_SEED_KEEP", "15")
    ctx.set_timing(True)
    ids, d = idx.search(qs, k=10, rerank=100)
    c = ctx.stage_counters()
    ctx.set_timing(False)
    assert c[5] == 1 and 0 < c[4] < len(qs)
    monkeypatch.delenv("VDB_SCAN_SEED_KEEP")
    ids2, d2 = idx.search(qs, k=10, rerank=100)
    monkeypatch.setenv("VDB_SCAN_SAMPLE", "0")
    plain = vdb_b200.Index.create(ctx, "sq8_flat", "cosine", base, 128)
    pi, pd_ = plain.search(qs, k=10, rerank=100)
    for a, b in ((ids, pi), (d, pd_), (ids2, pi), (d2, pd_)):
        np.testing.assert_array_equal(a, b)
    plain.free()
    idx.free()


def test_small_batches_over_many_row_slices(ctx):
    """A few queries over a large index spread over many row slices (unseeded), so a query's
    candidate lists hold more entries than finalize keeps in shared memory and the C best are
    selected over the lists in global memory, integer rows making ties on the pre-rank key at the
    cut. Exact against the oracle (flat), against the reference's SQ8 arithmetic (SQ8)."""
    import vdb_b200
    from vdb_b200 import synth
    base, qs = synth.flat_int(120_000, 40, dim=128, seed=13)
    idx = vdb_b200.Index.create(ctx, "flat", "l2", base, 128)
    orc = oracle.Oracle()
    for nq in (1, 7, 40):
        ids, d = idx.search(qs[:nq], k=10)
        oi, od = orc.flat_search(0, base, qs[:nq], 10)
        np.testing.assert_array_equal(ids, oi)
        np.testing.assert_array_equal(d, od)
    idx.free()
    base, qs = synth.sq8_cosine(200_000, 20, dim=128, seed=14)
    idx = vdb_b200.Index.create(ctx, "sq8_flat", "cosine", base, 128)
    ids, d = idx.search(qs, k=10, rerank=100)
    vmin, scale, codes = idx.sq8_export()
    oi, od = orc.sq8_scan_search(2, base, codes, vmin, scale, qs, k=10, depth=100)
    assert_same_neighbors(ids, d, oi, od)
    idx.free()
