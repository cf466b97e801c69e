"""The GPU IVF-PQ / PQ-flat builder against the reference's own build (IvfPqIndex::build and
PqFlatIndex::build with its seeded k-means): the index files must be identical, byte for byte.
The cases cover k-means++ and random initialisation, subsampled and full training sets, the
runtime kernel set's L2 (16-float sub-vectors) and L2SqAny distances, a clamped nlist, PQ-flat,
and fewer training points than centroids. Compared with a live reference build when
oracle/_ref is present, and with golden digests (tests/golden/make_ivfpq_build_golden.py)."""
import hashlib
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [
    {"name": "ivf_pp", "type": "ivf_pq", "n": 20000, "dim": 96, "nlist": 64, "pq_m": 48, "mppc": 64, "seed": 7},
    {"name": "ivf_random_init", "type": "ivf_pq", "n": 200000, "dim": 96, "nlist": 1024, "pq_m": 48, "mppc": 39,
     "seed": 42},
    {"name": "ivf_dsub16", "type": "ivf_pq", "n": 30000, "dim": 96, "nlist": 128, "pq_m": 6, "mppc": 256, "seed": 3},
    {"name": "ivf_clamped_odd_dim", "type": "ivf_pq", "n": 1000, "dim": 40, "nlist": 64, "pq_m": 8, "mppc": 256,
     "seed": 1},
    {"name": "pq_flat", "type": "pq_flat", "n": 20000, "dim": 96, "pq_m": 16, "mppc": 64, "seed": 5},
    {"name": "pq_flat_few_points", "type": "pq_flat", "n": 200, "dim": 32, "pq_m": 4, "mppc": 256, "seed": 9},
]


def case_rows(c):
    from vdb_b200 import synth
    return synth.mixture(c["n"], c["dim"], 1000, centres="uniform", lo=-1.0, hi=1.0, sigma=0.15,
                         seed=100 + c["seed"], stream=0)


def _golden():
    with open(os.path.join(HERE, "golden", "ivfpq_build.json")) as f:
        return json.load(f)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_gpu_build_is_the_reference_index(ctx, case):
    import oracle
    import vdb_b200
    rows = case_rows(case)
    ours = vdb_b200.build_ivfpq(ctx, rows, case["dim"], type=case["type"], nlist=case.get("nlist", 1),
                                pq_m=case["pq_m"], max_train_points_per_centroid=case["mppc"], seed=case["seed"])
    g = _golden()
    want = {c["name"]: c for c in g["cases"]}[case["name"]]
    orders = {"scalar": oracle.ORDER_SCALAR, "avx2": oracle.ORDER_AVX2, "avx512": oracle.ORDER_AVX512}
    if oracle.host_kernel_order() == orders.get(g["kernel_set"], -1):
        assert len(ours) == want["bytes"]
        assert hashlib.sha256(ours).hexdigest() == want["sha256"]
    if os.path.exists(oracle.REF_LIB):
        ref = oracle.Ref().build_index(4 if case["type"] == "ivf_pq" else 3, 0, rows, case["dim"],
                                       pq_m=case["pq_m"], nlist=case.get("nlist", 1),
                                       max_train_ppc=case["mppc"], seed=case["seed"], threads=0).save()
        assert ours == ref


@pytest.mark.gpu
def test_gpu_built_ivfpq_searches_like_the_reference(ctx):
    """The GPU-built file loads into the GPU index and searches to the reference's own results
    on it (ids and distances identical)."""
    import oracle
    import vdb_b200
    c = CASES[0]
    rows = case_rows(c)
    data = vdb_b200.build_ivfpq(ctx, rows, c["dim"], nlist=c["nlist"], pq_m=c["pq_m"],
                                max_train_points_per_centroid=c["mppc"], seed=c["seed"])
    q = case_rows(dict(c, n=300, seed=c["seed"] + 1))
    idx = vdb_b200.Index.load(ctx, data, "l2", rows, c["dim"])
    ids, d = idx.search(q, k=10, nprobe=8)
    orc = oracle.Oracle()
    f = oracle.parse_ivfpq(data)
    oi, od = orc.ivfpq_search(f, 0, rows, q, k=10, nprobe=8)[:2]
    np.testing.assert_array_equal(ids, oi)
    np.testing.assert_array_equal(d, od)
    idx.free()
