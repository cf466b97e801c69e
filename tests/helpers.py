"""Shared test helpers: regenerate the seeded inputs behind each golden fixture and check them."""
import hashlib
import os

import numpy as np

from conftest import golden  # noqa: F401  (re-exported)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def inputs(name, g):
    """(base, queries) of golden fixture `name`, regenerated and checked against its SHA-256."""
    from vdb_b200 import synth
    seed = int(g["seed"])
    n, nq = int(g["n"]), int(g["nq"])
    if name in ("flat_int", "hnsw", "hnsw_sq8"):
        b, q = synth.flat_int(n, nq, dim=128, seed=seed)
    elif name == "flat_float":
        b, q = synth.sharded_cosine(n, nq, dim=int(g["dim"]), seed=seed)
    elif name == "sq8_scan":
        b, q = synth.sq8_cosine(n, nq, dim=128, seed=seed)
    elif name in ("ivfpq", "pqflat"):
        b, q = synth.ivfpq_l2(n, nq, dim=96, seed=seed)
    else:
        raise KeyError(name)
    assert sha(b) == str(g["base_sha"]), f"{name}: regenerated base rows differ from the fixture's"
    assert sha(q) == str(g["query_sha"]), f"{name}: regenerated queries differ from the fixture's"
    return b, q


def assert_same_neighbors(ids_a, d_a, ids_b, d_b, rel=1e-4, exact_dist=True):
    """Ids identical except swaps inside distance ties (within rel); distances bit-equal where
    the ids agree when exact_dist."""
    import oracle
    assert ids_a.shape == ids_b.shape
    assert oracle.ids_match_up_to_ties(ids_a, d_a, ids_b, d_b, rel=rel)
    if exact_dist:
        same = ids_a == ids_b
        np.testing.assert_array_equal(d_a[same], d_b[same])


def extract_collection(g, dest):
    """Writes the collection directory stored in a coll_* fixture (keys "file:<relpath>") under
    dest and returns its path."""
    import os
    path = os.path.join(str(dest), "coll")
    for key in g:
        if not key.startswith("file:"):
            continue
        full = os.path.join(path, key[5:])
        os.makedirs(os.path.dirname(full), exist_ok=True)
        with open(full, "wb") as f:
            f.write(np.asarray(g[key]).tobytes())
    return path
