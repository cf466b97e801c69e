"""Fixture hnsw_gpu_built.npz: a graph built by the GPU builder, searched by the reference.

Two steps, because the builder needs a GPU and the reference is only present where it is
compiled:
    python tests/golden/make_gpu_graph_golden.py build OUT.bin     # on a GPU machine
    python tests/golden/make_gpu_graph_golden.py reference OUT.bin  # where oracle/_ref exists
The second step loads the file into the reference's HnswIndex (LoadIndex) and stores its search
results (ids, distances, distance computations) for ef 16 and 64 beside the file.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "hnsw-vector-db_b200"))

N, NQ, SEED, M = 8000, 200, 21, 16


def build(path):
    import vdb_b200
    from vdb_b200 import synth
    base, _ = synth.sharded_cosine(N, NQ, seed=SEED)
    ctx = vdb_b200.Context(0)
    with open(path, "wb") as f:
        f.write(vdb_b200.build_hnsw(ctx, "cosine", base, 128, M=M))


def reference(path):
    import oracle
    from vdb_b200 import synth
    base, qs = synth.sharded_cosine(N, NQ, seed=SEED)
    data = open(path, "rb").read()
    ref = oracle.Ref()
    idx = ref.load_index(data, oracle.COSINE, base, 128)
    out = {"index_file": np.frombuffer(data, np.uint8), "n": np.array(N), "nq": np.array(NQ),
           "seed": np.array(SEED)}
    for ef in (16, 64):
        ids, d, dc = idx.search(qs, k=10, ef=ef)
        out[f"ids_{ef}"], out[f"dist_{ef}"], out[f"dc_{ef}"] = ids, d, dc
    np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "hnsw_gpu_built.npz"), **out)
    print("wrote hnsw_gpu_built.npz")


if __name__ == "__main__":
    {"build": build, "reference": reference}[sys.argv[1]](sys.argv[2])
