"""Golden digests of index files built by the reference's own IvfPqIndex / PqFlatIndex (its seeded
k-means, src/index/quant/kmeans.cc) for the cases of tests/test_gpu_ivfpq_build.py: the GPU
builder must write the same bytes. Run from the repo root after `python __graft_entry__.py`
has built oracle/_ref; the digests depend on the host's distance kernel set, recorded with them."""
import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "hnsw-vector-db_b200")]

import oracle  # noqa: E402

sys.path.insert(0, os.path.dirname(HERE))
from test_gpu_ivfpq_build import CASES, case_rows  # noqa: E402


def main():
    ref = oracle.Ref()
    out = {"kernel_set": ref.kernel_set(), "cases": []}
    for c in CASES:
        rows = case_rows(c)
        idx = ref.build_index(4 if c["type"] == "ivf_pq" else 3, 0, rows, c["dim"], pq_m=c["pq_m"],
                              nlist=c.get("nlist", 1), max_train_ppc=c["mppc"], seed=c["seed"], threads=0)
        data = idx.save()
        out["cases"].append({"name": c["name"], "bytes": len(data), "sha256": hashlib.sha256(data).hexdigest()})
        print(c["name"], len(data), flush=True)
    with open(os.path.join(HERE, "ivfpq_build.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
