"""The drop-in boundary compiled and run: vdb::GpuIndex (hnsw-vector-db_b200/integration/gpu_index.*)
built against the reference's own src/index/index.h, handed to the reference's Segment::Open as each
segment's prebuilt index, and searched by the reference's own SearchDiskSegment
(src/engine/planner.cc:42-129) - planner, filter bitmaps, delete filter and ExactOverBitmap all the
reference's code. For every planner case and filter of the three collection fixtures the reference
wrote (HNSW / cosine, IVF-PQ / L2, flat / IP), per-segment hits and explains equal those of the same
segments opened with the reference's CPU indexes."""
import json

import numpy as np
import pytest

import oracle
from helpers import extract_collection, golden

pytestmark = pytest.mark.gpu

NAMES = ["coll_hnsw", "coll_ivfpq", "coll_flat"]


@pytest.mark.parametrize("name", NAMES)
def test_search_disk_segment_through_gpu_index(tmp_path, name):
    g = golden(name)
    path = extract_collection(g, tmp_path)
    cpu = oracle.GpuIndexHarness(path, use_gpu=False)
    gpu = oracle.GpuIndexHarness(path, use_gpu=True, device=0)
    assert cpu.nseg == gpu.nseg > 0
    filters = [str(f) for f in g["filters"]] + [None]
    bad = []
    for ci in range(len(g["cases"])):
        strategy, thr, ef, nprobe, k, alpha = json.loads(str(g["cases"][ci]))
        kw = dict(k=k, ef=ef, nprobe=nprobe, strategy=strategy, prefilter_threshold=thr, post_filter_alpha=alpha)
        for f in filters:
            for qi in range(0, g["queries"].shape[0], max(1, g["queries"].shape[0] // 6)):
                q = g["queries"][qi]
                cr, cd, cc, cex = cpu.search(q, filter=f, **kw)
                gr, gd, gc, gex = gpu.search(q, filter=f, **kw)
                if not (np.array_equal(cr, gr) and np.array_equal(cd, gd) and np.array_equal(cc, gc)):
                    bad.append(("hits", ci, f, qi))
                for a, b in zip(cex, gex):
                    for key in ("strategy", "matches", "live_rows", "ef", "distance_computations", "results"):
                        if a[key] != b[key]:
                            bad.append(("explain", ci, f, qi, key, a[key], b[key]))
    cpu.close()
    gpu.close()
    assert not bad, (name, len(bad), bad[:10])
