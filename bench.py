#!/usr/bin/env python
"""Benchmark of the batched search path on B200: batched QPS at fixed recall@10 (1/2/4/8 B200).

Default workload (config 4, the configuration the metric is quoted on at 1/2/4/8 GPUs): sharded
filtered multi-segment search over 100,000,000 x 128 cosine rows in 64 segments with year / tags
metadata, filter year >= 2020 AND tags contains a Zipf-drawn tag per query, the reference's auto
planner per (filter, segment), 10,000-query batches, k = 10. With N GPUs the segments shard by
manifest position (i % N); each rank searches and merges its own, then one NCCL exchange of the
k merged hit records per query (vdbgpu_shard_merge) and the merge on rank 0. Synthetic seeded data
stands in for the reference's public datasets.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c0..c4]

One JSON line on rank 0 (one per ef / variant for config 3). A step is one batched search of
10,000 queries. `value` is device-resident throughput (queries already in HBM); `e2e` is the same
call through the C ABI with host (pinned) buffers, copies included. Other workloads: c1 (SQ8
exhaustive scan + re-rank of the top 100 over 1M x 128, one segment: replicas only at N > 1), c0
(flat L2), c2 (IVF-PQ), c3 (HNSW on reference-built graphs).
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "hnsw-vector-db_b200"))

import numpy as np  # noqa: E402

METRIC = "batched QPS at fixed recall@10 (1/2/4/8 B200); % of HBM/tensor-core roofline"
N_ROWS, DIM, NQ, K, DEPTH = 1_000_000, 128, 10_000, 10, 100
WORKLOAD = ("config 1: SQ8 cosine exhaustive scan + fp32 re-rank of the top 100, "
            "1M x 128 rows, 10k-query batches, k=10")


C4_SEGMENTS, C4_SEG_ROWS, C4_EF = 64, 1_562_500, 64
C4_WORKLOAD = ("config 4: sharded filtered multi-segment search, {segs} segments x {rows} rows x 128 "
               "cosine (year int64 U[1990,2024], 1-5 Zipf(1.1) tags of 1000 words), HNSW M=16 per "
               "segment built on the GPU, filter year>=2020 AND tags contains a Zipf(1.1) tag per query "
               "(queries grouped by tag, one filter per group), auto planner, 10k-query batches, k=10, "
               "ef=64, per-GPU top-k merged after an NCCL all-gather")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--workload", default="c4", choices=["c0", "c1", "c2", "c3", "c4"])
    p.add_argument("--segments", type=int, default=C4_SEGMENTS)
    p.add_argument("--seg-rows", type=int, default=C4_SEG_ROWS)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--rows", type=int, default=N_ROWS)
    p.add_argument("--batch", type=int, default=NQ)
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--c2-rows", type=int, default=10_000_000,
                   help="config 2 rows (smaller only for profiling captures)")
    p.add_argument("--c3-ef", default="64,128,256", help="config 3 beam widths (comma-separated)")
    p.add_argument("--c3-variants", default="fp32,sq8", help="config 3 distance variants (fp32, sq8)")
    return p.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            m = json.load(f)
        return m["bf16_tflops_sustained"], m["bf16_tflops"], m["hbm_gbs"], "measured"
    return 1400.0, 1590.0, 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region (median SM clock under load, throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={device}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "50"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        # nvidia-smi takes a moment to start: wait (bounded) for its first sample so that the
        # samples cover the timed region that follows.
        t0 = time.time()
        while self.p is not None and time.time() - t0 < 3.0:
            if os.path.getsize(self.f.name) > 0:
                break
            time.sleep(0.01)

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.seek(0)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            c = [x.strip() for x in line.split(",")]
            if len(c) < 9:
                continue
            try:
                sm.append(float(c[1]))
                smax = float(c[2])
            except ValueError:
                continue
            for name, v in zip(names, c[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        os.unlink(self.f.name)
        load = [s for s in sm if smax and s > 0.5 * smax] or sm
        return {"sm_mhz": float(np.median(load)) if load else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_reference(base, qs_sample, threads=0):
    """The reference's own CPU implementation of this path (oracle/_ref, compiled from the
    reference sources): Sq8Quantizer + sq8_ip + TopK(100) + Rerank. Returns (ids, seconds)."""
    import oracle
    ref = oracle.Ref()
    vmin, scale, codes = ref.sq8_train_encode(base, DIM, threads=threads)
    ref.sq8_scan_search(2, base, codes, vmin, scale, qs_sample[:8], k=K, depth=DEPTH, threads=threads)
    t0 = time.perf_counter()
    ids, _ = ref.sq8_scan_search(2, base, codes, vmin, scale, qs_sample, k=K, depth=DEPTH, threads=threads)
    return ids, time.perf_counter() - t0, ref.kernel_set()


def sample_size(base, qs, seconds):
    """Queries of CPU work that take about `seconds` on all host threads (probe with 64)."""
    _, t, _ = cpu_reference(base, qs[:64])
    per_q = max(t / 64, 1e-6)
    return int(min(qs.shape[0], max(64, seconds / per_q)))


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    from vdb_b200 import synth
    base, qs = synth.sq8_cosine(args.rows, args.batch, dim=DIM, seed=1)
    cores = os.cpu_count()
    # Each step is a bounded sample of the batch, sized so the whole run ends in a few minutes.
    per_step = max(8, int(args.cpu_seconds * 2 / max(1, args.steps + args.warmup) /
                         max(1e-6, cpu_reference(base, qs[:32])[1] / 32)))
    per_step = min(per_step, args.batch)
    for w in range(args.warmup):
        cpu_reference(base, qs[:per_step])
    times = []
    for s in range(args.steps):
        off = (s * per_step) % max(1, args.batch - per_step + 1)
        _, t, ks = cpu_reference(base, qs[off:off + per_step])
        times.append(t)
    qps = per_step * len(times) / sum(times)
    out = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": WORKLOAD, "rows": args.rows, "dim": DIM,
                                        "batch": args.batch, "k": K, "rerank": DEPTH},
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": cores, "kind": "reference",
                         "sample": f"{per_step} of {args.batch} queries per step over {args.rows} rows "
                                   f"({cpu_model()}, kernel set {ks})"},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)
    return 0


def run_ours(args):
    import torch
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    import vdb_b200
    from vdb_b200 import synth
    base, qs = synth.sq8_cosine(args.rows, args.batch, dim=DIM, seed=1)
    if rank > 0:  # replicas: every rank its own query batch over the same index
        qs = synth.mixture(args.batch, DIM, 1000, centres="normal", sigma=0.3, normalize=True, seed=1,
                           stream=1 + 2 * rank)
    ctx = vdb_b200.Context(local)
    stream = torch.cuda.current_stream()
    ctx.set_stream(stream.cuda_stream)
    ctx.set_timing(True)
    idx = vdb_b200.Index.create(ctx, "sq8_flat", "cosine", base, DIM)
    nq = qs.shape[0]
    q_dev = torch.from_numpy(qs).cuda()
    ids_dev = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    d_dev = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    # prep_queries, scan_mma over the row sample, scan_seed, scan_mma, finalize (a seeded scan);
    # queries rescanned unseeded add gather, prep, scan, finalize and scatter launches.
    launches_per_step = 5

    def step():
        idx.search(q_dev, k=K, rerank=DEPTH, out=(ids_dev, d_dev))

    for _ in range(max(3, args.warmup)):
        step()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    scan_ms, stage, counters, resc_steps = [], np.zeros(3), np.zeros(7), 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
        st = ctx.stage_times()
        scan_ms.append(st[1])
        stage += np.array(st[:3])
        c = np.array(ctx.stage_counters()[:7], dtype=np.float64)
        counters += c
        resc_steps += int(c[4] > 0)
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    t = torch.tensor([ms], device="cuda")
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * nq / (ms_max / 1000.0)

    # e2e: the same call with pinned host buffers (H2D of the queries and D2H of the results
    # inside the timed region, every step).
    q_host = torch.from_numpy(qs).pin_memory()
    ids_host = torch.empty((nq, K), dtype=torch.int32).pin_memory()
    d_host = torch.empty((nq, K), dtype=torch.float32).pin_memory()
    for _ in range(2):
        idx.search(q_host, k=K, rerank=DEPTH, out=(ids_host, d_host))
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, args.steps // 2)
    e0.record(stream)
    for _ in range(e2e_steps):
        idx.search(q_host, k=K, rerank=DEPTH, out=(ids_host, d_host))
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / e2e_steps], device="cuda")
    if world > 1:
        torch.distributed.all_reduce(e2e_ms, op=torch.distributed.ReduceOp.MAX)
    e2e_value = world * nq / (float(e2e_ms.item()) / 1000.0)

    result = None
    if rank == 0:
        sustained, burst, hbm, src = peaks()
        scan_s = float(np.mean(scan_ms)) / 1000.0
        flops = 2.0 * nq * args.rows * DIM
        achieved = flops / scan_s / 1e12
        ids_gpu = ids_host.numpy().view(np.uint32).copy()
        # The dominant kernel is the full scan (stage 1); the sample scan that seeds it is timed in
        # stage 0 with the query preparation.
        # The scan is timed alone in a short loop at full clocks, so the burst peak is its
        # denominator; the power-capped sustained figure is reported beside it.
        roof = {"bound": "tensor", "kernel": "scan_mma_kernel", "achieved": achieved,
                "peak": burst, "unit": "TFLOP/s", "frac": achieved / burst,
                "peak_kind": f"{src} bf16 dense, burst",
                "frac_of_sustained": achieved / sustained,
                "traffic": traffic_per_launch(),
                "algorithmic": f"2*Q*N*d = {flops:.3e} FLOP per launch; codes operand "
                               f"{args.rows * DIM * 2 / 1e6:.0f} MB"}
        result = {
            "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 tensor-core pre-rank, f32 re-rank", "data": "synthetic",
            "config": {"workload": WORKLOAD, "rows": args.rows, "dim": DIM, "batch": nq, "k": K,
                       "rerank": DEPTH, "metric": "cosine",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2: 256 MB fp16 code operand + 512 MB fp32 rows"},
            "roofline": roof,
            "stage_ms": {"prep_and_seed": stage[0] / args.steps, "scan": stage[1] / args.steps,
                         "select_rerank": stage[2] / args.steps},
            "scan_counters_per_step": {"chunks": counters[0] / args.steps,
                                       "chunks_with_candidates": counters[1] / args.steps,
                                       "candidates_per_query": counters[2] / args.steps / nq,
                                       "compactions_per_query": counters[3] / args.steps / nq,
                                       "seeded": bool(counters[5] > 0),
                                       "seed_keep": counters[6] / max(counters[5], 1),
                                       "rescanned_queries": counters[4] / args.steps},
            "e2e": {"value": e2e_value, "unit": "queries/s", "h2d_bytes_per_step": nq * DIM * 4,
                    "d2h_bytes_per_step": nq * K * 8},
            "gpu_launches": launches_per_step * args.steps + 5 * resc_steps,
            "clocks": clk,
        }
        if world == 1:
            # CPU baseline: the reference's own implementation on the host cores, bounded sample.
            s = sample_size(base, qs, args.cpu_seconds)
            ref_ids, secs, ks = cpu_reference(base, qs[:s])
            agree = float(np.mean(np.all(ref_ids == ids_gpu[:s], axis=1)))
            rec = float(np.mean([len(set(a.tolist()) & set(b.tolist())) / K
                                 for a, b in zip(ids_gpu[:s], ref_ids)]))
            result["cpu_baseline"] = {"value": s / secs, "unit": "queries/s", "cores": os.cpu_count(),
                                      "kind": "reference",
                                      "sample": f"{s} of {nq} queries over {args.rows} rows "
                                                f"({cpu_model()}, kernel set {ks})"}
            result["recall_at_10_vs_reference"] = rec
            result["identical_ids_vs_reference"] = agree
        print(json.dumps(result), flush=True)
    idx.free()
    ctx.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def traffic_per_launch():
    """DRAM bytes of one scan launch from the committed ncu summary, if one exists."""
    path = os.path.join(ROOT, "profiles", "scan_mma_sq8_config1.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get("dram_bytes_per_launch")
    return None


# ------------------------------------------------------------------------------------- config 4

C4_OPTIONS = {"dim": DIM, "metric": "cosine", "index": {"type": "hnsw", "M": 16, "ef_construction": 200},
              "schema": [{"name": "year", "type": "int64"}, {"name": "tags", "type": "keyword_list"}]}


def c4_segment(s, seg_rows):
    from vdb_b200 import synth
    return synth.c4_segment(s, seg_rows)


def c4_queries(nq):
    from vdb_b200 import synth
    return synth.c4_queries(nq)


def c4_graph(ctx, s, rows_dev, seg_rows):
    """Segment s's HNSW graph (reference index.hnsw format) built on the GPU, cached in
    VDB_BENCH_CACHE (default the system temp directory) so that later runs on the same host (the
    next GPU count of a scaling run) load it instead. Returns (file bytes, build seconds or None)."""
    import shutil
    import vdb_b200
    cache = os.environ.get("VDB_BENCH_CACHE", tempfile.gettempdir())
    name = os.path.join(cache, f"vdb_c4_graph_{s}_{seg_rows}_m16_seed{42 + s}.hnsw")
    if os.path.exists(name):
        with open(name, "rb") as f:
            return f.read(), None
    t = time.time()
    graph = vdb_b200.build_hnsw(ctx, "cosine", rows_dev, DIM, M=16, seed=42 + s)
    build_s = time.time() - t
    try:
        if shutil.disk_usage(cache).free > 4 * len(graph) + (16 << 30):
            tmp = f"{name}.{os.getpid()}.part"
            with open(tmp, "wb") as f:
                f.write(graph)
            os.replace(tmp, name)
    except OSError:
        pass  # no cache: the next run builds again
    return graph, build_s


def run_c4_ours(args):
    import datetime
    from concurrent.futures import ThreadPoolExecutor
    import torch
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                             device_id=torch.device("cuda", local))
    import vdb_b200
    from vdb_b200 import sharded, synth
    ctx = vdb_b200.Context(local)
    stream = torch.cuda.current_stream()
    ctx.set_stream(stream.cuda_stream)
    coll = vdb_b200.Collection.create(ctx, C4_OPTIONS)
    t_setup = time.time()
    build_s, cached = 0.0, 0
    mine = [s for s in range(args.segments) if sharded.owner(s, world) == rank]
    # Host generation of the next segment overlaps the GPU graph build of the current one.
    with ThreadPoolExecutor(max_workers=1) as pool:
        nxt = pool.submit(c4_segment, mine[0], args.seg_rows) if mine else None
        for i, s in enumerate(mine):
            rows, ids, years, tags = nxt.result()
            nxt = pool.submit(c4_segment, mine[i + 1], args.seg_rows) if i + 1 < len(mine) else None
            rows_dev = torch.from_numpy(rows).cuda()
            graph, b = c4_graph(ctx, s, rows_dev, args.seg_rows)
            build_s += b or 0.0
            cached += b is None
            coll.add_segment(s, s, rows_dev, ids, synth.meta_payload(years, tags), graph)
            del rows_dev, graph
    setup_s = time.time() - t_setup
    # The exchange: the library's NCCL group (token from rank 0 over torch.distributed).
    group = vdb_b200.ShardGroup(ctx, sharded.share_token(), rank, world, timeout_ms=120000) if world > 1 else None
    qs, filters, qf = c4_queries(args.batch)
    nq = qs.shape[0]
    q_dev = torch.from_numpy(qs).cuda()
    hits = torch.empty(nq * K * 24, dtype=torch.uint8, device="cuda")
    ids_dev = torch.empty((nq, K), dtype=torch.int64, device="cuda")
    d_dev = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    phase = {"search": 0.0, "exchange": 0.0}

    def step(queries, out_ids, out_d, qfilt=qf, strategy="auto", hit_buf=hits):
        n = int(queries.shape[0])
        t0 = time.perf_counter()
        if world == 1:
            coll.search_grouped(queries, filters, qfilt, k=K, ef=C4_EF, strategy=strategy, out=(out_ids, out_d))
            phase["search"] += time.perf_counter() - t0
            return
        coll.search_grouped(queries, filters, qfilt, k=K, ef=C4_EF, strategy=strategy, out=False, hits=hit_buf)
        t1 = time.perf_counter()
        group.merge(hit_buf, n, K, root=0, out=(out_ids, out_d) if rank == 0 else None)
        phase["search"] += t1 - t0
        phase["exchange"] += time.perf_counter() - t1

    for _ in range(max(3, args.warmup)):
        step(q_dev, ids_dev, d_dev)
    coll.stats(enable=True)
    ctx.set_timing(True)
    step(q_dev, ids_dev, d_dev)
    # Graph-walk counters of that step: walks, expansions, front refills, pool slots scanned by
    # refills, merges into the front, result inserts, most expansions of one walk.
    wc = ctx.stage_counters()[:7]
    ctx.set_timing(False)
    st = coll.stats(enable=False)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    phase = {"search": 0.0, "exchange": 0.0}
    launches0 = vdb_b200.launch_count()
    clocks = Clocks(local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step(q_dev, ids_dev, d_dev)
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = vdb_b200.launch_count() - launches0
    t = torch.tensor([ev0.elapsed_time(ev1) / args.steps, 1000.0 * phase["search"] / args.steps,
                      1000.0 * phase["exchange"] / args.steps], device="cuda", dtype=torch.float64)
    lt = torch.tensor([launches], device="cuda", dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(lt, op=torch.distributed.ReduceOp.SUM)
    ms, search_ms, exchange_ms = (float(x) for x in t.tolist())
    # e2e: host queries and host results through the same calls.
    q_host = torch.from_numpy(qs).pin_memory()
    ids_host = torch.empty((nq, K), dtype=torch.int64).pin_memory()
    d_host = torch.empty((nq, K), dtype=torch.float32).pin_memory()
    step(q_host, ids_host, d_host)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_steps = max(2, args.steps // 2)
    for _ in range(e2e_steps):
        step(q_host, ids_host, d_host)
    e1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1) / e2e_steps], device="cuda")
    if world > 1:
        torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
    # Recall@10 against exact filtered search (the prefilter strategy forced on every segment) on
    # a query sample.
    ns = min(nq, 1000)
    sel = np.arange(0, nq, max(1, nq // ns))[:ns]
    qs_s = torch.from_numpy(np.ascontiguousarray(qs[sel])).cuda()
    qf_s = np.ascontiguousarray(qf[sel])
    hb = torch.empty(len(sel) * K * 24, dtype=torch.uint8, device="cuda")
    a_ids = torch.empty((len(sel), K), dtype=torch.int64, device="cuda")
    a_d = torch.empty((len(sel), K), dtype=torch.float32, device="cuda")
    e_ids = torch.empty((len(sel), K), dtype=torch.int64, device="cuda")
    e_d = torch.empty((len(sel), K), dtype=torch.float32, device="cuda")
    step(qs_s, a_ids, a_d, qf_s, "auto", hb)
    step(qs_s, e_ids, e_d, qf_s, "prefilter", hb)
    recall = None
    if rank == 0:
        ai, ei = a_ids.cpu().numpy(), e_ids.cpu().numpy()
        recall = float(np.mean([len(set(x[x >= 0].tolist()) & set(y[y >= 0].tolist())) / max(1, int((y >= 0).sum()))
                                for x, y in zip(ai, ei)]))
    # Work per step summed over ranks (rows gathered exactly or by graph walks, bitmap words), and
    # the phases of the busiest rank (host wall time of the synchronous phases of one step).
    w = torch.tensor([st["exact_rows"], st["index_distance_computations"], st["bitmap_words"],
                      st["prefilter_pairs"], st["graph_pairs"], st["empty_pairs"]], dtype=torch.float64,
                     device="cuda")
    ph = torch.tensor([st[k] / 1000.0 for k in ("us_bitmaps_plan", "us_exact", "us_index", "us_other")],
                      dtype=torch.float64, device="cuda")
    if world > 1:
        torch.distributed.all_reduce(w, op=torch.distributed.ReduceOp.SUM)
        torch.distributed.all_reduce(ph, op=torch.distributed.ReduceOp.MAX)
    w = w.cpu().numpy()
    ph = ph.cpu().numpy()
    if rank == 0:
        _, _, hbm, src = peaks()
        pd = 128
        row_bytes = (w[0] + w[1]) * pd * 4
        bitmap_bytes = w[2] * 4 * 3  # two leaf words read, one result word written
        achieved = (row_bytes + bitmap_bytes) / (ms / 1000.0) / 1e9 / world
        total_rows = args.segments * args.seg_rows
        # The dominant kernel of a step: the exact scoring of prefiltered rows (exact_rows_kernel)
        # or the filtered graph walks (hnsw_search_kernel), whichever phase takes longer.
        if ph[1] >= ph[2]:
            dom = {"kernel": "exact_rows_kernel (ExactOverBitmap)", "bytes": w[0] * pd * 4, "ms": ph[1],
                   "algorithmic": f"{w[0]:.3e} rows scored exactly x {pd * 4} B per step (all ranks)"}
        else:
            dom = {"kernel": "hnsw_search_kernel (filtered walks)", "bytes": w[1] * (pd * 4 + 4), "ms": ph[2],
                   "algorithmic": f"{w[1]:.3e} graph distance computations x {pd * 4 + 4} B per step (all ranks)"}
        dom_achieved = dom["bytes"] / world / (dom["ms"] / 1000.0) / 1e9 if dom["ms"] > 0 else None
        result = {
            "metric": METRIC, "value": nq / (ms / 1000.0), "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": C4_WORKLOAD.format(segs=args.segments, rows=args.seg_rows),
                       "rows": total_rows, "segments": args.segments, "dim": DIM, "batch": nq, "k": K,
                       "ef": C4_EF, "distinct_filters": len(filters),
                       "parallelism": f"segments sharded over {world} GPUs" if world > 1 else "single GPU",
                       "l2": f"inputs larger than L2: {total_rows * pd * 4 / 1e9:.1f} GB of fp32 rows"},
            "roofline": {"bound": "hbm", "kernel": dom["kernel"], "achieved": dom_achieved, "peak": hbm,
                         "unit": "GB/s", "frac": dom_achieved / hbm if dom_achieved else None,
                         "peak_kind": f"{src} copy bandwidth", "traffic": None,
                         "kernel_ms": dom["ms"], "algorithmic": dom["algorithmic"],
                         "timing": "the phase's host wall time in one step (synchronous phases), busiest rank",
                         "whole_step": {"achieved": achieved, "frac": achieved / hbm,
                                        "algorithmic": f"per step: {w[0]:.3e} rows scored exactly + {w[1]:.3e} "
                                                       f"graph distance computations (x {pd * 4} B) + {w[2]:.3e} "
                                                       "bitmap words (x 12 B), per GPU"}},
            "plan_per_step": {"prefilter_pairs": w[3], "graph_pairs": w[4], "empty_pairs": w[5]},
            "stage_ms_busiest_rank": {"bitmaps_plan": ph[0], "exact": ph[1], "graph_walks": ph[2],
                                      "merge_other": ph[3], "search_call": search_ms, "exchange": exchange_ms},
            "walk_counters_per_walk_rank0": ({"walks": wc[0], "expansions": wc[1] / wc[0],
                                              "front_refills": wc[2] / wc[0], "pool_slots_scanned": wc[3] / wc[0],
                                              "front_merges": wc[4] / wc[0], "result_inserts": wc[5] / wc[0],
                                              "max_expansions": wc[6]} if len(wc) >= 7 and wc[0] else None),
            "recall_at_10_vs_exact_filtered": recall,
            "e2e": {"value": nq / (float(te.item()) / 1000.0), "unit": "queries/s",
                    "h2d_bytes_per_step": nq * DIM * 4, "d2h_bytes_per_step": nq * K * 12},
            "gpu_launches": int(lt.item()),
            "clocks": clk,
            "setup_s": {"total_rank0": setup_s, "hnsw_build_rank0": build_s, "graphs_from_cache_rank0": cached},
        }
        if world == 1:
            # CPU baseline: the reference's own Collection on the host cores, one full segment it
            # bulk-loaded itself, a bounded query sample; QPS scaled to the 64 segments.
            qps_seg, n_timed, build = c4_reference_sample(args, 1, args.cpu_seconds)
            result["cpu_baseline"] = {
                "value": qps_seg / args.segments, "unit": "queries/s", "cores": os.cpu_count(), "kind": "reference",
                "sample": f"{n_timed} queries (grouped by tag, one SearchBatch per filter) over 1 full segment of "
                          f"{args.seg_rows} rows bulk-loaded by the reference; QPS scaled by 1/{args.segments} "
                          f"segments ({cpu_model()})"}
        print(json.dumps(result), flush=True)
    if group is not None:
        group.close()
    coll.free()
    ctx.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def c4_reference_collection(seg_rows, ref_segments):
    """A collection of `ref_segments` full-size config-4 segments bulk-loaded by the reference's own
    Collection (it builds each segment's HNSW graph itself), kept in VDB_BENCH_CACHE (default the
    system temp directory) so later runs on the same host reopen it. Returns (RefCollection,
    build seconds or None when reopened)."""
    import shutil
    import oracle
    cache = os.environ.get("VDB_BENCH_CACHE", tempfile.gettempdir())
    path = os.path.join(cache, f"vdb_c4_ref_{ref_segments}x{seg_rows}")
    if os.path.exists(os.path.join(path, "CURRENT")):
        try:
            return oracle.RefCollection.open(path, threads=os.cpu_count()), None
        except RuntimeError:
            shutil.rmtree(path, ignore_errors=True)
    tmp = f"{path}.{os.getpid()}.part"
    shutil.rmtree(tmp, ignore_errors=True)
    coll = oracle.RefCollection(tmp, DIM, metric="cosine", index=C4_OPTIONS["index"],
                                schema=C4_OPTIONS["schema"], threads=os.cpu_count())
    t = time.time()
    for s in range(ref_segments):
        rows, ids, years, tags = c4_segment(s, seg_rows)
        coll.bulk_load(ids, rows, years, tags)
    build = time.time() - t
    coll.close()
    try:
        os.replace(tmp, path)
        return oracle.RefCollection.open(path, threads=os.cpu_count()), build
    except OSError:
        return oracle.RefCollection.open(tmp, threads=os.cpu_count()), build


def c4_reference_sample(args, ref_segments, seconds):
    """The reference's Collection (oracle/_ref/libvdbref_engine.so, its own code) over
    `ref_segments` full-size config-4 segments it bulk-loaded itself, SearchBatch per filter group
    over a query sample of about `seconds` of CPU work. Returns (queries per second over those
    segments, queries timed, build seconds or None when the collection was reopened)."""
    coll, build = c4_reference_collection(args.seg_rows, ref_segments)
    qs, filters, qf = c4_queries(args.batch)
    order = np.argsort(qf, kind="stable")

    def run(qidx):
        groups = {}
        for i in qidx:
            groups.setdefault(int(qf[i]), []).append(i)
        t0 = time.perf_counter()
        for f, members in groups.items():
            coll.search(qs[members], k=K, ef=C4_EF, filter=filters[f])
        return time.perf_counter() - t0

    probe = order[:: max(1, len(order) // 64)][:64]
    per_q = max(run(probe) / len(probe), 1e-6)
    n = int(min(len(order), max(64, seconds / per_q)))
    sample = order[:: max(1, len(order) // n)][:n]
    secs = run(sample)
    coll.close()
    return len(sample) / secs, len(sample), build


def run_c4_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    ref_segments = 1
    qps_seg, nq_timed, build = c4_reference_sample(args, ref_segments, args.cpu_seconds)
    qps = qps_seg * ref_segments / args.segments  # every query searches every segment
    out = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s", "n_gpus": args.gpus,
        "steps": 1, "warmup": 1, "ms_per_step": 1000.0 * args.batch / qps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": C4_WORKLOAD.format(segs=args.segments, rows=args.seg_rows),
                   "rows": args.segments * args.seg_rows, "segments": args.segments, "batch": args.batch,
                   "k": K, "ef": C4_EF},
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": os.cpu_count(), "kind": "reference",
                         "sample": f"{nq_timed} queries (grouped by tag, one SearchBatch per filter) over "
                                   f"{ref_segments} full segment of {args.seg_rows} rows bulk-loaded by the reference "
                                   f"({'reopened' if build is None else f'built in {build:.0f} s'}); QPS scaled by "
                                   f"{ref_segments}/{args.segments} segments "
                                   f"({cpu_model()})"},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)
    return 0


# ---------------------------------------------------------------------------- configs 0 and 3

C0_WORKLOAD = ("config 0: exact flat L2 search, 100,000 x 128 integer rows (100-centre mixture, "
               "U[0,100] centres, sigma 10, clipped to [0,255] and rounded), 1,000-query batches, k=10")
C3_ROWS = 1_000_000
C3_WORKLOAD = ("config 3: HNSW batched search, 1,000,000 x 128 integer rows (config-0 mixture), L2, graph "
               "built by the reference (HnswIndex / HnswSq8Index M=16, ef_construction=200, seed 42) and "
               "loaded from its index file, {variant} distances, ef={ef}, 10,000-query batches, k=10")


def _timed(step, steps, warmup, stream, local):
    import torch
    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, clocks.stop()


def _recall(ids, gt):
    return float(np.mean([len(set(a.tolist()) & set(b.tolist())) / gt.shape[1] for a, b in zip(ids, gt)]))


def run_c0_c3(args):
    """Configs 0 and 3 on one GPU (single-segment configs: replicas only, so one line per GPU)."""
    import torch
    import oracle
    import vdb_b200
    from vdb_b200 import synth
    world, rank, local = dist_setup()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    ctx = vdb_b200.Context(local)
    stream = torch.cuda.current_stream()
    ctx.set_stream(stream.cuda_stream)
    sustained, burst, hbm, src = peaks()
    ref = oracle.Ref()
    if args.workload == "c0":
        base, qs = synth.flat_int(100_000, 1_000, seed=0)
        idx = vdb_b200.Index.create(ctx, "flat", "l2", base, DIM)
        q_dev = torch.from_numpy(qs).cuda()
        ids_dev = torch.empty((qs.shape[0], K), dtype=torch.int32, device="cuda")
        d_dev = torch.empty((qs.shape[0], K), dtype=torch.float32, device="cuda")
        ctx.set_timing(True)
        scan = []

        def step():
            idx.search(q_dev, k=K, out=(ids_dev, d_dev))
            scan.append(ctx.stage_times()[1])
        ms, clk = _timed(step, max(args.steps, 1000), args.warmup, stream, local)
        nq = qs.shape[0]
        flops = 2.0 * nq * base.shape[0] * DIM
        scan_s = float(np.median(scan)) / 1000.0
        ref_ids, _ = ref.flat_search_batch(oracle.L2, base, DIM, qs[:200], K, threads=0)
        t0 = time.perf_counter()
        ref_ids, _ = ref.flat_search_batch(oracle.L2, base, DIM, qs, K, threads=0)
        cpu_s = time.perf_counter() - t0
        gpu_ids = ids_dev.cpu().numpy().view(np.uint32)
        out = {"metric": METRIC, "value": nq / (ms / 1000.0), "unit": "queries/s", "n_gpus": 1, "steps": max(args.steps, 1000),
               "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "f16 tensor-core pre-rank (exact for these integer rows), f32 re-rank",
               "data": "synthetic", "config": {"workload": C0_WORKLOAD, "rows": base.shape[0], "batch": nq, "k": K,
                                              "l2": "inputs smaller than L2 (51 MB rows): repeated batches"},
               "roofline": {"bound": "tensor", "kernel": "scan_mma_kernel", "achieved": flops / scan_s / 1e12,
                            "peak": burst, "unit": "TFLOP/s", "frac": flops / scan_s / 1e12 / burst,
                            "peak_kind": f"{src} bf16 dense, burst", "traffic": None},
               "identical_ids_vs_reference": float(np.mean(np.all(gpu_ids == ref_ids, axis=1))),
               "cpu_baseline": {"value": nq / cpu_s, "unit": "queries/s", "cores": os.cpu_count(), "kind": "reference",
                                "sample": f"all {nq} queries (FlatSearchBatch, {cpu_model()}, kernel set {ref.kernel_set()})"},
               "clocks": clk}
        print(json.dumps(out), flush=True)
        return 0
    return run_c3(args, ctx, stream, local, ref, hbm, src)


def reference_graph(ref, type_, base, seed_rows):
    """index.hnsw (type 1) or index.hnsw_sq8 (type 2) for config 3, built once by the reference's
    own HnswIndex / HnswSq8Index {M=16, ef_construction=200, seed=42} on every host core and kept
    in a cache directory (VDB_BENCH_CACHE, default the system temp directory) so later runs on the
    same host load the same file. A parallel build is not deterministic; the GPU and the reference
    both search the one file. Returns (file bytes, build seconds or None when cached)."""
    cache = os.environ.get("VDB_BENCH_CACHE", tempfile.gettempdir())
    name = os.path.join(cache, f"vdb_c3_{'hnsw' if type_ == 1 else 'hnsw_sq8'}_{base.shape[0]}_s{seed_rows}_m16_efc200.idx")
    if os.path.exists(name):
        with open(name, "rb") as f:
            return f.read(), None
    import oracle
    t = time.time()
    data = ref.build_index(type_, oracle.L2, base, DIM, M=16, efc=200, seed=42, threads=0).save()
    build_s = time.time() - t
    tmp = name + f".{os.getpid()}.part"
    with open(tmp, "wb") as f:
        f.write(data)
    os.replace(tmp, name)
    return data, build_s


def run_c3(args, ctx, stream, local, ref, hbm, src):
    """Config 3: batched HNSW search over graphs the reference builds itself (fp32 and SQ8 distance
    variants) at ef 64 / 128 / 256. One JSON line per (variant, ef)."""
    import torch
    import oracle
    import vdb_b200
    from vdb_b200 import synth
    base, qs = synth.flat_int(C3_ROWS, args.batch, seed=0)
    b_dev = torch.from_numpy(base).cuda()
    flat = vdb_b200.Index.create(ctx, "flat", "l2", b_dev, DIM)
    q_dev = torch.from_numpy(qs).cuda()
    nq = qs.shape[0]
    gt_ids = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    gt_d = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    flat.search(q_dev, k=K, out=(gt_ids, gt_d))
    gt = gt_ids.cpu().numpy().view(np.uint32)
    flat.free()
    variants = [v for v in ((1, "fp32"), (2, "sq8")) if v[1] in args.c3_variants.split(",")]
    for type_, variant in variants:
        data, build_s = reference_graph(ref, type_, base, 0)
        idx = vdb_b200.Index.load(ctx, data, "l2", b_dev, DIM)
        rref = ref.load_index(data, oracle.L2, base, DIM)
        for ef in (int(x) for x in args.c3_ef.split(",")):
            ids_dev = torch.empty((nq, K), dtype=torch.int32, device="cuda")
            d_dev = torch.empty((nq, K), dtype=torch.float32, device="cuda")
            ctx.set_timing(True)
            walk_ms = []

            def step():
                idx.search(q_dev, k=K, ef=ef, out=(ids_dev, d_dev))
                walk_ms.append(ctx.stage_times()[1])
            ms, clk = _timed(step, args.steps, args.warmup, stream, local)
            # Walk counters of the last step: walks, expansions, front refills, pool slots scanned,
            # merges into the front, result inserts, most expansions of one walk.
            wc = ctx.stage_counters()[:7]
            ctx.set_timing(False)
            gpu_ids = ids_dev.cpu().numpy().view(np.uint32).copy()
            gpu_d = d_dev.cpu().numpy().copy()
            _, _, dc = idx.search(qs, k=K, ef=ef, stats=True)
            depth = max(ef, K)
            if variant == "fp32":
                bytes_per_q = float(dc.mean()) * (DIM * 4 + 4)
                formula = f"dc x (pd x 4 + 4) B per query (row + link id), dc = {dc.mean():.0f} (mean)"
            else:
                bytes_per_q = float(dc.mean()) * (DIM + 4) + depth * DIM * 4
                formula = (f"dc x (pd + 4) + depth x pd x 4 B per query (code + link id, re-ranked rows), "
                           f"dc = {dc.mean():.0f} (mean), depth = {depth}")
            kernel_ms = float(np.median(walk_ms)) if walk_ms and walk_ms[0] > 0 else ms
            achieved = bytes_per_q * nq / (kernel_ms / 1000.0) / 1e9
            # The reference's own index over the same file on every host core: all queries, for
            # the identity check, and as the timed CPU baseline.
            rref.search(qs[:200], k=K, ef=ef)
            t0 = time.perf_counter()
            r_ids, r_d, r_dc = rref.search(qs, k=K, ef=ef)
            cpu_s = time.perf_counter() - t0
            same = np.all(gpu_ids == r_ids, axis=1)
            out = {"metric": METRIC, "value": nq / (ms / 1000.0), "unit": "queries/s", "n_gpus": 1,
                   "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                   "scaling": "weak", "vs_baseline": None, "dtype": "f32" if variant == "fp32" else "u8 codes, f32 re-rank",
                   "data": "synthetic",
                   "config": {"workload": C3_WORKLOAD.format(variant=variant, ef=ef), "rows": C3_ROWS,
                              "batch": nq, "k": K, "ef": ef, "variant": variant,
                              "l2": "inputs larger than L2: 512 MB rows + 132 MB graph"},
                   "roofline": {"bound": "hbm", "kernel": "hnsw_search_kernel", "achieved": achieved, "peak": hbm,
                                "unit": "GB/s", "frac": achieved / hbm, "peak_kind": f"{src} copy bandwidth",
                                "kernel_ms": kernel_ms, "traffic": hnsw_traffic_per_launch(variant, ef, nq),
                                "algorithmic": formula},
                   "walk_counters_per_query": ({"expansions": wc[1] / nq, "front_refills": wc[2] / nq,
                                                "pool_slots_scanned": wc[3] / nq, "front_merges": wc[4] / nq,
                                                "result_inserts": wc[5] / nq, "max_expansions": wc[6]}
                                               if len(wc) >= 7 and wc[0] else None),
                   "recall_at_10_vs_exact": _recall(gpu_ids, gt),
                   "recall_at_10_reference_vs_exact": _recall(r_ids, gt),
                   "identical_ids_vs_reference_same_graph": float(np.mean(same)),
                   "identical_dists_vs_reference_same_graph": float(np.mean(np.all(gpu_d == r_d, axis=1))),
                   "identical_dist_computations_vs_reference": float(np.mean(dc == r_dc)),
                   "differing_queries": np.nonzero(~same)[0][:8].tolist(),
                   "e2e": None,
                   "gpu_launches": args.steps,
                   "cpu_baseline": {"value": nq / cpu_s, "unit": "queries/s", "cores": os.cpu_count(),
                                    "kind": "reference",
                                    "sample": f"all {nq} queries, the reference's {'HnswIndex' if variant == 'fp32' else 'HnswSq8Index'} "
                                              f"on the same index file ({cpu_model()}, kernel set {ref.kernel_set()})"},
                   "graph": {"built_by": "reference HnswIndex{M=16, ef_construction=200, seed=42}, all host cores",
                             "build_s": build_s, "file_bytes": len(data)},
                   "clocks": clk}
            # e2e: host queries and host results through the same C-ABI call.
            q_host = torch.from_numpy(qs).pin_memory()
            ids_host = torch.empty((nq, K), dtype=torch.int32).pin_memory()
            d_host = torch.empty((nq, K), dtype=torch.float32).pin_memory()
            idx.search(q_host, k=K, ef=ef, out=(ids_host, d_host))
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            e2e_steps = max(3, args.steps // 2)
            for _ in range(e2e_steps):
                idx.search(q_host, k=K, ef=ef, out=(ids_host, d_host))
            e1.record(stream)
            torch.cuda.synchronize()
            out["e2e"] = {"value": nq / (e0.elapsed_time(e1) / e2e_steps / 1000.0), "unit": "queries/s",
                          "h2d_bytes_per_step": nq * DIM * 4, "d2h_bytes_per_step": nq * K * 8}
            print(json.dumps(out), flush=True)
        idx.free()
    return 0


def hnsw_traffic_per_launch(variant, ef, nq):
    """DRAM bytes of one walk launch from the committed ncu summary, scaled to nq queries."""
    path = os.path.join(ROOT, "profiles", "hnsw_walk_config3.json")
    if os.path.exists(path):
        with open(path) as f:
            rec = json.load(f).get(f"{variant}_ef{ef}")
        if rec:
            return rec["dram_bytes_per_query"] * nq
    return None


# -------------------------------------------------------------------------------------- config 2

C2_ROWS, C2_DIM, C2_NLIST, C2_M, C2_PPC, C2_NPROBE = 10_000_000, 96, 4096, 48, 122, 32
C2_WORKLOAD = ("config 2: IVF-PQ L2 search, 10,000,000 x 96 rows (1,000-component mixture, centres U[-1,1]^96, "
               "sigma 0.15), nlist 4096, PQ M=48 x 8 bits, trained by the reference's seeded k-means on a "
               "499,712-row sample (122 points per centroid), replayed on the GPU (the reference's index file, "
               "byte for byte), nprobe 32, re-rank 100, 10,000-query batches, k=10")


def run_c2(args):
    """Config 2 on one GPU (one segment: replicas only). The index is built by the GPU builder; the
    reference loads the same file and is timed on the host cores over a query sample."""
    import torch
    import oracle
    import vdb_b200
    from vdb_b200 import synth
    world, rank, local = dist_setup()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    ctx = vdb_b200.Context(local)
    stream = torch.cuda.current_stream()
    sustained, burst, hbm, src = peaks()
    nq = args.batch
    n_rows = args.c2_rows
    rows = synth.mixture(n_rows, C2_DIM, 1000, centres="uniform", lo=-1.0, hi=1.0, sigma=0.15, seed=2, stream=0)
    qs = synth.mixture(nq, C2_DIM, 1000, centres="uniform", lo=-1.0, hi=1.0, sigma=0.15, seed=2, stream=1)
    t = time.time()
    data = vdb_b200.build_ivfpq(ctx, rows, C2_DIM, nlist=C2_NLIST, pq_m=C2_M,
                                max_train_points_per_centroid=C2_PPC, seed=42)
    build_s = time.time() - t
    b_dev = torch.from_numpy(rows).cuda()
    idx = vdb_b200.Index.load(ctx, data, "l2", b_dev, C2_DIM)
    q_dev = torch.from_numpy(qs).cuda()
    ids_dev = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    d_dev = torch.empty((nq, K), dtype=torch.float32, device="cuda")

    def step():
        idx.search(q_dev, k=K, nprobe=C2_NPROBE, out=(ids_dev, d_dev))
    ms, clk = _timed(step, args.steps, args.warmup, stream, local)
    gpu_ids = ids_dev.cpu().numpy().view(np.uint32).copy()
    # Launches per step, and the stages of the tensor-core path (marks: after the coarse probe,
    # after the nearest-list pass, after the scan of all probed lists, after the exact stage), from
    # separate timed steps.
    launches0 = vdb_b200.launch_count()
    step()
    torch.cuda.synchronize()
    launches_per_step = vdb_b200.launch_count() - launches0
    ctx.set_timing(True)
    st = np.zeros(3)
    for _ in range(3):
        step()
        st += np.array(ctx.stage_times()[:3])
    fc = ctx.stage_counters()
    ctx.set_timing(False)
    st /= 3
    # End to end through the C ABI from pinned host buffers.
    q_host = torch.from_numpy(qs).pin_memory()
    ids_host = torch.empty((nq, K), dtype=torch.int32).pin_memory()
    d_host = torch.empty((nq, K), dtype=torch.float32).pin_memory()
    for _ in range(2):
        idx.search(q_host, k=K, nprobe=C2_NPROBE, out=(ids_host, d_host))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_steps = max(3, args.steps // 2)
    for _ in range(e2e_steps):
        idx.search(q_host, k=K, nprobe=C2_NPROBE, out=(ids_host, d_host))
    torch.cuda.synchronize()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    _, _, dc = idx.search(qs[:1000], k=K, nprobe=C2_NPROBE, stats=True)
    # Algorithmic bytes per query: the codes and ids of the probed lists, one 1 KB table per
    # subquantizer per list, and the re-ranked rows.
    scanned = float(dc.mean()) - C2_NLIST - DEPTH
    bytes_per_q = scanned * (C2_M + 4) + C2_NPROBE * C2_M * 1024 + DEPTH * C2_DIM * 4
    achieved = bytes_per_q * nq / (ms / 1000.0) / 1e9
    tflops = 2.0 * C2_DIM * scanned * nq / (max(float(st[1]), 1e-6) / 1000.0) / 1e12
    # Exact ground truth on the GPU (flat index over the same rows).
    flat = vdb_b200.Index.create(ctx, "flat", "l2", b_dev, C2_DIM)
    gt_ids = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    gt_d = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    flat.search(q_dev, k=K, out=(gt_ids, gt_d))
    gt = gt_ids.cpu().numpy().view(np.uint32)
    flat.free()
    # The reference's own IvfPqIndex on the same file, all host threads, a bounded query sample.
    ref = oracle.Ref()
    rref = ref.load_index(data, oracle.L2, rows, C2_DIM, pq_m=C2_M)
    rref.search(qs[:50], k=K, nprobe=C2_NPROBE)
    t0 = time.perf_counter()
    sample = 0
    r_ids = []
    while sample < nq and time.perf_counter() - t0 < args.cpu_seconds:
        r, _, _ = rref.search(qs[sample:sample + 500], k=K, nprobe=C2_NPROBE)
        r_ids.append(r)
        sample += r.shape[0]
    cpu_s = time.perf_counter() - t0
    r_ids = np.concatenate(r_ids)
    out = {"metric": METRIC, "value": nq / (ms / 1000.0), "unit": "queries/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "f32 ADC tables, f32 re-rank", "data": "synthetic",
           "config": {"workload": C2_WORKLOAD if n_rows == C2_ROWS else f"config 2 shape at {n_rows} rows",
                      "rows": n_rows, "dim": C2_DIM, "batch": nq, "k": K,
                      "nlist": C2_NLIST, "pq_m": C2_M, "nprobe": C2_NPROBE, "rerank": DEPTH,
                      "l2": "inputs larger than L2: 520 MB of codes and ids + 3.8 GB rows"},
           # The dominant kernel is the list-mode scan of the probed lists (tensor-core pre-rank):
           # 2 x d FLOP per (query, probed row), over that stage's CUDA-event time. Beside it, the
           # bytes the reference's per-query ADC would read, over the whole step.
           "roofline": {"bound": "tensor", "kernel": "scan_mma_kernel<kKeyList> (scan of the probed lists)",
                        "achieved": tflops, "peak": burst, "unit": "TFLOP/s", "frac": tflops / burst,
                        "peak_kind": f"{src} bf16 dense, burst", "traffic": None,
                        "algorithmic": f"2 x {C2_DIM} x scanned FLOP per query, scanned = {scanned:.0f} rows "
                                       f"(mean), over the probed-lists stage ({st[1]:.3f} ms)",
                        "whole_step_reference_algorithm": {
                            "achieved_gbs": achieved, "frac_of_hbm": achieved / hbm,
                            "bytes": "scanned x (m + 4) + nprobe x m x 1 KB + 100 x pd x 4 B per query: the "
                                     "per-query ADC's reads; list tiles share each list's rows instead"}},
           "e2e": {"value": nq / e2e_s, "unit": "queries/s", "h2d_bytes_per_step": nq * C2_DIM * 4,
                   "d2h_bytes_per_step": nq * K * 8},
           "stage_ms": {"nearest_list_pass": float(st[0]), "probed_lists_scan": float(st[1]),
                        "exact_stage": float(st[2])},
           "exact_stage_per_query": {"entries_below_bound": fc[0] / nq, "radix_cut_fraction": fc[1] / nq,
                                     "warp_cycles_gather": fc[2] / nq, "warp_cycles_adc": fc[3] / nq,
                                     "warp_cycles_topk_rerank": fc[4] / nq} if len(fc) >= 5 else None,
           "gpu_launches": int(launches_per_step) * args.steps,
           "recall_at_10_vs_exact": _recall(gpu_ids, gt),
           "identical_ids_vs_reference_same_index": float(np.mean(np.all(gpu_ids[:sample] == r_ids, axis=1))),
           "cpu_baseline": {"value": sample / cpu_s, "unit": "queries/s", "cores": os.cpu_count(), "kind": "reference",
                            "sample": f"{sample} queries, the reference's IvfPqIndex on the same index file "
                                      f"({cpu_model()}, kernel set {ref.kernel_set()})"},
           "index_build_s_gpu": build_s, "index_bytes": len(data), "clocks": clk}
    print(json.dumps(out), flush=True)
    idx.free()
    return 0


def main():
    args = parse()
    if args.workload == "c2":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "config 2 times the reference inside the same "
                                                                  "run (cpu_baseline)"}))
            return 0
        return run_c2(args)
    if args.workload in ("c0", "c3"):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "configs 0 and 3 time the reference inside "
                                                                  "the same run (cpu_baseline)"}))
            return 0
        return run_c0_c3(args)
    if args.workload == "c4":
        if args.impl == "reference":
            return run_c4_reference(args)
        return run_c4_ours(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
