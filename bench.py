#!/usr/bin/env python
"""Benchmark of the batched search path on B200: batched QPS at fixed recall@10.

Workload (the configuration the headline metric is quoted on): an exhaustive SQ8 scan with an
fp32 re-rank of the top 100 over 1,000,000 unit-normalised 128-d vectors (1,000-centre Gaussian
mixture, sigma 0.3), 10,000-query batches, k = 10, cosine. Synthetic seeded data stands in for
the reference's public datasets.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line on rank 0. A step is one batched search of 10,000 queries. `value` is device-resident
throughput (queries already in HBM); `e2e` is the same call through the C ABI with host (pinned)
buffers, copies included. Multi-GPU runs are replicas (one full index per GPU, each rank its own
batch): the path has a single segment, so nothing shards and there is no collective.
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


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--rows", type=int, default=N_ROWS)
    p.add_argument("--batch", type=int, default=NQ)
    p.add_argument("--cpu-seconds", type=float, default=10.0)
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
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

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
    launches_per_step = 3  # prep_queries, scan_mma, finalize

    def step():
        idx.search(q_dev, k=K, rerank=DEPTH, out=(ids_dev, d_dev))

    for _ in range(max(3, args.warmup)):
        step()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    scan_ms, stage, counters = [], np.zeros(3), np.zeros(4)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
        st = ctx.stage_times()
        scan_ms.append(st[1])
        stage += np.array(st[:3])
        counters += np.array(ctx.stage_counters()[:4], dtype=np.float64)
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
        roof = {"bound": "tensor", "kernel": "scan_mma_kernel", "achieved": achieved,
                "peak": sustained, "unit": "TFLOP/s", "frac": achieved / sustained,
                "peak_kind": f"{src} bf16 dense, sustained (burst {burst})",
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
            "stage_ms": {"prep": stage[0] / args.steps, "scan": stage[1] / args.steps,
                         "select_rerank": stage[2] / args.steps},
            "scan_counters_per_step": {"chunks": counters[0] / args.steps,
                                       "chunks_with_candidates": counters[1] / args.steps,
                                       "candidates_per_query": counters[2] / args.steps / nq,
                                       "compactions_per_query": counters[3] / args.steps / nq},
            "e2e": {"value": e2e_value, "unit": "queries/s", "h2d_bytes_per_step": nq * DIM * 4,
                    "d2h_bytes_per_step": nq * K * 8},
            "gpu_launches": launches_per_step * args.steps,
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


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
