"""Generates the golden fixtures in tests/golden/ by running the reference itself.

The reference's index layer (vdb, compiled in place from its sources into oracle/_ref by
oracle/Makefile) builds indexes and answers queries on small seeded inputs; this script stores
its index files and outputs. Input rows are NOT stored: tests regenerate them with the seeded
generator (vdb_b200.synth) and check them against the SHA-256 recorded here.

Run from the repo root (needs oracle/_ref/libvdbref.so, i.e. the reference sources at build time):
    python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "hnsw-vector-db_b200"))

import oracle  # noqa: E402
from vdb_b200 import synth  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
FLAT, HNSW, HNSW_SQ8, PQ_FLAT, IVF_PQ = 0, 1, 2, 3, 4


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def save(name, **kw):
    np.savez_compressed(os.path.join(OUT, name + ".npz"), **kw)
    print("wrote", name, sum(v.nbytes for v in kw.values() if isinstance(v, np.ndarray)), "bytes")


def bits_of(mask):
    return np.asarray(__import__("vdb_b200").pack_bitset(mask))


def main():
    oracle.build(ref=True)
    ref = oracle.Ref()
    ks = ref.kernel_set()
    print("reference kernel set:", ks)

    # ---------------------------------------------------------------- distances + top-k pins
    rng = np.random.default_rng(7)
    dims = [1, 7, 16, 31, 32, 33, 48, 64, 96, 100, 112, 128, 200, 256, 1000]
    pairs = []
    for d in dims:
        pd = (d + 15) // 16 * 16
        a = np.zeros(pd, np.float32)
        b = np.zeros(pd, np.float32)
        a[:d] = rng.standard_normal(d).astype(np.float32)
        b[:d] = rng.standard_normal(d).astype(np.float32)
        pairs.append((a, b))
    dist_l2 = np.array([ref.distance(0, a, b) for a, b in pairs], np.float32)
    dist_dot = np.array([ref.distance(1, a, b) for a, b in pairs], np.float32)
    dist_ip = np.array([ref.distance(2, a, b) for a, b in pairs], np.float32)
    sq8_q, sq8_c, sq8_vmin, sq8_scale, sq8_l2, sq8_ip = [], [], [], [], [], []
    for d in [16, 100, 128, 384]:
        pd = (d + 15) // 16 * 16
        q = np.zeros(pd, np.float32)
        q[:d] = rng.uniform(-2, 2, d)
        vmin = np.zeros(pd, np.float32)
        vmin[:d] = rng.uniform(-2, 2, d)
        scale = np.zeros(pd, np.float32)
        scale[:d] = np.abs(rng.uniform(-2, 2, d)).astype(np.float32) / np.float32(255)
        c = np.zeros(pd, np.uint8)
        c[:d] = rng.integers(0, 256, d)
        sq8_q.append(q), sq8_c.append(c), sq8_vmin.append(vmin), sq8_scale.append(scale)
        sq8_l2.append(ref.sq8_distance(0, q, c, vmin, scale))
        sq8_ip.append(ref.sq8_distance(1, q, c, vmin, scale))
    # Metric convention pins (tests/distance_test.cc:86-91).
    ca = np.zeros(16, np.float32); ca[0] = 1
    cb = np.zeros(16, np.float32); cb[:2] = 0.5
    conv = np.array([ref.distance(0, ca, cb), ref.distance(2, ca, cb)], np.float32)
    # Top-k with heavy ties (tests/topk_test.cc:14-33).
    tk_d, tk_k, tk_out_i, tk_out_d, tk_n = [], [], [], [], []
    trng = np.random.default_rng(1)
    for trial in range(60):
        n = int(trng.integers(1, 500))
        k = int(trng.integers(1, 50))
        hi = 5 if trial % 2 == 0 else 1000
        d = trng.integers(0, hi + 1, n).astype(np.float32)
        ids = np.arange(n, dtype=np.uint32)
        oi, od = ref.topk(d, ids, k)
        tk_d.append(np.pad(d, (0, 500 - n), constant_values=np.nan)), tk_n.append(n), tk_k.append(k)
        tk_out_i.append(np.pad(oi, (0, 50 - oi.size), constant_values=2**32 - 1))
        tk_out_d.append(np.pad(od, (0, 50 - od.size), constant_values=np.inf))
    save("kernels", kernel_set=np.array(ks), dims=np.array(dims),
         pair_a=np.stack([np.pad(a, (0, 1008 - a.size)) for a, _ in pairs]),
         pair_b=np.stack([np.pad(b, (0, 1008 - b.size)) for _, b in pairs]),
         l2=dist_l2, dot=dist_dot, ip=dist_ip,
         sq8_q=np.stack([np.pad(x, (0, 384 - x.size)) for x in sq8_q]),
         sq8_c=np.stack([np.pad(x, (0, 384 - x.size)) for x in sq8_c]),
         sq8_vmin=np.stack([np.pad(x, (0, 384 - x.size)) for x in sq8_vmin]),
         sq8_scale=np.stack([np.pad(x, (0, 384 - x.size)) for x in sq8_scale]),
         sq8_dims=np.array([16, 100, 128, 384]), sq8_l2=np.array(sq8_l2, np.float32),
         sq8_ip=np.array(sq8_ip, np.float32), convention=conv,
         topk_d=np.stack(tk_d), topk_n=np.array(tk_n), topk_k=np.array(tk_k),
         topk_ids=np.stack(tk_out_i), topk_dists=np.stack(tk_out_d))

    # ---------------------------------------------------------------- flat (config-0 style)
    base, qs = synth.flat_int(4000, 64, dim=128, seed=10)
    ids, d = ref.flat_search_batch(0, base, 128, qs, 10)
    odd = (np.arange(base.shape[0]) % 2) == 1
    fidx = ref.build_index(FLAT, 0, base, 128)
    fids, fd, fdc = fidx.search(qs, k=50, allow=bits_of(odd))
    save("flat_int", base_sha=np.array(sha(base)), query_sha=np.array(sha(qs)), seed=np.array(10),
         n=np.array(4000), nq=np.array(64), ids=ids, dists=d, filt_ids=fids, filt_dists=fd,
         flat_file=np.frombuffer(fidx.save(), np.uint8))

    # flat over float rows with an odd dimension (100 -> 112), every metric
    fb, fq = synth.sharded_cosine(3000, 40, dim=100, seed=11)
    out = {}
    for m in (0, 1, 2):
        i, dd = ref.flat_search_batch(m, fb, 100, fq, 20)
        out[f"ids_m{m}"], out[f"dists_m{m}"] = i, dd
    save("flat_float", base_sha=np.array(sha(fb)), query_sha=np.array(sha(fq)), seed=np.array(11),
         n=np.array(3000), nq=np.array(40), dim=np.array(100), **out)

    # ---------------------------------------------------------------- SQ8 scan (config-1 style)
    sb, sq = synth.sq8_cosine(5000, 40, dim=128, seed=12)
    vmin, scale, codes = ref.sq8_train_encode(sb, 128)
    si, sd, spi, spd = ref.sq8_scan_search(2, sb, codes, vmin, scale, sq, k=10, depth=100, pre=True)
    save("sq8_scan", base_sha=np.array(sha(sb)), query_sha=np.array(sha(sq)), seed=np.array(12),
         n=np.array(5000), nq=np.array(40), vmin=vmin, scale=scale, codes=codes, ids=si, dists=sd,
         pre_ids=spi, pre_dists=spd)

    # ---------------------------------------------------------------- HNSW (config-3 style)
    hb, hq = synth.flat_int(6000, 64, dim=128, seed=13)
    hidx = ref.build_index(HNSW, 0, hb, 128, M=16, efc=100, seed=42, threads=1)
    hfile = hidx.save()
    res = {}
    for ef in (16, 64, 128):
        i, dd, dc = hidx.search(hq, k=10, ef=ef)
        res[f"ids_ef{ef}"], res[f"dists_ef{ef}"], res[f"dc_ef{ef}"] = i, dd, dc
    even = (np.arange(hb.shape[0]) % 2) == 0
    i, dd, dc = hidx.search(hq, k=10, ef=64, allow=bits_of(even))
    res["filt_ids"], res["filt_dists"], res["filt_dc"] = i, dd, dc
    save("hnsw", base_sha=np.array(sha(hb)), query_sha=np.array(sha(hq)), seed=np.array(13),
         n=np.array(6000), nq=np.array(64), index_file=np.frombuffer(hfile, np.uint8), **res)

    # HNSW-SQ8 over the same rows
    qidx = ref.build_index(HNSW_SQ8, 0, hb, 128, M=16, efc=100, seed=42, threads=1)
    qfile = qidx.save()
    res = {}
    for ef, rr in ((32, -1), (64, -1), (64, 0), (64, 20)):
        i, dd, dc = qidx.search(hq, k=10, ef=ef, rerank=rr)
        tag = f"ef{ef}_r{'auto' if rr < 0 else rr}"
        res[f"ids_{tag}"], res[f"dists_{tag}"], res[f"dc_{tag}"] = i, dd, dc
    save("hnsw_sq8", base_sha=np.array(sha(hb)), query_sha=np.array(sha(hq)), seed=np.array(13),
         n=np.array(6000), nq=np.array(64), index_file=np.frombuffer(qfile, np.uint8), **res)

    # ---------------------------------------------------------------- IVF-PQ / PQ-flat (config-2 style)
    ib, iq = synth.ivfpq_l2(6000, 48, dim=96, seed=14)
    iidx = ref.build_index(IVF_PQ, 0, ib, 96, pq_m=48, nlist=64, seed=42, threads=0)
    ifile = iidx.save()
    res = {}
    for nprobe, rr in ((4, -1), (16, -1), (16, 0)):
        i, dd, dc = iidx.search(iq, k=10, nprobe=nprobe, rerank=rr)
        tag = f"np{nprobe}_r{'auto' if rr < 0 else rr}"
        res[f"ids_{tag}"], res[f"dists_{tag}"], res[f"dc_{tag}"] = i, dd, dc
    gi, gd = ref.flat_search_batch(0, ib, 96, iq, 10)
    save("ivfpq", base_sha=np.array(sha(ib)), query_sha=np.array(sha(iq)), seed=np.array(14),
         n=np.array(6000), nq=np.array(48), index_file=np.frombuffer(ifile, np.uint8), gt_ids=gi, **res)
    pidx = ref.build_index(PQ_FLAT, 0, ib, 96, pq_m=48, seed=42, threads=0)
    pfile = pidx.save()
    i, dd, dc = pidx.search(iq, k=10, rerank=-1)
    save("pqflat", base_sha=np.array(sha(ib)), query_sha=np.array(sha(iq)), seed=np.array(14),
         n=np.array(6000), nq=np.array(48), index_file=np.frombuffer(pfile, np.uint8), ids=i, dists=dd,
         dc=dc)


if __name__ == "__main__":
    main()
