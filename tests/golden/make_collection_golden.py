"""Generates the collection fixtures (tests/golden/coll_*.npz) by running the reference's own
engine layer: Collection::Create / BulkLoad / SearchBatch / Search with explain, and
SegmentColumns::Evaluate for filter bitmaps (oracle/_ref/libvdbref_engine.so, built from the
reference sources by oracle/Makefile).

Each fixture holds a small collection directory exactly as the reference wrote it (CURRENT, the
manifest, and per segment vectors.f32 / ids.u64 / meta.bin / index.<type>), the raw queries,
the filters, and for every (case, filter) the reference's merged results, its per-segment
explain of query 0, and the filter bitmap of every segment.

Run from the repo root (needs the reference sources at build time):
    python tests/golden/make_collection_golden.py
"""
import json
import os
import shutil
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "hnsw-vector-db_b200"))

import oracle  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

SCHEMA = [{"name": "year", "type": "int64"}, {"name": "score", "type": "float64"},
          {"name": "lang", "type": "keyword"}, {"name": "tags", "type": "keyword_list"},
          {"name": "flag", "type": "bool"}]

FILTERS = [
    {"and": [{"field": "year", "gte": 2020}, {"field": "tags", "eq": "t0"}]},
    {"and": [{"field": "year", "gte": 2020}, {"field": "tags", "eq": "t5"}]},
    {"field": "tags", "in": ["t1", "t2", "t29"]},
    {"not": {"field": "lang", "eq": "en"}},
    {"field": "lang", "ne": "en"},
    {"or": [{"field": "score", "lt": -1.5}, {"field": "score", "gte": 2.0}]},
    {"and": [{"field": "flag", "eq": True}, {"field": "year", "exists": False}]},
    {"field": "flag", "ne": True},
    {"field": "score", "in": [0.5, -0.25, 1.0, 0.125]},
    {"field": "tags", "eq": "nope"},
    {"and": [{"field": "year", "lte": 2000}, {"not": {"field": "tags", "ne": "t0"}}]},
    {"field": "tags", "exists": True},
    {"field": "year", "eq": 2001},
    {"field": "tags", "ne": "t0"},
    {"or": [{"field": "lang", "in": ["de", "es"]}, {"field": "year", "gt": 2022}]},
    {"not": {"or": [{"field": "flag", "exists": True}, {"field": "score", "lte": 0}]}},
]

# (strategy, prefilter_threshold, ef, nprobe, k, post_filter_alpha)
CASES = [
    ("auto", 10000, 64, 16, 10, 10),
    ("auto", 100, 16, 2, 10, 10),
    ("graph", 10000, 32, 4, 10, 10),
    ("postfilter", 10000, 64, 16, 10, 10),
    ("prefilter", 10000, 64, 16, 7, 10),
]
# IVF-PQ re-ranks max(10 k, 100) candidates (RerankDepth, src/index/quant/ivf_pq.cc:16-19); the
# GPU path keeps at most 256, so its post-filter case searches k * 2.
CASES_IVF = CASES[:3] + [("postfilter", 10000, 64, 16, 10, 2)] + CASES[4:]


def metadata(rng, n, vocab=30):
    langs = ["en", "fr", "de", "es"]
    md = []
    for _ in range(n):
        m = {}
        if rng.random() > 0.1:
            m["year"] = int(rng.integers(1990, 2025))
        if rng.random() > 0.15:
            m["score"] = float(np.round(rng.normal(0, 2) * 8) / 8)  # repeated exact values
        if rng.random() > 0.2:
            m["lang"] = langs[int(rng.integers(0, 4))]
        if rng.random() > 0.1:
            nt = int(rng.integers(0, 5))  # 0 -> an empty list (present, no tags)
            m["tags"] = ["t%d" % min(vocab - 1, int(rng.zipf(1.3)) - 1) for _ in range(nt)]
        if rng.random() > 0.3:
            m["flag"] = bool(rng.random() < 0.5)
        md.append(m)
    return md


def rows_mixture(rng, n, dim, centres):
    c = centres[rng.integers(0, centres.shape[0], n)]
    return (c + 0.35 * rng.standard_normal((n, dim))).astype(np.float32)


def pack_dir(path):
    files = {}
    for dp, _, fns in os.walk(path):
        for fn in fns:
            full = os.path.join(dp, fn)
            rel = os.path.relpath(full, path)
            if rel.startswith("wal"):
                continue
            with open(full, "rb") as f:
                files["file:" + rel] = np.frombuffer(f.read(), dtype=np.uint8)
    return files


def make(name, dim, metric, index, sizes, seed, nq=24, filters=FILTERS, cases=CASES):
    rng = np.random.default_rng(seed)
    tmp = tempfile.mkdtemp(dir=OUT)  # scratch beside the fixtures, removed below
    path = os.path.join(tmp, "coll")
    coll = oracle.RefCollection(path, dim, metric=metric, index=index, schema=SCHEMA, threads=4)
    centres = rng.standard_normal((12, dim)).astype(np.float32)
    next_id = 1000
    for n in sizes:
        rows = rows_mixture(rng, n, dim, centres)
        ids = np.arange(next_id, next_id + n, dtype=np.uint64) * 3  # external ids, not row numbers
        next_id += n
        coll.bulk_load(ids, rows, metadata=metadata(rng, n))
    q = rows_mixture(rng, nq, dim, centres)
    out = {"queries": q, "dim": np.array(dim), "metric": np.array({"l2": 0, "ip": 1, "cosine": 2}[metric]),
           "filters": np.array([json.dumps(f) for f in filters]), "schema": np.array(json.dumps(SCHEMA)),
           "cases": np.array([json.dumps(c) for c in cases]), "sizes": np.array(sizes)}
    for ci, (strategy, thr, ef, nprobe, k, alpha) in enumerate(cases):
        for fi, f in enumerate(filters + [None]):
            ids, d = coll.search(q, k=k, ef=ef, nprobe=nprobe, strategy=strategy, filter=f,
                                 prefilter_threshold=thr, post_filter_alpha=alpha)
            out[f"ids_{ci}_{fi}"] = ids
            out[f"dist_{ci}_{fi}"] = d
            ex = coll.explain(q[0], k=k, ef=ef, nprobe=nprobe, strategy=strategy, filter=f,
                              prefilter_threshold=thr, post_filter_alpha=alpha)
            disk = [e for e in ex if e["kind"] == "disk"]
            out[f"explain_{ci}_{fi}"] = np.array(json.dumps(disk))
    segdirs = coll.segment_dirs()
    for fi, f in enumerate(filters):
        for si, (sd, n) in enumerate(zip(segdirs, sizes)):
            out[f"bitmap_{fi}_{si}"] = oracle.ref_segment_bitmap(sd, SCHEMA, json.dumps(f), n)
    out["segment_ids"] = np.array([int(os.path.basename(s)[4:]) for s in segdirs])
    coll.close()
    out.update(pack_dir(path))
    shutil.rmtree(tmp)
    np.savez_compressed(os.path.join(OUT, name + ".npz"), **out)
    print("wrote", name, os.path.getsize(os.path.join(OUT, name + ".npz")), "bytes")


# Filter texts for the parser pin: valid ones of every operator and type, and every error path of
# Parser::Node / Literal (src/meta/filter_parser.cc:51-138).
PARSE_CASES = [json.dumps(f) for f in FILTERS] + [
    'not json', '[]', '3', '{}', '{"and": []}', '{"and": {"field": "year"}}', '{"or": [1]}',
    '{"and": [{"field": "year", "gte": 1}], "x": 1}', '{"not": {"field": "year", "gte": 1}, "y": 2}',
    '{"field": "year"}', '{"field": 3, "eq": 1}', '{"field": "year", "eq": 1, "ne": 2}',
    '{"field": "nope", "eq": 1}', '{"field": "year", "between": 1}', '{"field": "year", "eq": "x"}',
    '{"field": "tags", "eq": 1}', '{"field": "flag", "eq": 1}', '{"field": "flag", "in": [true]}',
    '{"field": "lang", "gt": "a"}', '{"field": "year", "in": []}', '{"field": "year", "in": 5}',
    '{"field": "year", "exists": "yes"}', '{"field": "score", "eq": 1e400}',
    '{"field": "year", "in": [' + ",".join(["1"] * 1025) + ']}',
    '{"field": "score", "in": [1e-7, 123456789012345678, 0.1, -0.0, 5e-324, 1e16, 12345.678]}',
    '{"field": "lang", "eq": "quote\\"d \\u00e9 \\n"}',
    '{"field": "year", "eq": 18446744073709551615}', '{"field": "year", "eq": -9223372036854775808}',
    '{"field":"year","gte":2020,"field":"lang"}',
    '{"field": "year", "eq": 1} trailing',
    "{" * 40 + "}" * 40,
    '{"not": ' * 33 + '{"field": "year", "eq": 1}' + "}" * 33,
    '{"not": ' * 32 + '{"field": "year", "eq": 1}' + "}" * 32,
]


def parse_golden():
    codes, texts = [], []
    for c in PARSE_CASES:
        rc, t = oracle.ref_filter_parse(SCHEMA, c)
        codes.append(rc)
        texts.append(t)
    np.savez_compressed(os.path.join(OUT, "filter_parse.npz"), cases=np.array(PARSE_CASES),
                        codes=np.array(codes), texts=np.array(texts), schema=np.array(json.dumps(SCHEMA)))
    print("wrote filter_parse", len(PARSE_CASES), "cases")


def make_deletes(name="coll_deletes", dim=4, seed=14, nq=32):
    """A collection whose disk segments carry persisted delete sets (deletes-<n>.roar, written by
    Collection::Flush after RemoveBatch and UpsertBatch). Segment A (200,000 rows) spans four
    16-bit keys, and its set holds every container kind: scattered rows (array), two contiguous
    ranges (run), every other row of a key (bitmap), and a superseded row. Segment B's set has no
    run container (cookie 12346); segment C's is one run (cookie 12347 without offsets). Rows lie on
    a 1/16 grid to keep the fixture small; half the queries sit next to deleted rows."""
    rng = np.random.default_rng(seed)
    tmp = tempfile.mkdtemp(dir=OUT)  # scratch beside the fixtures, removed below
    path = os.path.join(tmp, "coll")
    coll = oracle.RefCollection(path, dim, metric="l2", index={"type": "flat"}, schema=[], threads=4)
    sizes = [200000, 5000, 3000]
    segs = []
    next_id = 10
    for n in sizes:
        rows = (rng.integers(-64, 64, (n, dim)) / 16).astype(np.float32)
        ids = np.arange(next_id, next_id + n, dtype=np.uint64) * 5
        next_id += n
        coll.bulk_load(ids, rows)
        segs.append((ids, rows))
    (ia, ra), (ib, _), (ic, _) = segs
    rows_a = np.concatenate([np.sort(rng.choice(65536, 700, replace=False)),   # key 0: array
                             np.arange(65536, 65600), np.arange(70000, 78000),  # key 1: two runs
                             131072 + 2 * np.arange(4500),                      # key 2: bitmap
                             np.arange(196608, 196700, 3)])                     # key 3: array
    removed = np.concatenate([ia[rows_a], ib[rng.choice(5000, 40, replace=False)], ic[100:1100],
                              np.array([7, 11], np.uint64)])                    # 7, 11: absent
    up_ids = np.array([ia[199999], 3], np.uint64)  # supersedes A's last row; a new id
    up_rows = (rng.integers(-64, 64, (2, dim)) / 16).astype(np.float32)
    live = coll.remove_flush(removed, up_ids, up_rows)
    near = ra[rng.choice(rows_a, nq // 2)] + rng.normal(0, 0.02, (nq // 2, dim)).astype(np.float32)
    q = np.concatenate([near, rng.normal(0, 2, (nq - nq // 2, dim))]).astype(np.float32)
    out = {"queries": q, "dim": np.array(dim), "sizes": np.array(sizes), "removed_live": np.array(live),
           "deleted_rows_a": rows_a.astype(np.int64)}
    for k in (10, 64):
        ids, d = coll.search(q, k=k)
        out[f"ids_{k}"], out[f"dist_{k}"] = ids, d
    segdirs = coll.segment_dirs()
    out["segment_ids"] = np.array([int(os.path.basename(s)[4:]) for s in segdirs])
    coll.close()
    out.update(pack_dir(path))
    coll = oracle.RefCollection.open(path, threads=4)  # Collection::Stats after the reference's recovery
    out["stats"] = np.array(json.dumps(coll.stats()))
    coll.close()
    shutil.rmtree(tmp)
    np.savez_compressed(os.path.join(OUT, name + ".npz"), **out)
    print("wrote", name, os.path.getsize(os.path.join(OUT, name + ".npz")), "bytes")


def make_mutable(name="coll_mutable", dim=24, seed=15, nq=24):
    """A collection left with an unflushed write-ahead log, as after a crash or a close without
    Flush. Disk segments: A (bulk load), B (the first upserts, flushed, with A's superseded rows as
    a persisted delete set) and D (a later bulk load). The log then holds upserts of new ids, of
    A's and B's ids, of one id twice, removals of disk rows, log rows and absent ids, and an id
    upserted and removed before D's bulk load brought it back (D's row is newer than both
    records), then more upserts and removals after D. The fixture holds the directory as closed;
    searches and explains (mutable part first) come from the reference's Collection::Open of it,
    which replays the log."""
    rng = np.random.default_rng(seed)
    tmp = tempfile.mkdtemp(dir=OUT)  # scratch beside the fixtures, removed below
    path = os.path.join(tmp, "coll")
    coll = oracle.RefCollection(path, dim, metric="cosine", index={"type": "hnsw", "M": 8, "ef_construction": 64},
                                schema=SCHEMA, threads=4)
    centres = rng.standard_normal((12, dim)).astype(np.float32)
    ids_a = np.arange(1000, 2500, dtype=np.uint64) * 3
    coll.bulk_load(ids_a, rows_mixture(rng, ids_a.size, dim, centres), metadata=metadata(rng, ids_a.size))
    ids_b = np.concatenate([np.arange(5000, 5300, dtype=np.uint64) * 3, ids_a[rng.choice(1500, 50, replace=False)]])
    coll.upsert(ids_b, rows_mixture(rng, ids_b.size, dim, centres), metadata(rng, ids_b.size))
    coll.flush()
    new = np.arange(9000, 9200, dtype=np.uint64) * 3
    again = new[:5]  # upserted twice in the log
    ups = np.concatenate([new, ids_a[rng.choice(1500, 30, replace=False)], ids_b[rng.choice(350, 20, replace=False)],
                          again])
    coll.upsert(ups, rows_mixture(rng, ups.size, dim, centres), metadata(rng, ups.size))
    gone = np.concatenate([ids_a[rng.choice(1500, 40, replace=False)], ids_b[rng.choice(350, 15, replace=False)],
                           new[rng.choice(200, 25, replace=False)], np.array([1, 2], np.uint64)])
    removed = coll.remove(gone)
    x = np.array([777777], np.uint64)
    coll.upsert(x, rows_mixture(rng, 1, dim, centres), metadata(rng, 1))
    coll.remove(x)
    ids_d = np.concatenate([x, np.arange(20000, 20299, dtype=np.uint64) * 3])
    coll.bulk_load(ids_d, rows_mixture(rng, ids_d.size, dim, centres), metadata=metadata(rng, ids_d.size))
    # After D: upserts of new ids and of A's and D's ids, then removals across A, D and the log.
    more = np.concatenate([np.arange(30000, 30020, dtype=np.uint64) * 3, ids_a[rng.choice(1500, 10, replace=False)],
                           ids_d[1 + rng.choice(299, 10, replace=False)]])
    coll.upsert(more, rows_mixture(rng, more.size, dim, centres), metadata(rng, more.size))
    coll.remove(np.concatenate([ids_a[rng.choice(1500, 8, replace=False)], ids_d[1 + rng.choice(299, 6, replace=False)],
                                new[rng.choice(200, 5, replace=False)], more[:3]]))
    last = np.array([900001, 900002, 900003], np.uint64)  # new ids: the log ends with three upserts
    coll.upsert(last, rows_mixture(rng, 3, dim, centres), [None, {"year": 2024}, {"tags": []}])
    coll.close()
    files = pack_dir_with_logs(path)  # the directory as the loader sees it
    coll = oracle.RefCollection.open(path, threads=4)  # the reference's own recovery of it
    q = rows_mixture(rng, nq, dim, centres)
    filters = FILTERS[:6] + [FILTERS[11], FILTERS[13]]
    out = {"queries": q, "dim": np.array(dim), "filters": np.array([json.dumps(f) for f in filters]),
           "schema": np.array(json.dumps(SCHEMA)), "cases": np.array([json.dumps(c) for c in CASES]),
           "removed_live": np.array(removed)}
    for ci, (strategy, thr, ef, nprobe, k, alpha) in enumerate(CASES):
        for fi, f in enumerate(filters + [None]):
            ids, d = coll.search(q, k=k, ef=ef, nprobe=nprobe, strategy=strategy, filter=f,
                                 prefilter_threshold=thr, post_filter_alpha=alpha)
            out[f"ids_{ci}_{fi}"] = ids
            out[f"dist_{ci}_{fi}"] = d
            ex = coll.explain(q[0], k=k, ef=ef, nprobe=nprobe, strategy=strategy, filter=f,
                              prefilter_threshold=thr, post_filter_alpha=alpha)
            out[f"explain_{ci}_{fi}"] = np.array(json.dumps(ex))
    out["stats"] = np.array(json.dumps(coll.stats()))
    coll.close()
    out.update(files)
    shutil.rmtree(tmp)
    np.savez_compressed(os.path.join(OUT, name + ".npz"), **out)
    print("wrote", name, os.path.getsize(os.path.join(OUT, name + ".npz")), "bytes")


def pack_dir_with_logs(path):
    files = {}
    for dp, _, fns in os.walk(path):
        for fn in fns:
            full = os.path.join(dp, fn)
            with open(full, "rb") as f:
                files["file:" + os.path.relpath(full, path)] = np.frombuffer(f.read(), dtype=np.uint8)
    return files


def fuzz_parse_golden(n=3000, seed=5):
    """Mutated filter texts (characters and tokens inserted, deleted, replaced in the PARSE_CASES),
    grammar-generated filters and comparisons against doubles of every magnitude, with the
    reference parser's code and text for each (tests/golden/filter_fuzz.npz), plus two integer
    literals whose double sits half-way between two shorter decimals."""
    rng = np.random.default_rng(seed)
    tokens = list('{}[]":,0123456789.-eE ') + [
        '"field"', '"and"', '"or"', '"not"', '"eq"', '"ne"', '"in"', '"gte"', '"lt"', '"exists"', 'true',
        'false', 'null', '"year"', '"tags"', '"score"', '"lang"', '"flag"', '\\u00e9', '\\"', '1e400', '-0',
        '18446744073709551616', '9223372036854775807']
    texts = ['{"field": "year", "eq": 144744073709551615}', '{"field":"year","eq": -92337203654775808}']
    codes, outs = [], []
    for t in texts:
        rc, o = oracle.ref_filter_parse(SCHEMA, t)
        codes.append(rc)
        outs.append(o)
    nvalid = n // 3  # a third of the cases parse, the rest exercise the error paths
    while len(texts) < n:
        b = list(PARSE_CASES[int(rng.integers(0, len(PARSE_CASES)))])
        for _ in range(int(rng.integers(1, 5))):
            i, op = int(rng.integers(0, len(b) + 1)), int(rng.integers(0, 3))
            if op == 0 and b:
                del b[min(i, len(b) - 1)]
            elif op == 1:
                b.insert(i, tokens[int(rng.integers(0, len(tokens)))])
            elif b:
                b[min(i, len(b) - 1)] = tokens[int(rng.integers(0, len(tokens)))]
        t = "".join(b)
        rc, o = oracle.ref_filter_parse(SCHEMA, t)
        if (rc == 0 and codes.count(0) >= nvalid) or (rc != 0 and len(codes) - codes.count(0) >= n - nvalid):
            continue
        texts.append(t)
        codes.append(rc)
        outs.append(o)
    # Filters generated from the grammar (nested and / or / not over every operator and type),
    # and single comparisons against doubles of every magnitude, random bit patterns included.
    types = {f["name"]: f["type"] for f in SCHEMA}

    def number():
        k = int(rng.integers(0, 4))
        if k == 0:
            return float(np.frombuffer(np.array([int(rng.integers(0, 2**63 - 2**52, dtype=np.uint64))], "<u8").tobytes(), "<f8")[0])
        if k == 1:
            return float(rng.normal() * 10.0 ** int(rng.integers(-30, 30)))
        if k == 2:
            return int(rng.integers(-2**62, 2**62))
        return float(np.float32(rng.normal() * 10.0 ** int(rng.integers(-10, 10))))

    def leaf():
        f = str(rng.choice(list(types)))
        t = types[f]
        ops = ["eq", "ne", "in", "exists"] + (["lt", "lte", "gt", "gte"] if t in ("int64", "float64") else [])
        op = str(rng.choice(ops))
        one = (number if t in ("int64", "float64") else
               (lambda: str(rng.choice(["en", "t0", "", "\u00e9", "a\"b"]))) if t != "bool" else (lambda: bool(rng.random() < .5)))
        v = bool(rng.random() < 0.5) if op == "exists" else ([one() for _ in range(int(rng.integers(1, 5)))] if op == "in" else one())
        return {"field": f, op: v}

    def node(d):
        r = rng.random()
        if d > 3 or r < 0.45:
            return leaf()
        if r < 0.85:
            return {"and" if r < 0.65 else "or": [node(d + 1) for _ in range(int(rng.integers(1, 4)))]}
        return {"not": node(d + 1)}

    extra = [json.dumps(node(0)) for _ in range(1500)]
    extra += ['{"field": "score", "eq": %s}' % repr(v) for v in (number() for _ in range(1500))
              if isinstance(v, int) or np.isfinite(v)]
    for t in extra:
        rc, o = oracle.ref_filter_parse(SCHEMA, t)
        texts.append(t)
        codes.append(rc)
        outs.append(o)
    # Schemas: the field list with names and types changed (type aliases included), fields
    # dropped, repeated or given extra keys, and the JSON text mutated; parsed with one filter.
    schemas, scodes, souts = [], [], []
    names = ["", "year", "a.b", "x" * 70, "\u00e9", "1abc", "a-b", "_x", "A"]
    stypes = ["int", "string", "double", "float", "tags", "keyword", "bool", "", "INT64", "int32"]
    while len(schemas) < 2000:
        if rng.random() < 0.6:
            sch = [dict(f) for f in SCHEMA if rng.random() < 0.8]
            for f in sch:
                if rng.random() < 0.15:
                    f["type"] = str(rng.choice(stypes))
                if rng.random() < 0.1:
                    f["name"] = str(rng.choice(names))
                if rng.random() < 0.05:
                    f["extra"] = 1
                if rng.random() < 0.05:
                    del f["type"]
            if rng.random() < 0.1:
                sch = sch + sch[:1]
            t = json.dumps(sch if rng.random() > 0.1 else {f.get("name", "?"): f.get("type", 0) for f in sch})
        else:
            b = list(json.dumps(SCHEMA))
            for _ in range(int(rng.integers(1, 4))):
                i, op = int(rng.integers(0, len(b) + 1)), int(rng.integers(0, 3))
                if op == 0 and b:
                    del b[min(i, len(b) - 1)]
                elif op == 1:
                    b.insert(i, tokens[int(rng.integers(0, len(tokens)))])
                elif b:
                    b[min(i, len(b) - 1)] = tokens[int(rng.integers(0, len(tokens)))]
            t = "".join(b)
        l = oracle._engine_lib()
        rc = l.ref_filter_parse(t.encode(), b'{"field": "year", "gte": 1}')
        schemas.append(t)
        scodes.append(rc)
        souts.append(l.ref_coll_last_error().decode())
    np.savez_compressed(os.path.join(OUT, "filter_fuzz.npz"), cases=np.array(texts), codes=np.array(codes),
                        texts=np.array(outs), schema=np.array(json.dumps(SCHEMA)), schemas=np.array(schemas),
                        schema_codes=np.array(scodes), schema_texts=np.array(souts))
    print("wrote filter_fuzz", len(texts), "cases,", sum(c == 0 for c in codes), "valid")


def main():
    oracle.build(ref=True)
    fuzz_parse_golden()
    make_mutable()
    make_deletes()
    parse_golden()
    make("coll_hnsw", 48, "cosine", {"type": "hnsw", "M": 8, "ef_construction": 64}, [900, 1300, 700], seed=11)
    make("coll_ivfpq", 32, "l2", {"type": "ivf_pq", "nlist": 16, "pq_m": 8}, [1000, 800], seed=12,
         filters=FILTERS[:6] + [FILTERS[13]], cases=CASES_IVF)
    make("coll_flat", 20, "ip", {"type": "flat"}, [600, 500, 400], seed=13,
         filters=FILTERS[:4] + [FILTERS[8], FILTERS[15]])


if __name__ == "__main__":
    main()
