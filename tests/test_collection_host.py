"""Host side of the collection read path, without a GPU: the filter parser against the
reference's FilterExpr::Parse (golden texts, and the live reference engine when it is built),
the collection fixtures' integrity, and the shard assignment of segments to ranks."""
import json
import os

import numpy as np
import pytest

from helpers import golden


def test_filter_parser_matches_reference_golden():
    import vdb_b200
    g = golden("filter_parse")
    schema = str(g["schema"])
    for case, code, text in zip(g["cases"], g["codes"], g["texts"]):
        assert vdb_b200.filter_describe(schema, str(case)) == (int(code), str(text)), str(case)[:80]


def test_filter_parser_matches_reference_on_fuzzed_texts():
    """6,000 texts with the reference parser's code and text: mutations of the golden texts (a
    third of them valid), grammar-generated filters, and comparisons against doubles of every
    magnitude. Covers error paths and messages, and numbers printed as the reference prints them
    (Grisu2's digits, which can differ from the correctly rounded shortest form)."""
    import vdb_b200
    g = golden("filter_fuzz")
    schema = str(g["schema"])
    bad = [str(c) for c, code, text in zip(g["cases"], g["codes"], g["texts"])
           if vdb_b200.filter_describe(schema, str(c)) != (int(code), str(text))]
    assert not bad, (len(bad), bad[:5])


def test_schema_parser_matches_reference_on_fuzzed_texts():
    """2,000 schemas (names and types changed, type aliases, dropped, repeated and extended
    fields, mutated JSON) parsed with one filter, against the reference's SchemaFromJson and
    FilterExpr::Parse (its schema messages carry the status name as a prefix)."""
    import vdb_b200
    g = golden("filter_fuzz")
    bad = []
    for sch, code, text in zip(g["schemas"], g["schema_codes"], g["schema_texts"]):
        want = str(text)
        for prefix in ("invalid_argument: ", "not_found: ", "corruption: "):
            if int(code) != 0 and want.startswith(prefix):
                want = want[len(prefix):]
        if vdb_b200.filter_describe(str(sch), '{"field": "year", "gte": 1}') != (int(code), want):
            bad.append(str(sch)[:120])
    assert not bad, (len(bad), bad[:4])


def test_filter_parser_matches_live_reference():
    import oracle
    import vdb_b200
    if not os.path.exists(oracle.REF_ENGINE_LIB):
        pytest.skip("the reference engine is not built here")
    schema = [{"name": "a", "type": "int64"}, {"name": "b", "type": "keyword_list"},
              {"name": "c", "type": "float64"}, {"name": "d", "type": "bool"}, {"name": "e", "type": "keyword"}]
    rng = np.random.default_rng(5)
    ops = ["eq", "ne", "in", "lt", "lte", "gt", "gte", "exists", "nope"]
    fields = ["a", "b", "c", "d", "e", "zz"]
    vals = [1, -2.5, "x", True, [1, 2], ["x", "y"], [], None, 1e300, "é"]

    def leaf():
        return {"field": fields[rng.integers(len(fields))], ops[rng.integers(len(ops))]: vals[rng.integers(len(vals))]}

    def node(d):
        r = rng.random()
        if d > 3 or r < 0.4:
            return leaf()
        if r < 0.6:
            return {"not": node(d + 1)}
        return {["and", "or"][rng.integers(2)]: [node(d + 1) for _ in range(rng.integers(1, 4))]}

    for _ in range(400):
        text = json.dumps(node(0))
        assert vdb_b200.filter_describe(schema, text) == oracle.ref_filter_parse(schema, text), text


@pytest.mark.parametrize("name", ["coll_hnsw", "coll_ivfpq", "coll_flat"])
def test_collection_fixture_is_the_reference_layout(name, tmp_path):
    """The stored directory is what Collection::Open reads: CURRENT names the manifest, every
    manifest segment has its four files."""
    from helpers import extract_collection
    g = golden(name)
    path = extract_collection(g, tmp_path)
    cur = open(os.path.join(path, "CURRENT")).read().strip()
    assert cur.startswith("MANIFEST-") and os.path.exists(os.path.join(path, cur))
    for sid in g["segment_ids"]:
        d = os.path.join(path, "segments", "seg-%06d" % int(sid))
        names = set(os.listdir(d))
        assert {"vectors.f32", "ids.u64", "meta.bin"} <= names
        assert any(n.startswith("index.") for n in names)


def test_shard_assignment_round_robin():
    """Segment ordinal i goes to rank i % world (the sharding of the collection read path)."""
    from vdb_b200 import sharded
    for world in (1, 2, 3, 8):
        owners = [sharded.owner(i, world) for i in range(64)]
        for r in range(world):
            mine = [i for i, o in enumerate(owners) if o == r]
            assert mine == list(range(r, 64, world))
