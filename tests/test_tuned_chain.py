"""The committed B200 tuned table (paia-project_b200/tuned/b200.json) and bench.py's decode-chain rule: every GEMV of
an INT4 decode chain (qkv, o, gate_up, down, lm_head) of a model resolves to one kernel instance, each chained entry
keeps its isolated per-shape pick, other shapes and formats keep theirs, and applying the rule again changes
nothing."""
import copy
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "paia-project_b200"))

import bench                                              # noqa: E402
from paia_gemv import synthetic                           # noqa: E402

KEYS = {"bf16": "shapes", "fp8": "fp8_shapes", "int4": "int4_shapes", "int4_asym": "int4_asym_shapes"}
CHAIN = synthetic.LAYER_SEQUENCE + ("lm_head",)


def table():
    return json.loads((ROOT / "paia-project_b200" / "tuned" / "b200.json").read_text())


def test_int4_chains_use_one_instance():
    t = table()
    for kind in bench.CHAIN_KINDS:
        for model, shapes in synthetic.SHAPES.items():
            vs = {json.dumps(t[KEYS[kind]]["{}x{}".format(*shapes[n])]["variant"], sort_keys=True) for n in CHAIN}
            assert len(vs) == 1, (kind, model, vs)
            for n in CHAIN:
                e = t[KEYS[kind]]["{}x{}".format(*shapes[n])]
                assert "isolated_best" in e and e["variant"]["R"] == 0, (kind, model, n)


def test_chain_rule_is_idempotent():
    t = table()
    again = copy.deepcopy(t)
    bench.chain_rule(again, KEYS, synthetic.SHAPES)
    assert again == t


def test_chain_rule_leaves_other_shapes_and_formats():
    t = table()
    chained = {"{}x{}".format(*s[n]) for s in synthetic.SHAPES.values() for n in CHAIN}
    for kind, key in KEYS.items():
        for shape, e in t[key].items():
            if kind not in bench.CHAIN_KINDS or shape not in chained:
                assert "chain" not in e, (kind, shape)


def test_chain_rule_prefers_the_lowest_summed_time():
    """A synthetic table: variant A is best on every shape but one, where it is missing from the top 5; B is in every
    top 5 but slower overall. The rule takes A (summed estimate) and keeps each isolated pick."""
    a = {"R": 0, "U": 4, "W": 8, "S": 0, "H": 1}
    b = {"R": 0, "U": 2, "W": 8, "S": 0, "H": 1}
    c = {"R": 0, "U": 2, "W": 16, "S": 0, "H": 1}
    shapes = {"m": {n: (100 + i, 128) for i, n in enumerate(CHAIN)}}
    t = {"int4_shapes": {}, "int4_asym_shapes": {}}
    for i, n in enumerate(CHAIN):
        top = [{"variant": a, "pct_of_best": 100.0}, {"variant": b, "pct_of_best": 90.0}]
        if i == 3:
            top = [{"variant": c, "pct_of_best": 100.0}, {"variant": b, "pct_of_best": 97.0}]
        t["int4_shapes"][f"{100 + i}x128"] = {"variant": top[0]["variant"], "us": 10.0, "top5": top}
    chosen = bench.chain_rule(t, KEYS, shapes)
    assert chosen[("int4", "m")] == a
    assert t["int4_shapes"]["103x128"]["isolated_best"]["variant"] == c


def test_every_tuned_variant_exists_in_the_library():
    """Every (R, U, W, S, H) the table names is in its format's variant table (the adapters and bench.py look tuples
    up by value and raise on a missing one); the library loads and answers variant_info without a GPU."""
    from paia_gemv import load_lib
    lib = load_lib()
    tables = {"bf16": lib.variants, "fp8": lib.variants_fp8, "int4": lib.variants_int4,
              "int4_asym": lib.variants_int4_asym}
    t = table()
    for kind, key in KEYS.items():
        have = {tuple(v[k] for k in "RUWSH") for v in tables[kind]}
        for shape, e in t[key].items():
            assert tuple(e["variant"][k] for k in "RUWSH") in have, (kind, shape, e["variant"])
