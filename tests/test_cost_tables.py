"""The committed planner cost tables (profiles/task_costs_*.csv, written by
`python -m fluidgpu_b200.profile_tasks` on a B200) in the format the
reference's planners read (planner.py:93-103 read_csv: name, prefill_us,
decode_us per kernel group). Its schedule_llm_layers.py plans every layer_*
row of a table, so a table holds one form of each layer: the reference's
attn / mlp task set (profile_llm_tasks.py:94-95), or for gpt-oss the MoE
groups (router / experts / combine) in place of mlp.

Plans the reference's planner made from these tables (tests/golden/plans,
written by tests/golden/make_plans.py) load with this package's plan loader."""
import csv
import json
from pathlib import Path

import pytest

from fluidgpu_b200.profile import load_profile, owned_layer_ids
from fluidgpu_b200.profile_tasks import coarse_rows

ROOT = Path(__file__).resolve().parent.parent
PLANS = ROOT / "tests" / "golden" / "plans"


def _read(name):
    with (ROOT / "profiles" / name).open(newline="") as f:
        rows = list(csv.DictReader(f))
    assert rows and list(rows[0].keys()) == ["name", "prefill_us", "decode_us"]
    return {r["name"]: (float(r["prefill_us"]), float(r["decode_us"])) for r in rows}, [r["name"] for r in rows]


@pytest.mark.parametrize("name,layers,groups", [
    ("task_costs_llama3_8b_b64_ctx4096.csv", 32, ("attn", "mlp")),
    ("task_costs_gptoss20b_b128_ctx4096.csv", 24, ("attn", "mlp")),
    ("task_costs_gptoss20b_b128_ctx4096_moe_groups.csv", 24, ("attn", "moe_router", "moe_experts", "moe_combine")),
])
def test_cost_table(name, layers, groups):
    table, order = _read(name)
    want = ["embed"] + [f"layer_{i}_{g}" for i in range(layers) for g in groups] + ["norm_lm_head"]
    assert order == want
    assert all(p > 0 and d > 0 for p, d in table.values())


def test_gptoss_tables_agree():
    """One measurement, two forms: each coarse mlp row is its layer's router +
    experts + combine, and every other row is shared."""
    coarse, _ = _read("task_costs_gptoss20b_b128_ctx4096.csv")
    fine, _ = _read("task_costs_gptoss20b_b128_ctx4096_moe_groups.csv")
    for i in range(24):
        for k in (0, 1):
            parts = sum(fine[f"layer_{i}_{g}"][k] for g in ("moe_router", "moe_experts", "moe_combine"))
            assert abs(coarse[f"layer_{i}_mlp"][k] - parts) <= 0.01
        assert coarse[f"layer_{i}_attn"] == fine[f"layer_{i}_attn"]
    for n in ("embed", "norm_lm_head"):
        assert coarse[n] == fine[n]


def test_coarse_rows():
    rows = [{"name": "embed", "prefill_us": "1.000", "decode_us": "2.000"},
            {"name": "layer_0_attn", "prefill_us": "3.000", "decode_us": "4.000"},
            {"name": "layer_0_moe_router", "prefill_us": "0.500", "decode_us": "0.250"},
            {"name": "layer_0_moe_experts", "prefill_us": "5.000", "decode_us": "6.000"},
            {"name": "layer_0_moe_combine", "prefill_us": "0.125", "decode_us": "1.000"},
            {"name": "norm_lm_head", "prefill_us": "7.000", "decode_us": "8.000"}]
    out = coarse_rows(rows)
    assert [r["name"] for r in out] == ["embed", "layer_0_attn", "layer_0_mlp", "norm_lm_head"]
    assert out[2] == {"name": "layer_0_mlp", "prefill_us": "5.625", "decode_us": "7.250"}
    dense = rows[:2] + [{"name": "layer_0_mlp", "prefill_us": "1.0", "decode_us": "1.0"}] + rows[-1:]
    assert coarse_rows(dense) == dense


def _plans():
    return sorted(PLANS.glob("plan_*.json"))


def test_reference_planner_fixtures_present():
    assert len(_plans()) >= 4, "run tests/golden/make_plans.py"


@pytest.mark.parametrize("path", _plans(), ids=lambda p: p.stem)
def test_reference_planner_output_loads(path):
    """A plan the reference's DP planner chose from a B200 cost table loads,
    validates, and places every kernel group of the table it came from."""
    raw = json.loads(path.read_text())
    prof = load_profile(path)
    meta = raw["fixture"]
    table, order = _read(meta["rank0_csv"])
    layer_tasks = [n for n in order if n.startswith("layer_")]
    assert [t.name for t in prof.tasks] == ["embed"] + layer_tasks + ["norm_lm_head"]
    ranks = [t.rank for t in prof.tasks]
    switches = sum(1 for a, b in zip([0, *ranks[1:-1]], [*ranks[1:-1], 0]) if a != b)
    assert switches == raw["predicted_cost_us"]["rank_switches"]
    if meta["expect_split"]:
        assert switches > 0 and owned_layer_ids(prof, 1)
    else:
        assert set(ranks) == {0}
