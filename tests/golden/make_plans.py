"""Generate placement plans with the reference's own planner from this
package's B200 cost tables, as fixtures for tests/test_cost_tables.py.

Run in a container that has the FluidGPU reference checkout (read-only is
fine); the plans it writes are committed, so the tests never need the
reference at run time:

  python tests/golden/make_plans.py <reference>

It runs the reference's examples/fluidgpu_torch/schedule_llm_layers.py (DP
solver, reading its two cost tables with planner.py:93-103) on:
  * the same B200 table for both ranks (two identical GPUs): every group on
    rank 0, since any hand-off only adds cost;
  * rank 1 given the same table with its feed-forward rows (mlp, or the MoE
    experts group) at half the cost, a stand-in for a second GPU that is
    faster at the FFN (this input is synthetic, the tables are measured):
    the planner moves feed-forward groups to rank 1.
Each plan carries a "fixture" entry naming its inputs and what it expects.

It also records what the reference's plan writer (profile.py:275-326
make_ranked_task_profile) emits for a few task assignments (attention /
FFN split, fine attention split, MoE groups, three ranks), in
reference_writer.json, and what the reference's loader (profile.py:97-167
profile_from_dict) decides on a set of valid and invalid plans, in
reference_validation.json, so the tests can compare this package's writer and
loader with them; and whether every plan the reference ships loads the same
way with both loaders (reference_shipped_plans.json, outcomes only).
"""
from __future__ import annotations

import csv
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
OUT = HERE / "plans"

MODELS = {
    "llama3_8b": dict(model="llama-3-8b", hidden=4096, kv=8, hd=128),
    "gptoss20b": dict(model="gpt-oss-20b", hidden=2880, kv=8, hd=64),
}
CASES = [
    ("llama3_8b", "task_costs_llama3_8b_b64_ctx4096.csv", None),
    ("llama3_8b", "task_costs_llama3_8b_b64_ctx4096.csv", "_mlp"),
    ("gptoss20b", "task_costs_gptoss20b_b128_ctx4096.csv", None),
    ("gptoss20b", "task_costs_gptoss20b_b128_ctx4096_moe_groups.csv", "_moe_experts"),
]


def _scaled_table(src: Path, suffix: str, dst: Path) -> None:
    with src.open(newline="") as f:
        rows = list(csv.DictReader(f))
    for r in rows:
        if r["name"].endswith(suffix):
            r["prefill_us"] = f"{float(r['prefill_us']) * 0.5:.3f}"
            r["decode_us"] = f"{float(r['decode_us']) * 0.5:.3f}"
    with dst.open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=["name", "prefill_us", "decode_us"])
        w.writeheader()
        w.writerows(rows)


def main(reference: Path) -> None:
    runtime = reference / "fluidgpu_runtime"
    script = runtime / "examples" / "fluidgpu_torch" / "schedule_llm_layers.py"
    assert script.exists(), f"no planner script at {script}"
    OUT.mkdir(exist_ok=True)
    env = {**os.environ, "PYTHONPATH": str(runtime)}
    with tempfile.TemporaryDirectory() as tmp:
        for key, table, faster in CASES:
            m = MODELS[key]
            rank0 = ROOT / "profiles" / table
            rank1 = rank0
            if faster:
                rank1 = Path(tmp) / f"rank1_{key}{faster}.csv"
                _scaled_table(rank0, faster, rank1)
            stem = table.replace("task_costs_", "plan_").replace(".csv", "") + (
                "_ffn_rank_faster" if faster else "_two_b200")
            out = OUT / f"{stem}.json"
            cmd = [sys.executable, str(script), "--rank0-csv", str(rank0), "--rank1-csv", str(rank1),
                   "--output", str(out), "--model", m["model"], "--hidden-size", str(m["hidden"]),
                   "--num-kv-heads", str(m["kv"]), "--head-dim", str(m["hd"]), "--max-seq-len", "5120",
                   "--comm-bw-gbps", "770", "--decode-weight", "32"]
            r = subprocess.run(cmd, env=env, capture_output=True, text=True, cwd=tmp)
            assert r.returncode == 0, r.stderr
            plan = json.loads(out.read_text())
            plan["fixture"] = {"rank0_csv": table, "rank1": f"same table, {faster} rows x 0.5" if faster
                               else "same table", "expect_split": bool(faster),
                               "planner": r.stdout.strip().splitlines()[-1]}
            out.write_text(json.dumps(plan, indent=1) + "\n")
            print(out.name, plan["fixture"]["planner"])


WRITER_CASES = [
    dict(model="m", hidden_size=64, num_kv_heads=2, head_dim=16, max_seq_len=128,
         task_assignments=[("layer_0_attn", 0), ("layer_0_mlp", 1), ("layer_1_attn", 0), ("layer_1_mlp", 1)]),
    dict(model="m", hidden_size=64, num_kv_heads=2, head_dim=16, max_seq_len=256,
         task_assignments=[("layer_0_qkv", 0), ("layer_0_sdpa", 1), ("layer_0_o_proj", 0),
                           ("layer_0_mlp_gate_up", 1), ("layer_0_mlp_down_proj", 1)]),
    dict(model="gpt-oss-20b", hidden_size=2880, num_kv_heads=8, head_dim=64, max_seq_len=5120,
         task_assignments=[("layer_0_attn", 0), ("layer_0_moe_router", 0), ("layer_0_moe_experts", 1),
                           ("layer_0_moe_combine", 0)]),
    dict(model="m", hidden_size=64, num_kv_heads=2, head_dim=16, max_seq_len=128, rank_count=3,
         task_assignments=[("layer_0_attn", 0), ("layer_0_mlp", 2)]),
]


def write_reference_writer_cases(runtime: Path) -> None:
    sys.path.insert(0, str(runtime))
    from fluidgpu_torch.profile import make_ranked_task_profile  # the reference's writer

    cases = [{"args": {k: (list(map(list, v)) if k == "task_assignments" else v) for k, v in c.items()},
              "profile": make_ranked_task_profile(**c)} for c in WRITER_CASES]
    (OUT / "reference_writer.json").write_text(json.dumps(cases, indent=1) + "\n")
    print("reference_writer.json", len(cases), "cases")


def _validation_cases(make) -> dict[str, dict]:
    """Plans, valid and invalid, for the loader's rules: fixed tasks on rank 0,
    dtype, per-layer task sequences (coarse, attn / mlp, fine attention,
    MoE groups), decode_rank placement, rank range, unique names, contiguous
    layers, suffixes."""
    def af():
        return make(model="m", task_assignments=[("layer_0_attn", 0), ("layer_0_mlp", 1), ("layer_1_attn", 0),
                                                 ("layer_1_mlp", 1)],
                    hidden_size=64, num_kv_heads=2, head_dim=16, max_seq_len=128)

    def fine():
        return make(model="m", task_assignments=[("layer_0_qkv", 0), ("layer_0_sdpa", 1), ("layer_0_o_proj", 0),
                                                 ("layer_0_mlp", 1)],
                    hidden_size=64, num_kv_heads=2, head_dim=16, max_seq_len=128)

    def moe():
        return make(model="m", task_assignments=[("layer_0_attn", 0), ("layer_0_moe_router", 0),
                                                 ("layer_0_moe_experts", 1), ("layer_0_moe_combine", 0)],
                    hidden_size=64, num_kv_heads=2, head_dim=16, max_seq_len=128)

    def renamed(r, i, name):
        r["tasks"][i] = {**r["tasks"][i], "name": name}

    def drop(r, i):
        r["tasks"].pop(i)
        r["task_count"] = len(r["tasks"])

    edits = {
        "valid_af": (af, lambda r: None),
        "valid_fine": (fine, lambda r: None),
        "valid_moe_groups": (moe, lambda r: None),
        "embed_on_rank1": (af, lambda r: r["tasks"][0].__setitem__("rank", 1)),
        "head_on_rank1": (af, lambda r: r["tasks"][-1].__setitem__("rank", 1)),
        "dtype_fp32": (af, lambda r: r.__setitem__("dtype", "float32")),
        "missing_mlp": (af, lambda r: drop(r, 2)),
        "decode_rank_on_attn": (af, lambda r: r["tasks"][1].__setitem__("decode_rank", 1)),
        "decode_rank_on_mlp": (af, lambda r: r["tasks"][2].__setitem__("decode_rank", 0)),
        "decode_rank_on_moe_experts": (moe, lambda r: r["tasks"][3].__setitem__("decode_rank", 0)),
        "mlp_before_attn": (af, lambda r: (renamed(r, 1, "layer_0_mlp"), renamed(r, 2, "layer_0_attn"))),
        "task_count_ignored": (af, lambda r: r.__setitem__("task_count", 99)),
        "rank_out_of_range": (af, lambda r: r["tasks"][2].__setitem__("rank", 2)),
        "duplicate_name": (af, lambda r: renamed(r, 3, "layer_0_attn")),
        "coarse_layer_tasks": (af, lambda r: (r.__setitem__("tasks", [
            r["tasks"][0], {"task_id": 1, "kernel_group_id": 1, "name": "layer_0", "rank": 0},
            {"task_id": 2, "kernel_group_id": 2, "name": "layer_1", "rank": 1},
            {**r["tasks"][-1], "task_id": 3, "kernel_group_id": 3}]), r.__setitem__("task_count", 4))),
        "fine_missing_sdpa": (fine, lambda r: drop(r, 2)),
        "task_id_gap": (af, lambda r: r["tasks"][2].__setitem__("task_id", 7)),
        "layer_gap": (af, lambda r: (renamed(r, 3, "layer_2_attn"), renamed(r, 4, "layer_2_mlp"))),
        "unknown_suffix": (af, lambda r: renamed(r, 2, "layer_0_ffn")),
        "mlp_and_moe_in_one_layer": (af, lambda r: r["tasks"].insert(
            3, {"task_id": 3, "kernel_group_id": 3, "name": "layer_0_moe_router", "rank": 1})),
    }
    out = {}
    for name, (base, edit) in edits.items():
        r = base()
        edit(r)
        out[name] = r
    return out


def write_reference_validation_cases(runtime: Path) -> None:
    sys.path.insert(0, str(runtime))
    from fluidgpu_torch.profile import make_ranked_task_profile, profile_from_dict  # the reference's

    cases = []
    for name, raw in _validation_cases(make_ranked_task_profile).items():
        try:
            profile_from_dict(json.loads(json.dumps(raw)))
            result = {"ok": True}
        except AssertionError as exc:
            result = {"ok": False, "error": "AssertionError", "message": str(exc)}
        cases.append({"name": name, "plan": raw, "reference": result})
    (OUT / "reference_validation.json").write_text(json.dumps(cases, indent=1) + "\n")
    print("reference_validation.json", len(cases), "cases")


def write_shipped_plan_check(reference: Path) -> None:
    """Load every plan the reference ships (its profiles/*.json and the
    validation artifact's profile.json) with its loader and with this
    package's, and record per file whether both accept it and expand it to
    the same (name, rank, decode_rank) tasks. Only the outcome is recorded;
    the plans stay in the reference checkout."""
    runtime = reference / "fluidgpu_runtime"
    sys.path.insert(0, str(runtime))
    sys.path.insert(0, str(ROOT))
    from fluidgpu_torch.profile import load_profile as reference_load

    from fluidgpu_b200.profile import load_profile as our_load

    def tasks(load, f):
        try:
            return [[t.name, t.rank, getattr(t, "decode_rank", None)] for t in load(f).tasks]
        except AssertionError as exc:
            return f"AssertionError: {exc}"

    files = sorted((runtime / "profiles").glob("*.json")) + sorted(
        (reference / "artifacts").rglob("profile.json"))
    rows = []
    for f in files:
        ref, ours = tasks(reference_load, f), tasks(our_load, f)
        rows.append({"file": str(f.relative_to(reference)), "reference_accepts": isinstance(ref, list),
                     "tasks": len(ref) if isinstance(ref, list) else 0, "identical": ref == ours})
    (OUT / "reference_shipped_plans.json").write_text(json.dumps(rows, indent=1) + "\n")
    print("reference_shipped_plans.json", sum(r["identical"] for r in rows), "of", len(rows), "identical")


if __name__ == "__main__":
    assert len(sys.argv) == 2, "usage: make_plans.py <reference checkout>"
    main(Path(sys.argv[1]))
    write_reference_writer_cases(Path(sys.argv[1]) / "fluidgpu_runtime")
    write_reference_validation_cases(Path(sys.argv[1]) / "fluidgpu_runtime")
    write_shipped_plan_check(Path(sys.argv[1]))
