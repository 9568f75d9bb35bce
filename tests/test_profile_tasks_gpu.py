"""Kernel-group cost table (fluidgpu_b200.profile_tasks): the CSV the
reference's planners read (profile_llm_tasks.py format: name, prefill_us,
decode_us), one row per kernel group, measured on the B200 kernels."""
import csv

import pytest

pytestmark = pytest.mark.gpu


def test_cost_table_rows(tmp_path):
    from fluidgpu_b200 import build, kernels
    from fluidgpu_b200.model import TINY_LLAMA
    from fluidgpu_b200.profile_tasks import measure, write_csv

    build.build()
    rows = measure(TINY_LLAMA.name, batch=4, context=64, decode_steps=3, warmup=1, prefill_len=8)
    names = [r["name"] for r in rows]
    L = TINY_LLAMA.num_layers
    assert names == ["embed"] + [f"layer_{i}_{s}" for i in range(L) for s in ("attn", "mlp")] + ["norm_lm_head"]
    assert all(float(r["decode_us"]) > 0 and float(r["prefill_us"]) > 0 for r in rows)
    out = tmp_path / "costs.csv"
    write_csv(rows, out)
    with out.open() as f:
        back = list(csv.DictReader(f))
    assert list(back[0].keys()) == ["name", "prefill_us", "decode_us"] and len(back) == len(rows)
    kernels.check_device("cost table")
