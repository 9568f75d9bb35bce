"""Kernel-group cost table for the placement planner, measured on the B200
kernels: the counterpart of the reference's kernel analyzer
(examples/fluidgpu_torch/profile_llm_tasks.py), writing the same CSV the
planners read (schedule_llm_layers.py): `name,prefill_us,decode_us`, one row
per kernel group of an all-on-one-GPU plan (embed, layer_i_*, norm_lm_head).

    python -m fluidgpu_b200.profile_tasks --model llama-3-8b --batch 64 \\
        --context 4096 --output llama3_8b_b200.csv

Differences from the reference's table, each forced by what is measured:
  * batch > 1 decodes together (the reference's runner is batch 1), and the
    KV pages hold `--context` tokens of synthetic values, so decode_us is the
    cost at that batch and context;
  * prefill_us is one batched prefill pass of a batch-1 prompt of
    `--prefill-len` positions (token-wise RoPE/KV append, causal prefill
    attention over the pages, GEMMs over every position), as the
    reference's whole-prompt HF forward;
  * for MoE models the measured groups are layer_i_moe_router /
    _moe_experts / _moe_combine. The table written by default has the
    reference's task set (attn and mlp rows, profile_llm_tasks.py:94-95),
    the mlp row being the sum of the three; `--groups moe` writes the three
    instead. The reference's schedule_llm_layers.py plans every layer_* row
    it reads, so a table never holds both forms of a layer.
Weights are random (no checkpoints here); decode cost does not depend on
their values.
"""
from __future__ import annotations

import argparse
import csv
import statistics
from pathlib import Path

import torch

from . import build
from .config import EngineConfig
from .engine import DecodeEngine
from .model import SPECS, ModelWeights
from .trace import TraceRecorder, install_trace_recorder


def _collect(rec: TraceRecorder) -> dict[str, list[float]]:
    out: dict[str, list[float]] = {}
    for r in rec.flush():
        if r.get("kind") == "compute":
            out.setdefault(str(r["name"]), []).append(float(r["elapsed_us"]))
    return out


def measure(model: str, batch: int, context: int, decode_steps: int = 8, warmup: int = 2,
            prefill_len: int = 64, device: str = "cuda:0", seed: int = 0) -> list[dict[str, str]]:
    spec = SPECS[model]
    dev = torch.device(device)
    weights = ModelWeights.random(spec, seed=seed, device=dev)
    rows: dict[str, dict[str, float]] = {}

    # decode: B sequences holding `context` tokens of synthetic KV
    total = context + warmup + decode_steps + 8
    eng = DecodeEngine(weights, EngineConfig(model_name=spec.name, max_seq_len=total, world_size=1,
                                             device=device, max_batch=batch))
    eng.start(batch, prompt_lens=[context] * batch, reserve_tokens=total)
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    if eng.kv_cache.pool is not None:
        eng.kv_cache.pool.normal_(0.0, 1.0, generator=g)
    tok = torch.randint(0, spec.vocab, (batch,), generator=g, device=dev)
    for _ in range(warmup):
        tok = eng.step_device(tok)
    torch.cuda.synchronize(dev)
    rec = TraceRecorder()
    install_trace_recorder(rec)
    try:
        for _ in range(decode_steps):
            tok = eng.step_device(tok)
        dec = _collect(rec)
        # prefill: a batch-1 prompt fed position by position
        eng1 = DecodeEngine(weights, EngineConfig(model_name=spec.name, max_seq_len=prefill_len + 8,
                                                  world_size=1, device=device, max_batch=1))
        prompt = torch.randint(0, spec.vocab, (1, prefill_len), generator=g, device=dev)
        eng1.start(1, reserve_tokens=prefill_len + 2)
        rec.flush()
        eng1.runner.prefill(prompt)
        pre = _collect(rec)
    finally:
        install_trace_recorder(None)
    names = ["embed"] + [n for n in eng.executor.task_index_by_name if n.startswith("layer_")] + ["norm_lm_head"]
    for n in names:
        d, p = dec.get(n, []), pre.get(n, [])
        assert len(d) == decode_steps, f"{n}: {len(d)} decode samples, expected {decode_steps}"
        rows[n] = {"decode_us": statistics.median(d), "prefill_us": sum(p)}
    return [{"name": n, "prefill_us": f"{rows[n]['prefill_us']:.3f}", "decode_us": f"{rows[n]['decode_us']:.3f}"}
            for n in names]


MOE_GROUPS = ("moe_router", "moe_experts", "moe_combine")


def coarse_rows(rows: list[dict[str, str]]) -> list[dict[str, str]]:
    """The reference's task set (embed, layer_i_attn, layer_i_mlp,
    norm_lm_head): each MoE layer's router / experts / combine rows become one
    layer_i_mlp row holding their sum. Dense tables pass through unchanged."""
    out: list[dict[str, str]] = []
    acc: dict[str, list[float]] = {}
    for r in rows:
        name = r["name"]
        parts = name.split("_", 2)
        if len(parts) == 3 and parts[0] == "layer" and parts[2] in MOE_GROUPS:
            a = acc.setdefault(parts[1], [0.0, 0.0])
            a[0] += float(r["prefill_us"])
            a[1] += float(r["decode_us"])
            if parts[2] == "moe_combine":
                out.append({"name": f"layer_{parts[1]}_mlp", "prefill_us": f"{a[0]:.3f}",
                            "decode_us": f"{a[1]:.3f}"})
        else:
            out.append(r)
    return out


def write_csv(rows: list[dict[str, str]], path: Path) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=["name", "prefill_us", "decode_us"])
        w.writeheader()
        w.writerows(rows)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", default="llama-3-8b", choices=sorted(SPECS))
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--decode-steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--prefill-len", type=int, default=64)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--output", type=Path, required=True)
    ap.add_argument("--groups", default="coarse", choices=["coarse", "moe"],
                    help="coarse: attn / mlp rows (the reference's task set); moe: an MoE layer's "
                         "router / experts / combine rows instead of its mlp row")
    a = ap.parse_args()
    assert torch.cuda.is_available(), "CUDA is required for kernel-group profiling"
    build.build()
    rows = measure(a.model, a.batch, a.context, a.decode_steps, a.warmup, a.prefill_len, a.device)
    if a.groups == "coarse":
        rows = coarse_rows(rows)
    write_csv(rows, a.output)
    print(f"profiled model={a.model} device={torch.cuda.get_device_name(a.device)} tasks={len(rows)} "
          f"batch={a.batch} context={a.context} output={a.output}")


if __name__ == "__main__":
    main()
