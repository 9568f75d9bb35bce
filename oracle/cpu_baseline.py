"""Timed CPU baseline of the decode step -- TEST/BENCH INFRASTRUCTURE ONLY.

Used by bench.py's cpu_baseline field and its `--impl reference` arm. It
runs the oracle's restatement of the reference algorithm (decode_ref.py:
RMSNorm, q/k/v linear, rotate-half RoPE, GQA attention over the whole
context with repeat_kv, o_proj + residual, SwiGLU MLP + residual,
norm + lm_head, greedy argmax) in float32 on the host cores.

A full Llama-3-8B step at batch 64 and context 4096 is minutes of CPU work,
so the measured sample is ONE decoder layer plus the norm/lm_head/argmax
tail at the full batch and context; the step time is scaled to the model as
num_layers * t_layer + t_head, and tokens/s = batch / step time. The
reference measures its per-group CPU costs the same way, one group at a time
at the target dims (examples/fluidgpu_torch/profile_llm_tasks.py:116-160).
"""
from __future__ import annotations

import math
import os
import time

import torch
import torch.nn.functional as F

from . import decode_ref as ref


def host_threads() -> int:
    """Host cores this process may use (len(os.sched_getaffinity(0)), the
    count the baseline reports beside its number)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


class LayerSample:
    """One dense decoder layer + head at (batch, context), fp32, random
    N(0,0.02): the reference's _run_attn + _run_mlp (runner.py:170-194,
    :349-352) and _norm_head + argmax (runner.py:167-168, engine.py:337-343)."""

    def __init__(self, hidden: int, n_q: int, n_kv: int, head_dim: int, intermediate: int,
                 vocab: int, rope_theta: float, batch: int, context: int, seed: int = 0) -> None:
        g = torch.Generator().manual_seed(seed)
        n = lambda *s: torch.randn(*s, generator=g) * 0.02  # noqa: E731
        self.H, self.nq, self.nkv, self.hd = hidden, n_q, n_kv, head_dim
        self.B, self.ctx = batch, context
        self.wq, self.wk, self.wv = n(n_q * head_dim, hidden), n(n_kv * head_dim, hidden), n(n_kv * head_dim, hidden)
        self.wo = n(hidden, n_q * head_dim)
        self.wg, self.wu, self.wd = n(intermediate, hidden), n(intermediate, hidden), n(hidden, intermediate)
        self.ln1 = torch.ones(hidden)
        self.ln2 = torch.ones(hidden)
        self.lm_head = n(vocab, hidden)
        self.final_norm = torch.ones(hidden)
        self.inv_freq = ref.default_inv_freq(head_dim, rope_theta)
        # contiguous cache with room for the new token
        self.k = torch.randn(batch, context + 1, n_kv, head_dim, generator=g)
        self.v = torch.randn(batch, context + 1, n_kv, head_dim, generator=g)
        self.h = torch.randn(batch, hidden, generator=g)

    def layer(self) -> torch.Tensor:
        """One decode step of the layer for the whole batch (runner.py:170-194
        attention group, :349-352 MLP group)."""
        B = self.B
        h = self.h
        x = ref.rms_norm(h, self.ln1, 1e-5)
        q = F.linear(x, self.wq).view(B, self.nq, self.hd)
        k = F.linear(x, self.wk).view(B, self.nkv, self.hd)
        v = F.linear(x, self.wv).view(B, self.nkv, self.hd)
        pos = torch.full((B,), self.ctx, dtype=torch.long)
        cos, sin = ref.rope_cos_sin(pos, self.inv_freq, 1.0, torch.float32)
        q = ref.apply_rope(q, cos, sin)
        k = ref.apply_rope(k, cos, sin)
        self.k[:, self.ctx] = k
        self.v[:, self.ctx] = v
        scale = 1.0 / math.sqrt(self.hd)
        outs = [ref.attention_one(q[b], self.k[b], self.v[b], scale).reshape(-1) for b in range(B)]
        h = h + F.linear(torch.stack(outs), self.wo)
        x = ref.rms_norm(h, self.ln2, 1e-5)
        return h + F.linear(ref.silu_mul(F.linear(x, self.wg), F.linear(x, self.wu)), self.wd)

    def head(self) -> torch.Tensor:
        """Final norm + lm_head + greedy argmax (runner.py:167-168,
        engine.py:337-343)."""
        x = ref.rms_norm(self.h, self.final_norm, 1e-5)
        return ref.argmax_lowest(F.linear(x, self.lm_head))


def time_sample(sample: LayerSample, num_layers: int, reps: int = 1) -> dict:
    """Median per-layer and head seconds over `reps`, scaled to one full step."""
    lt, ht = [], []
    with torch.inference_mode():
        for _ in range(reps):
            t0 = time.perf_counter()
            sample.layer()
            t1 = time.perf_counter()
            sample.head()
            t2 = time.perf_counter()
            lt.append(t1 - t0)
            ht.append(t2 - t1)
    lt.sort()
    ht.sort()
    t_layer, t_head = lt[len(lt) // 2], ht[len(ht) // 2]
    step = num_layers * t_layer + t_head
    return {"t_layer_s": t_layer, "t_head_s": t_head, "step_s": step,
            "tokens_per_s": sample.B / step, "threads": torch.get_num_threads()}
