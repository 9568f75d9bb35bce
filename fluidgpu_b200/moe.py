"""gpt-oss MoE feed-forward on the B200 kernels (router / experts / combine
groups of fluidgpu_torch.runner, runner.py:432-457).

Expert weights live on the device as MXFP4 (e2m1 values + one e8m0 scale per
32 inputs), packed into the 4352-byte tile records of fg_pack_mxfp4:
  w1: [E][2I/128][H/64] records of W1_e = the gate_up projection with rows
      interleaved in blocks of 64 (gate features 64j.., then up features 64j..),
      b1: [E][2I] in the same row order
  w2: [E][ceil(H/128)][I/64] records of the down projection, b2: [E][H]
Transformers keeps gate/up columns interleaved one by one (gate = 0::2,
up = 1::2, GptOssExperts._apply_gate); the 64-block order is what lets one
128-row tile finish SwiGLU-OAI in its epilogue.

Quantisation (weight preparation, not the decode path): scale =
2^ceil(log2(amax/6)) per 32 inputs, e2m1 value = round-to-nearest (ties to the
even code) of w / scale; MXFP4 weights that are already exact (a real
checkpoint, or dequantised ones) come back unchanged.
"""
from __future__ import annotations

from typing import Any

import torch

from . import _lib, kernels
from ._lib import call

_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


_MIDS = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])  # between e2m1 magnitudes


def _quantize_rows(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    *lead, K = w.shape
    blocks = w.float().reshape(*lead, K // 32, 32)
    amax = blocks.abs().amax(dim=-1, keepdim=True)
    exp = torch.ceil(torch.log2(torch.clamp(amax, min=2.0 ** -126) / 6.0)).clamp(-126, 127)
    scaled = blocks / torch.pow(2.0, exp)
    mag = scaled.abs()
    mids = _MIDS.to(w.device)
    code = torch.bucketize(mag, mids)  # ties land on the lower magnitude
    tie = (code < 7) & (mag == mids[code.clamp(max=6)])
    code = code + (tie & (code % 2 == 1)).long()  # ties go to the even code
    code = code + ((scaled < 0) & (code > 0)).long() * 8
    code = code.reshape(*lead, K)
    values = (code[..., 0::2] | (code[..., 1::2] << 4)).to(torch.uint8)
    scales = (exp.squeeze(-1) + 127).to(torch.uint8)
    return values, scales


def quantize_mxfp4(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """w [..., K] (K % 32 == 0) -> (values uint8 [..., K/2], scales uint8 [..., K/32]).
    Large tensors are processed one leading slice at a time."""
    *lead, K = w.shape
    assert K % 32 == 0, "MXFP4 needs K % 32 == 0"
    if w.ndim == 3 and w.numel() > (1 << 26):
        parts = [_quantize_rows(w[i]) for i in range(w.shape[0])]
        return torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts])
    return _quantize_rows(w)


def dequantize_mxfp4(values: torch.Tensor, scales: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    grid = torch.cat([_E2M1, -_E2M1]).to(values.device)
    codes = torch.stack([(values & 15).long(), (values >> 4).long()], dim=-1)
    codes = codes.reshape(*values.shape[:-1], values.shape[-1] * 2)
    v = grid[codes]
    *lead, K = v.shape
    s = torch.pow(2.0, scales.float() - 127.0).unsqueeze(-1)
    return (v.reshape(*lead, K // 32, 32) * s).reshape(*lead, K).to(dtype)


def interleave64(gate_up_rows: torch.Tensor) -> torch.Tensor:
    """[E, 2I, ...] with gate/up alternating row by row (transformers) ->
    [E, 2I, ...] with gate/up alternating in blocks of 64 rows."""
    E, N2 = gate_up_rows.shape[:2]
    I = N2 // 2
    assert I % 64 == 0, f"expert intermediate size {I} must be a multiple of 64"
    gate, up = gate_up_rows[:, 0::2], gate_up_rows[:, 1::2]
    rest = gate.shape[2:]
    return torch.stack([gate.reshape(E, I // 64, 64, *rest), up.reshape(E, I // 64, 64, *rest)],
                       dim=2).reshape(E, N2, *rest)


def pack_mxfp4(values: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    E, N, K2 = values.shape
    K = K2 * 2
    out = torch.empty(_lib.lib().fg_mxfp4_packed_bytes(E, N, K), dtype=torch.uint8, device=values.device)
    call("fg_pack_mxfp4", values.data_ptr(), scales.contiguous().data_ptr(), out.data_ptr(), E, N, K,
         kernels._stream(values.device))
    return out


def expert_range(E: int, shard: tuple[int, int] | None) -> tuple[int, int]:
    """Experts [lo, hi) held by expert-parallel shard (index, count): equal
    contiguous ranges."""
    if shard is None:
        return 0, E
    i, S = shard
    assert 0 <= i < S and E % S == 0, f"{E} experts do not split evenly over {S} shards"
    return E * i // S, E * (i + 1) // S


def _expert_tensors(w1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor, b2: torch.Tensor,
                    device: torch.device, shard: tuple[int, int] | None = None) -> dict[str, Any]:
    """w1 [E, 2I, H] (transformers' gate/up row order), b1 [E, 2I], w2 [E, H, I],
    b2 [E, H] (any float dtype) -> packed device tensors (of shard's experts)."""
    lo, hi = expert_range(w1.shape[0], shard)
    w1, b1, w2, b2 = w1[lo:hi], b1[lo:hi], w2[lo:hi], b2[lo:hi]
    E, N1, H = w1.shape
    I = N1 // 2
    w1 = interleave64(w1.to(device))
    b1 = interleave64(b1.to(device).unsqueeze(-1)).squeeze(-1)
    v1, s1 = quantize_mxfp4(w1)
    v2, s2 = quantize_mxfp4(w2.to(device))
    return {
        "moe_w1": pack_mxfp4(v1.contiguous(), s1.contiguous()),
        "moe_b1": b1.to(torch.bfloat16).contiguous(),
        "moe_w2": pack_mxfp4(v2.contiguous(), s2.contiguous()),
        "moe_b2": b2.to(device=device, dtype=torch.bfloat16).contiguous(),
        "moe_shape": (E, H, I),
        "moe_expert_range": (lo, hi),
    }


def random_expert_weights(spec, normal, device: torch.device, dtype: torch.dtype,
                          shard: tuple[int, int] | None = None) -> dict[str, Any]:
    E, H, I = spec.num_experts, spec.hidden, spec.intermediate
    out = {"router_w": normal(E, H), "router_b": torch.zeros(E, dtype=dtype, device=device)}
    w1 = normal(E, 2 * I, H)
    w2 = normal(E, H, I)
    out.update(_expert_tensors(w1, torch.zeros(E, 2 * I, device=device), w2,
                               torch.zeros(E, H, device=device), device, shard))
    return out


def expert_weights_from_hf(mlp: Any, device: torch.device, shard: tuple[int, int] | None = None) -> dict[str, Any]:
    """transformers GptOssMLP -> router + packed MXFP4 experts (of shard's experts)."""
    ex = mlp.experts
    bf = lambda t: t.detach().to(device=device, dtype=torch.bfloat16).contiguous()  # noqa: E731
    out = {"router_w": bf(mlp.router.weight), "router_b": bf(mlp.router.bias)}
    # transformers keeps x @ W: gate_up_proj [E, H, 2I], down_proj [E, I, H]
    out.update(_expert_tensors(ex.gate_up_proj.detach().transpose(1, 2).float(),
                               ex.gate_up_proj_bias.detach().float(),
                               ex.down_proj.detach().transpose(1, 2).float(),
                               ex.down_proj_bias.detach().float(), device, shard))
    return out


# ---------------------------------------------------------------------------
# the three kernel groups
# ---------------------------------------------------------------------------
def router_topk(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, k: int,
                logits: bool = False):
    T, H = x.shape
    E = w.shape[0]
    weights = torch.empty((T, k), dtype=torch.bfloat16, device=x.device)
    idx = torch.empty((T, k), dtype=torch.int32, device=x.device)
    lg = torch.empty((T, E), dtype=torch.bfloat16, device=x.device) if logits else None
    call("fg_moe_router_topk", x.data_ptr(), w.data_ptr(), None if b is None else b.data_ptr(), T, H,
         E, k, weights.data_ptr(), idx.data_ptr(), None if lg is None else lg.data_ptr(),
         kernels._stream(x.device))
    return (weights, idx, lg) if logits else (weights, idx)


class Routing:
    """Device buffers of one permutation (fg_moe_permute). expert_range limits
    the work items to an expert-parallel shard's experts [lo, hi)."""

    def __init__(self, idx: torch.Tensor, E: int, expert_range: tuple[int, int] | None = None) -> None:
        T, k = idx.shape
        lib = _lib.lib()
        dev = idx.device
        self.T, self.k, self.E = T, k, E
        self.lo, self.hi = expert_range if expert_range is not None else (0, E)
        self.BN = lib.fg_moe_tile_tokens(T, k, E)
        self.max_items = lib.fg_moe_max_items(T, k, E, self.BN)
        self.offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        self.perm_pair = torch.empty(T * k, dtype=torch.int32, device=dev)
        self.inv = torch.empty(T * k, dtype=torch.int32, device=dev)
        self.items = torch.empty(max(self.max_items, 1) * 2, dtype=torch.int32, device=dev)
        self.item_count = torch.empty(1, dtype=torch.int32, device=dev)
        call("fg_moe_permute", idx.data_ptr(), T, k, E, self.BN, self.lo, self.hi, self.offsets.data_ptr(),
             self.perm_pair.data_ptr(), self.inv.data_ptr(), self.items.data_ptr(),
             self.item_count.data_ptr(), kernels._stream(dev))


def grouped_gemm(x_perm: torch.Tensor, w_packed: torch.Tensor, bias: torch.Tensor | None,
                 routing: Routing, N: int, K: int, epilogue: int) -> torch.Tensor:
    """x_perm: f16 rows (fg_moe_gather's output, or a previous SwiGLU-OAI call's).
    Returns f16 [rows, N/2] after SwiGLU-OAI (bf16-rounded values), bf16 [rows, N]
    after a plain store."""
    assert x_perm.dtype == torch.float16, f"expert GEMM operands are f16 rows, got {x_perm.dtype}"
    rows = x_perm.shape[0]
    swiglu = epilogue == _lib.FG_EPI_SWIGLU_OAI
    n_out = N // 2 if swiglu else N
    out = torch.empty((rows, n_out), dtype=torch.float16 if swiglu else torch.bfloat16, device=x_perm.device)
    call("fg_moe_gemm_mxfp4", x_perm.data_ptr(), w_packed.data_ptr(),
         None if bias is None else bias.data_ptr(), routing.offsets.data_ptr(),
         routing.items.data_ptr(), routing.item_count.data_ptr(), routing.max_items,
         out.data_ptr(), rows, N, K, routing.BN, epilogue, routing.lo, kernels._stream(x_perm.device))
    return out


def experts_forward(x: torch.Tensor, idx: torch.Tensor, weights: torch.Tensor, W: dict, spec,
                    residual: torch.Tensor | None = None) -> torch.Tensor:
    """Routed experts for x [T, H] (post-norm): permute -> gate_up + SwiGLU-OAI
    -> down -> weighted un-permute (+ residual when given). Weights holding an
    expert-parallel shard (W["moe_expert_range"]) give that shard's fp32
    partial [T, H] (no residual) for fg_sum_partials."""
    T, H = x.shape
    E_local, H_, I = W["moe_shape"]
    E = spec.num_experts
    k = idx.shape[1]
    lo, hi = W.get("moe_expert_range", (0, E))
    assert hi - lo == E_local, f"packed experts {E_local} != range [{lo}, {hi})"
    partial = (lo, hi) != (0, E)
    assert not (partial and residual is not None), "an expert-parallel partial takes no residual"
    routing = Routing(idx, E, (lo, hi))
    x_perm = torch.empty((T * k, H), dtype=torch.float16, device=x.device)
    call("fg_moe_gather", x.data_ptr(), routing.perm_pair.data_ptr(), T, k, H, x_perm.data_ptr(),
         kernels._stream(x.device))
    act = grouped_gemm(x_perm, W["moe_w1"], W["moe_b1"], routing, 2 * I, H, _lib.FG_EPI_SWIGLU_OAI)
    y = grouped_gemm(act, W["moe_w2"], W["moe_b2"], routing, H, I, _lib.FG_EPI_STORE)
    out = torch.empty((T, H), dtype=torch.float32 if partial else torch.bfloat16, device=x.device)
    call("fg_moe_unpermute", y.data_ptr(), routing.inv.data_ptr(), idx.data_ptr(), weights.data_ptr(),
         None if residual is None else residual.data_ptr(), out.data_ptr(), T, k, H, lo, hi, int(partial),
         kernels._stream(x.device))
    return out


def residual_add(residual: torch.Tensor, y: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(residual)
    call("fg_add_bf16", residual.data_ptr(), y.data_ptr(), out.data_ptr(), residual.numel(),
         kernels._stream(residual.device))
    return out
