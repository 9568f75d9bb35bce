"""CPU oracle for the disaggregated decode step -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, and only as the checker or the timed CPU
baseline. The product path (fluidgpu_b200) never imports it.

It restates, in plain torch on the CPU, what the reference computes for one
decode step of a batch of requests. Reference anchors (FluidGPU project):
  fluidgpu_runtime/fluidgpu_torch/runner.py
    decode_step           :119-165  embed -> L x (attn, ffn) -> norm+lm_head
    _run_attn             :170-194  RMSNorm -> self_attn -> + residual
    _run_attn_qkv         :256-293  q/k/v proj, apply_rotary_pos_emb, KV update
    _run_attn_sdpa        :299-335  eager_attention_forward with mask and sinks
    _run_mlp              :349-352  RMSNorm -> mlp -> + residual
    _run_moe_router/experts/combine :432-457
    _attention_mask_for_layer / _sliding_window_mask :713-774 (kv > q - window)
    _attention_extra_kwargs :914-920 (sinks passed as s_aux)
    _norm_head            :167-168
  fluidgpu_runtime/fluidgpu_torch/engine.py:295-300, :337-343 greedy argmax
  fluidgpu_runtime/fluidgpu_torch/kv_cache.py:73-113 KV append at cache_position
Third-party semantics the reference calls into (transformers 5.5.0, the
version installed here; the reference pins >=4.56,<5.0):
  LlamaRMSNorm / GptOssRMSNorm, rotate-half RoPE (default and YaRN inv_freq),
  eager attention with gpt-oss sinks, SwiGLU / SwiGLU-OAI (alpha 1.702,
  limit 7), GptOssTopKRouter (linear -> topk -> softmax over the top-k).

Precision modes: "fp32" computes everything in float32 (the reference's
CPU configuration); "bf16" keeps every activation in bfloat16 exactly where
the reference's bf16 modules round (linear outputs, norm outputs, RoPE
products, softmax probabilities), so it reproduces the reference's bf16 path
on the CPU up to matmul summation order.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn.functional as F

# ---------------------------------------------------------------------------
# elementwise pieces
# ---------------------------------------------------------------------------


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, fp32_weight_mul: bool = False) -> torch.Tensor:
    """LlamaRMSNorm (weight * x_normed.to(dtype)) or GptOssRMSNorm
    ((weight * x_normed).to(dtype)): the layer's input_layernorm /
    post_attention_layernorm and the final norm the reference calls
    (runner.py:183, :351, :434, :167-168)."""
    dtype = x.dtype
    h = x.float()
    var = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(var + eps)
    if fp32_weight_mul:
        return (weight.float() * h).to(dtype)
    return weight * h.to(dtype)


def default_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """inv_freq[i] = theta^(-2i/d) (transformers' default rope init)."""
    exps = torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim
    return 1.0 / (theta ** exps)


def yarn_inv_freq(head_dim: int, theta: float, factor: float, original_max: int,
                  beta_fast: float = 32.0, beta_slow: float = 1.0,
                  truncate: bool = True) -> tuple[torch.Tensor, float]:
    """YaRN (Peng et al. 2023, "YaRN: Efficient Context Window Extension"):
    blend interpolated and extrapolated frequencies with a linear ramp between
    the dimensions whose wavelength makes beta_fast / beta_slow rotations over
    the original context; attention scaled by 0.1*ln(factor)+1."""
    pos_freqs = theta ** (torch.arange(0, head_dim, 2).float() / head_dim)
    extrap = 1.0 / pos_freqs
    interp = 1.0 / (factor * pos_freqs)

    def correction_dim(num_rot: float) -> float:
        return (head_dim * math.log(original_max / (num_rot * 2 * math.pi))) / (2 * math.log(theta))

    low = correction_dim(beta_fast)
    high = correction_dim(beta_slow)
    if truncate:
        low, high = math.floor(low), math.ceil(high)
    low, high = max(low, 0), min(high, head_dim - 1)
    if low == high:
        high += 0.001
    ramp = (torch.arange(head_dim // 2, dtype=torch.float32) - low) / (high - low)
    ramp = torch.clamp(ramp, 0, 1)
    extrap_factor = 1 - ramp
    inv_freq = interp * (1 - extrap_factor) + extrap * extrap_factor
    scaling = 0.1 * math.log(factor) + 1.0
    return inv_freq, scaling


def rope_cos_sin(positions: torch.Tensor, inv_freq: torch.Tensor, scaling: float,
                 dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin of shape [T, hd/2] computed in fp32, scaled, cast to dtype
    (the model's rotary_emb, which the reference calls at runner.py:786-801)."""
    freqs = positions.float()[:, None] * inv_freq.float()[None, :]
    return (freqs.cos() * scaling).to(dtype), (freqs.sin() * scaling).to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE on x[T, heads, hd] with cos/sin [T, hd/2]; each
    product and sum rounds to x.dtype like the reference's tensor ops
    (runner.py:892-903 _apply_rotary_pos_emb)."""
    x1, x2 = x.chunk(2, dim=-1)
    c = cos[:, None, :]
    s = sin[:, None, :]
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1)


def attention_one(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                  window: int = 0, sinks: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention of one sequence in fp32 (runner.py:299-335 with the
    window mask of :713-774 and the sinks of :914-920).
    q [nq, hd]; k, v [L, nkv, hd] (the whole cache incl. the new token).
    window > 0 keeps kv positions > (L-1) - window; sinks [nq] join the
    softmax denominator only (eager_attention_forward of gpt-oss)."""
    nq, hd = q.shape
    L, nkv, _ = k.shape
    G = nq // nkv
    kk = k.float().repeat_interleave(G, dim=1)  # [L, nq, hd]
    vv = v.float().repeat_interleave(G, dim=1)
    scores = torch.einsum("hd,lhd->hl", q.float(), kk) * scale  # [nq, L]
    if window > 0:
        pos = torch.arange(L)
        scores = scores.masked_fill((pos <= (L - 1) - window)[None, :], float("-inf"))
    if sinks is not None:
        logits = torch.cat([scores, sinks.float()[:, None]], dim=-1)
        logits = logits - logits.max(dim=-1, keepdim=True).values
        probs = torch.softmax(logits, dim=-1)[:, :-1]
    else:
        probs = torch.softmax(scores, dim=-1)
    return torch.einsum("hl,lhd->hd", probs, vv)


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """SiLU(gate) * up: the dense MLP the reference runs (runner.py:349-352,
    :416-430; LlamaMLP)."""
    return F.silu(gate) * up


def swiglu_oai(gate: torch.Tensor, up: torch.Tensor, alpha: float = 1.702, limit: float = 7.0) -> torch.Tensor:
    """GptOssExperts._apply_gate: clamp, gate*sigmoid(alpha*gate)*(up+1)
    (the experts module the reference calls at runner.py:444-452)."""
    gate = gate.clamp(min=None, max=limit)
    up = up.clamp(min=-limit, max=limit)
    glu = gate * torch.sigmoid(gate * alpha)
    return (up + 1) * glu


def argmax_lowest(logits: torch.Tensor) -> torch.Tensor:
    """Greedy token per row; ties resolve to the lowest index (torch argmax,
    as the reference's decode loop, engine.py:337-343)."""
    m = logits.max(dim=-1, keepdim=True).values
    idx = torch.arange(logits.shape[-1])
    big = torch.full_like(idx, logits.shape[-1])
    return torch.where(logits == m, idx, big).min(dim=-1).values


def topk_lowest(logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k by value, descending; equal values ordered by lower index
    (a stable descending sort): the router's top-k (runner.py:436;
    vllm_integration.py:462-464)."""
    order = torch.sort(logits, dim=-1, descending=True, stable=True)
    return order.values[..., :k], order.indices[..., :k]


# ---------------------------------------------------------------------------
# router with exactly rounded bf16 logits (GptOssTopKRouter: linear -> topk
# -> softmax over the top-k, the module the reference calls at
# runner.py:432-442; top-k then softmax as vllm_integration.py:462-464)
# ---------------------------------------------------------------------------
def round_bf16_f64(v: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """Nearest bf16 (ties to even) of float64 values, as float64.
    Returns (rounded, tie mask, k, q) where k = v / 2^q, 2^q the bf16
    quantum at v, so a tie is a k with fractional part exactly 1/2."""
    v = np.asarray(v, dtype=np.float64)
    _, ex = np.frexp(v)                      # v = m * 2^ex, 0.5 <= |m| < 1
    q = np.maximum(ex - 8, -133)             # 8 significant bits, or the subnormal quantum
    k = np.ldexp(v, -q)
    r = np.rint(k)                           # round half to even
    out = np.ldexp(r, q)
    out = np.where(np.abs(out) >= 2.0 ** 128, np.copysign(np.inf, v), out)
    tie = np.abs(k - np.trunc(k)) == 0.5
    return out, tie, k, q


def exact_linear_bf16(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
    """bf16(x @ w.T + b) rounded once from the exact real value (ties to
    even): x [T,H], w [E,H], b [E] bf16. Every bf16 x bf16 product is exact in
    float64; math.fsum returns the correctly rounded float64 of their exact
    sum, and its bf16 rounding equals the exact value's unless the float64
    lies exactly on a bf16 midpoint, which exact rational arithmetic then
    decides. This is the one value every bf16 linear with wider accumulation
    approximates; the B200 router kernel computes the same (exact sums)."""
    from fractions import Fraction

    x64 = x.to(torch.float64).numpy()
    w64 = w.to(torch.float64).numpy()
    b64 = b.to(torch.float64).numpy() if b is not None else np.zeros(w64.shape[0])
    T, E = x64.shape[0], w64.shape[0]
    S = np.empty((T, E))
    prods = x64[:, None, :] * w64[None, :, :]
    for t in range(T):
        for e in range(E):
            S[t, e] = math.fsum(prods[t, e].tolist() + [float(b64[e])])
    out, tie, k, q = round_bf16_f64(S)
    for t, e in zip(*np.nonzero(tie)):
        exact = sum(Fraction(p) for p in prods[t, e].tolist()) + Fraction(float(b64[e]))
        if exact != Fraction(float(S[t, e])):  # not a true tie: round towards the exact value
            r = math.ceil(k[t, e]) if exact > Fraction(float(S[t, e])) else math.floor(k[t, e])
            out[t, e] = math.ldexp(r, int(q[t, e]))
    return torch.from_numpy(out).to(torch.bfloat16)


def softmax_topk_bf16(top_v: torch.Tensor) -> torch.Tensor:
    """Softmax over the k selected logits (ordered by value): p_j =
    exp(v_j - v_0) and their sum in selection order in float64, each weight
    p_j / s rounded once to bf16 (GptOssTopKRouter's softmax in the router's
    dtype)."""
    v = top_v.to(torch.float64).numpy()
    p = np.exp(v - v[..., :1])
    s = np.zeros(v.shape[:-1])
    for j in range(v.shape[-1]):
        s = s + p[..., j]
    out = round_bf16_f64(p / s[..., None])[0]
    return torch.from_numpy(out).to(torch.bfloat16)


def router_topk_exact(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None,
                      k: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(weights bf16 [T,k], expert ids [T,k], logits bf16 [T,E]) of the
    router on bf16 inputs: exactly rounded logits, top-k by value with the
    lower expert id first on ties, softmax over the k."""
    logits = exact_linear_bf16(x, w, b)
    top_v, top_i = topk_lowest(logits.float(), k)
    return softmax_topk_bf16(top_v), top_i, logits


# ---------------------------------------------------------------------------
# MXFP4 (OCP microscaling: e2m1 values, one e8m0 scale per 32 elements)
# ---------------------------------------------------------------------------
E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                            -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def mxfp4_quantize(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """w [..., K] (K % 32 == 0) -> (packed uint8 [..., K/2] low nibble = even
    element, scales uint8 [..., K/32] e8m0). Scale = 2^ceil(log2(amax/6)),
    values rounded to the nearest e2m1 (ties to the even code). The layout is
    the checkpoint's, which the reference decodes at vllm_integration.py:503-513."""
    *lead, K = w.shape
    wb = w.float().reshape(*lead, K // 32, 32)
    amax = wb.abs().amax(dim=-1, keepdim=True)
    exp = torch.ceil(torch.log2(torch.clamp(amax, min=1e-30) / 6.0))
    exp = torch.where(amax > 0, exp, torch.full_like(exp, -127.0)).clamp(-127, 127)
    scaled = wb / torch.pow(2.0, exp)
    mags = E2M1_VALUES[:8]
    a = scaled.abs().unsqueeze(-1)
    dist = (a - mags).abs()
    best = dist.min(dim=-1, keepdim=True).values
    cand = (dist == best)
    # ties: prefer the even code (mantissa bit 0)
    codes = torch.arange(8)
    pref = torch.where(cand, (codes % 2) * 8 + codes, torch.full_like(codes, 1 << 20))
    code = pref.argmin(dim=-1)
    sign = (scaled < 0) & (code > 0)
    code = code + sign.long() * 8
    code = code.reshape(*lead, K)
    packed = (code[..., 0::2] | (code[..., 1::2] << 4)).to(torch.uint8)
    scales = (exp.squeeze(-1) + 127).to(torch.uint8)
    return packed, scales


def mxfp4_dequantize(packed: torch.Tensor, scales: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """e2m1 values (low nibble first) x 2^(e8m0 - 127), as
    transformers' convert_moe_packed_tensors (vllm_integration.py:503-513)."""
    lo = (packed & 0x0F).long()
    hi = (packed >> 4).long()
    codes = torch.stack([lo, hi], dim=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)
    vals = E2M1_VALUES[codes]
    *lead, K = vals.shape
    scale = torch.pow(2.0, scales.float() - 127.0)
    vals = vals.reshape(*lead, K // 32, 32) * scale.unsqueeze(-1)
    return vals.reshape(*lead, K).to(dtype)


# ---------------------------------------------------------------------------
# vLLM op boundary (fluidgpu_torch/vllm_integration.py)
# ---------------------------------------------------------------------------
def vllm_moe_experts(x: torch.Tensor, router_logits: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor,
                     w2: torch.Tensor, b2: torch.Tensor, top_k: int,
                     expert_range: tuple[int, int] | None = None) -> torch.Tensor:
    """The expert computation behind the reference's vLLM MoE forward_impl
    (MarlinExpertsOnDevice.forward_on_device, vllm_integration.py:452-485):
    top-k of the router logits (lowest expert id first on ties), softmax over
    the k selected in fp32, per selected expert gu = x W1^T + b1 with gate =
    gu[:, 0::2], up = gu[:, 1::2] (the checkpoint's interleaved rows),
    SwiGLU-OAI, y = act W2^T + b2, weighted sum over the k. fp32 throughout.
    w1 [E, 2I, H], b1 [E, 2I], w2 [E, H, I], b2 [E, H]. With expert_range
    only experts in [lo, hi) contribute (expert_map, :371-390), so two ranges
    that cover all experts add up to the full result (:1052-1093)."""
    x = x.float()
    top_v, top_i = topk_lowest(router_logits.float(), top_k)
    wts = torch.softmax(top_v, dim=-1)
    lo, hi = expert_range if expert_range is not None else (0, w1.shape[0])
    out = torch.zeros(x.shape[0], w2.shape[1], dtype=torch.float32)
    for e in range(lo, hi):
        tok, slot = torch.where(top_i == e)
        if tok.numel() == 0:
            continue
        gu = x[tok] @ w1[e].float().T + b1[e].float()
        act = swiglu_oai(gu[:, 0::2], gu[:, 1::2])
        y = act @ w2[e].float().T + b2[e].float()
        out.index_add_(0, tok, y * wts[tok, slot, None])
    return out


def vllm_dense_mlp(x: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    """RemoteDenseMLP._mlp (vllm_integration.py:1305-1311): w_gate_up is the
    merged [gate; up] weight [2I, H]; down(SiLU(gate) * up) in fp32."""
    gu = x.float() @ w_gate_up.float().T
    gate, up = gu.chunk(2, dim=-1)
    return (F.silu(gate) * up) @ w_down.float().T


# ---------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------
@dataclass
class OracleSpec:
    num_layers: int
    hidden: int
    n_q: int
    n_kv: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float
    eps: float = 1e-5
    # gpt-oss
    moe: bool = False
    num_experts: int = 0
    top_k: int = 0
    attn_bias: bool = False
    sinks: bool = False
    layer_windows: list[int] = field(default_factory=list)  # 0 = full
    rope_yarn: dict | None = None
    fp32_weight_mul: bool = False


class OracleModel:
    """Batched decode over per-request contiguous caches (no paging: the
    page layout is a device detail, checked separately).

    weights: dict with
      embed [V,H], final_norm [H], lm_head [V,H],
      per layer i: ln1, ln2 [H]; wq [nq*hd,H], wk, wv [nkv*hd,H] (+bq,bk,bv);
      wo [H, nq*hd] (+bo); dense: wg, wu [I,H], wd [H,I];
      moe: router_w [E,H], router_b [E], w_gate_up [E, 2I, H] (gate/up rows
      interleaved as in the HF parameter: row 2j gate, 2j+1 up), b_gate_up
      [E,2I], w_down [E,H,I], b_down [E,H]; sinks [nq].
    Keys are f"{i}.{name}" for layer tensors.
    """

    def __init__(self, spec: OracleSpec, weights: dict[str, torch.Tensor], dtype: torch.dtype) -> None:
        self.spec = spec
        self.w = {k: v.to(dtype) if v.is_floating_point() else v for k, v in weights.items()}
        self.dtype = dtype
        s = spec
        if s.rope_yarn:
            y = s.rope_yarn
            self.inv_freq, self.rope_scaling = yarn_inv_freq(
                s.head_dim, s.rope_theta, y["factor"], y["original_max_position_embeddings"],
                y.get("beta_fast", 32.0), y.get("beta_slow", 1.0), y.get("truncate", True))
        else:
            self.inv_freq, self.rope_scaling = default_inv_freq(s.head_dim, s.rope_theta), 1.0
        self.k_cache: list[list[torch.Tensor]] = []
        self.v_cache: list[list[torch.Tensor]] = []
        self.lengths: list[int] = []
        self.router_indices: list[torch.Tensor] = []  # per layer, last step
        # per layer, last step: each token's gap between its k-th and (k+1)-th
        # router logit (a small gap is a near tie that rounding may flip)
        self.router_margins: list[torch.Tensor] = []
        # per layer, last step: the router's input x (normalised hidden), kept
        # when record_router_inputs is set
        self.record_router_inputs = False
        self.router_inputs: list[torch.Tensor] = []

    def reset(self, batch: int) -> None:
        L = self.spec.num_layers
        e = torch.empty(0, self.spec.n_kv, self.spec.head_dim, dtype=self.dtype)
        self.k_cache = [[e.clone() for _ in range(L)] for _ in range(batch)]
        self.v_cache = [[e.clone() for _ in range(L)] for _ in range(batch)]
        self.lengths = [0] * batch

    def _linear(self, x: torch.Tensor, w: str, b: str | None = None) -> torch.Tensor:
        bias = self.w.get(b) if b else None
        return F.linear(x, self.w[w], bias)

    def _attention(self, i: int, h: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        s = self.spec
        B = h.shape[0]
        x = rms_norm(h, self.w[f"{i}.ln1"], s.eps, s.fp32_weight_mul)
        bias = s.attn_bias
        q = self._linear(x, f"{i}.wq", f"{i}.bq" if bias else None).view(B, s.n_q, s.head_dim)
        k = self._linear(x, f"{i}.wk", f"{i}.bk" if bias else None).view(B, s.n_kv, s.head_dim)
        v = self._linear(x, f"{i}.wv", f"{i}.bv" if bias else None).view(B, s.n_kv, s.head_dim)
        cos, sin = rope_cos_sin(positions, self.inv_freq, self.rope_scaling, self.dtype)
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        window = s.layer_windows[i] if s.layer_windows else 0
        sinks = self.w.get(f"{i}.sinks") if s.sinks else None
        outs = []
        for b in range(B):
            self.k_cache[b][i] = torch.cat([self.k_cache[b][i], k[b : b + 1]], dim=0)
            self.v_cache[b][i] = torch.cat([self.v_cache[b][i], v[b : b + 1]], dim=0)
            o = attention_one(q[b], self.k_cache[b][i], self.v_cache[b][i],
                              1.0 / math.sqrt(s.head_dim), window, sinks)
            outs.append(o.reshape(-1))
        attn = torch.stack(outs).to(self.dtype)
        o = self._linear(attn, f"{i}.wo", f"{i}.bo" if bias else None)
        return h + o

    def _dense_ffn(self, i: int, h: torch.Tensor) -> torch.Tensor:
        s = self.spec
        x = rms_norm(h, self.w[f"{i}.ln2"], s.eps, s.fp32_weight_mul)
        act = silu_mul(self._linear(x, f"{i}.wg"), self._linear(x, f"{i}.wu"))
        return h + self._linear(act, f"{i}.wd")

    def _moe_ffn(self, i: int, h: torch.Tensor) -> torch.Tensor:
        s = self.spec
        x = rms_norm(h, self.w[f"{i}.ln2"], s.eps, s.fp32_weight_mul)
        if self.dtype == torch.bfloat16:
            # bf16 router logits rounded once from their exact value (the
            # order-independent result of the bf16 linear), softmax rounded once
            scores, top_i, logits = router_topk_exact(x, self.w[f"{i}.router_w"], self.w.get(f"{i}.router_b"),
                                                      s.top_k)
        else:
            logits = self._linear(x, f"{i}.router_w", f"{i}.router_b")
            top_v, top_i = topk_lowest(logits, s.top_k)
            scores = torch.softmax(top_v, dim=-1)
        if self.record_router_inputs:
            self.router_inputs.append(x.clone())
        self.router_indices.append(top_i.clone())
        if s.top_k < s.num_experts:
            kk = torch.topk(logits.float(), s.top_k + 1, dim=-1).values
            self.router_margins.append(kk[:, s.top_k - 1] - kk[:, s.top_k])
        out = torch.zeros_like(x)
        wgu = self.w[f"{i}.w_gate_up"]
        bgu = self.w[f"{i}.b_gate_up"]
        wd = self.w[f"{i}.w_down"]
        bd = self.w[f"{i}.b_down"]
        for e in range(s.num_experts):
            tok, kpos = torch.where(top_i == e)
            if tok.numel() == 0:
                continue
            gu = F.linear(x[tok], wgu[e], bgu[e])
            act = swiglu_oai(gu[:, 0::2], gu[:, 1::2])
            y = F.linear(act, wd[e], bd[e])
            out.index_add_(0, tok, (y * scores[tok, kpos, None]).to(x.dtype))
        return h + out

    def step(self, tokens: torch.Tensor) -> torch.Tensor:
        """Append one token per request; returns logits [B, V] (model dtype):
        the reference's decode_step (runner.py:119-165) for every request."""
        s = self.spec
        B = tokens.numel()
        if not self.lengths:
            self.reset(B)
        positions = torch.tensor(self.lengths, dtype=torch.long)
        h = self.w["embed"][tokens.reshape(-1)]
        self.router_indices = []
        self.router_margins = []
        self.router_inputs = []
        for i in range(s.num_layers):
            h = self._attention(i, h, positions)
            h = self._moe_ffn(i, h) if s.moe else self._dense_ffn(i, h)
        self.lengths = [n + 1 for n in self.lengths]
        x = rms_norm(h, self.w["final_norm"], s.eps, s.fp32_weight_mul)
        return F.linear(x, self.w["lm_head"])

    def prefill(self, prompts: torch.Tensor) -> torch.Tensor:
        """Full-prompt prefill of prompts [B, S] with a causal (and, per layer,
        sliding-window) mask, as the reference's prefill does
        (runner.py:66-116); fills the caches and returns the last logits."""
        s = self.spec
        B, S = prompts.shape
        self.reset(B)
        pos = torch.arange(S)
        cos, sin = rope_cos_sin(pos, self.inv_freq, self.rope_scaling, self.dtype)
        h = self.w["embed"][prompts.reshape(-1)].view(B, S, s.hidden)
        scale = 1.0 / math.sqrt(s.head_dim)
        G = s.n_q // s.n_kv
        for i in range(s.num_layers):
            x = rms_norm(h, self.w[f"{i}.ln1"], s.eps, s.fp32_weight_mul)
            bias = s.attn_bias
            q = self._linear(x, f"{i}.wq", f"{i}.bq" if bias else None).view(B * S, s.n_q, s.head_dim)
            k = self._linear(x, f"{i}.wk", f"{i}.bk" if bias else None).view(B * S, s.n_kv, s.head_dim)
            v = self._linear(x, f"{i}.wv", f"{i}.bv" if bias else None).view(B, S, s.n_kv, s.head_dim)
            q = apply_rope(q, cos.repeat(B, 1), sin.repeat(B, 1)).view(B, S, s.n_q, s.head_dim)
            k = apply_rope(k, cos.repeat(B, 1), sin.repeat(B, 1)).view(B, S, s.n_kv, s.head_dim)
            for b in range(B):
                self.k_cache[b][i] = k[b].clone()
                self.v_cache[b][i] = v[b].clone()
            kk = k.float().repeat_interleave(G, dim=2)
            vv = v.float().repeat_interleave(G, dim=2)
            sc = torch.einsum("bqhd,bkhd->bhqk", q.float(), kk) * scale
            mask = pos[None, :] > pos[:, None]
            window = s.layer_windows[i] if s.layer_windows else 0
            if window > 0:
                mask = mask | (pos[None, :] <= pos[:, None] - window)
            sc = sc.masked_fill(mask, float("-inf"))
            if s.sinks:
                sk = self.w[f"{i}.sinks"].float()[None, :, None, None].expand(B, -1, S, 1)
                lg = torch.cat([sc, sk], dim=-1)
                lg = lg - lg.max(dim=-1, keepdim=True).values
                probs = torch.softmax(lg, dim=-1)[..., :-1]
            else:
                probs = torch.softmax(sc, dim=-1)
            o = torch.einsum("bhqk,bkhd->bqhd", probs, vv).reshape(B, S, -1).to(self.dtype)
            h = h + self._linear(o, f"{i}.wo", f"{i}.bo" if bias else None)
            flat = h.reshape(B * S, s.hidden)
            flat = self._moe_ffn(i, flat) if s.moe else self._dense_ffn(i, flat)
            h = flat.view(B, S, s.hidden)
        self.lengths = [S] * B
        x = rms_norm(h[:, -1], self.w["final_norm"], s.eps, s.fp32_weight_mul)
        return F.linear(x, self.w["lm_head"])

    def prefill_stepwise(self, prompts: torch.Tensor) -> torch.Tensor:
        """Feed prompts [B, S] one position at a time (causal attention makes
        this equal to a full prefill, runner.py:66-116); returns the last
        logits [B, V]."""
        self.reset(prompts.shape[0])
        logits = None
        for t in range(prompts.shape[1]):
            logits = self.step(prompts[:, t])
        return logits

    def generate(self, prompts: torch.Tensor, steps: int) -> tuple[torch.Tensor, list[torch.Tensor]]:
        """Greedy decode: returns tokens [B, steps] and the logits of every step
        (the reference's loop, engine.py:275-357)."""
        logits = self.prefill(prompts)
        toks, all_logits = [], []
        for _ in range(steps):
            all_logits.append(logits)
            nxt = argmax_lowest(logits.float())
            toks.append(nxt)
            logits = self.step(nxt)
        return torch.stack(toks, dim=1), all_logits


# ---------------------------------------------------------------------------
# weights straight from a transformers model (the reference runs HF modules)
# ---------------------------------------------------------------------------
def spec_from_hf(cfg) -> OracleSpec:
    """Shapes and options of an HF Llama / GptOss config, as the reference
    reads them from the model (runner.py:923-941 head counts and sizes)."""
    gpt = cfg.model_type == "gpt_oss"
    hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    params = getattr(cfg, "rope_parameters", None) or {}
    kind = params.get("rope_type", "default")
    windows = []
    if gpt:
        windows = [int(cfg.sliding_window) if t == "sliding_attention" else 0 for t in cfg.layer_types]
    return OracleSpec(
        num_layers=cfg.num_hidden_layers, hidden=cfg.hidden_size, n_q=cfg.num_attention_heads,
        n_kv=cfg.num_key_value_heads, head_dim=hd, intermediate=cfg.intermediate_size,
        vocab=cfg.vocab_size, rope_theta=float(params.get("rope_theta", getattr(cfg, "rope_theta", 10000.0))),
        eps=float(cfg.rms_norm_eps), moe=gpt, num_experts=int(getattr(cfg, "num_local_experts", 0) or 0),
        top_k=int(getattr(cfg, "num_experts_per_tok", 0) or 0) if gpt else 0,
        attn_bias=bool(getattr(cfg, "attention_bias", False)), sinks=gpt, layer_windows=windows,
        rope_yarn=dict(params) if kind == "yarn" else None, fp32_weight_mul=gpt)


def weights_from_hf(model) -> dict[str, torch.Tensor]:
    """The tensors of an HF model the reference's runner uses
    (runner.py:15-25 extract_components)."""
    m = model.model
    w: dict[str, torch.Tensor] = {"embed": m.embed_tokens.weight.detach(),
                                  "final_norm": m.norm.weight.detach(),
                                  "lm_head": model.lm_head.weight.detach()}
    for i, layer in enumerate(m.layers):
        a = layer.self_attn
        w[f"{i}.ln1"] = layer.input_layernorm.weight.detach()
        w[f"{i}.ln2"] = layer.post_attention_layernorm.weight.detach()
        for n in ("q", "k", "v", "o"):
            w[f"{i}.w{n}"] = getattr(a, f"{n}_proj").weight.detach()
            b = getattr(a, f"{n}_proj").bias
            if b is not None:
                w[f"{i}.b{n}"] = b.detach()
        if hasattr(a, "sinks"):
            w[f"{i}.sinks"] = a.sinks.detach()
        mlp = layer.mlp
        if hasattr(mlp, "router"):
            w[f"{i}.router_w"] = mlp.router.weight.detach()
            w[f"{i}.router_b"] = mlp.router.bias.detach()
            ex = mlp.experts
            # HF keeps [E, H, 2I] / [E, I, H] (x @ W); the oracle uses [out, in]
            w[f"{i}.w_gate_up"] = ex.gate_up_proj.detach().transpose(1, 2).contiguous()
            w[f"{i}.b_gate_up"] = ex.gate_up_proj_bias.detach()
            w[f"{i}.w_down"] = ex.down_proj.detach().transpose(1, 2).contiguous()
            w[f"{i}.b_down"] = ex.down_proj_bias.detach()
        else:
            w[f"{i}.wg"] = mlp.gate_proj.weight.detach()
            w[f"{i}.wu"] = mlp.up_proj.weight.detach()
            w[f"{i}.wd"] = mlp.down_proj.weight.detach()
    return w
