"""Model architecture specs and device weights in the layouts the kernels use.

Layouts (all bf16 unless noted, row-major, K contiguous so every GEMM
operand is a K-major TMA source):
  embed        [V, H]
  lm_head      [V, H]            (tied models share embed)
  ln1, ln2     [H]               final_norm [H]
  wqkv         [(nq + 2 nkv) hd, H]    q rows, then k rows, then v rows
  bqkv         [(nq + 2 nkv) hd]       (gpt-oss attention bias)
  wo           [H, nq hd]        bo [H]
  w_gate_up    [2 I, H]          gate and up rows interleaved in blocks of 64
                                 (rows 128j..128j+63 = gate rows 64j..64j+63,
                                 rows 128j+64..128j+127 = up rows 64j..64j+63),
                                 so one 128-row GEMM tile holds matching
                                 gate/up features for the fused SwiGLU epilogue
  w_down       [H, I]
  sinks        [nq] fp32         (gpt-oss)
  MoE (gpt-oss): router_w [E, H], router_b [E]; experts in MXFP4
  (see fluidgpu_b200.moe for the packed layout).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch

from . import _lib
from . import rope as rope_mod


@dataclass(frozen=True)
class ModelSpec:
    name: str
    family: str                    # "llama" | "gpt_oss"
    num_layers: int
    hidden: int
    n_q: int
    n_kv: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float
    eps: float = 1e-5
    rope: dict[str, Any] | None = None      # None = default RoPE
    attn_bias: bool = False
    sinks: bool = False
    sliding_window: int = 0
    layer_types: tuple[str, ...] = ()        # "full_attention" / "sliding_attention"
    num_experts: int = 0
    top_k: int = 0
    tie_embeddings: bool = False

    @property
    def moe(self) -> bool:
        return self.num_experts > 0

    @property
    def norm_mode(self) -> int:
        return _lib.FG_NORM_FP32MUL if self.family == "gpt_oss" else _lib.FG_NORM_LLAMA

    @property
    def qkv_width(self) -> int:
        return (self.n_q + 2 * self.n_kv) * self.head_dim

    def window(self, layer: int) -> int:
        if self.layer_types and self.layer_types[layer] == "sliding_attention":
            return self.sliding_window
        return 0

    def rope_tables(self) -> tuple[torch.Tensor, float]:
        if not self.rope:
            return rope_mod.default(self.head_dim, self.rope_theta)
        kind = self.rope["rope_type"]
        if kind == "yarn":
            r = self.rope
            return rope_mod.yarn(self.head_dim, self.rope_theta, r["factor"],
                                 r["original_max_position_embeddings"], r.get("beta_fast", 32.0),
                                 r.get("beta_slow", 1.0), r.get("truncate", True),
                                 r.get("attention_factor"))
        if kind == "llama3":
            r = self.rope
            return rope_mod.llama3(self.head_dim, self.rope_theta, r["factor"], r["low_freq_factor"],
                                   r["high_freq_factor"], r["original_max_position_embeddings"])
        return rope_mod.default(self.head_dim, self.rope_theta)


# Config 1 of the benchmark description (CPU-runnable reference case).
TINY_LLAMA = ModelSpec(name="tiny-llama-c1", family="llama", num_layers=4, hidden=1024, n_q=16,
                       n_kv=4, head_dim=64, intermediate=2816, vocab=32000, rope_theta=10000.0,
                       eps=1e-6)
# Config 2: Llama-3-8B architecture.
LLAMA3_8B = ModelSpec(name="llama-3-8b", family="llama", num_layers=32, hidden=4096, n_q=32,
                      n_kv=8, head_dim=128, intermediate=14336, vocab=128256,
                      rope_theta=500000.0, eps=1e-5)
# Config 3: gpt-oss-20b architecture.
GPT_OSS_20B = ModelSpec(
    name="gpt-oss-20b", family="gpt_oss", num_layers=24, hidden=2880, n_q=64, n_kv=8, head_dim=64,
    intermediate=2880, vocab=201088, rope_theta=150000.0, eps=1e-5,
    rope={"rope_type": "yarn", "factor": 32.0, "original_max_position_embeddings": 4096,
          "beta_fast": 32.0, "beta_slow": 1.0, "truncate": False},
    attn_bias=True, sinks=True, sliding_window=128,
    layer_types=tuple("sliding_attention" if i % 2 == 0 else "full_attention" for i in range(24)),
    num_experts=32, top_k=4)

SPECS = {s.name: s for s in (TINY_LLAMA, LLAMA3_8B, GPT_OSS_20B)}


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[I,H] gate and up -> [2I,H] with 64-row blocks alternating gate/up."""
    I, H = gate.shape
    assert I % 64 == 0, f"intermediate size {I} must be a multiple of 64"
    return torch.stack([gate.view(I // 64, 64, H), up.view(I // 64, 64, H)], dim=1).reshape(2 * I, H)


def shard_dense_ffn(w_gate_up: torch.Tensor, w_down: torch.Tensor,
                    shard: tuple[int, int]) -> tuple[torch.Tensor, torch.Tensor]:
    """Tensor-parallel slice (index, count) of a dense FFN over the intermediate
    dimension: features [I*i/S, I*(i+1)/S) (a multiple of 64, so the 64-row
    gate/up interleave stays whole) -> (gate_up rows, down columns)."""
    i, S = shard
    I = w_down.shape[1]
    assert 0 <= i < S and I % (64 * S) == 0, f"intermediate {I} does not split into {S} shards of 64-multiples"
    lo, hi = I * i // S, I * (i + 1) // S
    return w_gate_up[2 * lo:2 * hi].contiguous(), w_down[:, lo:hi].contiguous()


@dataclass
class ModelWeights:
    spec: ModelSpec
    embed: torch.Tensor
    final_norm: torch.Tensor
    lm_head: torch.Tensor
    layers: list[dict[str, torch.Tensor]] = field(default_factory=list)
    inv_freq: torch.Tensor | None = None
    rope_scaling: float = 1.0
    # (index, count) when this rank holds one shard of every feed-forward
    # group: the intermediate slice of a dense FFN, or a range of experts
    ffn_shard: tuple[int, int] | None = None

    @property
    def device(self) -> torch.device:
        return self.embed.device

    GEMM_WEIGHTS = ("wqkv", "wo", "w_gate_up", "w_down")

    def finalize(self, pack: bool = True) -> "ModelWeights":
        """RoPE tables, and (pack=True) every GEMM weight converted to the
        packed 16 KB tile layout the weight-streaming GEMM reads; the
        row-major copies are released (the embedding table stays row-major
        for the gather; a tied lm_head gets its own packed copy)."""
        inv, sc = self.spec.rope_tables()
        self.inv_freq = inv.to(device=self.device, dtype=torch.float32).contiguous()
        self.rope_scaling = float(sc)
        if pack and self.device.type == "cuda":
            from .kernels import PackedWeight

            for L in self.layers:
                for k in self.GEMM_WEIGHTS:
                    if k in L and isinstance(L[k], torch.Tensor):
                        L[k] = PackedWeight(L[k])
            if isinstance(self.lm_head, torch.Tensor):
                self.lm_head = PackedWeight(self.lm_head)
        return self

    # -- constructors --------------------------------------------------------
    @classmethod
    def random(cls, spec: ModelSpec, seed: int = 0, device: str | torch.device = "cuda",
               std: float = 0.02, layers: list[int] | None = None,
               dtype: torch.dtype = torch.bfloat16,
               ffn_shard: tuple[int, int] | None = None) -> "ModelWeights":
        """N(0, std) weights from a seeded generator on `device` (norm weights 1,
        biases 0, as transformers initialises them). `layers` limits which
        layers get weights (the others stay empty dicts). `ffn_shard` keeps one
        tensor-/expert-parallel shard of the FFNs (the same draws as the whole
        model, then sliced)."""
        device = torch.device(device)
        g = torch.Generator(device=device).manual_seed(seed)

        def normal(*shape):
            t = torch.empty(shape, dtype=torch.float32, device=device)
            t.normal_(0.0, std, generator=g)
            return t.to(dtype)

        H, I = spec.hidden, spec.intermediate
        embed = normal(spec.vocab, H)
        lm_head = embed if spec.tie_embeddings else normal(spec.vocab, H)
        out = cls(spec=spec, embed=embed, final_norm=torch.ones(H, dtype=dtype, device=device),
                  lm_head=lm_head)
        want = set(range(spec.num_layers)) if layers is None else set(layers)
        for i in range(spec.num_layers):
            if i not in want:
                out.layers.append({})
                continue
            L: dict[str, torch.Tensor] = {
                "ln1": torch.ones(H, dtype=dtype, device=device),
                "ln2": torch.ones(H, dtype=dtype, device=device),
                "wqkv": normal(spec.qkv_width, H),
                "wo": normal(H, spec.n_q * spec.head_dim),
            }
            if spec.attn_bias:
                L["bqkv"] = torch.zeros(spec.qkv_width, dtype=dtype, device=device)
                L["bo"] = torch.zeros(H, dtype=dtype, device=device)
            if spec.sinks:
                L["sinks"] = normal(spec.n_q).float()
            if spec.moe:
                from . import moe

                L.update(moe.random_expert_weights(spec, normal, device, dtype, ffn_shard))
            else:
                L["w_gate_up"] = interleave_gate_up(normal(I, H), normal(I, H))
                L["w_down"] = normal(H, I)
                if ffn_shard is not None:
                    L["w_gate_up"], L["w_down"] = shard_dense_ffn(L["w_gate_up"], L["w_down"], ffn_shard)
            out.layers.append(L)
        out.ffn_shard = ffn_shard
        return out.finalize()

    @classmethod
    def from_hf(cls, hf_model: Any, device: str | torch.device,
                ffn_shard: tuple[int, int] | None = None) -> "ModelWeights":
        """Import an HF LlamaForCausalLM / GptOssForCausalLM (any dtype);
        `ffn_shard` as in random()."""
        cfg = hf_model.config
        device = torch.device(device)
        bf = lambda t: t.detach().to(device=device, dtype=torch.bfloat16).contiguous()  # noqa: E731
        family = "gpt_oss" if cfg.model_type == "gpt_oss" else "llama"
        hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        params = getattr(cfg, "rope_parameters", None) or {}
        kind = params.get("rope_type", "default")
        rope = None if kind == "default" else dict(params)
        spec = ModelSpec(
            name=getattr(cfg, "name_or_path", "") or cfg.model_type, family=family,
            num_layers=cfg.num_hidden_layers, hidden=cfg.hidden_size, n_q=cfg.num_attention_heads,
            n_kv=cfg.num_key_value_heads, head_dim=hd, intermediate=cfg.intermediate_size,
            vocab=cfg.vocab_size, rope_theta=float(params.get("rope_theta", getattr(cfg, "rope_theta", 10000.0))),
            eps=float(cfg.rms_norm_eps), rope=rope,
            attn_bias=bool(getattr(cfg, "attention_bias", False)),
            sinks=family == "gpt_oss",
            sliding_window=int(getattr(cfg, "sliding_window", 0) or 0) if family == "gpt_oss" else 0,
            layer_types=tuple(getattr(cfg, "layer_types", ()) or ()) if family == "gpt_oss" else (),
            num_experts=int(getattr(cfg, "num_local_experts", 0) or 0),
            top_k=int(getattr(cfg, "num_experts_per_tok", 0) or 0) if family == "gpt_oss" else 0,
            tie_embeddings=bool(getattr(cfg, "tie_word_embeddings", False)),
        )
        m = hf_model.model
        embed = bf(m.embed_tokens.weight)
        lm_head = embed if spec.tie_embeddings else bf(hf_model.lm_head.weight)
        out = cls(spec=spec, embed=embed, final_norm=bf(m.norm.weight), lm_head=lm_head)
        for layer in m.layers:
            a = layer.self_attn
            L = {
                "ln1": bf(layer.input_layernorm.weight),
                "ln2": bf(layer.post_attention_layernorm.weight),
                "wqkv": torch.cat([bf(a.q_proj.weight), bf(a.k_proj.weight), bf(a.v_proj.weight)]),
                "wo": bf(a.o_proj.weight),
            }
            if spec.attn_bias:
                L["bqkv"] = torch.cat([bf(a.q_proj.bias), bf(a.k_proj.bias), bf(a.v_proj.bias)])
                L["bo"] = bf(a.o_proj.bias)
            if spec.sinks:
                L["sinks"] = a.sinks.detach().to(device=device, dtype=torch.float32).contiguous()
            if spec.moe:
                from . import moe

                L.update(moe.expert_weights_from_hf(layer.mlp, device, ffn_shard))
            else:
                mlp = layer.mlp
                L["w_gate_up"] = interleave_gate_up(bf(mlp.gate_proj.weight), bf(mlp.up_proj.weight))
                L["w_down"] = bf(mlp.down_proj.weight)
                if ffn_shard is not None:
                    L["w_gate_up"], L["w_down"] = shard_dense_ffn(L["w_gate_up"], L["w_down"], ffn_shard)
            out.layers.append(L)
        out.ffn_shard = ffn_shard
        return out.finalize()


