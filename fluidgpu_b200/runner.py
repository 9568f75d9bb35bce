"""Batched decode runner with the interface of fluidgpu_torch.runner.CausalLMRunner
(fluidgpu_runtime/fluidgpu_torch/runner.py:26-165).

The task walk is the reference's: embed -> per layer (attention group, FFN
group) -> norm_lm_head, each group run through LayerExecutor.run_kernel_group
so the placement plan decides which rank executes it and where the hidden
state is handed off. The override points keep the reference's names and
keyword arguments (_run_attn, _run_mlp, _norm_head); their bodies call the
sm_100a kernels of libfgb200.so instead of HF modules:

  _run_attn  : fg_rmsnorm -> fg_gemm_bf16 (qkv, + bias) -> fg_rope_kv_append
               -> fg_paged_decode_attn (window, sinks) -> fg_gemm_bf16 (o_proj,
               residual epilogue)
  _run_mlp   : fg_rmsnorm -> fg_gemm_bf16 (gate|up, SwiGLU epilogue)
               -> fg_gemm_bf16 (down, residual epilogue)
  MoE FFN    : fg_rmsnorm -> router top-k -> expert grouped GEMMs (moe.py)
  _norm_head : fg_rmsnorm -> fg_gemm_bf16 (lm_head)

Fine-grained plans split the groups as the reference does (runner.py:196-254,
:362-414): layer_i_{qkv,sdpa,o_proj}, layer_i_{mlp_gate_up,mlp_down_proj},
layer_i_{moe_router,moe_experts,moe_combine}. The value on the main path is
the reference's (qkv and gate_up pass the normalised hidden on, sdpa the
attention output); what a later group needs from an earlier one on another
rank travels as aux tensors in a fixed order (runner.py:462-654):
  qkv -> sdpa        : projected qkv row [B, (n_q + 2 n_kv) hd], residual [B, H]
  sdpa -> o_proj     : residual
  gate_up -> down    : SwiGLU intermediate [B, I], residual
  router -> experts  : top-k weights [B, k] bf16, expert ids [B, k] int32, residual
  experts -> combine : residual
A feed-forward group sharded over several ranks (plan extension shard_ranks,
see executor.py) runs here on this rank's slice: a dense FFN on its
intermediate columns (fp32 partial; shard 0 adds the residual), the MoE
experts on its expert range (fp32 partial of the weighted sum; the router
sends top-k weights and ids to every shard and keeps the residual for the
combine group).
The reference ships q plus the whole K/V view from qkv to sdpa; here the KV
pages live on the sdpa rank (profile.kv_layer_ids) and RoPE + append run
there, so only the new token's projection crosses.

Generalisations over the reference: a batch of B requests decodes together
(hidden [B, 1, H], the reference asserts batch 1 at runner.py:67, :120), and
the KV cache is paged (kv_cache.PagedKVCache). prefill() feeds the prompt
position by position through the decode kernels (causal attention makes the
result identical to a full-sequence prefill).

Drop-in: the runner also runs under the reference's own objects. Its
executor may be fluidgpu_torch.executor.LayerExecutor (which forwards every
extra keyword to the kernel-group callable and has no shard or hand-off
extensions; then a batch larger than 1 only works where no hidden state
crosses ranks, its receive buffers being [1, 1, H]), its cfg
fluidgpu_torch.config.EngineConfig (no max_batch: one sequence), and the
override points take the reference's keywords: `layer` as the HF decoder
layer or its index, attention_mask / position_ids / past_key_value /
use_cache / cache_position / position_embeddings (accepted and unused: the
masks are implicit in the attention kernels, positions live in the paged
cache), layer_id for the fine-grained groups.
"""
from __future__ import annotations

from typing import Any

import torch

from . import _lib, kernels
from .config import EngineConfig
from .executor import LayerExecutor
from .kv_cache import PagedKVCache
from .model import ModelWeights
from .profile import has_fine_groups


class FluidRunner:
    def __init__(self, hf_model: Any, tokenizer: Any, executor: LayerExecutor, cfg: EngineConfig,
                 owned_layer_ids: list[int], *, num_blocks: int | None = None) -> None:
        self.weights = hf_model if isinstance(hf_model, ModelWeights) else \
            ModelWeights.from_hf(hf_model, cfg.torch_device)
        self.spec = self.weights.spec
        self.tokenizer = tokenizer
        self.executor = executor
        self.cfg = cfg
        self.device = cfg.torch_device
        self.hidden_size = self.spec.hidden
        self.layers = list(range(self.spec.num_layers))
        self.kv_cache = PagedKVCache(
            num_layers=self.spec.num_layers, owned_layer_ids=owned_layer_ids,
            max_seq_len=cfg.max_seq_len, num_kv_heads=self.spec.n_kv, head_dim=self.spec.head_dim,
            dtype=cfg.dtype, device=self.device, max_batch=getattr(cfg, "max_batch", 1), num_blocks=num_blocks,
            allocation=getattr(cfg, "kv_allocation", "vllm"))
        self._mode, self._n = "decode", 1
        self._moe_states: dict[int, dict[str, torch.Tensor]] = {}
        self._attn_states: dict[int, dict[str, torch.Tensor]] = {}
        self._mlp_states: dict[int, dict[str, torch.Tensor]] = {}
        # scratch slots of this runner (runners on other streams use their own)
        self.slot = f"runner{id(self):x}"
        # positions per sequence in one prefill pass (bounded by activation memory)
        self.prefill_chunk = 1024
        # MoE routing of the last step per layer (tests compare it with the oracle)
        self.record_routing = False
        self.last_routing: dict[int, torch.Tensor] = {}
        # with record_routing: every pass's (layer, positions per sequence,
        # indices [B * n, k], router input [B * n, H] or None where the ids
        # came from another rank) in order, when this is a list
        self.routing_log: list[tuple[int, int, torch.Tensor, torch.Tensor | None]] | None = None
        # with record_routing: the router's input of the last pass per layer
        # (the normalised hidden [B * n, H]), so a test can evaluate another
        # router on exactly the rows this one saw
        self.last_router_input: dict[int, torch.Tensor] = {}

    # -- sequence admission ---------------------------------------------------
    def start(self, batch: int, prompt_lens: list[int] | None = None,
              reserve_tokens: int | list[int] | None = None) -> None:
        """Open a batch: sequences start at prompt_lens (0 = empty) and
        reserve pages for reserve_tokens tokens each."""
        lens = prompt_lens if prompt_lens is not None else [0] * batch
        self.kv_cache.start_batch(lens, reserve_tokens if reserve_tokens is not None
                                  else self.cfg.max_seq_len)

    # -- reference entry points -----------------------------------------------
    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor, chunk: int | None = None) -> torch.Tensor | None:
        """Prompts [B, S] (equal lengths) -> logits of the last position [B, 1, V].

        The prompt runs in chunks of `chunk` positions (default prefill_chunk),
        each chunk one pass of every kernel group over its B*chunk tokens:
        token-wise RoPE + KV append, causal attention over the pages
        (fg_prefill_attn, earlier chunks included), GEMMs over all the tokens.
        Plans with fine-grained attention / FFN splits feed the prompt one
        position at a time through the decode path instead."""
        assert input_ids.ndim == 2, "input_ids must be [batch, seq]"
        B, S = input_ids.shape
        assert S <= self.cfg.max_seq_len, f"prompt length {S} exceeds max_seq_len {self.cfg.max_seq_len}"
        if self.kv_cache.batch != B or self.kv_cache.get_seq_length() != 0:
            self.start(B)
        ids = input_ids.to(self.device)
        step = 1 if has_fine_groups(self.executor.profile) else max(1, chunk or self.prefill_chunk)
        cap = self.executor.message_capacity() if hasattr(self.executor, "message_capacity") else None
        if cap is not None and self.executor.profile.rank_count > 1:
            # every hand-off of a chunk must fit one mailbox slot
            step = max(1, min(step, cap // self.max_message_bytes(B)))
        out = None
        for t in range(0, S, step):
            n = min(step, S - t)
            out = self._step(ids[:, t : t + n], want_logits=(t + n == S))
        return out

    @torch.inference_mode()
    def decode_step(self, token_id: torch.Tensor) -> torch.Tensor | None:
        """Tokens [B, 1] (or [B]) -> logits [B, 1, V] on the norm_lm_head rank, None elsewhere."""
        tok = token_id.reshape(-1, 1)
        if self.kv_cache.batch == 0:
            self.start(tok.shape[0])
        assert tok.shape[0] == self.kv_cache.batch, (
            f"decode batch {tok.shape[0]} != started batch {self.kv_cache.batch}"
        )
        return self._step(tok.to(self.device), want_logits=True)

    # -- step -------------------------------------------------------------------
    def _step(self, tokens: torch.Tensor, *, want_logits: bool) -> torch.Tensor | None:
        """tokens [B, n]: one decode step (n == 1) or one prefill chunk."""
        B, n = tokens.shape
        mode = "decode" if n == 1 else "prefill"
        self._mode, self._n = mode, n  # the kernel groups of this pass run in this mode
        ex = self.executor
        self.kv_cache.prepare_step(n)  # blocks for these tokens (no-op inside a graph capture)
        hidden = ex.run_stage("embed", self._embed, tokens, mode=mode, seq_len=n, batch=B)
        for i in self.layers:
            hidden = self._run_attention_tasks(i, hidden, B)
            hidden = self._run_feed_forward_tasks(i, hidden, B)
        self.kv_cache.advance(n)
        head = self._norm_head if want_logits else self._skip_head
        return ex.run_stage("norm_lm_head", head, hidden, mode=mode, seq_len=n, batch=B)

    def _has_task(self, name: str) -> bool:
        return name in self.executor.task_index_by_name

    def _run_attention_tasks(self, i: int, hidden: torch.Tensor | None, B: int) -> torch.Tensor | None:
        if not self._has_task(f"layer_{i}_qkv"):
            out = self.executor.run_kernel_group(f"layer_{i}_attn", self._run_attn, hidden, mode=self._mode,
                                                 seq_len=self._n, batch=B, layer=i)
            return out if out is not None else hidden
        s = self.spec
        for suffix, fn in (("qkv", self._run_attn_qkv), ("sdpa", self._run_attn_sdpa),
                           ("o_proj", self._run_attn_o_proj)):
            kw = {"recv_width": s.n_q * s.head_dim} if suffix == "o_proj" else {}
            out = self.executor.run_kernel_group(f"layer_{i}_{suffix}", fn, hidden, mode=self._mode,
                                                 seq_len=self._n, batch=B, layer=i, **kw)
            if out is not None:
                hidden = out
                if suffix == "qkv":
                    self._after_attn_qkv(i)
                elif suffix == "sdpa":
                    self._after_attn_sdpa(i)
        return hidden

    def _run_feed_forward_tasks(self, i: int, hidden: torch.Tensor | None, B: int) -> torch.Tensor | None:
        if self._has_task(f"layer_{i}_mlp_gate_up"):
            for suffix, fn in (("mlp_gate_up", self._run_mlp_gate_up), ("mlp_down_proj", self._run_mlp_down_proj)):
                out = self.executor.run_kernel_group(f"layer_{i}_{suffix}", fn, hidden, mode=self._mode,
                                                     seq_len=self._n, batch=B, layer=i)
                if out is not None:
                    hidden = out
                    if suffix == "mlp_gate_up":
                        self._after_mlp_gate_up(i)
            return hidden
        if self._has_task(f"layer_{i}_mlp"):
            out = self.executor.run_kernel_group(f"layer_{i}_mlp", self._run_mlp, hidden,
                                                 mode=self._mode, seq_len=self._n, batch=B, layer=i)
            return out if out is not None else hidden
        for suffix, fn in (("moe_router", self._run_moe_router), ("moe_experts", self._run_moe_experts),
                           ("moe_combine", self._run_moe_combine)):
            out = self.executor.run_kernel_group(f"layer_{i}_{suffix}", fn, hidden, mode=self._mode,
                                                 seq_len=self._n, batch=B, layer=i)
            if out is not None:
                hidden = out
                if suffix == "moe_router":
                    self._after_moe_router(i)
                elif suffix == "moe_experts":
                    self._after_moe_experts(i)
        return hidden

    # -- kernel groups (override points of the reference runner) ---------------
    # `out`: where the group's result must land (the next rank's slot of a
    # zero-copy hand-off); the group's last kernel writes there directly
    def _embed(self, tokens: torch.Tensor, out: torch.Tensor | None = None, **_: Any) -> torch.Tensor:
        B, n = tokens.shape
        o = kernels.embed(tokens.reshape(-1).contiguous(), self.weights.embed,
                          out=None if out is None else out.view(B * n, -1))
        return o.view(B, n, -1) if out is None else out

    def _run_attn(self, hidden: torch.Tensor, *, layer: Any, out: torch.Tensor | None = None,
                  attention_mask: Any = None, position_ids: Any = None, past_key_value: Any = None,
                  use_cache: bool = True, cache_position: Any = None, position_embeddings: Any = None,
                  **_: Any) -> torch.Tensor:
        """The attention group (runner.py:170-194, same keywords)."""
        layer = _layer_index(layer)
        s = self.spec
        W = self.weights.layers[layer]
        kv = self.kv_cache
        B, n = hidden.shape[0], hidden.shape[1]
        T = B * n
        h = hidden.reshape(T, s.hidden)
        x = kernels.rmsnorm(h, W["ln1"], s.eps, s.norm_mode)
        qkv = kernels.gemm(x, W["wqkv"], bias=W.get("bqkv"), slot=self.slot + ".gemm")
        kp, vp = kv.layer_pages(layer)
        bt = kv.block_table[:B]
        if n == 1:
            q = kernels.rope_kv_append(qkv, kv.positions[:B], self.weights.inv_freq,
                                       self.weights.rope_scaling, bt, kp, vp, s.n_q, s.n_kv, s.head_dim)
            a = kernels.paged_decode_attn(q, kp, vp, bt, kv.seq_lens[:B], kv.plan_len(),
                                          window=s.window(layer), sinks=W.get("sinks"),
                                          slot=self.slot + ".attn")
        else:
            seq_ids, pos = self._chunk_tokens(B, n)
            q = kernels.rope_kv_append_tokens(qkv, seq_ids, pos, self.weights.inv_freq,
                                              self.weights.rope_scaling, kv.block_table, kp, vp,
                                              s.n_q, s.n_kv, s.head_dim)
            a = kernels.prefill_attn(q, kp, vp, kv.block_table, kv.positions[:B], n,
                                     window=s.window(layer), sinks=W.get("sinks")).view(T, -1)
        o = kernels.gemm(a, W["wo"], epilogue=_lib.FG_EPI_RESIDUAL, residual=h, bias=W.get("bo"),
                         out=None if out is None else out.view(T, s.hidden), slot=self.slot + ".gemm")
        return o.view(B, n, s.hidden) if out is None else out

    def _chunk_tokens(self, B: int, n: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(sequence id, position) of every token of a prefill chunk of n
        positions per sequence, from the device position counters."""
        seq = torch.arange(B, device=self.device, dtype=torch.int32).repeat_interleave(n)
        pos = (self.kv_cache.positions[:B, None]
               + torch.arange(n, device=self.device, dtype=torch.int32)[None, :]).reshape(-1)
        return seq, pos.to(torch.int32).contiguous()

    # fine attention groups (runner.py:256-347)
    def _run_attn_qkv(self, hidden: torch.Tensor, *, layer: Any, layer_id: int | None = None,
                      **_: Any) -> torch.Tensor:
        layer = _layer_index(layer, layer_id)
        s = self.spec
        W = self.weights.layers[layer]
        B = hidden.shape[0]
        h = hidden.reshape(B, s.hidden)
        x = kernels.rmsnorm(h, W["ln1"], s.eps, s.norm_mode)
        qkv = kernels.gemm(x, W["wqkv"], bias=W.get("bqkv"), slot=self.slot + ".gemm")
        self._attn_states[layer] = {"residual": h, "qkv": qkv}
        return x.view(B, 1, s.hidden)

    def _run_attn_sdpa(self, hidden: torch.Tensor, *, layer: Any, layer_id: int | None = None,
                       **_: Any) -> torch.Tensor:
        layer = _layer_index(layer, layer_id)
        s = self.spec
        W = self.weights.layers[layer]
        kv = self.kv_cache
        B = hidden.shape[0]
        st = self._ensure_attn_qkv_state(layer, B)
        kp, vp = kv.layer_pages(layer)
        bt = kv.block_table[:B]
        q = kernels.rope_kv_append(st["qkv"], kv.positions[:B], self.weights.inv_freq,
                                   self.weights.rope_scaling, bt, kp, vp, s.n_q, s.n_kv, s.head_dim)
        a = kernels.paged_decode_attn(q, kp, vp, bt, kv.seq_lens[:B], kv.plan_len(),
                                      window=s.window(layer), sinks=W.get("sinks"),
                                      slot=self.slot + ".attn")
        return a.view(B, 1, s.n_q * s.head_dim)

    def _run_attn_o_proj(self, hidden: torch.Tensor, *, layer: Any, layer_id: int | None = None,
                         **_: Any) -> torch.Tensor:
        layer = _layer_index(layer, layer_id)
        s = self.spec
        W = self.weights.layers[layer]
        B = hidden.shape[0]
        self._ensure_residual(self._attn_states, layer, B, src=self._rank_of(layer, "sdpa"))
        st = self._attn_states.pop(layer)
        a = hidden.reshape(B, s.n_q * s.head_dim)
        out = kernels.gemm(a, W["wo"], epilogue=_lib.FG_EPI_RESIDUAL, residual=st["residual"],
                           bias=W.get("bo"), slot=self.slot + ".gemm")
        return out.view(B, 1, s.hidden)

    def _after_attn_qkv(self, layer: int) -> None:
        dst = self._rank_of(layer, "sdpa")
        if dst == self._rank_of(layer, "qkv"):
            return
        st = self._attn_states.pop(layer)
        self._send_aux(st["qkv"], dst)
        self._send_aux(st["residual"], dst)

    def _after_attn_sdpa(self, layer: int) -> None:
        st = self._attn_states.get(layer)
        if st is None:
            return
        st.pop("qkv", None)
        dst = self._rank_of(layer, "o_proj")
        if dst == self._rank_of(layer, "sdpa"):
            return
        self._send_aux(st["residual"], dst)
        self._attn_states.pop(layer, None)

    def _ensure_attn_qkv_state(self, layer: int, B: int) -> dict[str, torch.Tensor]:
        st = self._attn_states.setdefault(layer, {})
        if "qkv" not in st:
            src = self._rank_of(layer, "qkv")
            st["qkv"] = self._recv_aux((B, self.spec.qkv_width), torch.bfloat16, src)
            st["residual"] = self._recv_aux((B, self.spec.hidden), torch.bfloat16, src)
        return st

    def _run_mlp(self, hidden: torch.Tensor, *, layer: Any, shard: tuple[int, int] | None = None,
                 out: torch.Tensor | None = None, **_: Any) -> torch.Tensor:
        """The FFN group (runner.py:349-352, same keywords)."""
        layer = _layer_index(layer)
        s = self.spec
        W = self.weights.layers[layer]
        B0, n = hidden.shape[0], hidden.shape[1]
        B = B0 * n  # token rows
        h = hidden.reshape(B, s.hidden)
        x = kernels.rmsnorm(h, W["ln2"], s.eps, s.norm_mode)
        act = kernels.gemm(x, W["w_gate_up"], epilogue=_lib.FG_EPI_SWIGLU, slot=self.slot + ".gemm")
        if shard is not None:
            # tensor-parallel slice: fp32 partial of the down projection, the
            # first shard carrying the residual; the consumer adds them up
            assert self.weights.ffn_shard == shard, (
                f"layer {layer}: plan shard {shard} != weights shard {self.weights.ffn_shard}")
            out = kernels.gemm(act, W["w_down"], epilogue=_lib.FG_EPI_F32,
                               residual=h if shard[0] == 0 else None, slot=self.slot + ".gemm")
            return out.view(B0, n, s.hidden)
        o = kernels.gemm(act, W["w_down"], epilogue=_lib.FG_EPI_RESIDUAL, residual=h,
                         out=None if out is None else out.view(B, s.hidden), slot=self.slot + ".gemm")
        return o.view(B0, n, s.hidden) if out is None else out

    # fine dense FFN groups (runner.py:416-430)
    def _run_mlp_gate_up(self, hidden: torch.Tensor, *, layer: Any, layer_id: int | None = None,
                         **_: Any) -> torch.Tensor:
        layer = _layer_index(layer, layer_id)
        s = self.spec
        W = self.weights.layers[layer]
        B = hidden.shape[0]
        h = hidden.reshape(B, s.hidden)
        x = kernels.rmsnorm(h, W["ln2"], s.eps, s.norm_mode)
        act = kernels.gemm(x, W["w_gate_up"], epilogue=_lib.FG_EPI_SWIGLU, slot=self.slot + ".gemm")
        self._mlp_states[layer] = {"residual": h, "intermediate": act}
        return x.view(B, 1, s.hidden)

    def _run_mlp_down_proj(self, hidden: torch.Tensor, *, layer: Any, layer_id: int | None = None,
                           **_: Any) -> torch.Tensor:
        layer = _layer_index(layer, layer_id)
        s = self.spec
        W = self.weights.layers[layer]
        B = hidden.shape[0]
        st = self._mlp_states.setdefault(layer, {})
        if "intermediate" not in st:
            src = self._rank_of(layer, "mlp_gate_up")
            st["intermediate"] = self._recv_aux((B, s.intermediate), torch.bfloat16, src)
            st["residual"] = self._recv_aux((B, s.hidden), torch.bfloat16, src)
        st = self._mlp_states.pop(layer)
        out = kernels.gemm(st["intermediate"], W["w_down"], epilogue=_lib.FG_EPI_RESIDUAL,
                           residual=st["residual"], slot=self.slot + ".gemm")
        return out.view(B, 1, s.hidden)

    def _after_mlp_gate_up(self, layer: int) -> None:
        dst = self._rank_of(layer, "mlp_down_proj")
        if dst == self._rank_of(layer, "mlp_gate_up"):
            return
        st = self._mlp_states.pop(layer)
        self._send_aux(st["intermediate"], dst)
        self._send_aux(st["residual"], dst)

    def _run_moe_router(self, hidden: torch.Tensor, *, layer: Any, layer_id: int | None = None,
                        **_: Any) -> torch.Tensor:
        from . import moe

        layer = _layer_index(layer, layer_id)
        s = self.spec
        W = self.weights.layers[layer]
        B0, n = hidden.shape[0], hidden.shape[1]
        B = B0 * n  # token rows
        h = hidden.reshape(B, s.hidden)
        x = kernels.rmsnorm(h, W["ln2"], s.eps, s.norm_mode)
        weights, idx = moe.router_topk(x, W["router_w"], W.get("router_b"), s.top_k)
        self._moe_states[layer] = {"residual": h, "weights": weights, "indices": idx}
        if self.record_routing:
            self._record_routing(layer, idx, x)
        return x.view(B0, n, s.hidden)

    def _run_moe_experts(self, hidden: torch.Tensor, *, layer: Any, shard: tuple[int, int] | None = None,
                         layer_id: int | None = None, **_: Any) -> torch.Tensor:
        from . import moe

        layer = _layer_index(layer, layer_id)
        s = self.spec
        B0, n = hidden.shape[0], hidden.shape[1]
        B = B0 * n  # token rows
        if shard is not None:
            # expert-parallel shard: fp32 partial over this rank's experts
            assert self.weights.ffn_shard == shard, (
                f"layer {layer}: plan shard {shard} != weights shard {self.weights.ffn_shard}")
            src = self._rank_of(layer, "moe_router")
            wts = self._recv_aux((B, s.top_k), torch.bfloat16, src)
            idx = self._recv_aux((B, s.top_k), torch.int32, src)
            if self.record_routing:
                self._record_routing(layer, idx)
            y = moe.experts_forward(hidden.reshape(B, s.hidden), idx, wts, self.weights.layers[layer], s)
            return y.view(B0, n, s.hidden)
        st = self._moe_states.setdefault(layer, {})
        if "indices" not in st:
            src = self._rank_of(layer, "moe_router")
            st["weights"] = self._recv_aux((B, s.top_k), torch.bfloat16, src)
            st["indices"] = self._recv_aux((B, s.top_k), torch.int32, src)
            st["residual"] = self._recv_aux((B, s.hidden), torch.bfloat16, src)
            if self.record_routing:
                self._record_routing(layer, st["indices"])
        # the combine group's residual add is fused when it runs here too (not
        # under zero-copy hand-offs, where the combine writes the peer's slot)
        fuse = (self._rank_of(layer, "moe_combine") == self.executor.my_rank
                and not getattr(self.executor, "_direct", False))
        y = moe.experts_forward(hidden.reshape(B, s.hidden), st["indices"], st["weights"],
                                self.weights.layers[layer], s,
                                residual=st["residual"] if fuse else None)
        st["fused"] = fuse
        return y.view(B0, n, s.hidden)

    def _record_routing(self, layer: int, idx: torch.Tensor, x: torch.Tensor | None = None) -> None:
        self.last_routing[layer] = idx
        if x is not None:
            self.last_router_input[layer] = x.clone()
        if self.routing_log is not None:
            self.routing_log.append((layer, self._n, idx.clone(), None if x is None else x.clone()))

    def _run_moe_combine(self, hidden: torch.Tensor, *, layer: Any, out: torch.Tensor | None = None,
                         layer_id: int | None = None, **_: Any) -> torch.Tensor:
        from . import moe

        layer = _layer_index(layer, layer_id)
        B0, n = hidden.shape[0], hidden.shape[1]
        B = B0 * n  # token rows
        self._ensure_residual(self._moe_states, layer, B, src=self._rank_of(layer, "moe_experts"))
        st = self._moe_states.pop(layer)
        if st.get("fused"):
            assert out is None, "a fused combine has no output of its own to place"
            return hidden
        o = moe.residual_add(st["residual"], hidden.reshape(B, -1),
                             out=None if out is None else out.view(B, -1))
        return o.view(B0, n, -1) if out is None else out

    def _after_moe_router(self, layer: int) -> None:
        shards = self._shards_of(layer, "moe_experts")
        if shards is not None:
            # every shard needs the routing; the residual stays here for the
            # combine group (same rank, checked by the plan validation)
            st = self._moe_states[layer]
            for r in shards:
                self._send_aux(st["weights"], r)
                self._send_aux(st["indices"], r)
            return
        dst = self._rank_of(layer, "moe_experts")
        if dst == self._rank_of(layer, "moe_router"):
            return
        st = self._moe_states.pop(layer)
        self._send_aux(st["weights"], dst)
        self._send_aux(st["indices"], dst)
        self._send_aux(st["residual"], dst)

    def _after_moe_experts(self, layer: int) -> None:
        if self._shards_of(layer, "moe_experts") is not None:
            return  # partials go to the combine rank through the executor
        st = self._moe_states.get(layer)
        if st is None:
            return
        st.pop("weights", None)
        st.pop("indices", None)
        dst = self._rank_of(layer, "moe_combine")
        if dst == self._rank_of(layer, "moe_experts"):
            return
        self._send_aux(st["residual"], dst)
        self._moe_states.pop(layer, None)

    # -- aux routing (runner.py:462-670) ----------------------------------------
    def _rank_of(self, layer: int, suffix: str) -> int:
        ex = self.executor
        return ex.tasks[ex.task_index_by_name[f"layer_{layer}_{suffix}"]].rank_for("decode")

    def _shards_of(self, layer: int, suffix: str) -> tuple[int, ...] | None:
        ex = self.executor
        return getattr(ex.tasks[ex.task_index_by_name[f"layer_{layer}_{suffix}"]], "shard_ranks", None)

    def _send_aux(self, t: torch.Tensor, dst: int) -> None:
        self.executor.send_aux_tensor(t if t.is_contiguous() else t.contiguous(), dst=dst)

    def _recv_aux(self, shape: tuple[int, ...], dtype: torch.dtype, src: int) -> torch.Tensor:
        out = torch.empty(shape, dtype=dtype, device=self.device)
        self.executor.recv_aux_tensor(out, src=src)
        return out

    def _ensure_residual(self, states: dict, layer: int, B: int, *, src: int) -> None:
        st = states.setdefault(layer, {})
        if "residual" not in st:
            st["residual"] = self._recv_aux((B, self.spec.hidden), torch.bfloat16, src)

    def _norm_head(self, hidden: torch.Tensor, **_: Any) -> torch.Tensor:
        s = self.spec
        B = hidden.shape[0]
        if hidden.dim() == 3 and hidden.shape[1] > 1:  # a prefill chunk: the last position only
            hidden = hidden[:, -1].contiguous()
        x = kernels.rmsnorm(hidden.reshape(B, s.hidden), self.weights.final_norm, s.eps, s.norm_mode)
        return kernels.gemm(x, self.weights.lm_head, slot=self.slot + ".gemm").view(B, 1, s.vocab)

    def _skip_head(self, hidden: torch.Tensor, **_: Any) -> torch.Tensor:
        return hidden

    def max_message_bytes(self, batch: int) -> int:
        """Largest tensor this plan sends between two ranks in a decode step of
        `batch` sequences (the P2PComm slot must hold it); a prefill chunk of
        n positions sends n times as much."""
        s = self.spec
        names = self.executor.task_index_by_name
        sizes = [batch * s.hidden * 2]
        if any(n.endswith("_qkv") for n in names):
            sizes += [batch * s.qkv_width * 2, batch * s.n_q * s.head_dim * 2]
        if any(n.endswith("_mlp_gate_up") for n in names):
            sizes.append(batch * s.intermediate * 2)
        if any(getattr(t, "shard_ranks", None) is not None for t in self.executor.tasks):
            sizes.append(batch * s.hidden * 4)  # fp32 partials
        return max(sizes)

    def reserve_workspaces(self, batch: int, plan_len: int) -> None:
        """Allocate this runner's scratch at the size a step of `batch`
        sequences planned for `plan_len` tokens needs (before graph capture)."""
        s = self.spec
        lib = _lib.lib()
        windows = {s.window(i) for i in self.layers}
        attn = max(lib.fg_attn_workspace_bytes(batch, s.n_q, s.n_kv, s.head_dim, plan_len, w)
                   for w in windows)
        kernels.Workspace.get(attn, self.device, self.slot + ".attn")
        shapes = [(s.qkv_width, s.hidden), (s.hidden, s.n_q * s.head_dim), (s.vocab, s.hidden)]
        if not s.moe:
            shapes += [(2 * s.intermediate, s.hidden), (s.hidden, s.intermediate)]
        gemm = max(lib.fg_gemm_workspace_bytes(batch, n, k, 0) for n, k in shapes)
        kernels.Workspace.get(gemm, self.device, self.slot + ".gemm")


def _layer_index(layer: Any, layer_id: int | None = None) -> int:
    """Layer index from the override point's arguments: an int (this
    runner's walk), layer_id (the reference's fine-grained groups), or the
    HF decoder layer the reference's walk passes (its self_attn.layer_idx)."""
    if isinstance(layer, int):
        return layer
    if layer_id is not None:
        return int(layer_id)
    idx = getattr(getattr(layer, "self_attn", None), "layer_idx", None)
    assert idx is not None, f"cannot tell the layer index of {type(layer).__name__}"
    return int(idx)
