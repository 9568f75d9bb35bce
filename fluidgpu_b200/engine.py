"""Greedy decode loop over FluidRunner, the role of fluidgpu_torch.engine.LLMEngine's
decode loops (fluidgpu_runtime/fluidgpu_torch/engine.py:275-357).

Two entry points per step:
  step(tokens_host) -> next tokens on the host. The public call: copies the
      step's tokens host->device (pinned), runs the decode step and the
      greedy argmax (fg_argmax, on the device like the reference's sync-free
      loop, engine.py:328-348) and copies the next tokens back.
  step_device(tokens) -> next tokens on the device, no host round trip.

With EngineConfig.cuda_graph_decode the whole step (embed .. argmax, KV
append and position advance included) is captured once per attention length
bucket (powers of two from 256 up to max_seq_len) and replayed: the device
counters advance inside the graph, the host mirror advances after each
replay, and the next-token buffer feeds the following replay directly. This
is the B200 form of the reference's graphed decode segments
(graph_decode.py:57-153), without the per-segment host send/recv.
"""
from __future__ import annotations

from typing import Any

import torch

from . import kernels
from .comm import LocalComm
from .config import EngineConfig
from .executor import LayerExecutor
from .model import ModelWeights
from .profile import RuntimeProfile, colocated_profile, kv_layer_ids, profile_from_dict
from .runner import FluidRunner


class DecodeEngine:
    def __init__(self, weights: ModelWeights, cfg: EngineConfig, profile: RuntimeProfile | None = None,
                 comm: Any = None, num_blocks: int | None = None) -> None:
        s = weights.spec
        if profile is None:
            profile = profile_from_dict(colocated_profile(s.name, s.num_layers, s.hidden, s.n_kv,
                                                          s.head_dim, cfg.max_seq_len, moe=s.moe))
        self.comm = comm if comm is not None else LocalComm()
        self.rank = self.comm.get_rank()
        self.profile = profile
        self.executor = LayerExecutor(profile, cfg, self.comm)
        self.runner = FluidRunner(weights, None, self.executor, cfg,
                                  kv_layer_ids(profile, self.rank), num_blocks=num_blocks)
        self.cfg = cfg
        self.device = cfg.torch_device
        self._tok_dev: torch.Tensor | None = None
        self._tok_host: torch.Tensor | None = None
        self._next_dev: torch.Tensor | None = None
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.use_graph = bool(cfg.cuda_graph_decode)

    @property
    def kv_cache(self):
        return self.runner.kv_cache

    def start(self, batch: int, prompt_lens: list[int] | None = None,
              reserve_tokens: int | list[int] | None = None) -> None:
        self.runner.start(batch, prompt_lens, reserve_tokens)
        self._tok_dev = torch.zeros(batch, dtype=torch.int64, device=self.device)
        self._next_dev = torch.zeros(batch, dtype=torch.int64, device=self.device)
        self._tok_host = torch.zeros(batch, dtype=torch.int64).pin_memory()
        self._graphs.clear()

    @torch.inference_mode()
    def step_device(self, tokens: torch.Tensor) -> torch.Tensor | None:
        logits = self.runner.decode_step(tokens)
        if logits is None:
            return None
        return kernels.argmax(logits.reshape(logits.shape[0], -1))

    # -- CUDA graph decode ------------------------------------------------------
    def bucket(self, n: int) -> int:
        return self.kv_cache.bucket(n)

    def capture(self, bucket: int) -> torch.cuda.CUDAGraph:
        """Capture one decode step planned for `bucket` tokens. The graph reads
        its tokens from, and writes the next tokens back to, a static buffer."""
        if bucket in self._graphs:
            return self._graphs[bucket]
        kv = self.kv_cache
        B = kv.batch
        self.runner.reserve_workspaces(B, bucket)
        snap = kv.snapshot_host()
        kv.plan_len_override = bucket
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        try:
            with torch.cuda.stream(s), torch.inference_mode():
                with torch.cuda.graph(g, stream=s):
                    logits = self.runner.decode_step(self._tok_dev)
                    if logits is not None:  # the norm_lm_head rank closes the loop
                        kernels.argmax(logits.reshape(B, -1), out=self._next_dev)
                        self._tok_dev.copy_(self._next_dev)
        finally:
            kv.plan_len_override = None
            kv.restore_host(snap)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self._graphs[bucket] = g
        return g

    def replay(self) -> torch.Tensor:
        """One graphed decode step from the static token buffer; returns the
        static next-token buffer (also the next replay's input)."""
        self.kv_cache.prepare_step(1)  # block-table entries the step needs (before any capture)
        g = self.capture(self.bucket(self.kv_cache.max_attended()))
        g.replay()
        self.kv_cache.host_advance(1)
        return self._next_dev

    @torch.inference_mode()
    def step_static(self) -> torch.Tensor | None:
        """One greedy step from the static token buffer into the static
        next-token buffer, which also feeds the following step: a graph
        replay when CUDA graphs are on, eager launches otherwise. Returns the
        next-token buffer on the norm_lm_head rank, None elsewhere."""
        assert self._tok_dev is not None, "call start() first"
        if self.use_graph:
            nxt = self.replay()
            return nxt if self.runner.executor.task_rank("norm_lm_head", "decode") == self.rank else None
        logits = self.runner.decode_step(self._tok_dev)
        if logits is None:
            return None
        kernels.argmax(logits.reshape(logits.shape[0], -1), out=self._next_dev)
        self._tok_dev.copy_(self._next_dev)
        return self._next_dev

    def set_tokens(self, tokens: torch.Tensor) -> None:
        """Load the static token buffer (the next step's input) from tokens [B]."""
        assert self._tok_dev is not None, "call start() first"
        self._tok_dev.copy_(tokens.reshape(-1), non_blocking=True)

    @torch.inference_mode()
    def step(self, tokens_host: torch.Tensor) -> torch.Tensor | None:
        """One greedy step from host tokens [B] to host tokens [B]."""
        assert self._tok_dev is not None, "call start() first"
        self._tok_dev.copy_(tokens_host, non_blocking=True)
        if self.use_graph:
            nxt = self.replay() if self.rank == 0 else (self.replay(), None)[1]
        else:
            nxt = self.step_device(self._tok_dev)
        if nxt is None:
            return None
        self._tok_host.copy_(nxt, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self._tok_host.clone()

    @torch.inference_mode()
    def generate(self, prompts: torch.Tensor, max_new_tokens: int) -> tuple[torch.Tensor, list[torch.Tensor]]:
        """Greedy generation for prompts [B, S]; returns tokens [B, n] and the
        logits [B, V] that chose each token (rank 0)."""
        B, S = prompts.shape
        self.start(B, reserve_tokens=S + max_new_tokens + 1)
        logits = self.runner.prefill(prompts.to(self.device))
        toks, all_logits = [], []
        for _ in range(max_new_tokens):
            lg = logits.reshape(B, -1)
            all_logits.append(lg.float().cpu())
            nxt = kernels.argmax(lg)
            toks.append(nxt)
            logits = self.runner.decode_step(nxt)
        return torch.stack(toks, dim=1).cpu(), all_logits
