"""Greedy decode loop over FluidRunner, the role of fluidgpu_torch.engine.LLMEngine's
decode loops (fluidgpu_runtime/fluidgpu_torch/engine.py:275-357).

Two entry points per step:
  step(tokens_host) -> next tokens on the host. The public call: copies the
      step's tokens host->device (pinned), runs the decode step and the
      greedy argmax (fg_argmax, on the device like the reference's sync-free
      loop, engine.py:328-348) and copies the next tokens back.
  step_device(tokens) -> next tokens on the device, no host round trip.
"""
from __future__ import annotations

from typing import Any

import torch

from . import kernels
from .comm import LocalComm
from .config import EngineConfig
from .executor import LayerExecutor
from .model import ModelWeights
from .profile import RuntimeProfile, colocated_profile, owned_layer_ids, profile_from_dict
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
                                  owned_layer_ids(profile, self.rank), num_blocks=num_blocks)
        self.cfg = cfg
        self.device = cfg.torch_device
        self._tok_dev: torch.Tensor | None = None
        self._tok_host: torch.Tensor | None = None

    @property
    def kv_cache(self):
        return self.runner.kv_cache

    def start(self, batch: int, prompt_lens: list[int] | None = None,
              reserve_tokens: int | list[int] | None = None) -> None:
        self.runner.start(batch, prompt_lens, reserve_tokens)
        self._tok_dev = torch.zeros(batch, dtype=torch.int64, device=self.device)
        self._tok_host = torch.zeros(batch, dtype=torch.int64).pin_memory()

    @torch.inference_mode()
    def step_device(self, tokens: torch.Tensor) -> torch.Tensor | None:
        logits = self.runner.decode_step(tokens)
        if logits is None:
            return None
        return kernels.argmax(logits.reshape(logits.shape[0], -1))

    @torch.inference_mode()
    def step(self, tokens_host: torch.Tensor) -> torch.Tensor | None:
        """One greedy step from host tokens [B] to host tokens [B]."""
        assert self._tok_dev is not None, "call start() first"
        self._tok_dev.copy_(tokens_host, non_blocking=True)
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
