"""Micro-batched ping-pong decode across attention and FFN ranks.

The B200 form of the reference's pipelined schedules: vLLM dual-batch
overlap with the expert GPU (`_overlapped_remote`, vllm_integration.py:
1141-1237, per-micro-batch streams :838-867, staggered priorities :824-835)
and the native engine's concurrent workers with private comm groups and
priority streams (engine.py:168-216, async_engine.py:194-214).

M micro-batches each own a FluidRunner (their own paged-KV slice on the
attention rank), a P2PComm channel set (their own mailboxes, so sequence
numbers never mix) and a CUDA stream; the weights are shared. Each rank
replays one captured decode-step graph per micro-batch on that
micro-batch's stream (or, with EngineConfig.cuda_graph_decode off, launches
the step's kernels eagerly on it). Within a rank the streams only meet at the SMs: while
micro-batch A waits in its receive kernel for the FFN rank, micro-batch B's
attention runs, and the FFN rank works on A while the attention rank works
on B. Earlier micro-batches get higher stream priority, as in the reference.
"""
from __future__ import annotations

from typing import Any, Callable

import torch

from .config import EngineConfig
from .engine import DecodeEngine
from .model import ModelWeights
from .profile import RuntimeProfile


class PingPongEngine:
    def __init__(self, weights: ModelWeights, cfg: EngineConfig, profile: RuntimeProfile,
                 make_comm: Callable[[int], Any], micro_batches: int = 2) -> None:
        assert micro_batches >= 1
        self.device = cfg.torch_device
        # lower number = higher priority; torch clamps to the device's range
        self.streams = [torch.cuda.Stream(self.device, priority=-(micro_batches - 1 - m))
                        for m in range(micro_batches)]
        self.engines = [DecodeEngine(weights, cfg, profile=profile, comm=make_comm(m))
                        for m in range(micro_batches)]
        self.rank = self.engines[0].rank

    def start(self, batch: int, prompt_lens: list[int] | None = None,
              reserve_tokens: int | list[int] | None = None) -> None:
        for eng in self.engines:
            eng.start(batch, prompt_lens, reserve_tokens)

    def capture(self) -> None:
        """Capture every micro-batch's graph for the current length bucket now
        (ranks capture before any of them replays, so no receive waits on a
        peer that is still capturing)."""
        for eng in self.engines:
            eng.kv_cache.prepare_step(1)
            eng.capture(eng.bucket(eng.kv_cache.max_attended()))

    @property
    def kv_caches(self):
        return [e.kv_cache for e in self.engines]

    def step(self) -> list[torch.Tensor | None]:
        """One decode step of every micro-batch, interleaved on their streams;
        returns each micro-batch's next-token buffer on the norm_lm_head rank
        (None elsewhere)."""
        outs = []
        cur = torch.cuda.current_stream(self.device)
        for s in self.streams:
            s.wait_stream(cur)
        for eng, s in zip(self.engines, self.streams):
            with torch.cuda.stream(s):
                outs.append(eng.step_static())
        for s in self.streams:
            cur.wait_stream(s)
        return outs
