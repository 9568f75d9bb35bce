"""Comm backends with the duck-typed interface of fluidgpu_torch.comm
(ProcessGroupComm, fluidgpu_runtime/fluidgpu_torch/comm.py:14-61):
get_rank(), send_tensor(t, dst), recv_tensor(out, src), broadcast_tensor(t, src).

LocalComm   : one rank, everything co-located; any send/recv is a plan error.
QueueComm   : ranks as threads joined by queues (the reference tests' pattern,
              test_fine_dense_runtime.py:14-27), for host-side tests; every
              get() is bounded by a timeout.
P2PComm     : ranks as processes on one NVLink node; see handoff.py.
"""
from __future__ import annotations

import queue
from dataclasses import dataclass, field

import torch


@dataclass
class LocalComm:
    rank: int = 0

    def get_rank(self) -> int:
        return self.rank

    def get_world_size(self) -> int:
        return 1

    def send_tensor(self, t: torch.Tensor, dst: int) -> None:
        raise AssertionError(f"single-rank plan tried to send to rank {dst}")

    def recv_tensor(self, out: torch.Tensor, src: int) -> None:
        raise AssertionError(f"single-rank plan tried to receive from rank {src}")

    def broadcast_tensor(self, t: torch.Tensor, src: int = 0) -> None:
        return None


@dataclass
class QueueComm:
    rank: int
    channels: dict = field(default_factory=dict)
    timeout_s: float = 5.0

    @staticmethod
    def make_channels(world: int) -> dict:
        return {(a, b): queue.Queue() for a in range(world) for b in range(world) if a != b}

    def get_rank(self) -> int:
        return self.rank

    def send_tensor(self, t: torch.Tensor, dst: int) -> None:
        assert t.is_contiguous(), "send requires a contiguous tensor"
        self.channels[(self.rank, dst)].put(t.detach().clone())

    def recv_tensor(self, out: torch.Tensor, src: int) -> None:
        assert out.is_contiguous(), "recv requires a contiguous tensor"
        try:
            value = self.channels[(src, self.rank)].get(timeout=self.timeout_s)
        except queue.Empty as exc:
            raise TimeoutError(f"rank {self.rank}: no tensor from rank {src} within {self.timeout_s}s") from exc
        assert value.shape == out.shape, f"recv shape {tuple(value.shape)} != buffer {tuple(out.shape)}"
        out.copy_(value)

    def broadcast_tensor(self, t: torch.Tensor, src: int = 0) -> None:
        return None
