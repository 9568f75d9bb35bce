"""Comm backends with the duck-typed interface of fluidgpu_torch.comm
(ProcessGroupComm, fluidgpu_runtime/fluidgpu_torch/comm.py:14-61):
get_rank(), send_tensor(t, dst), recv_tensor(out, src), broadcast_tensor(t, src).

LocalComm   : one rank, everything co-located; any send/recv is a plan error.
QueueComm   : ranks as threads joined by queues (the reference tests' pattern,
              test_fine_dense_runtime.py:14-27), for host-side tests; every
              get() is bounded by a timeout.
P2PComm     : ranks as processes on one NVLink node. Sends are stores into
              the receiver's mailbox over NVLink plus a sequence flag
              (fg_handoff_put / fg_handoff_recv), no NCCL on the data path.
"""
from __future__ import annotations

import ctypes
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


class P2PComm:
    """Comm backend over NVLink peer memory.

    Every rank owns one mailbox in its HBM (fg_mailbox_bytes: per sender
    `nslot` slots of `slot_bytes`, sequence flags and acks); peers map it once
    through CUDA IPC, exchanging handles with torch.distributed. send_tensor
    stores straight into the destination's slot and releases a flag;
    recv_tensor waits for the flag (bounded by timeout_ms, reported through the
    device status) and copies the slot out. Both are ordinary launches on the
    current stream (CUDA-graph capturable). `tag` names an independent channel
    set (one per micro-batch in the ping-pong schedule).
    """

    def __init__(self, slot_bytes: int, *, nslot: int = 2, timeout_ms: int = 2000, group=None,
                 tag: int = 0, device: torch.device | None = None) -> None:
        import torch.distributed as dist

        from . import _lib

        assert dist.is_available() and dist.is_initialized(), "P2PComm needs torch.distributed"
        self._dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.slot_bytes = (int(slot_bytes) + 15) // 16 * 16
        self.nslot = nslot
        self.timeout_ms = timeout_ms
        self.tag = tag
        lib = _lib.lib()
        nbytes = lib.fg_mailbox_bytes(self.world, nslot, self.slot_bytes)
        self.mailbox = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        torch.cuda.synchronize(self.device)
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_size_t(0)
        _lib.call("fg_ipc_export", self.mailbox.data_ptr(), handle, ctypes.byref(off))
        mine = (self.rank, bytes(handle.raw), off.value)
        allh: list = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        self.peers: dict[int, tuple[int, int]] = {}
        for r, h, o in allh:
            if r == self.rank:
                continue
            ptr = ctypes.c_void_p()
            _lib.call("fg_ipc_import", h, o, ctypes.byref(ptr))
            self.peers[r] = (ptr.value, o)
        dist.barrier(group=group)

    def get_rank(self) -> int:
        return self.rank

    def get_world_size(self) -> int:
        return self.world

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def send_tensor(self, t: torch.Tensor, dst: int) -> None:
        from ._lib import call

        assert t.is_contiguous(), "send requires a contiguous tensor"
        assert t.is_cuda, f"send requires a CUDA tensor, got {t.device}"
        nbytes = t.numel() * t.element_size()
        call("fg_handoff_put", t.data_ptr(), nbytes, self.mailbox.data_ptr(), self.peers[dst][0],
             self.world, self.rank, dst, self.nslot, self.slot_bytes, self.timeout_ms, self._stream())

    def recv_tensor(self, out: torch.Tensor, src: int) -> None:
        from ._lib import call

        assert out.is_contiguous(), "recv requires a contiguous tensor"
        assert out.is_cuda, f"recv requires a CUDA tensor, got {out.device}"
        nbytes = out.numel() * out.element_size()
        call("fg_handoff_recv", out.data_ptr(), nbytes, self.mailbox.data_ptr(), self.peers[src][0],
             self.world, self.rank, src, self.nslot, self.slot_bytes, self.timeout_ms, self._stream())

    def broadcast_tensor(self, t: torch.Tensor, src: int = 0) -> None:
        # src is a rank of this comm's group
        g = src if self.group is None else self._dist.get_global_rank(self.group, src)
        self._dist.broadcast(t, src=g, group=self.group)

    def close(self) -> None:
        from ._lib import call

        torch.cuda.synchronize(self.device)
        for ptr, off in self.peers.values():
            call("fg_ipc_close", ptr, off)
        self.peers.clear()
