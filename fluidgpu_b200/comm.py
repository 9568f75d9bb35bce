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
ProcessGroupComm : the reference's own backend, torch.distributed send /
              recv / broadcast on a process group (NCCL for CUDA tensors, the
              baseline the NVLink hand-off replaces; gloo for CPU tensors, so
              the multi-process protocol is testable without a GPU).
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


class _PeerMailbox:
    """One mailbox per rank in its own HBM (fg_mailbox_bytes geometry), mapped
    by every peer through CUDA IPC (handles exchanged with all_gather_object)."""

    def __init__(self, dist, group, rank: int, world: int, nslot: int, slot_bytes: int,
                 device: torch.device) -> None:
        from . import _lib

        lib = _lib.lib()
        nbytes = lib.fg_mailbox_bytes(world, nslot, slot_bytes)
        assert nbytes > 0, f"bad mailbox geometry world={world} nslot={nslot} slot={slot_bytes}"
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        torch.cuda.synchronize(device)
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_size_t(0)
        _lib.call("fg_ipc_export", self.buf.data_ptr(), handle, ctypes.byref(off))
        allh: list = [None] * world
        dist.all_gather_object(allh, (rank, bytes(handle.raw), off.value), group=group)
        self.peers: dict[int, tuple[int, int]] = {}
        for r, h, o in allh:
            if r == rank:
                continue
            ptr = ctypes.c_void_p()
            _lib.call("fg_ipc_import", h, o, ctypes.byref(ptr))
            self.peers[r] = (ptr.value, o)

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    def close(self) -> None:
        from ._lib import call

        for ptr, off in self.peers.values():
            call("fg_ipc_close", ptr, off)
        self.peers.clear()


class _LocalMailbox:
    """A mailbox in this process's device memory whose peers are other
    _LocalMailbox objects of the same process and device (plain device
    pointers, no IPC): the mailbox set of P2PComm.same_device_group."""

    def __init__(self, world: int, nslot: int, slot_bytes: int, device: torch.device) -> None:
        from . import _lib

        nbytes = _lib.lib().fg_mailbox_bytes(world, nslot, slot_bytes)
        assert nbytes > 0, f"bad mailbox geometry world={world} nslot={nslot} slot={slot_bytes}"
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        self.peers: dict[int, tuple[int, int]] = {}

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    def close(self) -> None:
        self.peers.clear()


def _preload(device: torch.device) -> None:
    """Load every kernel of the library on `device` before this rank's
    kernels start waiting on other ranks (fg_preload)."""
    from ._lib import call

    with torch.cuda.device(device):
        call("fg_preload")


class _DeviceArray:
    """A CUDA array interface over a raw device pointer (a peer's slot), so
    torch can wrap it without copying."""

    def __init__(self, ptr: int, shape: tuple[int, ...], dtype: torch.dtype) -> None:
        typestr = {torch.bfloat16: "<i2", torch.float16: "<f2", torch.float32: "<f4"}[dtype]  # bf16 as i2, viewed
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


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

    direct=True adds a second, one-slot mailbox for zero-copy hand-offs of the
    main path (direct_out / direct_signal on the sender, direct_wait /
    direct_in on the receiver): the sender's producing kernel writes straight
    into the peer's slot and the receiver's kernels read it in place
    (fg_handoff_signal / fg_handoff_wait; the header states when that is safe).
    """

    def __init__(self, slot_bytes: int, *, nslot: int = 2, timeout_ms: int = 2000, group=None,
                 tag: int = 0, device: torch.device | None = None, direct: bool = False) -> None:
        import torch.distributed as dist

        assert dist.is_available() and dist.is_initialized(), "P2PComm needs torch.distributed"
        device = device or torch.device("cuda", torch.cuda.current_device())
        _preload(device)
        slot = (int(slot_bytes) + 15) // 16 * 16
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        mb = _PeerMailbox(dist, group, rank, world, nslot, slot, device)
        dmb = _PeerMailbox(dist, group, rank, world, 1, slot, device) if direct else None
        self._setup(dist, group, rank, world, mb, dmb, slot, nslot, timeout_ms, tag, device)
        dist.barrier(group=group)

    def _setup(self, dist, group, rank: int, world: int, mb, dmb, slot_bytes: int, nslot: int,
               timeout_ms: int, tag: int, device: torch.device) -> None:
        self._dist = dist
        self.group = group
        self.rank = rank
        self.world = world
        self.device = device
        self.slot_bytes = slot_bytes
        self.nslot = nslot
        self.timeout_ms = timeout_ms
        self.tag = tag
        self._mb = mb
        self.mailbox = mb.buf
        self.peers = mb.peers
        self.direct = dmb is not None
        self._dmb = dmb
        self._views: dict[tuple, torch.Tensor] = {}

    @classmethod
    def same_device_group(cls, world: int, slot_bytes: int, *, nslot: int = 2, timeout_ms: int = 2000,
                          device: torch.device | None = None, direct: bool = False) -> list["P2PComm"]:
        """`world` ranks in one process on one device, one comm per rank:
        each rank's mailbox lives in that device's memory and the others
        address it directly (no IPC, no torch.distributed). The hand-off
        kernels use the same slots, flags and sequence numbers as between
        GPUs. Ranks that share a GPU must be ordered by the host: a rank's
        receive (or wait) may only be enqueued behind the matching send (or
        signal) through a CUDA event or the same stream, because two launches
        on one GPU are not guaranteed to run at the same time, so a receive
        left to spin on a send that has not started would only end at its
        timeout. This serves single-GPU tests and debugging of multi-rank
        plans."""
        device = device or torch.device("cuda", torch.cuda.current_device())
        slot = (int(slot_bytes) + 15) // 16 * 16
        mbs = [_LocalMailbox(world, nslot, slot, device) for _ in range(world)]
        dmbs = [_LocalMailbox(world, 1, slot, device) for _ in range(world)] if direct else None
        for boxes in (mbs, dmbs or []):
            for r, box in enumerate(boxes):
                box.peers.update({p: (boxes[p].ptr, 0) for p in range(world) if p != r})
        comms = []
        for r in range(world):
            c = cls.__new__(cls)
            c._setup(None, None, r, world, mbs[r], dmbs[r] if dmbs else None, slot, nslot, timeout_ms, 0, device)
            comms.append(c)
        return comms

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

    # -- direct (zero-copy) main-path hand-off --------------------------------
    def _slot_view(self, mailbox_ptr: int, src: int, shape: tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
        from . import _lib

        key = (mailbox_ptr, src, tuple(shape), dtype)
        v = self._views.get(key)
        if v is None:
            nbytes = torch.Size(shape).numel() * torch.empty((), dtype=dtype).element_size()
            assert nbytes <= self.slot_bytes, f"{nbytes} bytes do not fit the {self.slot_bytes}-byte slot"
            ptr = _lib.lib().fg_mailbox_slot(mailbox_ptr, self.world, 1, self.slot_bytes, src, 0)
            assert ptr, "fg_mailbox_slot failed"
            v = torch.as_tensor(_DeviceArray(ptr, shape, dtype), device=self.device)
            if dtype == torch.bfloat16:
                v = v.view(torch.bfloat16)
            self._views[key] = v
        return v

    def direct_out(self, dst: int, shape: tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
        """This rank's slot in dst's direct mailbox (peer memory): write the
        message there, then direct_signal(dst)."""
        assert self.direct, "P2PComm(direct=True) is required"
        return self._slot_view(self._dmb.peers[dst][0], self.rank, shape, dtype)

    def direct_signal(self, dst: int) -> None:
        from ._lib import call

        call("fg_handoff_signal", self._dmb.ptr, self._dmb.peers[dst][0], self.world, self.rank, dst,
             self.slot_bytes, self._stream())

    def direct_wait(self, src: int) -> None:
        from ._lib import call

        call("fg_handoff_wait", self._dmb.ptr, self.world, self.rank, src, self.slot_bytes, self.timeout_ms,
             self._stream())

    def direct_in(self, src: int, shape: tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
        """src's slot in this rank's direct mailbox (read after direct_wait)."""
        assert self.direct, "P2PComm(direct=True) is required"
        return self._slot_view(self._dmb.ptr, src, shape, dtype)

    def broadcast_tensor(self, t: torch.Tensor, src: int = 0) -> None:
        # src is a rank of this comm's group
        assert self._dist is not None, "a same-device group has no process group to broadcast over"
        g = src if self.group is None else self._dist.get_global_rank(self.group, src)
        self._dist.broadcast(t, src=g, group=self.group)

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        self._views.clear()
        self._mb.close()
        if self._dmb is not None:
            self._dmb.close()


@dataclass(frozen=True)
class ProcessGroupComm:
    """torch.distributed point-to-point comm (fluidgpu_torch/comm.py:14-61).
    Ranks are global ranks, as the plan's are; `group` restricts the
    collective (broadcast) and names the group the sends use."""

    group: object = None

    def get_rank(self) -> int:
        return torch.distributed.get_rank()

    def get_world_size(self) -> int:
        return torch.distributed.get_world_size(self.group)

    def send_tensor(self, t: torch.Tensor, dst: int) -> None:
        assert t.is_contiguous(), "send requires a contiguous tensor"
        torch.distributed.send(t, dst=dst, group=self.group)

    def recv_tensor(self, out: torch.Tensor, src: int) -> None:
        assert out.is_contiguous(), "recv requires a contiguous tensor"
        torch.distributed.recv(out, src=src, group=self.group)

    def broadcast_tensor(self, t: torch.Tensor, src: int = 0) -> None:
        assert t.is_contiguous(), "broadcast requires a contiguous tensor"
        torch.distributed.broadcast(t, src=src, group=self.group)
