"""Kernel-group executor with the interface of fluidgpu_torch.executor.LayerExecutor
(fluidgpu_runtime/fluidgpu_torch/executor.py:15-167).

Per task: return None when the task is placed on another rank; receive the
hidden state when the previous task ran elsewhere; run the task; send the
output when the next task runs elsewhere. The rank switch is where the
reference does NCCL send/recv; here it goes to whatever comm backend is
plugged in (P2PComm for the NVLink handoff, LocalComm on one GPU, or any
object with get_rank / send_tensor / recv_tensor).

Sharded feed-forward groups (TaskSpec.shard_ranks, a plan-format extension):
the rank of the task before the group sends its output to every shard rank;
each shard runs the group on its slice (the callable gets shard=(index,
count)) and sends an fp32 partial to the rank of the task after the group,
which receives the partials in shard order and adds them up (fg_sum_partials)
before running that task: the reduce-by-consumer that replaces an
all-reduce.

Batch generalisation: the reference preallocates decode receive buffers of
[1, 1, H] (executor.py:29-41); this executor keeps one [B, 1, H] buffer per
batch size B seen, since the B200 step decodes a batch of requests.
"""
from __future__ import annotations

from collections.abc import Callable
from typing import Any

import torch

from .config import EngineConfig
from .profile import RuntimeProfile
from .trace import trace_region


class LayerExecutor:
    def __init__(self, profile: RuntimeProfile, cfg: EngineConfig, comm_backend: Any) -> None:
        self.profile = profile
        self.cfg = cfg
        self.tasks = list(profile.tasks)
        self.task_index_by_name = profile.task_index_by_name
        self.my_rank = comm_backend.get_rank()
        self._comm = comm_backend
        self.device = cfg.torch_device
        self._decode_bufs: dict[int, torch.Tensor] = {}
        self._prefill_buf: torch.Tensor | None = None
        self._wide_bufs: dict[tuple, torch.Tensor] = {}
        self._partial_bufs: dict[tuple, tuple[torch.Tensor, torch.Tensor]] = {}
        # zero-copy main path (P2PComm(direct=True)): only for plans whose main
        # path alternates strictly between ranks at coarse task boundaries, so
        # a received slot is never read after this rank has sent the value on
        self._direct = bool(getattr(comm_backend, "direct", False)) and _direct_safe(profile)
        self._accepts_out: dict[Any, bool] = {}
        if cfg.preallocate_recv_buffers:
            self._decode_bufs[cfg.max_batch] = torch.empty(
                (cfg.max_batch, 1, profile.hidden_size), dtype=cfg.dtype, device=self.device)

    # -- the reference's public surface ------------------------------------
    def run_stage(self, task_name: str, fn: Callable[..., Any], value: torch.Tensor | None, *,
                  mode: str, seq_len: int | None = None, **kwargs: Any) -> torch.Tensor | None:
        return self._run(task_name, fn, value, mode=mode, seq_len=seq_len, **kwargs)

    def run_layer(self, task_name: str, layer: Callable[..., Any], hidden: torch.Tensor | None, *,
                  mode: str, seq_len: int | None = None, **kwargs: Any) -> torch.Tensor | None:
        def layer_fn(hidden_states: torch.Tensor, **kw: Any) -> Any:
            return layer(hidden_states=hidden_states, **kw)

        return self._run(task_name, layer_fn, hidden, mode=mode, seq_len=seq_len, **kwargs)

    def run_kernel_group(self, task_name: str, fn: Callable[..., Any], hidden: torch.Tensor | None,
                         *, mode: str, seq_len: int | None = None,
                         **kwargs: Any) -> torch.Tensor | None:
        return self._run(task_name, fn, hidden, mode=mode, seq_len=seq_len, **kwargs)

    def message_capacity(self) -> int | None:
        """Largest tensor (bytes) the comm backend carries in one hand-off;
        None when it has no fixed slot size."""
        cap = getattr(self._comm, "slot_bytes", None)
        return None if cap is None else int(cap)

    def send_aux_tensor(self, tensor: torch.Tensor, *, dst: int) -> None:
        self._comm.send_tensor(tensor, dst=dst)

    def recv_aux_tensor(self, tensor: torch.Tensor, *, src: int) -> None:
        self._comm.recv_tensor(tensor, src=src)

    # -- internals -----------------------------------------------------------
    def task_rank(self, task_name: str, mode: str) -> int:
        return self.tasks[self.task_index_by_name[task_name]].rank_for(mode)

    def _run(self, task_name: str, fn: Callable[..., Any], value: torch.Tensor | None, *, mode: str,
             seq_len: int | None, batch: int | None = None, recv_width: int | None = None,
             **kwargs: Any) -> torch.Tensor | None:
        """`recv_width`: last dimension of the incoming value when it is not the
        hidden size (the sdpa -> o_proj edge carries n_q * head_dim features)."""
        assert mode in ("prefill", "decode"), f"invalid mode {mode}"
        idx = self.task_index_by_name[task_name]
        task = self.tasks[idx]
        if task.shard_ranks is not None:
            # a sharded feed-forward group: every shard rank runs it on its slice
            if self.my_rank not in task.shard_ranks:
                return None
            kwargs["shard"] = (task.shard_ranks.index(self.my_rank), len(task.shard_ranks))
        elif task.rank_for(mode) != self.my_rank:
            return None
        b = batch if batch is not None else (value.shape[0] if value is not None else 1)
        prev = self.tasks[idx - 1] if idx > 0 else None
        if prev is not None and prev.shard_ranks is not None:
            # consumer of a sharded group: add up the shards' fp32 partials
            value = self._recv_partials(prev.shard_ranks, mode=mode, batch=b,
                                        seq_len=self._seq_len(value, seq_len))
        elif prev is not None and prev.rank_for(mode) != self.my_rank:
            sl = self._seq_len(value, seq_len)
            if self._direct and mode == "decode" and recv_width is None:
                # zero-copy: wait for the sender's flag and read its slot in place
                src = prev.rank_for(mode)
                self._comm.direct_wait(src)
                value = self._comm.direct_in(src, (b, sl, self.profile.hidden_size), self.cfg.dtype)
            else:
                value = self._recv(mode=mode, batch=b, seq_len=sl, src=prev.rank_for(mode), width=recv_width)
        assert value is not None, f"rank {self.my_rank} entered {task_name} without input"
        nxt = self.tasks[idx + 1] if idx < len(self.tasks) - 1 else None
        direct_dst = None
        if (self._direct and mode == "decode" and nxt is not None and nxt.shard_ranks is None
                and nxt.rank_for(mode) != self.my_rank):
            assert self._takes_out(fn), f"{task_name}: a direct hand-off needs a kernel group that takes out="
            # zero-copy: the group's last kernel writes straight into the peer's slot
            direct_dst = nxt.rank_for(mode)
            kwargs["out"] = self._comm.direct_out(direct_dst, (b, self._seq_len(value, seq_len),
                                                               self.profile.hidden_size), self.cfg.dtype)
        with trace_region(kind="compute", name=task_name, device=self.device, mode=mode):
            out = _first_tensor(fn(value, **kwargs))
        if direct_dst is not None:
            assert out.data_ptr() == kwargs["out"].data_ptr(), f"{task_name} did not write its output in place"
            self._comm.direct_signal(direct_dst)
            return out
        if nxt is not None:
            if not out.is_contiguous():
                out = out.contiguous()
            if nxt.shard_ranks is not None:
                for r in nxt.shard_ranks:  # scatter the group's input to every shard
                    self._comm.send_tensor(out, dst=r)
            elif nxt.rank_for(mode) != self.my_rank:
                self._comm.send_tensor(out, dst=nxt.rank_for(mode))
        return out

    def _takes_out(self, fn: Callable[..., Any]) -> bool:
        key = getattr(fn, "__func__", fn)
        ok = self._accepts_out.get(key)
        if ok is None:
            import inspect

            try:
                ok = "out" in inspect.signature(fn).parameters
            except (TypeError, ValueError):
                ok = False
            self._accepts_out[key] = ok
        return ok

    def _recv(self, *, mode: str, batch: int, seq_len: int, src: int, width: int | None = None) -> torch.Tensor:
        buf = self._recv_buffer(mode=mode, batch=batch, seq_len=seq_len, width=width)
        self._comm.recv_tensor(buf, src=src)
        return buf

    def _recv_partials(self, shard_ranks: tuple[int, ...], *, mode: str, batch: int,
                       seq_len: int) -> torch.Tensor:
        """Receive each shard's fp32 partial [batch, seq_len, H] (shard order)
        and return bf16(sum) (fg_sum_partials)."""
        from . import kernels

        H = self.profile.hidden_size
        S = len(shard_ranks)
        key = (S, batch, seq_len, mode)
        bufs = self._partial_bufs.get(key)
        if bufs is None:
            bufs = (torch.empty((S, batch, seq_len, H), dtype=torch.float32, device=self.device),
                    torch.empty((batch, seq_len, H), dtype=self.cfg.dtype, device=self.device))
            self._partial_bufs[key] = bufs
        parts, total = bufs
        for i, r in enumerate(shard_ranks):
            self._comm.recv_tensor(parts[i], src=r)
        return kernels.sum_partials(parts, out=total)

    def _recv_buffer(self, *, mode: str, batch: int, seq_len: int, width: int | None = None) -> torch.Tensor:
        assert seq_len > 0, f"seq_len must be positive, got {seq_len}"
        H = self.profile.hidden_size
        if width is not None and width != H:
            # a second buffer per (batch, width): the o_proj input of a split attention
            key = (batch, seq_len, width, mode)
            buf = self._wide_bufs.get(key)
            if buf is None:
                buf = torch.empty((batch, seq_len, width), dtype=self.cfg.dtype, device=self.device)
                self._wide_bufs[key] = buf
            return buf
        if mode == "decode":
            assert seq_len == 1, f"decode seq_len must be 1, got {seq_len}"
            buf = self._decode_bufs.get(batch)
            if buf is None:
                buf = torch.empty((batch, 1, H), dtype=self.cfg.dtype, device=self.device)
                self._decode_bufs[batch] = buf
            return buf
        assert seq_len <= self.cfg.max_seq_len, (
            f"prefill seq_len {seq_len} exceeds max_seq_len {self.cfg.max_seq_len}"
        )
        need = batch * seq_len * H
        if self._prefill_buf is None or self._prefill_buf.numel() < need:
            self._prefill_buf = torch.empty(need, dtype=self.cfg.dtype, device=self.device)
        return self._prefill_buf[:need].view(batch, seq_len, H)

    def _seq_len(self, value: torch.Tensor | None, seq_len: int | None) -> int:
        if value is not None:
            assert value.ndim >= 2, f"expected [batch, seq, hidden], got {tuple(value.shape)}"
            return int(value.shape[1])
        assert seq_len is not None, "seq_len is required when receiving into an empty value"
        return seq_len


def _direct_safe(profile: RuntimeProfile) -> bool:
    """The zero-copy hand-off needs a main path that alternates between ranks
    only at coarse attention / FFN boundaries, with no fine-grained split (aux
    tensors), no sharded group and no phase-dependent rank; MoE groups must
    share a rank."""
    from .profile import parse_layer_task

    for t in profile.tasks:
        if t.shard_ranks is not None or t.decode_rank is not None:
            return False
        p = parse_layer_task(t.name)
        if p is not None and p[1] not in ("attn", "mlp", "moe_router", "moe_experts", "moe_combine"):
            return False
    by_name = profile.task_by_name
    for t in profile.tasks:
        p = parse_layer_task(t.name)
        if p is not None and p[1] == "moe_router":
            ranks = {by_name[f"layer_{p[0]}_{s}"].rank for s in ("moe_router", "moe_experts", "moe_combine")}
            if len(ranks) != 1:
                return False
    return True


def _first_tensor(value: Any) -> torch.Tensor:
    if isinstance(value, torch.Tensor):
        return value
    if isinstance(value, tuple):
        assert value, "layer returned an empty tuple"
        assert isinstance(value[0], torch.Tensor), (
            f"expected first tuple item to be Tensor, got {type(value[0])}"
        )
        return value[0]
    raise TypeError(f"expected Tensor or tuple[Tensor, ...], got {type(value)}")


KernelGroupExecutor = LayerExecutor
