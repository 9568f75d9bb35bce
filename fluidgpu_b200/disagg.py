"""Disaggregated decode step over the GPUs of one NVLink node, with merged
feed-forward batches and hand-offs fused into the kernels on either side.

The B200 form of FluidGPU's attention/FFN disaggregation (the placement of
benchmark configs 2 and 4: attention on some GPUs, the FFN on others; the
reference hands the hidden state over with NCCL send/recv at every task
boundary, executor.py:104-123, and pipelines micro-batches with the remote
FFN, vllm_integration.py:1141-1237).

Roles (A attention ranks, S FFN ranks, M micro-batches of b sequences on
every attention rank):
  attention rank a : embed; per layer RMSNorm -> QKV GEMM -> RoPE + paged KV
                     append -> paged attention -> O-proj GEMM (+ residual);
                     final norm -> lm_head -> argmax. Each micro-batch has its
                     own paged KV cache, stream and CUDA graph, so one
                     micro-batch's attention runs while another's FFN is away.
  FFN rank j       : the FFN of layer l for micro-batch m of ALL A attention
                     ranks at once: their rows form one batch of A*b tokens
                     (one RMSNorm, one gate/up GEMM with the SwiGLU epilogue,
                     one down GEMM), over its slice j of the intermediate
                     dimension (tensor-parallel, S shards). One graph per
                     step walks (layer, micro-batch) in order.

Hand-offs (per layer and micro-batch; no NCCL and no copy kernels):
  a -> every j : the O-proj epilogue stores its b rows of h (bf16) into
                 in[m] rows [a*b, (a+1)*b) of every FFN rank (broadcast
                 route), and its last CTA raises in_flag[m][a] there.
  j -> every a : the down-proj epilogue stores rows [a*b, (a+1)*b) of its
                 result into rank a's ret[m] (split route) and raises
                 ret_flag[m][j] there: with S == 1 the finished residual
                 stream bf16(h + FFN(h)); with S > 1 an fp32 partial (shard 0
                 adds h), summed in shard order by the consumer.
  The first kernel reading a message waits for its flag itself
  (fg_rmsnorm_wait / fg_sum_rmsnorm_wait). Flag values are epoch * L +
  layer + 1, where each side counts its own finished steps (fg_counter_add
  at the end of its graph), so no flag is ever reset and no acknowledgement
  travels back: a buffer is rewritten only after its reader has answered a
  later message, which it sends after its last read.

Memory: every rank owns one mailbox (data, then flags 128 bytes apart) in its
own HBM; the other role's ranks map it through CUDA IPC. In one process on
one device (tests), Fabric.local wires the same buffers by plain pointers.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Any

import torch

from . import _lib, kernels
from ._lib import call, ptr_array
from .kv_cache import PagedKVCache
from .model import ModelWeights

FLAG_STRIDE = 128  # bytes between flags (one per cache line)


@dataclass(frozen=True)
class DisaggLayout:
    """Global ranks of the two roles, micro-batches per attention rank,
    sequences per micro-batch, and how the hidden state reaches the FFN ranks:
    "pull" (the O-proj GEMM stores it in the attention GPU's own memory and
    the FFN ranks' waiting RMSNorm reads it over NVLink) or "push" (the O-proj
    GEMM's epilogue stores it into every FFN rank's memory)."""

    attn_ranks: tuple[int, ...]
    ffn_ranks: tuple[int, ...]
    micro_batches: int
    rows: int
    handoff: str = "pull"

    def __post_init__(self) -> None:
        assert self.handoff in ("pull", "push"), f"unknown hand-off {self.handoff!r}"
        assert self.attn_ranks and self.ffn_ranks, "need at least one attention and one FFN rank"
        assert not set(self.attn_ranks) & set(self.ffn_ranks), "a rank has one role"
        assert len(self.attn_ranks) <= 8 and len(self.ffn_ranks) <= 8, "at most 8 ranks per role"
        assert self.micro_batches >= 1 and self.rows >= 1

    @property
    def A(self) -> int:
        return len(self.attn_ranks)

    @property
    def S(self) -> int:
        return len(self.ffn_ranks)

    @property
    def world(self) -> int:
        return self.A + self.S

    def role(self, rank: int) -> tuple[str, int]:
        if rank in self.attn_ranks:
            return "attn", self.attn_ranks.index(rank)
        assert rank in self.ffn_ranks, f"rank {rank} has no role"
        return "ffn", self.ffn_ranks.index(rank)

    @classmethod
    def split(cls, world: int, micro_batches: int, rows: int, handoff: str = "pull") -> "DisaggLayout":
        """First half of the ranks attention, second half FFN (one of each for 2)."""
        assert world >= 2 and world % 2 == 0, f"a split layout needs an even world, got {world}"
        h = world // 2
        return cls(tuple(range(h)), tuple(range(h, world)), micro_batches, rows, handoff)


class _Mailbox:
    """`data_bytes` of message rows, then `n_flags` u32 flags, zeroed, in this
    GPU's memory."""

    def __init__(self, data_bytes: int, n_flags: int, device: torch.device) -> None:
        self.data_bytes = (data_bytes + 255) // 256 * 256
        self.buf = torch.zeros(self.data_bytes + n_flags * FLAG_STRIDE, dtype=torch.uint8, device=device)

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()


def _flag(base: int, data_bytes: int, i: int) -> int:
    return base + data_bytes + i * FLAG_STRIDE


class _Rank:
    """State shared by both roles: layout, weights, mailbox, peers' mailbox
    base addresses (filled by a Fabric), hooks."""

    def __init__(self, layout: DisaggLayout, rank: int, weights: ModelWeights, device: torch.device,
                 timeout_ms: int) -> None:
        self.layout = layout
        self.rank = rank
        self.role, self.index = layout.role(rank)
        self.w = weights
        self.spec = weights.spec
        self.device = device
        self.timeout_ms = timeout_ms
        self.L = self.spec.num_layers
        self.peer_base: dict[int, int] = {}  # global rank -> its mailbox base address as seen here
        # host-side ordering hooks for ranks that share a GPU (tests); None on
        # separate GPUs, where the flags alone order the ranks
        self.hooks: Any = None

    # mailbox geometry of each role (identical on every rank)
    def ffn_geometry(self) -> tuple[int, int]:
        lay, H = self.layout, self.spec.hidden
        data = lay.micro_batches * lay.A * lay.rows * H * 2
        return (data + 255) // 256 * 256, lay.micro_batches * lay.A

    def attn_geometry(self) -> tuple[int, int]:
        """Return buffers ret[m] (then, pulling, send buffers send[m]) and
        one flag per (micro-batch, FFN rank)."""
        lay, H = self.layout, self.spec.hidden
        data = self.attn_send_offset()
        if lay.handoff == "pull":
            data += lay.micro_batches * lay.rows * H * 2
        return (data + 255) // 256 * 256, lay.micro_batches * lay.S

    def attn_send_offset(self) -> int:
        """Byte offset of send[0] in an attention rank's mailbox (pull)."""
        lay, H = self.layout, self.spec.hidden
        elem = 4 if lay.S > 1 else 2
        data = lay.micro_batches * lay.S * lay.rows * H * elem
        return (data + 255) // 256 * 256

    def _hook(self, what: str, *args) -> None:
        if self.hooks is not None:
            getattr(self.hooks, what)(self, *args)


class AttentionRank(_Rank):
    """One attention rank: M micro-batches of b sequences, each with its own
    paged KV cache, buffers, stream and graph."""

    def __init__(self, layout: DisaggLayout, rank: int, weights: ModelWeights, max_seq_len: int, *,
                 device: torch.device, timeout_ms: int = 10000, schedule: str = "interleaved") -> None:
        super().__init__(layout, rank, weights, device, timeout_ms)
        assert self.role == "attn"
        assert schedule in ("interleaved", "streams"), f"unknown schedule {schedule!r}"
        self.schedule = schedule
        self._graphs: dict[str, tuple[torch.cuda.CUDAGraph, tuple[int, ...]]] = {}
        s, lay = self.spec, layout
        data, nflag = self.attn_geometry()
        self.mailbox = _Mailbox(data, nflag, device)
        self.max_seq_len = max_seq_len
        b, H = lay.rows, s.hidden
        qkv_w = weights.layers[0]["wqkv"].shape[0]
        vocab = weights.lm_head.shape[0]
        self.mbs = []
        for m in range(lay.micro_batches):
            kv = PagedKVCache(num_layers=s.num_layers, owned_layer_ids=list(range(s.num_layers)),
                              max_seq_len=max_seq_len, num_kv_heads=s.n_kv, head_dim=s.head_dim,
                              dtype=torch.bfloat16, device=device, max_batch=b)
            self.mbs.append({
                "kv": kv,
                "tok": torch.zeros(b, dtype=torch.int64, device=device),
                "next": torch.zeros(b, dtype=torch.int64, device=device),
                "h": torch.empty(b, H, dtype=torch.bfloat16, device=device),
                "x": torch.empty(b, H, dtype=torch.bfloat16, device=device),
                "epoch": torch.zeros(1, dtype=torch.int32, device=device),
                "tickets": torch.zeros(s.num_layers, dtype=torch.int32, device=device),
                # per-layer buffers: a step allocates nothing (see step())
                "qkv": torch.empty(b, qkv_w, dtype=torch.bfloat16, device=device),
                "q": torch.empty(b, s.n_q, s.head_dim, dtype=torch.bfloat16, device=device),
                "a": torch.empty(b, s.n_q * s.head_dim, dtype=torch.bfloat16, device=device),
                "logits": torch.empty(b, vocab, dtype=torch.bfloat16, device=device),
                "slot": f"disagg{id(self):x}.{m}",
                "graph": None,
            })
        self.streams = [torch.cuda.Stream(device, priority=-(lay.micro_batches - 1 - m))
                        for m in range(lay.micro_batches)]

    # -- views of this rank's mailbox -------------------------------------
    def ret_view(self, m: int) -> torch.Tensor:
        """This rank's return buffer of micro-batch m: [S, b, H] fp32 (S > 1)
        or [b, H] bf16 (S == 1)."""
        lay, H = self.layout, self.spec.hidden
        if lay.S > 1:
            plane = lay.rows * H
            flat = self.mailbox.buf[: self.mailbox.data_bytes].view(torch.float32)
            return flat[m * lay.S * plane:(m + 1) * lay.S * plane].view(lay.S, lay.rows, H)
        flat = self.mailbox.buf[: self.mailbox.data_bytes].view(torch.bfloat16)
        return flat[m * lay.rows * H:(m + 1) * lay.rows * H].view(lay.rows, H)

    def ret_flags(self, m: int) -> list[int]:
        return [_flag(self.mailbox.ptr, self.mailbox.data_bytes, m * self.layout.S + j)
                for j in range(self.layout.S)]

    def send_view(self, m: int) -> torch.Tensor:
        """send[m], [b, H] bf16: micro-batch m's hidden state after the O-proj,
        which the FFN ranks read (pull)."""
        lay, H = self.layout, self.spec.hidden
        off = self.attn_send_offset() + m * lay.rows * H * 2
        return self.mailbox.buf[off:off + lay.rows * H * 2].view(torch.bfloat16).view(lay.rows, H)

    def ffn_in_rows(self, m: int) -> list[int]:
        """Address of this rank's row block of in[m] on every FFN rank."""
        lay, H = self.layout, self.spec.hidden
        out = []
        for r in lay.ffn_ranks:
            base = self.peer_base[r]
            out.append(base + (m * lay.A * lay.rows) * H * 2)
        return out

    def ffn_in_flags(self, m: int) -> list[int]:
        data, _ = self.ffn_geometry()
        return [_flag(self.peer_base[r], data, m * self.layout.A + self.index) for r in self.layout.ffn_ranks]

    # -- batch --------------------------------------------------------------
    def start(self, prompt_lens: list[list[int]], reserve_tokens: int) -> None:
        """prompt_lens[m]: cached tokens of micro-batch m's b sequences."""
        for mb, lens in zip(self.mbs, prompt_lens):
            assert len(lens) == self.layout.rows
            mb["kv"].start_batch(lens, reserve_tokens)
        self.release_graphs()

    def set_tokens(self, m: int, tokens: torch.Tensor) -> None:
        self.mbs[m]["tok"].copy_(tokens.reshape(-1))

    # -- one decode step of micro-batch m, enqueued on the current stream ----
    def _norm_in(self, m: int, layer: int, weight: torch.Tensor) -> None:
        """x = RMSNorm(h) of the residual stream after the FFN of `layer - 1`
        (waiting for the FFN ranks' message)."""
        s, lay, mb = self.spec, self.layout, self.mbs[m]
        self._hook("before_wait", "ret", m, layer - 1)
        flags = ptr_array(self.ret_flags(m))
        stream = kernels._stream(self.device)
        if lay.S == 1:
            ret = self.ret_view(m)
            call("fg_rmsnorm_wait", ret.data_ptr(), weight.data_ptr(), mb["x"].data_ptr(), lay.rows, s.hidden,
                 float(s.eps), s.norm_mode, flags, 1, lay.rows, mb["epoch"].data_ptr(), self.L, layer,
                 self.timeout_ms, stream)
        else:
            call("fg_sum_rmsnorm_wait", self.ret_view(m).data_ptr(), lay.S, mb["h"].data_ptr(),
                 weight.data_ptr(), mb["x"].data_ptr(), lay.rows, s.hidden, float(s.eps), s.norm_mode, flags,
                 lay.S, mb["epoch"].data_ptr(), self.L, layer, self.timeout_ms, stream)

    def _residual(self, m: int) -> torch.Tensor:
        """The residual stream h of micro-batch m (in the return buffer when
        one FFN rank sends it finished)."""
        if self.layout.S == 1:
            return self.ret_view(m)
        return self.mbs[m]["h"]

    def step_mb(self, m: int, standalone: bool = False) -> None:
        """Enqueue one decode step of micro-batch m on the current stream.
        standalone=True runs the same attention-side kernels with the FFN
        left out (no hand-offs, the O-proj result is the next layer's input):
        a timing reference for how much of the step the hand-offs and the
        remote FFN add, not a model computation."""
        for _ in self._enqueue(m, standalone):
            pass

    def step_interleaved(self, standalone: bool = False) -> None:
        """Enqueue one decode step of every micro-batch on the current stream,
        layer by layer: micro-batch 0's layer l, micro-batch 1's layer l, ...,
        then layer l + 1. While one micro-batch's attention runs here, the FFN
        GPUs work on the one before it, and its answer is back by the time
        this stream reaches that micro-batch's next layer."""
        gens = [self._enqueue(m, standalone) for m in range(len(self.mbs))]
        while gens:
            gens = [g for g in gens if next(g, StopIteration) is not StopIteration]

    def _enqueue(self, m: int, standalone: bool):
        """Generator enqueuing micro-batch m's step; it yields after each
        layer's hand-off to the FFN ranks (the points where another
        micro-batch's layer may be enqueued)."""
        s, lay, mb, W = self.spec, self.layout, self.mbs[m], self.w
        kv = mb["kv"]
        b = lay.rows
        kernels.embed(mb["tok"], W.embed, out=mb["h"])
        kernels.rmsnorm(mb["h"], W.layers[0]["ln1"], s.eps, s.norm_mode, out=mb["x"])
        pull = lay.handoff == "pull"
        if standalone:
            dsts = sigs = None
        else:
            dsts = ptr_array([self.send_view(m).data_ptr()] if pull else self.ffn_in_rows(m))
            sigs = ptr_array(self.ffn_in_flags(m))
        n_dst, row0 = (1, 0) if pull else (lay.S, self.index * b)
        for i in range(s.num_layers):
            stream = kernels._stream(self.device)
            L = W.layers[i]
            h = mb["h"] if (i == 0 or standalone) else self._residual(m)
            if i > 0:
                if standalone:
                    kernels.rmsnorm(mb["h"], L["ln1"], s.eps, s.norm_mode, out=mb["x"])
                else:
                    self._norm_in(m, i, L["ln1"])
            qkv = kernels.gemm(mb["x"], L["wqkv"], bias=L.get("bqkv"), out=mb["qkv"], slot=mb["slot"] + ".gemm")
            kp, vp = kv.layer_pages(i)
            q = kernels.rope_kv_append(qkv, kv.positions[:b], W.inv_freq, W.rope_scaling, kv.block_table[:b],
                                       kp, vp, s.n_q, s.n_kv, s.head_dim, q_out=mb["q"])
            a = kernels.paged_decode_attn(q, kp, vp, kv.block_table[:b], kv.seq_lens[:b], kv.plan_len(),
                                          window=s.window(i), sinks=L.get("sinks"), out=mb["a"],
                                          slot=mb["slot"] + ".attn")
            if standalone:
                kernels.gemm(a, L["wo"], epilogue=_lib.FG_EPI_RESIDUAL, residual=h, bias=L.get("bo"), out=mb["h"],
                             slot=mb["slot"] + ".gemm")
            else:
                wo = L["wo"]
                call("fg_gemm_bf16_packed_routed", a.data_ptr(), wo.data.data_ptr(), h.data_ptr(),
                     None if L.get("bo") is None else L["bo"].data_ptr(), b, s.hidden, s.n_q * s.head_dim,
                     _lib.FG_EPI_RESIDUAL, _lib.FG_ROUTE_BROADCAST, dsts, n_dst, b, row0, sigs, lay.S,
                     mb["epoch"].data_ptr(), self.L, i + 1, mb["tickets"][i:i + 1].data_ptr(), stream)
                self._hook("after_send", "in", m, i)
            yield
        stream = kernels._stream(self.device)
        if standalone:
            kernels.rmsnorm(mb["h"], W.final_norm, s.eps, s.norm_mode, out=mb["x"])
        else:
            self._norm_in(m, s.num_layers, W.final_norm)
        logits = kernels.gemm(mb["x"], W.lm_head, out=mb["logits"], slot=mb["slot"] + ".gemm")
        kernels.argmax(logits, out=mb["next"])
        mb["tok"].copy_(mb["next"])
        kernels.advance(kv.positions[:b], kv.seq_lens[:b])
        if not standalone:
            call("fg_counter_add", mb["epoch"].data_ptr(), 1, stream)

    # -- graphs -----------------------------------------------------------------
    def reserve(self, m: int) -> None:
        """Scratch at the size the current length bucket needs, for the
        attention and for every GEMM of the step (before a capture or an
        eager step: a step must not allocate)."""
        s, mb, W = self.spec, self.mbs[m], self.w
        kv = mb["kv"]
        lib = _lib.lib()
        b = self.layout.rows
        plan = kv.plan_len()
        need = max(lib.fg_attn_workspace_bytes(b, s.n_q, s.n_kv, s.head_dim, plan, s.window(i))
                   for i in range(s.num_layers))
        kernels.Workspace.get(need, self.device, mb["slot"] + ".attn")
        shapes = [W.layers[0]["wqkv"].shape, W.lm_head.shape, W.layers[0]["wo"].shape]
        gneed = max(lib.fg_gemm_workspace_bytes(b, n, k, 0) for n, k in shapes)
        kernels.Workspace.get(gneed, self.device, mb["slot"] + ".gemm")

    def _bucket_for_step(self, m: int) -> int:
        kv = self.mbs[m]["kv"]
        return kv.bucket(kv.max_attended())

    def _capture(self, ms: list[int], standalone: bool) -> tuple[torch.cuda.CUDAGraph, tuple[int, ...]]:
        """Capture the step of micro-batches `ms` (one of them: that
        micro-batch's step; all of them: the interleaved step) for their
        current length buckets, on the first one's stream."""
        buckets = []
        snaps = []
        for m in ms:
            kv = self.mbs[m]["kv"]
            kv.prepare_step(1)
            self.reserve(m)
            buckets.append(self._bucket_for_step(m))
            snaps.append(kv.snapshot_host())
            kv.plan_len_override = buckets[-1]
        g = torch.cuda.CUDAGraph()
        s = self.streams[ms[0]]
        s.wait_stream(torch.cuda.current_stream(self.device))
        try:
            with torch.cuda.stream(s), torch.inference_mode():
                with torch.cuda.graph(g, stream=s):
                    if len(ms) == 1:
                        self.step_mb(ms[0], standalone)
                    else:
                        self.step_interleaved(standalone)
        finally:
            for m, snap in zip(ms, snaps):
                kv = self.mbs[m]["kv"]
                kv.plan_len_override = None
                kv.restore_host(snap)
        torch.cuda.current_stream(self.device).wait_stream(s)
        return g, tuple(buckets)

    def capture(self, m: int, standalone: bool = False) -> None:
        """Capture micro-batch m's step for its current length bucket. Capture
        synchronises this GPU: call it only while no replay of this rank
        waits on the FFN GPUs for a micro-batch not yet launched (step()
        captures all micro-batches before replaying any)."""
        key = "alone" if standalone else "graph"
        mb = self.mbs[m]
        mb[key], (mb[key + "_bucket"],) = self._capture([m], standalone)

    def step(self, graphs: bool = True, standalone: bool = False) -> list[torch.Tensor]:
        """One decode step of every micro-batch; returns the next-token buffers.

        schedule "interleaved" (the default): one stream, micro-batches
        alternating layer by layer (step_interleaved), one graph for all.
        schedule "streams": each micro-batch on a stream and graph of its own,
        the GPU interleaving them as their waits allow.

        Once a micro-batch is launched its kernels may wait on the FFN GPUs,
        which go on only when the others are launched too. So nothing between
        the launches may wait for this GPU to go idle: the step allocates no
        device memory (buffers above, scratch reserved first) and launches no
        kernel for the first time (the library's kernels are loaded when the
        mailboxes are mapped)."""
        cur = torch.cuda.current_stream(self.device)
        for s in self.streams:
            s.wait_stream(cur)
        key = "alone" if standalone else "graph"
        if not graphs:
            for m, mb in enumerate(self.mbs):
                mb["kv"].prepare_step(1)
                self.reserve(m)
        if self.schedule == "interleaved":
            s = self.streams[0]
            with torch.cuda.stream(s):
                for mb in self.mbs:
                    mb["kv"].prepare_step(1)
                if graphs:
                    want = tuple(self._bucket_for_step(m) for m in range(len(self.mbs)))
                    if self._graphs.get(key, (None, None))[1] != want:
                        self._graphs[key] = self._capture(list(range(len(self.mbs))), standalone)
                    self._graphs[key][0].replay()
                else:
                    with torch.inference_mode():
                        self.step_interleaved(standalone)
                for mb in self.mbs:
                    mb["kv"].host_advance(1)
        else:
            if graphs:
                # capture every micro-batch's graph before replaying any: a capture
                # synchronises the device, and a replayed micro-batch can only
                # finish after the FFN GPUs have processed the others' messages
                for m, (mb, s) in enumerate(zip(self.mbs, self.streams)):
                    with torch.cuda.stream(s):
                        mb["kv"].prepare_step(1)
                        if mb.get(key) is None or self._bucket_for_step(m) != mb[key + "_bucket"]:
                            self.capture(m, standalone)
            for m, (mb, s) in enumerate(zip(self.mbs, self.streams)):
                kv = mb["kv"]
                with torch.cuda.stream(s):
                    kv.prepare_step(1)
                    if graphs:
                        mb[key].replay()
                    else:
                        with torch.inference_mode():
                            self.step_mb(m, standalone)
                    kv.host_advance(1)
        for s in self.streams:
            cur.wait_stream(s)
        return [mb["next"] for mb in self.mbs]

    def step_serial_standalone(self) -> None:
        """Every micro-batch's attention-side step with the FFN left out, one
        after another on the current stream (kernels timed one at a time)."""
        with torch.inference_mode():
            for m, mb in enumerate(self.mbs):
                mb["kv"].prepare_step(1)
                self.step_mb(m, standalone=True)
                mb["kv"].host_advance(1)

    def release_graphs(self) -> None:
        self._graphs.clear()
        for mb in self.mbs:
            mb["graph"] = None
            mb["alone"] = None


class FFNRank(_Rank):
    """One FFN rank: shard `index` of every layer's dense FFN, applied to the
    merged rows of all attention ranks, micro-batch by micro-batch."""

    def __init__(self, layout: DisaggLayout, rank: int, weights: ModelWeights, *, device: torch.device,
                 timeout_ms: int = 10000) -> None:
        super().__init__(layout, rank, weights, device, timeout_ms)
        assert self.role == "ffn"
        assert not self.spec.moe, "the merged-FFN rank serves dense FFNs"
        if layout.S > 1:
            assert weights.ffn_shard == (self.index, layout.S), (
                f"FFN rank {self.index} needs the weights of shard ({self.index}, {layout.S})")
        data, nflag = self.ffn_geometry()
        self.mailbox = _Mailbox(data, nflag, device)
        T = layout.A * layout.rows
        self.x = torch.empty(T, self.spec.hidden, dtype=torch.bfloat16, device=device)
        gu = weights.layers[0]["w_gate_up"]
        self.act = torch.empty(T, gu.shape[0] // 2, dtype=torch.bfloat16, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.tickets = torch.zeros(self.spec.num_layers * layout.micro_batches, dtype=torch.int32, device=device)
        self.slot = f"disagg-ffn{id(self):x}"
        kernels.Workspace.get(_lib.lib().fg_gemm_workspace_bytes(T, gu.shape[0], gu.shape[1], 0), device,
                              self.slot)
        self.stream = torch.cuda.Stream(device)
        self.graph = None

    def in_view(self, m: int) -> torch.Tensor:
        lay, H = self.layout, self.spec.hidden
        T = lay.A * lay.rows
        flat = self.mailbox.buf[: self.mailbox.data_bytes].view(torch.bfloat16)
        return flat[m * T * H:(m + 1) * T * H].view(T, H)

    def in_flags(self, m: int) -> list[int]:
        return [_flag(self.mailbox.ptr, self.mailbox.data_bytes, m * self.layout.A + a)
                for a in range(self.layout.A)]

    def attn_send_rows(self, m: int) -> list[int]:
        """Address of send[m] on every attention rank (pull)."""
        lay, H = self.layout, self.spec.hidden
        off = self.attn_send_offset() + m * lay.rows * H * 2
        return [self.peer_base[r] + off for r in lay.attn_ranks]

    def ret_rows(self, m: int) -> list[int]:
        """Address of this shard's plane of ret[m] on every attention rank."""
        lay, H = self.layout, self.spec.hidden
        out = []
        for r in lay.attn_ranks:
            base = self.peer_base[r]
            if lay.S > 1:
                out.append(base + ((m * lay.S + self.index) * lay.rows * H) * 4)
            else:
                out.append(base + (m * lay.rows * H) * 2)
        return out

    def ret_flags(self, m: int) -> list[int]:
        data, _ = self.attn_geometry()
        return [_flag(self.peer_base[r], data, m * self.layout.S + self.index) for r in self.layout.attn_ranks]

    def step(self, graphs: bool = True) -> None:
        if graphs:
            if self.graph is None:
                self.capture()
            self.graph.replay()
        else:
            with torch.inference_mode():
                self._step()

    def _step(self) -> None:
        s, lay, W = self.spec, self.layout, self.w
        T = lay.A * lay.rows
        stream = kernels._stream(self.device)
        epi = _lib.FG_EPI_RESIDUAL if lay.S == 1 else _lib.FG_EPI_F32
        for i in range(s.num_layers):
            L = W.layers[i]
            for m in range(lay.micro_batches):
                self._hook("before_wait", "in", m, i)
                inp = self.in_view(m)
                if lay.handoff == "pull":  # read the attention ranks' send[m] over NVLink into in[m]
                    call("fg_rmsnorm_gather_wait", ptr_array(self.attn_send_rows(m)), lay.A, lay.rows,
                         inp.data_ptr(), L["ln2"].data_ptr(), self.x.data_ptr(), T, s.hidden, float(s.eps),
                         s.norm_mode, ptr_array(self.in_flags(m)), lay.A, lay.rows, self.epoch.data_ptr(), self.L,
                         i + 1, self.timeout_ms, stream)
                else:
                    call("fg_rmsnorm_wait", inp.data_ptr(), L["ln2"].data_ptr(), self.x.data_ptr(), T, s.hidden,
                         float(s.eps), s.norm_mode, ptr_array(self.in_flags(m)), lay.A, lay.rows,
                         self.epoch.data_ptr(), self.L, i + 1, self.timeout_ms, stream)
                act = kernels.gemm(self.x, L["w_gate_up"], epilogue=_lib.FG_EPI_SWIGLU, out=self.act, slot=self.slot)
                wd = L["w_down"]
                res = inp if (lay.S == 1 or self.index == 0) else None
                t = i * lay.micro_batches + m
                call("fg_gemm_bf16_packed_routed", act.data_ptr(), wd.data.data_ptr(),
                     None if res is None else res.data_ptr(), None, T, s.hidden, wd.K, epi, _lib.FG_ROUTE_SPLIT,
                     ptr_array(self.ret_rows(m)), lay.A, lay.rows, 0, ptr_array(self.ret_flags(m)), lay.A,
                     self.epoch.data_ptr(), self.L, i + 1, self.tickets[t:t + 1].data_ptr(), stream)
                self._hook("after_send", "ret", m, i)
        call("fg_counter_add", self.epoch.data_ptr(), 1, stream)

    def time_standalone(self, reps: int = 3) -> float:
        """Device milliseconds of this rank's own FFN work for one (layer,
        micro-batch): RMSNorm, gate/up GEMM with SwiGLU, down GEMM, over every
        layer and micro-batch with no waits and no hand-offs (the down GEMM
        writes a local buffer), replayed from a CUDA graph. A timing reference
        for the FFN GPUs' roofline, not a model computation; call it only
        while no other rank waits on this one."""
        s, lay, W = self.spec, self.layout, self.w
        T = lay.A * lay.rows
        epi = _lib.FG_EPI_RESIDUAL if lay.S == 1 else _lib.FG_EPI_F32
        out = torch.empty(T, s.hidden, dtype=torch.bfloat16 if lay.S == 1 else torch.float32, device=self.device)
        wd0 = W.layers[0]["w_down"]
        kernels.Workspace.get(_lib.lib().fg_gemm_workspace_bytes(T, s.hidden, wd0.K, 0), self.device,
                              self.slot + ".alone")

        def body():
            for i in range(s.num_layers):
                L = W.layers[i]
                for m in range(lay.micro_batches):
                    inp = self.in_view(m)
                    kernels.rmsnorm(inp, L["ln2"], s.eps, s.norm_mode, out=self.x)
                    act = kernels.gemm(self.x, L["w_gate_up"], epilogue=_lib.FG_EPI_SWIGLU, out=self.act,
                                       slot=self.slot)
                    kernels.gemm(act, L["w_down"], epilogue=epi, residual=inp if epi == _lib.FG_EPI_RESIDUAL else None,
                                 out=out, slot=self.slot + ".alone")

        g = torch.cuda.CUDAGraph()
        st = self.stream
        st.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(st), torch.inference_mode():
            with torch.cuda.graph(g, stream=st):
                body()
            g.replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                g.replay()
            e1.record()
        e1.synchronize()
        torch.cuda.current_stream(self.device).wait_stream(st)
        del g
        return e0.elapsed_time(e1) / (reps * s.num_layers * lay.micro_batches)

    def capture(self) -> None:
        g = torch.cuda.CUDAGraph()
        s = self.stream
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s), torch.inference_mode():
            with torch.cuda.graph(g, stream=s):
                self._step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.graph = g

    def release_graphs(self) -> None:
        self.graph = None


def preload(device: torch.device) -> None:
    """Load every kernel of the library on `device` before ranks start
    waiting on each other (fg_preload: under lazy loading a kernel's first
    launch waits for the device's work in flight, and a kernel spinning on
    another GPU's flag can be part of it)."""
    with torch.cuda.device(device):
        call("fg_preload")


class Fabric:
    """Makes every rank's mailbox reachable from the ranks of the other role
    (and loads the library's kernels on each rank's device first)."""

    @staticmethod
    def local(ranks: list[_Rank]) -> None:
        """Ranks of one process on one device: plain device pointers."""
        for d in {r.device for r in ranks}:
            preload(d)
        bases = {r.rank: r.mailbox.ptr for r in ranks}
        for r in ranks:
            r.peer_base = dict(bases)

    @staticmethod
    def ipc(rank: _Rank, group=None) -> "Fabric._Imports":
        """Ranks in separate processes: export this rank's mailbox through
        CUDA IPC, gather every rank's handle (torch.distributed), import the
        mailboxes of the other role. Returns the imports (close() them)."""
        import torch.distributed as dist

        preload(rank.device)
        torch.cuda.synchronize(rank.device)
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_size_t(0)
        call("fg_ipc_export", rank.mailbox.ptr, handle, ctypes.byref(off))
        world = dist.get_world_size(group)
        allh: list = [None] * world
        dist.all_gather_object(allh, (rank.rank, rank.role, bytes(handle.raw), off.value), group=group)
        imports = Fabric._Imports()
        rank.peer_base = {rank.rank: rank.mailbox.ptr}
        for r, role, h, o in allh:
            if r == rank.rank or role == rank.role:
                continue
            p = ctypes.c_void_p()
            call("fg_ipc_import", h, o, ctypes.byref(p))
            rank.peer_base[r] = p.value
            imports.items.append((p.value, o))
        dist.barrier(group=group)
        return imports

    class _Imports:
        def __init__(self) -> None:
            self.items: list[tuple[int, int]] = []

        def close(self) -> None:
            for ptr, off in self.items:
                call("fg_ipc_close", ptr, off)
            self.items.clear()


def nvlink_bytes_per_step(layout: DisaggLayout, hidden: int, layers: int) -> int:
    """Bytes every step moves between GPUs: per layer and micro-batch, each
    attention rank's h rows to every FFN rank (bf16) and every FFN rank's
    result rows back (bf16 with one FFN rank, fp32 partials otherwise)."""
    lay = layout
    out = lay.A * lay.S * lay.rows * hidden * 2
    back = lay.A * lay.S * lay.rows * hidden * (4 if lay.S > 1 else 2)
    return (out + back) * lay.micro_batches * layers
