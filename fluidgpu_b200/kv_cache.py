"""Paged KV cache with the surface of fluidgpu_torch.kv_cache.LayerKVCache
(fluidgpu_runtime/fluidgpu_torch/kv_cache.py:21-166): owned, static_mode,
max_seq_len, update, get_seq_length, get_mask_sizes, advance, reset.

Layout in HBM. Every owned layer has K and V page pools
  [num_blocks, n_kv, 16, head_dim] bf16
held in one allocation [n_owned, 2, num_blocks, n_kv, 16, head_dim], so a
page of one KV head is a contiguous 2-4 KB run (what the attention kernel's
TMA box fetches). All layers share one block table [max_batch, max_blocks]
int32: sequence b's page p lives in block block_table[b, p] of every layer.
Device-side per-sequence counters:
  positions[b] = tokens already cached = position of the next token
  seq_lens[b]  = positions[b] + 1       = tokens attended during a step
Both advance on the device (fg_advance), so a decode step needs no host
round trip; a host mirror tracks the same counts for planning.

Block allocation (allocation="vllm", the default) follows vLLM's BlockPool
(vllm/v1/core/block_pool.py, the allocator behind the reference's vLLM
integration): block 0 is the reserved null block, free blocks form a FIFO
queue (lowest id first), a sequence gets the blocks its prompt needs when the
batch starts and one more block whenever a step would run past its last one
(prepare_step, sequences in batch order), and a finished sequence returns its
blocks tail-first. The block tables therefore equal vLLM's for the same
requests (tests/test_block_table_vllm.py runs vLLM's own BlockPool beside
it). allocation="reserve" instead reserves each sequence's whole expected
length up front (lowest ids first, no null block).
"""
from __future__ import annotations

import collections
from typing import Any

import torch

from . import kernels

BLOCK = 16


class BlockAllocator:
    """FIFO free-list of physical block ids (deterministic). With null_block,
    block 0 is never handed out (vLLM's placeholder block)."""

    def __init__(self, num_blocks: int, null_block: bool = False) -> None:
        self.num_blocks = num_blocks
        self._free = collections.deque(range(1 if null_block else 0, num_blocks))

    @property
    def num_free(self) -> int:
        return len(self._free)

    def allocate(self, n: int) -> list[int]:
        assert n <= len(self._free), f"out of KV blocks: need {n}, have {len(self._free)}"
        return [self._free.popleft() for _ in range(n)]

    def free(self, blocks: list[int]) -> None:
        self._free.extend(blocks)


class PagedKVCache:
    def __init__(self, num_layers: int, owned_layer_ids: list[int] | tuple[int, ...],
                 max_seq_len: int, num_kv_heads: int, head_dim: int, dtype: torch.dtype,
                 device: torch.device | str, *, max_batch: int = 1,
                 num_blocks: int | None = None, allocation: str = "vllm") -> None:
        assert dtype is torch.bfloat16, "the paged cache holds bf16"
        assert allocation in ("vllm", "reserve"), f"unknown allocation policy {allocation}"
        self.allocation = allocation
        self.num_layers = num_layers
        self.owned = set(owned_layer_ids)
        self.max_seq_len = max_seq_len
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        self.max_batch = max_batch
        self.max_blocks = (max_seq_len + BLOCK - 1) // BLOCK
        null = allocation == "vllm"
        self.num_blocks = num_blocks if num_blocks is not None else max_batch * self.max_blocks + int(null)
        self.static_mode = False
        self._slot = {lid: i for i, lid in enumerate(sorted(self.owned))}
        n_owned = len(self._slot)
        self.pool = torch.zeros((max(n_owned, 1), 2, self.num_blocks, num_kv_heads, BLOCK, head_dim),
                                dtype=dtype, device=self.device) if n_owned else None
        self.block_table = torch.full((max_batch, self.max_blocks), -1, dtype=torch.int32,
                                      device=self.device)
        # host mirror of the block table (pinned), copied to the device in one
        # asynchronous copy when a step adds blocks; entries only grow until
        # the next batch, so a copy that runs late still holds every entry
        # the kernels before it read
        self._bt_host = torch.full((max_batch, self.max_blocks), -1, dtype=torch.int32,
                                   pin_memory=self.device.type == "cuda")
        self.positions = torch.zeros(max_batch, dtype=torch.int32, device=self.device)
        self.seq_lens = torch.ones(max_batch, dtype=torch.int32, device=self.device)
        self.allocator = BlockAllocator(self.num_blocks, null_block=null)
        self._blocks: list[list[int]] = [[] for _ in range(max_batch)]
        self._host_pos = [0] * max_batch
        self.batch = 0
        # attention split plan length used while capturing a CUDA graph (the
        # captured launch must stay valid as sequences grow within a bucket)
        self.plan_len_override: int | None = None

    # -- layout ----------------------------------------------------------------
    def layer_pages(self, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        assert layer_idx in self.owned, f"layer {layer_idx} not owned by this rank"
        s = self._slot[layer_idx]
        return self.pool[s, 0], self.pool[s, 1]

    def host_block_table(self) -> list[list[int]]:
        return [list(b) for b in self._blocks[: self.batch]]

    # -- request admission -----------------------------------------------------
    def start_batch(self, lengths: list[int], reserve: list[int] | int) -> None:
        """Begin a batch of len(lengths) sequences with lengths[b] tokens already
        cached, reserving pages for reserve[b] total tokens each."""
        self.reset()
        B = len(lengths)
        assert 1 <= B <= self.max_batch, f"batch {B} exceeds max_batch {self.max_batch}"
        res = [reserve] * B if isinstance(reserve, int) else list(reserve)
        table = torch.full((self.max_batch, self.max_blocks), -1, dtype=torch.int32)
        for b in range(B):
            total = max(res[b], lengths[b] + 1)
            assert total <= self.max_seq_len, f"exceed max_seq_len: {total} > {self.max_seq_len}"
            if self.allocation == "vllm":
                total = lengths[b]  # the prompt's blocks; the rest come step by step
            nb = (total + BLOCK - 1) // BLOCK
            self._blocks[b] = self.allocator.allocate(nb)
            table[b, :nb] = torch.tensor(self._blocks[b], dtype=torch.int32)
        self._bt_host.copy_(table)
        self.block_table.copy_(table)
        pos = torch.zeros(self.max_batch, dtype=torch.int32)
        pos[:B] = torch.tensor(lengths, dtype=torch.int32)
        self.positions.copy_(pos)
        self.seq_lens.copy_(pos + 1)
        self._host_pos = list(lengths) + [0] * (self.max_batch - B)
        self.batch = B

    def prepare_step(self, n: int = 1) -> None:
        """Give every sequence the blocks its next n tokens need (vLLM order:
        sequences in batch order, one FIFO allocation each), writing the new
        block-table entries on the current stream. Not while a CUDA graph is
        being captured (the graph must not hold these host copies)."""
        if self.allocation != "vllm" or (self.block_table.is_cuda and torch.cuda.is_current_stream_capturing()):
            return
        dirty = False
        for b in range(self.batch):
            need = (self._host_pos[b] + n + BLOCK - 1) // BLOCK
            have = len(self._blocks[b])
            if need > have:
                assert need <= self.max_blocks, f"exceed max_seq_len: {self._host_pos[b] + n}"
                new = self.allocator.allocate(need - have)
                self._blocks[b].extend(new)
                for j, blk in enumerate(new):
                    self._bt_host[b, have + j] = blk
                dirty = True
        if dirty:
            self.block_table.copy_(self._bt_host, non_blocking=True)

    # -- LayerKVCache surface --------------------------------------------------
    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: dict[str, Any] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Append key/value states [B, n_kv, S, hd] at each sequence's current
        position (or cache_kwargs['cache_position'] for batch 1); returns the
        layer's page pools (read through the block table)."""
        assert layer_idx in self.owned, f"layer {layer_idx} not owned by this rank"
        assert key_states.shape == value_states.shape, "key/value shapes must match"
        B, nkv, S, hd = key_states.shape
        assert nkv == self.num_kv_heads, f"num_kv_heads mismatch: got {nkv}, expected {self.num_kv_heads}"
        assert hd == self.head_dim, f"head_dim mismatch: got {hd}, expected {self.head_dim}"
        if B > self.batch:
            self.start_batch([0] * B, self.max_seq_len)
        self.prepare_step(S)
        cp = None if cache_kwargs is None else cache_kwargs.get("cache_position")
        if cp is not None and B == 1:
            pos = cp.flatten().to(device=self.device, dtype=torch.int32)
        else:
            base = self.positions[:B].to(torch.int32)
            pos = (base[:, None] + torch.arange(S, device=self.device, dtype=torch.int32)[None, :]).reshape(-1)
        seq = torch.arange(B, device=self.device, dtype=torch.int32).repeat_interleave(S)
        k = key_states.permute(0, 2, 1, 3).reshape(B * S, nkv, hd).contiguous()
        v = value_states.permute(0, 2, 1, 3).reshape(B * S, nkv, hd).contiguous()
        kp, vp = self.layer_pages(layer_idx)
        kernels.kv_append(k, v, seq, pos, self.block_table, kp, vp)
        return kp, vp

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return max(self._host_pos[: max(self.batch, 1)])

    def seq_lengths(self) -> list[int]:
        return list(self._host_pos[: self.batch])

    def get_max_length(self) -> int:
        return self.max_seq_len

    def get_max_cache_shape(self) -> int:
        return self.max_seq_len

    def get_mask_sizes(self, cache_position: torch.Tensor, layer_idx: int | None = None) -> tuple[int, int]:
        assert cache_position.numel() > 0, "cache_position must not be empty"
        if self.static_mode:
            return self.max_seq_len, 0
        kv_length = int(cache_position.flatten()[-1].item()) + 1
        assert kv_length <= self.max_seq_len, f"exceed max_seq_len: {kv_length} > {self.max_seq_len}"
        return kv_length, 0

    def get_usable_length(self, new_seq_length: int, layer_idx: int = 0) -> int:
        """Cached tokens a step of new_seq_length more can still attend to
        (kv_cache.py:135-138), for the longest sequence of the batch."""
        cur = self.get_seq_length(layer_idx)
        if cur + new_seq_length <= self.max_seq_len:
            return cur
        return self.max_seq_len - new_seq_length

    def advance(self, seq_len: int) -> None:
        assert seq_len > 0, f"seq_len must be positive, got {seq_len}"
        for b in range(self.batch):
            nxt = self._host_pos[b] + seq_len
            assert nxt <= self.max_seq_len, f"exceed max_seq_len: {nxt} > {self.max_seq_len}"
            assert nxt < len(self._blocks[b]) * BLOCK + 1, "sequence ran past its reserved pages"
            self._host_pos[b] = nxt
        if seq_len == 1:
            kernels.advance(self.positions, self.seq_lens)
        else:  # a prefill chunk: one counter update on the device
            self.positions[: self.batch] += seq_len
            self.seq_lens[: self.batch] += seq_len

    def max_attended(self) -> int:
        """Longest attention span of the coming step (host mirror)."""
        return max(self._host_pos[: max(self.batch, 1)]) + 1

    def bucket(self, n: int) -> int:
        """Power-of-two length bucket (>= 256, <= max_seq_len) holding n tokens."""
        b = 256
        while b < n:
            b *= 2
        return min(b, self.max_seq_len)

    def plan_len(self) -> int:
        """Length the attention kernels plan their page splits for: the bucket
        of the coming step's longest sequence, so eager steps and CUDA graphs
        captured for that bucket launch identical plans (identical results)."""
        if self.plan_len_override is not None:
            return self.plan_len_override
        return self.bucket(self.max_attended())

    def host_advance(self, seq_len: int) -> None:
        """Advance only the host mirror (after a replayed CUDA graph advanced
        the device counters)."""
        for b in range(self.batch):
            self._host_pos[b] += seq_len
            assert self._host_pos[b] < len(self._blocks[b]) * BLOCK + 1, "sequence ran past its reserved pages"

    def snapshot_host(self) -> list[int]:
        return list(self._host_pos)

    def restore_host(self, snap: list[int]) -> None:
        self._host_pos = list(snap)

    def reset(self) -> None:
        for b in range(self.max_batch):
            if self._blocks[b]:
                # vLLM frees a finished request's blocks tail-first
                self.allocator.free(self._blocks[b][::-1] if self.allocation == "vllm" else self._blocks[b])
                self._blocks[b] = []
        self._host_pos = [0] * self.max_batch
        self.batch = 0
        if self.block_table.is_cuda:  # a pending table copy may still read the host mirror
            torch.cuda.current_stream(self.device).synchronize()
        self._bt_host.fill_(-1)
        if self.positions.is_cuda:
            self.positions.zero_()
            self.seq_lens.fill_(1)
            self.block_table.fill_(-1)

    def reorder_cache(self, beam_idx: torch.LongTensor) -> None:
        raise NotImplementedError("beam search is not supported")
