"""Engine configuration, field-compatible with fluidgpu_torch.config.EngineConfig
(fluidgpu_runtime/fluidgpu_torch/config.py:15-67).

Differences, each because the B200 path generalises the reference:
  - world_size may be 1 (co-located attention + FFN on one GPU);
  - max_batch sizes the batched decode buffers (the reference is batch 1);
  - block_size is the paged-KV page (16 tokens).
The reference's bf16-only assertion is kept.
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Literal

import torch


@dataclass(frozen=True)
class EngineConfig:
    model_name: str
    profiling_json: str | Path | None = None
    dtype: torch.dtype = torch.bfloat16
    max_seq_len: int = 2048
    master_addr: str = "127.0.0.1"
    master_port: int = 29500
    rank_override: int | None = None
    device_id: int = 0
    device: str | None = None
    world_size: int = 2
    preallocate_recv_buffers: bool = True
    cuda_graph_decode: bool = False
    strict_transformers_version: bool = True
    monitor_output: str | Path | None = None
    comm_transport: Literal["auto", "rdma", "nvlink"] = "auto"
    nccl_socket_ifname: str | None = None
    nccl_ib_hca: str | None = None
    rdma_hca_by_rank: tuple[str, ...] = ("<set-rank0-ib-hca>", "<set-rank1-ib-hca>")
    nccl_ib_gid_index: int | None = None
    max_batch: int = 1
    block_size: int = 16
    # paged-KV block allocation: "vllm" (vLLM BlockPool order, blocks added as
    # sequences grow) or "reserve" (each sequence's expected length up front)
    kv_allocation: str = "vllm"

    def __post_init__(self) -> None:
        assert self.dtype is torch.bfloat16, f"dtype must be torch.bfloat16, got {self.dtype}"
        assert self.max_seq_len > 0, f"max_seq_len must be positive, got {self.max_seq_len}"
        assert self.world_size >= 1, f"world_size must be >= 1, got {self.world_size}"
        assert self.device_id >= 0, f"device_id must be non-negative, got {self.device_id}"
        assert self.comm_transport in ("auto", "rdma", "nvlink"), (
            f"comm_transport must be auto, rdma or nvlink, got {self.comm_transport}"
        )
        assert self.max_batch >= 1, f"max_batch must be >= 1, got {self.max_batch}"
        assert self.block_size == 16, f"block_size must be 16, got {self.block_size}"
        assert self.kv_allocation in ("vllm", "reserve"), f"bad kv_allocation {self.kv_allocation}"
        if self.rank_override is not None:
            assert 0 <= self.rank_override < self.world_size, (
                f"rank_override must be in [0, {self.world_size}), got {self.rank_override}"
            )

    @property
    def torch_device(self) -> torch.device:
        if self.device is not None:
            return torch.device(self.device)
        return torch.device(f"cuda:{self.device_id}")

    @property
    def profiling_path(self) -> Path:
        assert self.profiling_json is not None, "profiling_json is required"
        return Path(self.profiling_json)
