"""Placement plans: the reference's profile.json format, parsed and validated
with the same rules, so plans written by planner.py / milp_planner.py /
schedule_llm_layers.py load unchanged.

Format (fluidgpu_runtime/fluidgpu_torch/profile.py:333-357): {model,
rank_count, task_count, hidden_size, num_kv_heads, head_dim, dtype,
max_seq_len, tasks: [{task_id, kernel_group_id, name, rank, decode_rank?}],
decode_weight?, predicted_cost_us?}. Task names: "embed", "norm_lm_head",
"layer_<i>" (expanded into layer_<i>_attn + layer_<i>_mlp), or
"layer_<i>_<suffix>" with the suffix sequences of profile.py:369-393.
Validation mirrors validate_profile (:108-167), except that rank_count may
be 1 (a co-located single-GPU plan).
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Iterable

import torch

ATTN_COARSE = ("attn",)
ATTN_FINE = ("qkv", "sdpa", "o_proj")
MLP_COARSE = ("mlp",)
MLP_FINE = ("mlp_gate_up", "mlp_down_proj")
MOE = ("moe_router", "moe_experts", "moe_combine")
VALID_SUFFIXES = set(ATTN_COARSE) | set(ATTN_FINE) | set(MLP_COARSE) | set(MLP_FINE) | set(MOE)
VALID_SEQUENCES = (
    ATTN_COARSE + MLP_COARSE,
    ATTN_FINE + MLP_COARSE,
    ATTN_COARSE + MLP_FINE,
    ATTN_FINE + MLP_FINE,
    ATTN_COARSE + MOE,
    ATTN_FINE + MOE,
)


SHARDABLE = ("mlp", "moe_experts")


@dataclass(frozen=True)
class TaskSpec:
    task_id: int
    kernel_group_id: int
    name: str
    rank: int
    decode_rank: int | None = None
    # Extension of the reference's plan format: a feed-forward group run by
    # several ranks at once, each on one shard (dense `mlp`: a slice of the
    # intermediate dimension; `moe_experts`: a range of experts). The rank of
    # the task before it sends it its input, every shard returns an fp32
    # partial, and the same rank, which runs the task after it, adds the
    # partials up (reduce-by-consumer). `rank` is then shard_ranks[0].
    shard_ranks: tuple[int, ...] | None = None

    def rank_for(self, mode: str) -> int:
        if mode == "decode" and self.decode_rank is not None:
            return self.decode_rank
        return self.rank


@dataclass(frozen=True)
class RuntimeProfile:
    model: str
    rank_count: int
    task_count: int
    tasks: tuple[TaskSpec, ...]
    hidden_size: int
    num_kv_heads: int
    head_dim: int
    dtype: torch.dtype
    max_seq_len: int
    decode_weight: float | None = None
    predicted_cost_us: dict[str, float] | None = None

    @property
    def task_by_name(self) -> dict[str, TaskSpec]:
        return {t.name: t for t in self.tasks}

    @property
    def task_index_by_name(self) -> dict[str, int]:
        return {t.name: i for i, t in enumerate(self.tasks)}


def dtype_from_name(name: str) -> torch.dtype:
    key = name.replace("torch.", "")
    table = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}
    assert key in table, f"unsupported dtype {name}"
    return table[key]


def dtype_name(dtype: torch.dtype) -> str:
    names = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}
    assert dtype in names, f"unsupported dtype {dtype}"
    return names[dtype]


def parse_layer_task(name: str) -> tuple[int, str] | None:
    if not name.startswith("layer_"):
        return None
    parts = name.split("_")
    assert len(parts) >= 2 and parts[1].isdigit(), f"invalid layer task name {name}"
    if len(parts) == 2:
        return int(parts[1]), "layer"
    suffix = "_".join(parts[2:])
    assert suffix in VALID_SUFFIXES, f"invalid layer task suffix in {name}"
    return int(parts[1]), suffix


def _parse_tasks(raw: list[dict[str, Any]]) -> tuple[TaskSpec, ...]:
    out: list[TaskSpec] = []
    for item in raw:
        name = str(item["name"])
        rank = int(item["rank"])
        decode_rank = item.get("decode_rank")
        layer = parse_layer_task(name)
        if decode_rank is not None:
            decode_rank = int(decode_rank)
            suffix = layer[1] if layer is not None else name
            # only the coarse FFN group may change rank between phases: fine
            # FFN groups route their aux tensors by the prefill rank
            assert suffix == "mlp", (
                "decode_rank is only supported on the coarse 'mlp' feed-forward group "
                f"(got {name})"
            )
        if layer is not None and layer[1] == "layer":
            for suffix in ("attn", "mlp"):
                tid = len(out)
                out.append(TaskSpec(tid, tid, f"layer_{layer[0]}_{suffix}", rank,
                                    decode_rank if suffix == "mlp" else None))
            continue
        shard_ranks = item.get("shard_ranks")
        if shard_ranks is not None:
            shard_ranks = tuple(int(r) for r in shard_ranks)
            suffix = layer[1] if layer is not None else name
            assert suffix in SHARDABLE, f"shard_ranks is only supported on {SHARDABLE} (got {name})"
            assert decode_rank is None, f"{name}: shard_ranks and decode_rank cannot be combined"
            assert len(shard_ranks) >= 1 and len(set(shard_ranks)) == len(shard_ranks), (
                f"{name}: shard_ranks must be distinct, got {shard_ranks}")
            assert rank == shard_ranks[0], f"{name}: rank must be shard_ranks[0]"
        tid = len(out)
        out.append(TaskSpec(tid, tid, name, rank, decode_rank, shard_ranks))
    return tuple(out)


def profile_from_dict(raw: dict[str, Any], *, model_name: str | None = None,
                      hf_config: Any | None = None) -> RuntimeProfile:
    tasks = _parse_tasks(raw["tasks"])
    hidden = int(raw.get("hidden_size", getattr(hf_config, "hidden_size", 0)))
    nkv = int(raw.get("num_kv_heads", getattr(hf_config, "num_key_value_heads", 0)))
    default_hd = hf_config.hidden_size // hf_config.num_attention_heads if hf_config is not None else 0
    head_dim = int(raw.get("head_dim", default_hd))
    assert hidden > 0, "profile hidden_size is required"
    assert nkv > 0, "profile num_kv_heads is required"
    assert head_dim > 0, "profile head_dim is required"
    prof = RuntimeProfile(
        model=str(raw["model"]), rank_count=int(raw["rank_count"]), task_count=len(tasks),
        tasks=tasks, hidden_size=hidden, num_kv_heads=nkv, head_dim=head_dim,
        dtype=dtype_from_name(str(raw.get("dtype", "bfloat16"))),
        max_seq_len=int(raw.get("max_seq_len", 2048)), decode_weight=raw.get("decode_weight"),
        predicted_cost_us=raw.get("predicted_cost_us"),
    )
    validate_profile(prof, model_name=model_name, hf_config=hf_config)
    return prof


def load_profile(path: str | Path, *, model_name: str | None = None,
                 hf_config: Any | None = None) -> RuntimeProfile:
    return profile_from_dict(json.loads(Path(path).read_text()), model_name=model_name,
                             hf_config=hf_config)


def _layer_ids(names: Iterable[str]) -> list[int]:
    return sorted({p[0] for n in names if (p := parse_layer_task(n)) is not None})


def validate_profile(profile: RuntimeProfile, *, model_name: str | None = None,
                     hf_config: Any | None = None) -> None:
    assert profile.rank_count >= 1, f"rank_count must be >= 1, got {profile.rank_count}"
    assert profile.task_count == len(profile.tasks), (
        f"task_count {profile.task_count} != len(tasks) {len(profile.tasks)}"
    )
    assert profile.dtype is torch.bfloat16, f"profile dtype must be bfloat16, got {profile.dtype}"
    assert profile.max_seq_len > 0, f"max_seq_len must be positive, got {profile.max_seq_len}"
    if model_name is not None:
        assert profile.model == model_name, f"profile model {profile.model} != requested {model_name}"
    names = [t.name for t in profile.tasks]
    assert len(names) == len(set(names)), "task names must be unique"
    assert names.count("embed") == 1, "profile must contain exactly one embed task"
    assert names.count("norm_lm_head") == 1, "profile must contain exactly one norm_lm_head task"
    for i, t in enumerate(profile.tasks):
        assert t.task_id == i, f"tasks must be sorted by task_id; index {i} has {t.task_id}"
        assert t.kernel_group_id == t.task_id, "kernel_group_id must match task_id"
        assert 0 <= t.rank < profile.rank_count, (
            f"invalid rank {t.rank} for {t.name} under rank_count={profile.rank_count}"
        )
        if t.decode_rank is not None:
            assert 0 <= t.decode_rank < profile.rank_count, f"invalid decode_rank for {t.name}"
        if t.shard_ranks is not None:
            assert all(0 <= r < profile.rank_count for r in t.shard_ranks), (
                f"invalid shard_ranks {t.shard_ranks} for {t.name} under rank_count={profile.rank_count}")
            assert 0 < i < len(profile.tasks) - 1, f"{t.name}: a sharded group needs a task before and after"
            before, after = profile.tasks[i - 1], profile.tasks[i + 1]
            assert before.shard_ranks is None and after.shard_ranks is None, (
                f"{t.name}: neighbouring tasks of a sharded group must not be sharded")
            assert before.decode_rank is None and after.decode_rank is None, (
                f"{t.name}: neighbouring tasks of a sharded group must keep one rank")
            assert before.rank == after.rank and before.rank not in t.shard_ranks, (
                f"{t.name}: the tasks before and after a sharded group must run on one rank outside it "
                "(it scatters the input and adds up the partials)")
    by_name = profile.task_by_name
    assert by_name["embed"].rank == 0, "embed must be assigned to rank 0"
    assert by_name["norm_lm_head"].rank == 0, "norm_lm_head must be assigned to rank 0"
    layer_ids = _layer_ids(names)
    assert layer_ids == list(range(len(layer_ids))), f"layers must be contiguous from 0, got {layer_ids}"
    index = profile.task_index_by_name
    for lid in layer_ids:
        seq = tuple(p[1] for t in profile.tasks if (p := parse_layer_task(t.name)) and p[0] == lid)
        assert seq in VALID_SEQUENCES, (
            f"layer_{lid} must use a supported attention/feed-forward task sequence, got {seq}"
        )
        idx = [index[f"layer_{lid}_{s}"] for s in seq]
        assert idx == list(range(idx[0], idx[0] + len(idx))), f"layer_{lid} tasks must be adjacent and ordered"
    if hf_config is not None:
        assert len(layer_ids) == hf_config.num_hidden_layers, "profile layer count != model layer count"
        assert profile.hidden_size == hf_config.hidden_size, "profile hidden_size != model hidden_size"
        assert profile.num_kv_heads == hf_config.num_key_value_heads, "profile num_kv_heads mismatch"
        hd = getattr(hf_config, "head_dim", None) or hf_config.hidden_size // hf_config.num_attention_heads
        assert profile.head_dim == hd, f"profile head_dim {profile.head_dim} != model head_dim {hd}"


def owned_layer_ids(profile: RuntimeProfile, rank: int) -> list[int]:
    """Layers whose KV cache lives on `rank` (the rank of attn / qkv)."""
    owned = []
    for t in profile.tasks:
        p = parse_layer_task(t.name)
        if p is not None and p[1] in ("attn", "qkv") and t.rank == rank:
            owned.append(p[0])
    return owned


def ffn_shard_of(profile: RuntimeProfile, rank: int) -> tuple[int, int] | None:
    """(index, count) of the feed-forward shard `rank` holds in this plan (the
    same for every sharded group), or None."""
    found = None
    for t in profile.tasks:
        if t.shard_ranks is not None and rank in t.shard_ranks:
            s = (t.shard_ranks.index(rank), len(t.shard_ranks))
            assert found in (None, s), f"rank {rank} holds different shards in different layers"
            found = s
    return found


def has_fine_groups(profile: RuntimeProfile) -> bool:
    """True when a layer's attention or dense FFN is split into sub-groups
    (qkv / sdpa / o_proj, mlp_gate_up / mlp_down_proj). Such plans prefill
    one position per pass through the decode kernels; the others prefill
    chunks of positions."""
    return any(n.endswith(("_qkv", "_mlp_gate_up")) for n in profile.task_index_by_name)


def kv_layer_ids(profile: RuntimeProfile, rank: int) -> list[int]:
    """Layers whose paged KV lives on `rank`: where the attention reads it
    (attn, or sdpa in a split plan). Equal to owned_layer_ids except when
    qkv and sdpa sit on different ranks: the reference then appends on the
    qkv rank and ships q plus the whole K/V view to sdpa every step
    (runner.py:284-296, :462-472); here the qkv rank ships only the new
    token's projected qkv row and the sdpa rank appends it to its own pages."""
    owned = []
    for t in profile.tasks:
        p = parse_layer_task(t.name)
        if p is not None and p[1] in ("attn", "sdpa") and t.rank == rank:
            owned.append(p[0])
    return owned


def make_ranked_task_profile(*, model: str, task_assignments: list[tuple[str, Any]],
                             hidden_size: int, num_kv_heads: int, head_dim: int,
                             max_seq_len: int = 2048, dtype: torch.dtype = torch.bfloat16,
                             rank_count: int | None = None) -> dict[str, Any]:
    """Plan dict with embed/norm_lm_head on rank 0 around the given tasks. A
    rank given as a list makes the task a sharded group over those ranks."""
    def ranks_of(r: Any) -> list[int]:
        return list(r) if isinstance(r, (list, tuple)) else [r]

    top = max((x for _, r in task_assignments for x in ranks_of(r)), default=0)
    n_ranks = rank_count if rank_count is not None else max(1, top + 1)
    tasks = [{"task_id": 0, "kernel_group_id": 0, "name": "embed", "rank": 0}]
    for name, rank in task_assignments:
        rs = ranks_of(rank)
        assert all(0 <= x < n_ranks for x in rs), f"invalid rank {rank} for {name} under rank_count={n_ranks}"
        tid = len(tasks)
        t = {"task_id": tid, "kernel_group_id": tid, "name": name, "rank": rs[0]}
        if isinstance(rank, (list, tuple)):
            t["shard_ranks"] = rs
        tasks.append(t)
    tid = len(tasks)
    tasks.append({"task_id": tid, "kernel_group_id": tid, "name": "norm_lm_head", "rank": 0})
    return {"model": model, "rank_count": n_ranks, "task_count": len(tasks),
            "hidden_size": hidden_size, "num_kv_heads": num_kv_heads, "head_dim": head_dim,
            "dtype": dtype_name(dtype), "max_seq_len": max_seq_len, "tasks": tasks}


def sharded_ffn_profile(model: str, num_layers: int, hidden_size: int, num_kv_heads: int,
                        head_dim: int, max_seq_len: int, shard_ranks: list[int],
                        moe: bool = False) -> dict[str, Any]:
    """Attention (and embed, head, MoE router and combine) on rank 0, every
    layer's feed-forward group sharded over shard_ranks: the tensor-parallel
    FFN of config 4 (intermediate split) or the expert-parallel MoE of
    config 3 (experts split)."""
    tasks: list[tuple[str, Any]] = []
    for i in range(num_layers):
        tasks.append((f"layer_{i}_attn", 0))
        if moe:
            tasks += [(f"layer_{i}_moe_router", 0), (f"layer_{i}_moe_experts", list(shard_ranks)),
                      (f"layer_{i}_moe_combine", 0)]
        else:
            tasks.append((f"layer_{i}_mlp", list(shard_ranks)))
    return make_ranked_task_profile(model=model, task_assignments=tasks, hidden_size=hidden_size,
                                    num_kv_heads=num_kv_heads, head_dim=head_dim, max_seq_len=max_seq_len,
                                    rank_count=1 + max(shard_ranks))


def colocated_profile(model: str, num_layers: int, hidden_size: int, num_kv_heads: int,
                      head_dim: int, max_seq_len: int, moe: bool = False) -> dict[str, Any]:
    """Every task on rank 0 (the 1-GPU configuration)."""
    tasks = []
    for i in range(num_layers):
        tasks.append((f"layer_{i}_attn", 0))
        if moe:
            tasks += [(f"layer_{i}_moe_router", 0), (f"layer_{i}_moe_experts", 0), (f"layer_{i}_moe_combine", 0)]
        else:
            tasks.append((f"layer_{i}_mlp", 0))
    return make_ranked_task_profile(model=model, task_assignments=tasks, hidden_size=hidden_size,
                                    num_kv_heads=num_kv_heads, head_dim=head_dim,
                                    max_seq_len=max_seq_len, rank_count=1)


def attn_ffn_profile(model: str, num_layers: int, hidden_size: int, num_kv_heads: int,
                     head_dim: int, max_seq_len: int, attn_rank: int = 0, ffn_rank: int = 1,
                     moe: bool = False) -> dict[str, Any]:
    """Attention on attn_rank, FFN on ffn_rank: the AF placement of configs 1-2."""
    tasks = []
    for i in range(num_layers):
        tasks.append((f"layer_{i}_attn", attn_rank))
        if moe:
            tasks += [(f"layer_{i}_moe_router", ffn_rank), (f"layer_{i}_moe_experts", ffn_rank),
                      (f"layer_{i}_moe_combine", ffn_rank)]
        else:
            tasks.append((f"layer_{i}_mlp", ffn_rank))
    return make_ranked_task_profile(model=model, task_assignments=tasks, hidden_size=hidden_size,
                                    num_kv_heads=num_kv_heads, head_dim=head_dim,
                                    max_seq_len=max_seq_len, rank_count=max(attn_rank, ffn_rank) + 1)
