"""Placement plans and the executor's rank-boundary protocol, on CPU.

Mirrors the reference's own tests of the same behaviour:
  test_profile.py / test_per_phase_placement.py (plan validation),
  test_executor_boundary.py:27-56 (send/recv shapes and order per rank),
  test_fine_dense_runtime.py:103-141 (two ranks as threads, bounded joins).
"""
import json
import threading

import pytest
import torch

from fluidgpu_b200.comm import QueueComm
from fluidgpu_b200.config import EngineConfig
from fluidgpu_b200.executor import LayerExecutor
from fluidgpu_b200.profile import (attn_ffn_profile, colocated_profile, load_profile,
                                   make_ranked_task_profile, owned_layer_ids, profile_from_dict)


class FakeComm:
    def __init__(self, rank):
        self.rank = rank
        self.send_log, self.recv_log = [], []

    def get_rank(self):
        return self.rank

    def send_tensor(self, tensor, dst):
        self.send_log.append((tuple(tensor.shape), dst))

    def recv_tensor(self, tensor, src):
        self.recv_log.append((tuple(tensor.shape), src))
        tensor.fill_(src + 1)


def _cfg(**kw):
    base = dict(model_name="m", device="cpu", max_seq_len=8, dtype=torch.bfloat16, max_batch=3)
    base.update(kw)
    return EngineConfig(**base)


def _run_layers(ex, B, layers):
    calls = []
    h = torch.zeros(B, 1, 4, dtype=torch.bfloat16)
    h = ex.run_stage("embed", lambda x: x, h, mode="decode", seq_len=1)
    for i in range(layers):
        for suffix in ("attn", "mlp"):
            name = f"layer_{i}_{suffix}"

            def fn(x, name=name):
                calls.append(name)
                return x + 1

            out = ex.run_kernel_group(name, fn, h, mode="decode", seq_len=1, batch=B)
            h = out if out is not None else h
    ex.run_stage("norm_lm_head", lambda x: x, h, mode="decode", seq_len=1, batch=B)
    return calls


def test_af_split_boundaries_batched():
    """Attention on rank 0, FFN on rank 1: one hand-off each way per layer,
    with [B,1,H] hidden states (the reference hands off [1,1,H])."""
    prof = profile_from_dict(attn_ffn_profile("m", 2, 4, 2, 2, 8))
    ex0 = LayerExecutor(prof, _cfg(), FakeComm(0))
    ex1 = LayerExecutor(prof, _cfg(), FakeComm(1))
    calls0 = _run_layers(ex0, 3, 2)
    calls1 = _run_layers(ex1, 3, 2)
    assert calls0 == ["layer_0_attn", "layer_1_attn"]
    assert calls1 == ["layer_0_mlp", "layer_1_mlp"]
    c0, c1 = ex0._comm, ex1._comm
    assert c0.send_log == [((3, 1, 4), 1), ((3, 1, 4), 1)]
    assert c0.recv_log == [((3, 1, 4), 1), ((3, 1, 4), 1)]
    assert c1.send_log == [((3, 1, 4), 0), ((3, 1, 4), 0)]
    assert c1.recv_log == [((3, 1, 4), 0), ((3, 1, 4), 0)]


def test_colocated_plan_never_hands_off():
    prof = profile_from_dict(colocated_profile("m", 3, 4, 2, 2, 8))
    ex = LayerExecutor(prof, _cfg(), FakeComm(0))
    calls = _run_layers(ex, 2, 3)
    assert len(calls) == 6 and not ex._comm.send_log and not ex._comm.recv_log
    assert owned_layer_ids(prof, 0) == [0, 1, 2]


def test_reference_layer_plan_format_loads(tmp_path):
    """A plan in the reference's coarse "layer_<i>" form (profiles/*.json) loads
    and expands to attn + mlp tasks."""
    raw = {"model": "m", "rank_count": 2, "task_count": 4, "hidden_size": 4, "num_kv_heads": 2,
           "head_dim": 2, "dtype": "bfloat16", "max_seq_len": 8,
           "tasks": [{"task_id": 0, "kernel_group_id": 0, "name": "embed", "rank": 0},
                     {"task_id": 1, "kernel_group_id": 1, "name": "layer_0", "rank": 0},
                     {"task_id": 2, "kernel_group_id": 2, "name": "layer_1", "rank": 1},
                     {"task_id": 3, "kernel_group_id": 3, "name": "norm_lm_head", "rank": 0}]}
    p = tmp_path / "plan.json"
    p.write_text(json.dumps(raw))
    prof = load_profile(p)
    names = [t.name for t in prof.tasks]
    assert names == ["embed", "layer_0_attn", "layer_0_mlp", "layer_1_attn", "layer_1_mlp", "norm_lm_head"]
    assert owned_layer_ids(prof, 0) == [0] and owned_layer_ids(prof, 1) == [1]
    # as in the reference (profile.py:403-421), decode_rank is refused on the
    # coarse layer task and on fine FFN groups, and honoured on "mlp"
    raw["tasks"][1]["decode_rank"] = 1
    with pytest.raises(AssertionError, match="decode_rank is only supported"):
        profile_from_dict(raw)
    per_phase = make_ranked_task_profile(model="m", task_assignments=[
        ("layer_0_attn", 0), ("layer_0_mlp", 0)], hidden_size=4, num_kv_heads=2, head_dim=2,
        rank_count=2)
    per_phase["tasks"][2]["decode_rank"] = 1
    prof = profile_from_dict(per_phase)
    mlp = prof.task_by_name["layer_0_mlp"]
    assert mlp.rank_for("decode") == 1 and mlp.rank_for("prefill") == 0
    # KV ownership follows the attention task, never decode_rank
    # (test_per_phase_placement.py:48-53 in the reference)
    assert owned_layer_ids(prof, 0) == [0] and owned_layer_ids(prof, 1) == []


@pytest.mark.parametrize("mutate,msg", [
    (lambda r: r["tasks"].__setitem__(0, {**r["tasks"][0], "rank": 1}), "embed must be assigned to rank 0"),
    (lambda r: r.__setitem__("dtype", "float32"), "bfloat16"),
    (lambda r: r["tasks"].pop(1), "supported attention/feed-forward task sequence"),
    (lambda r: r["tasks"][1].__setitem__("decode_rank", 1), "decode_rank is only supported"),
])
def test_plan_validation_errors(mutate, msg):
    raw = attn_ffn_profile("m", 1, 4, 2, 2, 8)
    mutate(raw)
    with pytest.raises(AssertionError, match=msg):
        profile_from_dict(raw)


def test_fine_sequence_rules():
    ok = make_ranked_task_profile(model="m", task_assignments=[
        ("layer_0_qkv", 0), ("layer_0_sdpa", 1), ("layer_0_o_proj", 0),
        ("layer_0_mlp_gate_up", 1), ("layer_0_mlp_down_proj", 0)], hidden_size=4, num_kv_heads=2, head_dim=2)
    profile_from_dict(ok)
    bad = make_ranked_task_profile(model="m", task_assignments=[
        ("layer_0_qkv", 0), ("layer_0_mlp", 0), ("layer_0_sdpa", 0)], hidden_size=4, num_kv_heads=2, head_dim=2)
    with pytest.raises(AssertionError, match="supported attention/feed-forward task sequence"):
        profile_from_dict(bad)


def test_two_ranks_as_threads_no_deadlock():
    """Two executors in two threads exchanging real tensors through bounded
    queues: both finish, values flow attn(+1) -> mlp(+1) per layer."""
    prof = profile_from_dict(attn_ffn_profile("m", 3, 4, 2, 2, 8))
    ch = QueueComm.make_channels(2)
    exs = [LayerExecutor(prof, _cfg(), QueueComm(r, ch)) for r in (0, 1)]
    results, errors = {}, []

    def go(r):
        try:
            h = torch.zeros(2, 1, 4, dtype=torch.bfloat16)
            h = exs[r].run_stage("embed", lambda x: x, h, mode="decode", seq_len=1)
            for i in range(3):
                for suffix in ("attn", "mlp"):
                    out = exs[r].run_kernel_group(f"layer_{i}_{suffix}", lambda x: x + 1, h,
                                                  mode="decode", seq_len=1, batch=2)
                    h = out if out is not None else h
            results[r] = exs[r].run_stage("norm_lm_head", lambda x: x, h, mode="decode", seq_len=1, batch=2)
        except BaseException as exc:  # noqa: BLE001
            errors.append(exc)

    ts = [threading.Thread(target=go, args=(r,)) for r in (0, 1)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=10)
    assert not errors and all(not t.is_alive() for t in ts)
    assert results[1] is None
    assert torch.equal(results[0], torch.full((2, 1, 4), 6.0, dtype=torch.bfloat16))


def test_lost_message_times_out_on_host():
    """A peer that never sends: the receiver fails with a bounded timeout
    instead of hanging (host-side failure detection)."""
    ch = QueueComm.make_channels(2)
    c = QueueComm(1, ch, timeout_s=0.2)
    with pytest.raises(TimeoutError):
        c.recv_tensor(torch.zeros(2, 1, 4), src=0)


def test_fine_attention_edge_widths_and_kv_placement():
    """A split attention: qkv and o_proj on rank 0, sdpa on rank 1. Rank 0
    receives the sdpa output at its own width (n_q * head_dim, here 6 while the
    hidden size is 4); the KV pages live where sdpa reads them."""
    from fluidgpu_b200.profile import kv_layer_ids

    prof = profile_from_dict(make_ranked_task_profile(model="m", task_assignments=[
        ("layer_0_qkv", 0), ("layer_0_sdpa", 1), ("layer_0_o_proj", 0), ("layer_0_mlp", 1)],
        hidden_size=4, num_kv_heads=2, head_dim=2))
    assert owned_layer_ids(prof, 0) == [0]  # the reference's rule: the qkv rank
    assert kv_layer_ids(prof, 0) == [] and kv_layer_ids(prof, 1) == [0]
    comm = FakeComm(0)
    ex = LayerExecutor(prof, _cfg(), comm)
    h = torch.zeros(3, 1, 4, dtype=torch.bfloat16)
    seen = {}
    for name, width in (("layer_0_qkv", None), ("layer_0_sdpa", None), ("layer_0_o_proj", 6)):
        kw = {"recv_width": width} if width else {}
        def fn(x, name=name):
            seen[name] = x.clone()
            return torch.zeros(3, 1, 4, dtype=torch.bfloat16)

        out = ex.run_kernel_group(name, fn, h, mode="decode", seq_len=1, batch=3, **kw)
        h = out if out is not None else h
    assert "layer_0_sdpa" not in seen
    assert tuple(seen["layer_0_o_proj"].shape) == (3, 1, 6)
    assert comm.send_log == [((3, 1, 4), 1), ((3, 1, 4), 1)]  # qkv -> sdpa, o_proj -> mlp
    assert comm.recv_log == [((3, 1, 6), 1)]


def test_sharded_group_plan_rules():
    from fluidgpu_b200.profile import ffn_shard_of, sharded_ffn_profile

    prof = profile_from_dict(sharded_ffn_profile("m", 2, 4, 2, 2, 8, shard_ranks=[1, 2, 3]))
    assert prof.rank_count == 4
    assert [ffn_shard_of(prof, r) for r in range(4)] == [None, (0, 3), (1, 3), (2, 3)]
    assert owned_layer_ids(prof, 0) == [0, 1]
    moe = profile_from_dict(sharded_ffn_profile("m", 1, 4, 2, 2, 8, shard_ranks=[1, 2], moe=True))
    assert moe.task_by_name["layer_0_moe_experts"].shard_ranks == (1, 2)
    bad = [
        ([("layer_0_attn", 0), ("layer_0_mlp", [0, 1])], "outside it"),        # producer among the shards
        ([("layer_0_attn", 1), ("layer_0_mlp", [2, 3])], "outside it"),        # producer 1, consumer 0
        ([("layer_0_attn", [0, 1]), ("layer_0_mlp", 0)], "only supported on"),  # attention cannot shard
    ]
    for tasks, msg in bad:
        raw = make_ranked_task_profile(model="m", task_assignments=tasks, hidden_size=4, num_kv_heads=2,
                                       head_dim=2, rank_count=4)
        with pytest.raises(AssertionError, match=msg):
            profile_from_dict(raw)


def test_sharded_group_scatter_and_reduce(monkeypatch):
    """Rank 0 runs attention, ranks 1 and 2 each run a shard of the FFN: both
    shards receive rank 0's output, each returns an fp32 partial, and rank 0
    adds them up (shard order) before the next task."""
    from fluidgpu_b200 import kernels
    from fluidgpu_b200.profile import sharded_ffn_profile

    def sum_partials(parts, out=None):
        total = parts.sum(0).to(torch.bfloat16)
        if out is not None:
            out.copy_(total)
            return out
        return total

    monkeypatch.setattr(kernels, "sum_partials", sum_partials)
    prof = profile_from_dict(sharded_ffn_profile("m", 2, 4, 2, 2, 8, shard_ranks=[1, 2]))
    ch = QueueComm.make_channels(3)
    exs = [LayerExecutor(prof, _cfg(), QueueComm(r, ch)) for r in range(3)]
    seen, results, errors = [], {}, []

    def go(r):
        try:
            h = torch.zeros(2, 1, 4, dtype=torch.bfloat16)
            h = exs[r].run_stage("embed", lambda x: x, h, mode="decode", seq_len=1)
            for i in range(2):
                out = exs[r].run_kernel_group(f"layer_{i}_attn", lambda x: x + 1, h, mode="decode",
                                              seq_len=1, batch=2)
                h = out if out is not None else h

                def mlp(x, shard, r=r, i=i):
                    seen.append((r, i, shard))
                    return (x.float() * (shard[0] + 1))  # partial of shard k = (k+1) * input

                out = exs[r].run_kernel_group(f"layer_{i}_mlp", mlp, h, mode="decode", seq_len=1, batch=2)
                h = out if out is not None else h
            results[r] = exs[r].run_stage("norm_lm_head", lambda x: x, h, mode="decode", seq_len=1, batch=2)
        except BaseException as exc:  # noqa: BLE001
            errors.append(exc)

    ts = [threading.Thread(target=go, args=(r,)) for r in range(3)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=10)
    assert not errors and all(not t.is_alive() for t in ts), errors
    assert sorted(seen) == [(1, 0, (0, 2)), (1, 1, (0, 2)), (2, 0, (1, 2)), (2, 1, (1, 2))]
    assert results[1] is None and results[2] is None
    # layer 0: attn 0 -> 1, mlp 1*1 + 2*1 = 3; layer 1: attn 4, mlp 4 + 8 = 12
    assert torch.equal(results[0], torch.full((2, 1, 4), 12.0, dtype=torch.bfloat16))


def test_plan_writer_matches_reference():
    """make_ranked_task_profile writes the same plan JSON as the reference's
    (profile.py:275-326) for two- and three-rank assignments, fine attention
    splits and MoE groups (fixture: tests/golden/plans/reference_writer.json,
    from tests/golden/make_plans.py), and the plans validate here."""
    from pathlib import Path

    cases = json.loads((Path(__file__).parent / "golden" / "plans" / "reference_writer.json").read_text())
    assert len(cases) >= 4
    for case in cases:
        args = dict(case["args"])
        args["task_assignments"] = [tuple(a) for a in args["task_assignments"]]
        ours = make_ranked_task_profile(**args)
        assert ours == case["profile"], args
        profile_from_dict(ours)


def test_plan_loader_decisions_match_reference():
    """Valid and invalid plans (fixed tasks off rank 0, dtype, broken per-layer
    task sequences, decode_rank on the wrong group, rank range, duplicate
    names, layer gaps, unknown suffixes, coarse layer tasks, MoE groups): this
    loader accepts exactly the plans the reference's profile_from_dict
    accepts, and rejects the others with the same AssertionError text
    (fixture from tests/golden/make_plans.py)."""
    from pathlib import Path

    cases = json.loads((Path(__file__).parent / "golden" / "plans" / "reference_validation.json").read_text())
    assert len(cases) >= 20
    for case in cases:
        ref = case["reference"]
        if ref["ok"]:
            profile_from_dict(case["plan"])
        else:
            with pytest.raises(AssertionError) as info:
                profile_from_dict(case["plan"])
            head = ref["message"][:48]
            assert str(info.value)[:48] == head, (case["name"], str(info.value), ref["message"])
