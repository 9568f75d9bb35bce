"""NVLink hand-off (fg_handoff_put / fg_handoff_recv, P2PComm).

- A receive whose flag nobody sets gives up after its bound, records the
  peer-flag-timeout status and leaves the context usable (single GPU).
- Two ranks as two processes on two GPUs: round trips through the mailboxes
  with slot reuse, the same exchange replayed from CUDA graphs, and two
  disaggregated decodes whose logits equal a co-located run bit for bit:
  attention + head on rank 0 with the FFN on rank 1, and a fine-grained plan
  (qkv / sdpa / o_proj and gate_up / down_proj on alternating ranks, with
  their aux tensors crossing over NVLink).
- Three ranks: a tensor-parallel FFN over two ranks, partials added up on the
  attention rank, within the bf16 tolerance of a co-located run.
Multi-GPU cases are skipped on a box with fewer GPUs."""
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_recv_times_out_cleanly():
    from fluidgpu_b200 import _lib, build, kernels

    build.build()
    lib = _lib.lib()
    slot = 4096
    mb = torch.zeros(lib.fg_mailbox_bytes(2, 2, slot), dtype=torch.uint8, device="cuda")
    out = torch.empty(slot, dtype=torch.uint8, device="cuda")
    kernels.device_status(reset=True)
    # rank 0 waits for a message from rank 1 that is never sent (its own
    # mailbox stands in for the peer's: only the final ack lands there)
    _lib.call("fg_handoff_recv", out.data_ptr(), slot, mb.data_ptr(), mb.data_ptr(), 2, 0, 1, 2, slot,
              200, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    st = kernels.device_status(reset=True)
    assert st & 0xFF == 2, f"expected a peer flag timeout, got status {st:#x}"
    # the context is still usable
    x = torch.arange(10, device="cuda")
    assert int(x.sum().item()) == 45


# ---------------------------------------------------------------------------
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _roundtrip(rank, comm):
    sizes = [16, 4096, 65536, 128 * 1024, 16, 100 * 16]
    for it in range(24):
        n = sizes[it % len(sizes)] // 2
        if rank == 0:
            x = (torch.arange(n, device="cuda", dtype=torch.float32) + it).to(torch.bfloat16)
            comm.send_tensor(x, 1)
            y = torch.empty_like(x)
            comm.recv_tensor(y, 1)
            torch.cuda.synchronize()
            assert torch.equal(y.float(), x.float() * 2), f"iteration {it}"
        else:
            z = torch.empty(n, dtype=torch.bfloat16, device="cuda")
            comm.recv_tensor(z, 0)
            comm.send_tensor(z * 2, 0)
            torch.cuda.synchronize()


def _graphed(rank, comm):
    n = 8192
    x = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros_like(x)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            if rank == 0:
                comm.send_tensor(x, 1)
                comm.recv_tensor(y, 1)
            else:
                comm.recv_tensor(y, 0)
                x.copy_(y + 1)
                comm.send_tensor(x, 0)
    torch.cuda.current_stream().wait_stream(s)
    for it in range(10):
        if rank == 0:
            x.fill_(float(it))
        g.replay()
        torch.cuda.synchronize()
        if rank == 0:
            assert torch.equal(y, torch.full_like(y, float(it + 1))), f"replay {it}"
    del g


def _attn_ffn_plan():
    from fluidgpu_b200.profile import attn_ffn_profile

    return attn_ffn_profile("disagg", 3, 512, 2, 64, 64)


def _fine_plan():
    from fluidgpu_b200.profile import make_ranked_task_profile

    return make_ranked_task_profile(model="disagg", task_assignments=[
        ("layer_0_qkv", 0), ("layer_0_sdpa", 1), ("layer_0_o_proj", 0),
        ("layer_0_mlp_gate_up", 1), ("layer_0_mlp_down_proj", 0),
        ("layer_1_qkv", 1), ("layer_1_sdpa", 0), ("layer_1_o_proj", 1), ("layer_1_mlp", 0),
        ("layer_2_attn", 1), ("layer_2_mlp_gate_up", 0), ("layer_2_mlp_down_proj", 1),
    ], hidden_size=512, num_kv_heads=2, head_dim=64, max_seq_len=64, rank_count=2)


def _disaggregated(rank, comm, plan=_attn_ffn_plan):
    from transformers.models.llama import LlamaConfig, LlamaForCausalLM

    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import ModelWeights
    from fluidgpu_b200.profile import has_fine_groups, profile_from_dict

    torch.manual_seed(0)
    cfg = LlamaConfig(num_hidden_layers=3, vocab_size=2048, hidden_size=512, intermediate_size=1024,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=256)
    model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    B, prompt, steps = 4, 10, 6
    ecfg = EngineConfig(model_name="disagg", max_seq_len=64, world_size=2, device=f"cuda:{rank}",
                        max_batch=B)
    prof = profile_from_dict(plan())
    eng = DecodeEngine(ModelWeights.from_hf(model, f"cuda:{rank}"), ecfg, profile=prof, comm=comm)
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, 2048, (B, prompt), generator=g)
    eng.start(B, reserve_tokens=prompt + steps + 2)
    logits = []
    out = eng.runner.prefill(prompts.cuda())
    tok = torch.zeros(B, dtype=torch.int64)
    for _ in range(steps):
        if rank == 0:
            logits.append(out.reshape(B, -1).float().cpu())
            tok = logits[-1].argmax(-1)
        out = eng.runner.decode_step(tok.cuda())
    torch.cuda.synchronize()
    if rank == 1:
        assert out is None
        return
    # co-located reference on the same GPU, same kernels
    ref = DecodeEngine(ModelWeights.from_hf(model, "cuda:0"),
                       EngineConfig(model_name="colo", max_seq_len=64, world_size=1, device="cuda:0",
                                    max_batch=B))
    ref.start(B, reserve_tokens=prompt + steps + 2)
    out = ref.runner.prefill(prompts.cuda(), chunk=1 if has_fine_groups(prof) else None)
    for s in range(steps):
        lg = out.reshape(B, -1).float().cpu()
        assert torch.equal(lg, logits[s]), f"step {s}: disaggregated logits differ"
        out = ref.runner.decode_step(lg.argmax(-1).cuda())


def _sharded(rank, comm):
    """Attention on rank 0, every layer's FFN tensor-parallel over ranks 1 and 2
    (fp32 partials over NVLink, added up on rank 0): logits within the bf16
    tolerance of a co-located run."""
    from transformers.models.llama import LlamaConfig, LlamaForCausalLM

    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import ModelWeights
    from fluidgpu_b200.profile import ffn_shard_of, profile_from_dict, sharded_ffn_profile

    torch.manual_seed(0)
    cfg = LlamaConfig(num_hidden_layers=3, vocab_size=2048, hidden_size=512, intermediate_size=1024,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=256)
    model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    B, prompt, steps = 4, 10, 6
    prof = profile_from_dict(sharded_ffn_profile("tp", 3, 512, 2, 64, 64, shard_ranks=[1, 2]))
    eng = DecodeEngine(ModelWeights.from_hf(model, f"cuda:{rank}", ffn_shard=ffn_shard_of(prof, rank)),
                       EngineConfig(model_name="tp", max_seq_len=64, world_size=3, device=f"cuda:{rank}",
                                    max_batch=B), profile=prof, comm=comm)
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, 2048, (B, prompt), generator=g)
    eng.start(B, reserve_tokens=prompt + steps + 2)
    logits = []
    out = eng.runner.prefill(prompts.cuda())
    tok = torch.zeros(B, dtype=torch.int64)
    for _ in range(steps):
        if rank == 0:
            logits.append(out.reshape(B, -1).float().cpu())
            tok = logits[-1].argmax(-1)
        out = eng.runner.decode_step(tok.cuda())
    torch.cuda.synchronize()
    if rank != 0:
        assert out is None
        return
    ref = DecodeEngine(ModelWeights.from_hf(model, "cuda:0"),
                       EngineConfig(model_name="colo", max_seq_len=64, world_size=1, device="cuda:0",
                                    max_batch=B))
    ref.start(B, reserve_tokens=prompt + steps + 2)
    out = ref.runner.prefill(prompts.cuda())
    for s in range(steps):
        lg = out.reshape(B, -1).float().cpu()
        assert ((logits[s] - lg).abs() <= 2e-2 + 1e-2 * lg.abs()).all(), f"step {s}"
        out = ref.runner.decode_step(logits[s].argmax(-1).cuda())


def _direct_graphed(rank, comm):
    """Zero-copy hand-offs (the o_proj / down GEMM writes the peer's slot, the
    peer reads it in place), replayed from per-rank CUDA graphs: greedy tokens
    and logits equal a co-located run bit for bit."""
    from transformers.models.llama import LlamaConfig, LlamaForCausalLM

    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import ModelWeights
    from fluidgpu_b200.profile import profile_from_dict

    assert comm.direct
    torch.manual_seed(0)
    cfg = LlamaConfig(num_hidden_layers=3, vocab_size=2048, hidden_size=512, intermediate_size=1024,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=256)
    model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    B, prompt, steps = 4, 10, 8
    ecfg = EngineConfig(model_name="disagg", max_seq_len=64, world_size=2, device=f"cuda:{rank}",
                        max_batch=B, cuda_graph_decode=True)
    eng = DecodeEngine(ModelWeights.from_hf(model, f"cuda:{rank}"), ecfg, profile=profile_from_dict(_attn_ffn_plan()),
                       comm=comm)
    assert eng.executor._direct
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, 2048, (B, prompt), generator=g)
    eng.start(B, reserve_tokens=prompt + steps + 2)
    out = eng.runner.prefill(prompts.cuda())  # eager steps through the direct channel
    tok = out.reshape(B, -1).float().argmax(-1).cpu() if rank == 0 else torch.zeros(B, dtype=torch.int64)
    toks = []
    for _ in range(steps):  # graphed steps
        nxt = eng.step(tok)
        if rank == 0:
            toks.append(nxt)
            tok = nxt
    torch.cuda.synchronize()
    if rank != 0:
        return
    ref = DecodeEngine(ModelWeights.from_hf(model, "cuda:0"),
                       EngineConfig(model_name="colo", max_seq_len=64, world_size=1, device="cuda:0",
                                    max_batch=B, cuda_graph_decode=True))
    ref.start(B, reserve_tokens=prompt + steps + 2)
    out = ref.runner.prefill(prompts.cuda())
    tok = out.reshape(B, -1).float().argmax(-1).cpu()
    for s in range(steps):
        tok = ref.step(tok)
        assert torch.equal(tok, toks[s]), f"step {s}: direct hand-off tokens differ"


CASES = {"roundtrip": _roundtrip, "graphed": _graphed, "disaggregated": _disaggregated,
         "fine_split": lambda rank, comm: _disaggregated(rank, comm, _fine_plan), "sharded": _sharded,
         "direct": _disaggregated, "direct_graphed": _direct_graphed}


def _worker(rank, world, port, case, q):
    try:
        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        from fluidgpu_b200 import build, kernels
        from fluidgpu_b200.comm import P2PComm

        build.build()
        comm = P2PComm(slot_bytes=1 << 20, nslot=2, timeout_ms=5000, direct=case.startswith("direct"))
        CASES[case](rank, comm)
        torch.cuda.synchronize()
        kernels.check_device(f"{case} rank {rank}")
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, True, ""))
    except BaseException:  # noqa: BLE001
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.parametrize("case", [c for c in CASES if c != "sharded"])
def test_two_ranks(case):
    _spawn(case, 2)


def test_three_ranks_tensor_parallel_ffn():
    _spawn("sharded", 3)


def _spawn(case, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for _ in procs:
        results.append(q.get(timeout=300))
    for p in procs:
        p.join(timeout=60)
    for rank, ok, msg in sorted(results):
        assert ok, f"rank {rank} failed:\n{msg}"
