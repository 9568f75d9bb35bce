"""Feed-forward groups sharded over several ranks (plan extension shard_ranks):
the tensor-parallel dense FFN of config 4 (intermediate dimension split, fp32
partials, the first carrying the residual) and the expert-parallel MoE of
config 3 (experts split, router and combine on the attention rank). The
consumer adds the partials up (fg_sum_partials), so the sum order differs
from one GEMM over the whole intermediate dimension: logits are compared with
the co-located plan within the bf16 tolerance, greedy tokens exactly where
the top-2 margin is clear of it, and the router's expert ids exactly.

Ranks are threads on one GPU joined by QueueComm (the reference's own split
test pattern, test_fine_dense_runtime.py:14-27)."""
import threading

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from fluidgpu_b200 import build

    build.build()
    yield
    from fluidgpu_b200 import kernels

    kernels.check_device("sharded ffn tests")


def _tiny_llama():
    from transformers.models.llama import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(num_hidden_layers=3, vocab_size=2048, hidden_size=512, intermediate_size=1024,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=256)
    return LlamaForCausalLM(cfg).to(torch.bfloat16).eval()


def _tiny_gptoss():
    from transformers.models.gpt_oss import GptOssConfig, GptOssForCausalLM

    from fluidgpu_b200 import moe

    torch.manual_seed(0)
    cfg = GptOssConfig(num_hidden_layers=2, num_local_experts=8, vocab_size=1024, hidden_size=384,
                       intermediate_size=256, head_dim=64, num_attention_heads=8, num_key_value_heads=2,
                       sliding_window=16, num_experts_per_tok=2,
                       layer_types=["sliding_attention", "full_attention"], max_position_embeddings=4096)
    cfg._attn_implementation = "eager"
    model = GptOssForCausalLM(cfg).to(torch.bfloat16).eval()
    with torch.no_grad():
        for layer in model.model.layers:
            ex = layer.mlp.experts
            for name in ("gate_up_proj", "down_proj"):  # MXFP4-exact experts, as a real checkpoint
                p = getattr(ex, name)
                v, s = moe.quantize_mxfp4(p.data.transpose(1, 2).float())
                p.data.copy_(moe.dequantize_mxfp4(v, s).transpose(1, 2).to(p.dtype))
            layer.mlp.router.weight.data.normal_(0, 0.2)
            layer.self_attn.sinks.data.normal_(0, 1.0)
    return model


def _decode(weights, prof, comm, B, prompts, steps, rank, out, routing=None):
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine

    eng = DecodeEngine(weights, EngineConfig(model_name=prof.model, max_seq_len=64,
                                             world_size=prof.rank_count, device=DEV, max_batch=B),
                       profile=prof, comm=comm)
    eng.runner.record_routing = routing is not None
    eng.start(B, reserve_tokens=prompts.shape[1] + steps + 2)
    logits = []
    o = eng.runner.prefill(prompts.to(DEV))
    for _ in range(steps):
        if o is not None:
            logits.append(o.reshape(B, -1).float().cpu())
            tok = logits[-1].argmax(-1)
        else:
            tok = torch.zeros(B, dtype=torch.int64)
        o = eng.runner.decode_step(tok.to(DEV))
        if routing is not None:
            routing.append({k: v.cpu().clone() for k, v in eng.runner.last_routing.items()})
    torch.cuda.synchronize()
    out[rank] = logits


def _run_sharded(model, shards, moe, B=4, prompt=9, steps=5):
    from fluidgpu_b200.comm import LocalComm, QueueComm
    from fluidgpu_b200.model import ModelWeights
    from fluidgpu_b200.profile import colocated_profile, ffn_shard_of, profile_from_dict, sharded_ffn_profile

    full = ModelWeights.from_hf(model, DEV)
    s = full.spec
    prof = profile_from_dict(sharded_ffn_profile("sharded", s.num_layers, s.hidden, s.n_kv, s.head_dim, 64,
                                                 shard_ranks=shards, moe=moe))
    world = prof.rank_count
    weights = {r: (full if ffn_shard_of(prof, r) is None else
                   ModelWeights.from_hf(model, DEV, ffn_shard=ffn_shard_of(prof, r))) for r in range(world)}
    prompts = torch.randint(0, s.vocab, (B, prompt), generator=torch.Generator().manual_seed(1))
    chans = QueueComm.make_channels(world)
    results, errors, routes = {}, {}, {r: [] for r in range(world)}

    def worker(rank):
        try:
            with torch.inference_mode():
                _decode(weights[rank], prof, QueueComm(rank, chans, timeout_s=60.0), B, prompts, steps, rank,
                        results, routes[rank] if moe else None)
        except BaseException as exc:  # noqa: BLE001
            errors[rank] = exc

    threads = [threading.Thread(target=worker, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not any(t.is_alive() for t in threads), "a rank did not finish"
    for r, exc in errors.items():
        raise AssertionError(f"rank {r} failed") from exc
    ref, ref_routes = {}, [[]]
    colo = profile_from_dict(colocated_profile("colo", s.num_layers, s.hidden, s.n_kv, s.head_dim, 64, moe=moe))
    _decode(full, colo, LocalComm(), B, prompts, steps, 0, ref, ref_routes[0] if moe else None)
    for step, (a, b) in enumerate(zip(results[0], ref[0])):
        err = (a - b).abs()
        assert (err <= ATOL + RTOL * b.abs()).all(), f"step {step}: max |delta| {err.max().item():.4f}"
        top2 = b.topk(2, dim=-1).values
        clear = (top2[:, 0] - top2[:, 1]) > 2 * (ATOL + RTOL * top2[:, 0].abs())
        assert torch.equal(a.argmax(-1)[clear], b.argmax(-1)[clear]), f"step {step}: greedy tokens differ"
    if moe:
        # each expert shard saw the router's ids; they equal the co-located ones
        for r in shards:
            for step, (got, want) in enumerate(zip(routes[r], ref_routes[0])):
                for layer in want:
                    assert torch.equal(got[layer], want[layer]), f"rank {r} step {step} layer {layer}"


@pytest.mark.parametrize("shards", [[1, 2], [1, 2, 3, 4]])
def test_tensor_parallel_dense_ffn(shards):
    _run_sharded(_tiny_llama(), shards, moe=False)


def test_expert_parallel_moe():
    _run_sharded(_tiny_gptoss(), [1, 2], moe=True)
