"""Fine-grained placements: the attention group split into qkv / sdpa /
o_proj, the dense FFN into gate_up / down_proj and the MoE FFN into router /
experts / combine, each piece on either of two ranks (reference runner.py:
196-254, :362-414, aux routing :462-670). Every split decodes to the logits
of the co-located plan bit for bit: the same kernels run on the same inputs,
only the rank that runs them changes.

The two ranks are two threads on one GPU joined by QueueComm, the pattern of
the reference's own split tests (test_fine_dense_runtime.py:14-27); the
NVLink form of a split (two processes, P2PComm) is in test_handoff_gpu.py."""
import threading

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from fluidgpu_b200 import build

    build.build()
    yield
    from fluidgpu_b200 import kernels

    kernels.check_device("split plan tests")


def _tiny_llama():
    from transformers.models.llama import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    # head_dim 128 with 8 heads: the attention output (1024 wide) differs from
    # the hidden size (512), as in gpt-oss, so the sdpa -> o_proj edge carries
    # a wider tensor than the other edges
    cfg = LlamaConfig(num_hidden_layers=3, vocab_size=2048, hidden_size=512, intermediate_size=1024,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                      max_position_embeddings=256)
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
            for name in ("gate_up_proj", "down_proj"):
                p = getattr(ex, name)
                v, s = moe.quantize_mxfp4(p.data.transpose(1, 2).float())
                p.data.copy_(moe.dequantize_mxfp4(v, s).transpose(1, 2).to(p.dtype))
            layer.mlp.router.weight.data.normal_(0, 0.2)
            layer.self_attn.sinks.data.normal_(0, 1.0)
    return model


def _decode(weights, prof, comm, B, prompts, steps, rank, out, feed=None, chunk=None):
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine

    eng = DecodeEngine(weights, EngineConfig(model_name=prof.model, max_seq_len=64,
                                             world_size=prof.rank_count, device=DEV, max_batch=B),
                       profile=prof, comm=comm)
    eng.start(B, reserve_tokens=prompts.shape[1] + steps + 2)
    logits = []
    o = eng.runner.prefill(prompts.to(DEV), chunk=chunk)
    for s in range(steps):
        if o is not None:
            logits.append(o.reshape(B, -1).float().cpu())
            tok = logits[-1].argmax(-1)
        else:
            tok = torch.zeros(B, dtype=torch.int64)
        o = eng.runner.decode_step(tok.to(DEV))
    torch.cuda.synchronize()
    out[rank] = logits


def _run_split(model, assignments, B=4, prompt=9, steps=5):
    from fluidgpu_b200.comm import QueueComm
    from fluidgpu_b200.model import ModelWeights
    from fluidgpu_b200.profile import (colocated_profile, has_fine_groups, make_ranked_task_profile,
                                       profile_from_dict)

    weights = ModelWeights.from_hf(model, DEV)
    s = weights.spec
    prompts = torch.randint(0, s.vocab, (B, prompt), generator=torch.Generator().manual_seed(1))
    prof = profile_from_dict(make_ranked_task_profile(
        model="split", task_assignments=assignments, hidden_size=s.hidden, num_kv_heads=s.n_kv,
        head_dim=s.head_dim, max_seq_len=64, rank_count=2))
    chans = QueueComm.make_channels(2)
    results, errors = {}, {}

    def worker(rank):
        try:
            with torch.inference_mode():
                _decode(weights, prof, QueueComm(rank, chans, timeout_s=60.0), B, prompts, steps, rank,
                        results)
        except BaseException as exc:  # noqa: BLE001
            errors[rank] = exc

    threads = [threading.Thread(target=worker, args=(r,)) for r in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not any(t.is_alive() for t in threads), "a rank did not finish"
    for r, exc in errors.items():
        raise AssertionError(f"rank {r} failed") from exc
    assert results[1] == [], "only the norm_lm_head rank returns logits"
    colo = profile_from_dict(colocated_profile("colo", s.num_layers, s.hidden, s.n_kv, s.head_dim, 64,
                                               moe=s.moe))
    ref = {}
    from fluidgpu_b200.comm import LocalComm

    # a plan with sub-groups prefills position by position: the co-located
    # run does the same, so every kernel sees the same rows
    _decode(weights, colo, LocalComm(), B, prompts, steps, 0, ref, chunk=1 if has_fine_groups(prof) else None)
    for step, (a, b) in enumerate(zip(results[0], ref[0])):
        assert torch.equal(a, b), f"step {step}: split logits differ from co-located"


def test_llama_attention_and_ffn_splits():
    _run_split(_tiny_llama(), [
        ("layer_0_qkv", 0), ("layer_0_sdpa", 1), ("layer_0_o_proj", 0),
        ("layer_0_mlp_gate_up", 1), ("layer_0_mlp_down_proj", 0),
        ("layer_1_qkv", 1), ("layer_1_sdpa", 1), ("layer_1_o_proj", 0),
        ("layer_1_mlp", 1),
        ("layer_2_attn", 0),
        ("layer_2_mlp_gate_up", 0), ("layer_2_mlp_down_proj", 1),
    ])


def test_llama_sdpa_home_projections_remote():
    _run_split(_tiny_llama(), [
        ("layer_0_qkv", 1), ("layer_0_sdpa", 0), ("layer_0_o_proj", 1),
        ("layer_0_mlp", 0),
        ("layer_1_qkv", 0), ("layer_1_sdpa", 0), ("layer_1_o_proj", 1),
        ("layer_1_mlp_gate_up", 1), ("layer_1_mlp_down_proj", 1),
        ("layer_2_attn", 1), ("layer_2_mlp", 0),
    ])


def test_gpt_oss_moe_router_experts_combine_split():
    _run_split(_tiny_gptoss(), [
        ("layer_0_qkv", 0), ("layer_0_sdpa", 1), ("layer_0_o_proj", 1),
        ("layer_0_moe_router", 0), ("layer_0_moe_experts", 1), ("layer_0_moe_combine", 0),
        ("layer_1_attn", 1),
        ("layer_1_moe_router", 1), ("layer_1_moe_experts", 0), ("layer_1_moe_combine", 1),
    ])
