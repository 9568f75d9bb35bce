"""Pin the CPU oracle to the reference: its outputs must reproduce the golden
fixtures tests/golden/make_golden.py recorded from the reference's own
CausalLMRunner (Llama) and from transformers' GptOssForCausalLM (gpt-oss)."""
from pathlib import Path

import torch

from oracle import decode_ref as ref
from tests.golden import make_golden as mg

GOLD = Path(__file__).resolve().parent / "golden"


def _oracle(model, dtype):
    return ref.OracleModel(ref.spec_from_hf(model.config), ref.weights_from_hf(model), dtype)


def test_config1_fp32_matches_reference_runner():
    """Benchmark config 1 (fp32, disaggregated reference run): every greedy
    token identical, top-64 logits within 1e-4."""
    gold = torch.load(GOLD / "llama_c1_fp32.pt")
    model = mg.c1_model(torch.float32)
    oracle = _oracle(model, torch.float32)
    prompts = mg.c1_prompts()
    with torch.inference_mode():
        toks, logits = oracle.generate(prompts, mg.C1["steps"])
    assert torch.equal(toks, gold["tokens"])
    for s in range(mg.C1["steps"]):
        got = logits[s].float().gather(1, gold["top_indices"][:, s].long())
        assert (got - gold["top_values"][:, s]).abs().max().item() <= 1e-4, s


def test_tiny_bf16_matches_reference_runner():
    gold = torch.load(GOLD / "llama_tiny_bf16.pt")
    model = mg.tiny_llama_bf16()
    oracle = _oracle(model, torch.bfloat16)
    with torch.inference_mode():
        pre = oracle.prefill(torch.tensor([[1, 2, 3, 4]])).float().reshape(-1)
        dec = oracle.step(torch.tensor([5])).float().reshape(-1)
    for got, exp in ((pre, gold["prefill_logits"]), (dec, gold["decode_logits"])):
        assert ((got - exp).abs() <= 2e-2 + 1e-2 * exp.abs()).all()


def test_stepwise_prefill_equals_full_prefill():
    model = mg.tiny_llama_bf16().float()
    oracle = _oracle(model, torch.float32)
    ids = torch.tensor([[1, 2, 3, 4, 9, 30], [5, 6, 7, 8, 1, 0]])
    with torch.inference_mode():
        a = oracle.prefill(ids)
        b = oracle.prefill_stepwise(ids)
    assert (a - b).abs().max().item() <= 1e-5


def _gptoss_positions(model, dtype, prompt):
    oracle = _oracle(model, dtype)
    oracle.reset(1)
    logits, routers = [], []
    with torch.inference_mode():
        for t in range(prompt.shape[1]):
            logits.append(oracle.step(prompt[:, t]).float()[0])
            routers.append(torch.stack(oracle.router_indices)[:, 0])  # [layers, k]
    return torch.stack(logits), torch.stack(routers, dim=1)  # [T, V], [layers, T, k]


def test_gptoss_fp32_logits_and_router_indices():
    gold = torch.load(GOLD / "gptoss_tiny.pt")
    model = mg.tiny_gptoss(torch.float32)
    logits, routers = _gptoss_positions(model, torch.float32, gold["prompt"])
    g = gold["fp32"]
    assert (logits - g["logits"]).abs().max().item() <= 1e-4
    # top-k expert sets identical per token and layer (ordered by score)
    assert torch.equal(routers.to(torch.int32), g["router_indices"])


def test_gptoss_bf16_logits_and_router_indices():
    gold = torch.load(GOLD / "gptoss_tiny.pt")
    model = mg.tiny_gptoss(torch.bfloat16)
    logits, routers = _gptoss_positions(model, torch.bfloat16, gold["prompt"])
    g = gold["bf16"]
    assert ((logits - g["logits"]).abs() <= 2e-2 + 1e-2 * g["logits"].abs()).all()
    assert torch.equal(torch.sort(routers.to(torch.int32), dim=-1).values,
                       torch.sort(g["router_indices"], dim=-1).values)


def test_mxfp4_roundtrip_and_grid():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(8, 64, generator=g) * 0.02
    packed, scales = ref.mxfp4_quantize(w)
    assert packed.shape == (8, 32) and scales.shape == (8, 2)
    deq = ref.mxfp4_dequantize(packed, scales, torch.float32)
    # every dequantised value is an e2m1 grid point times its block scale
    blk = deq.view(8, 2, 32) / torch.pow(2.0, scales.float() - 127).unsqueeze(-1)
    grid = ref.E2M1_VALUES.abs().unique()
    assert torch.isin(blk.abs(), grid).all()
    # round-to-nearest: error at most half the widest e2m1 step (2) = 1 block-scale unit
    scale = torch.pow(2.0, scales.float() - 127).unsqueeze(-1)
    assert ((deq.view(8, 2, 32) - w.view(8, 2, 32)).abs() <= scale + 1e-12).all()
    # and the block maximum lands on the grid top (amax/scale in (3, 6])
    amax = w.view(8, 2, 32).abs().amax(-1, keepdim=True)
    assert ((amax / scale > 3) & (amax / scale <= 6)).all()
