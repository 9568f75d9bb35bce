"""End-to-end decode parity: FluidRunner on the B200 against the CPU oracle on
the same HF-initialised weights (bf16), teacher-forced on identical tokens.

Tolerance (north star, bf16): |logit - oracle| <= 2e-2 + 1e-2 * |oracle|
elementwise; the greedy token must agree wherever the oracle's top-2 margin
exceeds twice that bound (a closer call is a bf16 tie that summation order
may break either way)."""
import pytest
import torch

from oracle import decode_ref as ref

pytestmark = pytest.mark.gpu


def _tiny_llama(layers=4, hidden=1024, heads=16, kv=4, inter=2816, vocab=32000, theta=10000.0):
    from transformers.models.llama import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(num_hidden_layers=layers, vocab_size=vocab, hidden_size=hidden,
                      intermediate_size=inter, num_attention_heads=heads, num_key_value_heads=kv,
                      max_position_embeddings=4096, rope_theta=theta)
    return LlamaForCausalLM(cfg).to(torch.bfloat16).eval()


def _engine(model, batch, max_seq_len):
    from fluidgpu_b200 import build
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import ModelWeights

    build.build()
    w = ModelWeights.from_hf(model, "cuda")
    cfg = EngineConfig(model_name="tiny", max_seq_len=max_seq_len, world_size=1, device="cuda:0",
                       max_batch=batch)
    return DecodeEngine(w, cfg)


ATOL, RTOL = 2e-2, 1e-2


def _check_step(got, exp, step):
    got = got.float().cpu()
    exp = exp.float()
    excess = ((got - exp).abs() - (ATOL + RTOL * exp.abs())).max().item()
    assert excess <= 0, f"step {step}: logits outside atol {ATOL} / rtol {RTOL} by {excess}"
    top2 = exp.topk(2, dim=-1).values
    decided = (top2[:, 0] - top2[:, 1]) > 2 * (ATOL + RTOL * top2[:, 0].abs())
    g_tok = ref.argmax_lowest(got)
    e_tok = ref.argmax_lowest(exp)
    assert torch.equal(g_tok[decided], e_tok[decided]), f"step {step}: greedy token mismatch"


@pytest.mark.parametrize("batch,prompt,steps", [(8, 24, 32), (3, 5, 8)])
def test_llama_decode_matches_oracle(batch, prompt, steps):
    from fluidgpu_b200 import kernels

    model = _tiny_llama()
    eng = _engine(model, batch, prompt + steps + 2)
    oracle = ref.OracleModel(ref.spec_from_hf(model.config), ref.weights_from_hf(model), torch.bfloat16)
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, model.config.vocab_size, (batch, prompt), generator=g)
    eng.start(batch, reserve_tokens=prompt + steps + 2)
    got = eng.runner.prefill(prompts.cuda()).reshape(batch, -1)
    exp = oracle.prefill_stepwise(prompts)
    _check_step(got, exp, "prefill")
    for s in range(steps):
        tok = ref.argmax_lowest(exp.float())  # teacher forcing on the oracle's choice
        got = eng.runner.decode_step(tok.cuda()).reshape(batch, -1)
        exp = oracle.step(tok)
        _check_step(got, exp, s)
    kernels.check_device("llama decode")


def test_greedy_generate_tokens_match_oracle():
    """Free-running greedy decode for 32 steps (config-1 model shape, batch 8)."""
    model = _tiny_llama()
    batch, prompt, steps = 8, 16, 32
    eng = _engine(model, batch, prompt + steps + 2)
    oracle = ref.OracleModel(ref.spec_from_hf(model.config), ref.weights_from_hf(model), torch.bfloat16)
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, model.config.vocab_size, (batch, prompt), generator=g)
    toks, logits = eng.generate(prompts, steps)
    exp_toks, exp_logits = oracle.generate(prompts, steps)
    # tokens agree until the first step whose oracle decision is within tolerance
    for b in range(batch):
        for s in range(steps):
            if toks[b, s] != exp_toks[b, s]:
                e = exp_logits[s][b].float()
                top2 = e.topk(2).values
                assert (top2[0] - top2[1]).item() <= 2 * (ATOL + RTOL * top2[0].abs().item()), (
                    f"seq {b} step {s}: token {int(toks[b, s])} vs oracle {int(exp_toks[b, s])}")
                break
