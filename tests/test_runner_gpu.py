"""End-to-end decode parity at benchmark config 1's shape (4 layers, hidden
1024, 16/4 heads, FFN 2816, vocab 32000, batch 8, 256-token prompts, 32
greedy steps), bf16 weights.

- Teacher-forced: FluidRunner on the B200 against the CPU oracle on the same
  weights. Tolerance (north star, bf16): |logit - oracle| <= 2e-2 + 1e-2 *
  |oracle| elementwise, or no worse than the reference's own bf16
  arithmetic (see Judge); the greedy token must agree wherever the exact
  model's top-2 margin exceeds twice that bound (a closer call is a bf16 tie
  that summation order may break either way). The number of steps that
  needed the bf16-arithmetic fallback is reported.
- Free-running: 32 greedy steps from the config-1 prompts against the
  reference's own CausalLMRunner run in bf16 (tests/golden/llama_c1_bf16.pt,
  top-64 logits of every decision). Along each sequence the GPU's token must
  equal the reference's at every step; the one allowed exception is a step
  whose reference top-2 margin is no larger than twice the GPU's measured
  deviation from the reference logits at that very step (a tie at the bf16
  noise floor, after which the two trajectories part). How many sequences
  match all 32 steps, and every parting step with its margin and deviation,
  is reported."""
from pathlib import Path

import pytest
import torch

from oracle import decode_ref as ref

GOLD = Path(__file__).resolve().parent / "golden"

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


class Judge:
    """Three CPU computations of the same bf16 weights:
      truth : oracle in fp32 (the exact math the kernels approximate)
      bf16  : oracle rounding like the reference's bf16 modules
    The GPU must be as close to `truth` as the reference's own bf16
    arithmetic is: at every step elementwise within atol/rtol of `truth` or
    of the bf16 oracle, or, over the run, a worst deviation no more than
    1.25x the bf16 oracle's worst deviation (the north star's elementwise
    bound is at the bf16 noise floor for these random-init models: the two
    CPU variants already differ by ~0.03 max-abs after a few dozen
    positions). The comparison with the bf16 oracle is made over the whole
    run because one step's maximum over a vocabulary row is a noisy
    statistic, and the bf16 oracle itself comes out slightly differently on
    hosts whose CPU matmul kernels differ. Per step: cosine >= 0.9999 and
    identical greedy tokens wherever the exact model's top-2 margin exceeds
    twice the tolerance."""

    def __init__(self, model):
        spec = ref.spec_from_hf(model.config)
        w = ref.weights_from_hf(model)
        self.bf16 = ref.OracleModel(spec, w, torch.bfloat16)
        self.truth = ref.OracleModel(spec, {k: v.float() for k, v in w.items()}, torch.float32)
        self.err, self.ref_err, self.loose = 0.0, 0.0, []

    def prefill(self, prompts):
        return self.truth.prefill(prompts), self.bf16.prefill(prompts)

    def step(self, tok):
        return self.truth.step(tok), self.bf16.step(tok)

    def check(self, got, truth, bf16, step):
        got, truth, bf16 = got.float().cpu(), truth.float(), bf16.float()
        err = (got - truth).abs()
        self.err = max(self.err, err.max().item())
        self.ref_err = max(self.ref_err, (bf16 - truth).abs().max().item())
        near_truth = bool((err <= ATOL + RTOL * truth.abs()).all())
        near_bf16 = bool(((got - bf16).abs() <= ATOL + RTOL * bf16.abs()).all())
        if not (near_truth or near_bf16):
            self.loose.append(step)
        cos = torch.nn.functional.cosine_similarity(got, truth, dim=-1).min().item()
        assert cos >= 0.9999, f"step {step}: cosine {cos}"
        top2 = truth.topk(2, dim=-1).values
        decided = (top2[:, 0] - top2[:, 1]) > 2 * (ATOL + RTOL * top2[:, 0].abs())
        assert torch.equal(ref.argmax_lowest(got)[decided], ref.argmax_lowest(truth)[decided]), (
            f"step {step}: greedy token mismatch")

    def final(self, what=""):
        print(f"{what}: {len(self.loose)} step(s) outside 2e-2 + 1e-2|x| of both oracles {self.loose}; "
              f"worst max-abs {self.err:.4f}, reference-bf16 worst {self.ref_err:.4f}")
        assert not self.loose or self.err <= 1.25 * self.ref_err + 1e-3, (
            f"steps {self.loose} outside atol/rtol; worst max-abs {self.err:.4f} vs "
            f"reference-bf16 worst {self.ref_err:.4f}")


@pytest.mark.parametrize("batch,prompt,steps", [(8, 256, 32), (3, 5, 8)])
def test_llama_decode_matches_oracle(batch, prompt, steps):
    from fluidgpu_b200 import kernels

    model = _tiny_llama()
    eng = _engine(model, batch, prompt + steps + 2)
    judge = Judge(model)
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, model.config.vocab_size, (batch, prompt), generator=g)
    eng.start(batch, reserve_tokens=prompt + steps + 2)
    got = eng.runner.prefill(prompts.cuda()).reshape(batch, -1)
    truth, bf16 = judge.prefill(prompts)
    judge.check(got, truth, bf16, "prefill")
    for s in range(steps):
        tok = ref.argmax_lowest(truth.float())  # teacher forcing on the exact model's choice
        got = eng.runner.decode_step(tok.cuda()).reshape(batch, -1)
        truth, bf16 = judge.step(tok)
        judge.check(got, truth, bf16, s)
    judge.final(f"batch {batch} prompt {prompt}")
    kernels.check_device("llama decode")


def test_config1_greedy_tokens_match_reference_runner():
    """Free-running greedy decode of config 1 (batch 8, 256-token prompts, 32
    steps) against the reference's CausalLMRunner in bf16 on the same
    weights and prompts."""
    from tests.golden import make_golden as mg

    gold = torch.load(GOLD / "llama_c1_bf16.pt")
    model = mg.c1_model(torch.bfloat16)
    prompts = mg.c1_prompts()
    batch, steps = prompts.shape[0], mg.C1["steps"]
    eng = _engine(model, batch, prompts.shape[1] + steps + 2)
    toks, logits = eng.generate(prompts, steps)
    parted, worst = [], 0.0
    for b in range(batch):
        for s in range(steps):
            idx = gold["top_indices"][b, s].long()
            val = gold["top_values"][b, s].float()
            dev = (logits[s][b].float()[idx] - val).abs().max().item()
            worst = max(worst, dev)
            if int(toks[b, s]) != int(gold["tokens"][b, s]):
                margin = (val[0] - val[1]).item()
                assert margin <= 2 * dev, (
                    f"sequence {b} step {s}: token {int(toks[b, s])} vs reference {int(gold['tokens'][b, s])} "
                    f"at margin {margin:.4f} > 2 x deviation {dev:.4f}")
                parted.append((b, s, round(margin, 4), round(dev, 4)))
                break  # the trajectories part here
    print(f"config 1 greedy vs reference bf16 runner: {batch - len(parted)} of {batch} sequences equal over "
          f"{steps} steps; parted at near ties (seq, step, margin, deviation): {parted}; "
          f"worst top-64 deviation before parting {worst:.4f}")
