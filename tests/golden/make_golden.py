"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container that has the FluidGPU reference checkout (read-only is
fine); the fixtures it writes are committed, so the tests never need the
reference at run time:

  PYTHONPATH=<reference>/fluidgpu_runtime python tests/golden/make_golden.py <reference>

Fixtures (all small):
  llama_c1_fp32.pt   Benchmark config 1 through the reference's own
                     CausalLMRunner + LayerExecutor, disaggregated exactly as
                     the reference's tests run it (attention tasks on rank 0,
                     MLP tasks on rank 1, ranks as threads joined by queues,
                     fluidgpu_runtime/test/fluidgpu_torch/test_fine_dense_runtime.py:14-27),
                     fp32 (EngineConfig asserts bf16, config.py:41, so the
                     dtype field is overridden after construction). 8 requests,
                     256-token prompts, 32 greedy steps, one request at a time
                     (the reference runner is batch 1, runner.py:67, :120).
                     Saved: greedy tokens [8, 32] and the top-64 logits
                     (values, indices) of every decision [8, 32, 64].
  llama_c1_bf16.pt   The same config-1 run with the weights cast to bf16 and
                     the runner in bf16 (EngineConfig's own dtype): the
                     reference's bf16 path, which the B200 kernels' greedy
                     tokens are compared with.
  llama_tiny_bf16.pt The reference tests' tiny bf16 Llama
                     (test_fine_dense_runtime.py:150-168) through the runner
                     with a split fine-grained plan: prefill logits of
                     [[1,2,3,4]] and decode logits after token 5.
  gptoss_tiny.pt     gpt-oss through HF GptOssForCausalLM eager (the
                     reference runner's gpt-oss path fails under the installed
                     transformers 5.5, so HF is the reference there): logits of
                     every prompt position and each layer's router top-k
                     indices, fp32 and bf16.
Weights are regenerated from the seeds by transformers' own initialisation,
so the fixtures hold only inputs' seeds and outputs.
"""
from __future__ import annotations

import json
import sys
import tempfile
from pathlib import Path
from queue import Queue
from threading import Thread

import torch

HERE = Path(__file__).resolve().parent

C1 = dict(layers=4, hidden=1024, heads=16, kv=4, inter=2816, vocab=32000, theta=10000.0,
          batch=8, prompt=256, steps=32, topk=64)


def c1_model(dtype=torch.float32):
    from transformers.models.llama import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(num_hidden_layers=C1["layers"], vocab_size=C1["vocab"], hidden_size=C1["hidden"],
                      intermediate_size=C1["inter"], num_attention_heads=C1["heads"],
                      num_key_value_heads=C1["kv"], max_position_embeddings=4096,
                      rope_theta=C1["theta"])
    return LlamaForCausalLM(cfg).to(dtype).eval()


def c1_prompts():
    g = torch.Generator().manual_seed(0)
    return torch.randint(0, C1["vocab"], (C1["batch"], C1["prompt"]), generator=g)


def tiny_llama_bf16():
    from transformers.models.llama import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(num_hidden_layers=1, vocab_size=128, hidden_size=64, intermediate_size=128,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=16)
    return LlamaForCausalLM(cfg).to(torch.bfloat16).eval()


def tiny_gptoss(dtype):
    from transformers.models.gpt_oss import GptOssConfig, GptOssForCausalLM

    torch.manual_seed(0)
    cfg = GptOssConfig(num_hidden_layers=2, num_local_experts=4, vocab_size=256, hidden_size=64,
                       intermediate_size=64, head_dim=16, num_attention_heads=4,
                       num_key_value_heads=2, sliding_window=4, num_experts_per_tok=2,
                       layer_types=["sliding_attention", "full_attention"],
                       max_position_embeddings=4096)
    cfg._attn_implementation = "eager"
    return GptOssForCausalLM(cfg).to(dtype).eval()


GPTOSS_PROMPT = [[3, 17, 250, 9, 44, 101, 7, 7, 200, 31, 5, 66]]


class _QueueComm:
    def __init__(self, rank, channels):
        self._rank, self._channels = rank, channels

    def get_rank(self):
        return self._rank

    def send_tensor(self, tensor, dst):
        self._channels[(self._rank, dst)].put(tensor.detach().clone())

    def recv_tensor(self, tensor, src):
        tensor.copy_(self._channels[(src, self._rank)].get(timeout=60))

    def broadcast_tensor(self, t, src=0):
        pass


def _two_rank_runners(model, assignments, max_seq_len, dtype, tmp: Path, name: str):
    from fluidgpu_torch.config import EngineConfig
    from fluidgpu_torch.executor import LayerExecutor
    from fluidgpu_torch.profile import load_profile, make_ranked_task_profile, owned_layer_ids
    from fluidgpu_torch.runner import CausalLMRunner

    cfgm = model.config
    hd = getattr(cfgm, "head_dim", None) or cfgm.hidden_size // cfgm.num_attention_heads
    raw = make_ranked_task_profile(model=name, task_assignments=assignments,
                                   hidden_size=cfgm.hidden_size, num_kv_heads=cfgm.num_key_value_heads,
                                   head_dim=hd, max_seq_len=max_seq_len)
    path = tmp / f"{name}.json"
    path.write_text(json.dumps(raw))
    profile = load_profile(path, model_name=name, hf_config=cfgm)
    cfg = EngineConfig(model_name=name, profiling_json=path, max_seq_len=max_seq_len, device="cpu")
    object.__setattr__(cfg, "dtype", dtype)
    channels = {(0, 1): Queue(), (1, 0): Queue()}
    return [CausalLMRunner(model, tokenizer=None,
                           executor=LayerExecutor(profile, cfg, comm_backend=_QueueComm(r, channels)),
                           cfg=cfg, owned_layer_ids=owned_layer_ids(profile, r)) for r in (0, 1)]


def _run_both(runners, method, arg):
    results, errors = {}, []

    def go(r):
        try:
            results[r] = getattr(runners[r], method)(arg)
        except BaseException as exc:  # noqa: BLE001
            errors.append(exc)

    ts = [Thread(target=go, args=(r,)) for r in (0, 1)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=600)
    assert not errors, errors
    assert results[1] is None and results[0] is not None
    return results[0]


def make_c1(tmp: Path, dtype=torch.float32) -> dict:
    model = c1_model(dtype)
    assign = []
    for i in range(C1["layers"]):
        assign += [(f"layer_{i}_attn", 0), (f"layer_{i}_mlp", 1)]
    runners = _two_rank_runners(model, assign, 512, dtype, tmp, "c1")
    prompts = c1_prompts()
    tokens = torch.zeros(C1["batch"], C1["steps"], dtype=torch.int64)
    vals = torch.zeros(C1["batch"], C1["steps"], C1["topk"])
    idxs = torch.zeros(C1["batch"], C1["steps"], C1["topk"], dtype=torch.int32)
    for b in range(C1["batch"]):
        logits = _run_both(runners, "prefill", prompts[b : b + 1])
        for s in range(C1["steps"]):
            row = logits.reshape(-1).float()
            top = row.topk(C1["topk"])
            vals[b, s], idxs[b, s] = top.values, top.indices.to(torch.int32)
            tok = int(row.argmax())
            tokens[b, s] = tok
            if s + 1 < C1["steps"]:
                logits = _run_both(runners, "decode_step", torch.tensor([[tok]]))
    name = "fp32" if dtype == torch.float32 else "bf16"
    return {"config": C1, "tokens": tokens, "top_values": vals, "top_indices": idxs,
            "source": f"fluidgpu_torch.runner.CausalLMRunner, 2 ranks (attn rank 0, mlp rank 1), {name}"}


def make_tiny_bf16(tmp: Path) -> dict:
    model = tiny_llama_bf16()
    assign = [("layer_0_qkv", 0), ("layer_0_sdpa", 1), ("layer_0_o_proj", 0),
              ("layer_0_mlp_gate_up", 1), ("layer_0_mlp_down_proj", 0)]
    runners = _two_rank_runners(model, assign, 8, torch.bfloat16, tmp, "tiny-llama")
    with torch.inference_mode():
        pre = _run_both(runners, "prefill", torch.tensor([[1, 2, 3, 4]]))
        dec = _run_both(runners, "decode_step", torch.tensor([[5]]))
    return {"prefill_logits": pre.float().reshape(-1), "decode_logits": dec.float().reshape(-1),
            "source": "fluidgpu_torch.runner.CausalLMRunner, split fine plan, bf16"}


def make_gptoss() -> dict:
    out = {}
    ids = torch.tensor(GPTOSS_PROMPT)
    for name, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        model = tiny_gptoss(dtype)
        router = []
        hooks = [layer.mlp.router.register_forward_hook(
            lambda mod, inp, outp: router.append(outp[2].clone())) for layer in model.model.layers]
        with torch.inference_mode():
            logits = model(ids).logits[0].float()
        for h in hooks:
            h.remove()
        out[name] = {"logits": logits, "router_indices": torch.stack(router).to(torch.int32)}
    out["prompt"] = torch.tensor(GPTOSS_PROMPT)
    out["source"] = "transformers 5.5 GptOssForCausalLM eager"
    return out


def main(only: str | None = None) -> None:
    with tempfile.TemporaryDirectory() as d:
        tmp = Path(d)
        jobs = {"llama_tiny_bf16.pt": lambda: make_tiny_bf16(tmp), "gptoss_tiny.pt": make_gptoss,
                "llama_c1_fp32.pt": lambda: make_c1(tmp),
                "llama_c1_bf16.pt": lambda: make_c1(tmp, torch.bfloat16)}
        for name, job in jobs.items():
            if only is None or only == name:
                torch.save(job(), HERE / name)
    for p in sorted(HERE.glob("*.pt")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    # make_golden.py <reference checkout> [fixture name]
    if len(sys.argv) > 1:
        sys.path.insert(0, str(Path(sys.argv[1]) / "fluidgpu_runtime"))
    main(sys.argv[2] if len(sys.argv) > 2 else None)
