#!/usr/bin/env python
"""Decode-step benchmark (Llama-3-8B architecture, batch 64, context 4096,
paged KV, bf16) on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl fgb200|reference]

One "step" = one greedy decode step of the whole model for the batch: every
sequence appends one token (embed -> 32 x (attention, SwiGLU FFN) -> norm ->
lm_head -> argmax). Weights are random N(0, 0.02) bf16 from a seed, the KV
cache is filled with synthetic N(0,1) values for the 4096-token prompts
(the timed work does not depend on the values), and the KV pool (~35 GB)
and weights (~16 GB) are far larger than L2, so no flush is needed.

value : tokens/s over all ranks, inputs resident in HBM, device-timed; each
        step is one replay of the CUDA graph holding the whole decode step.
e2e   : tokens/s through DecodeEngine.step (host tokens in pinned memory,
        H2D copy + step + argmax + D2H read per step), device-timed.
roofline: paged attention (the dominant kernel, ~60% of the step), its
        duration from CUDA event pairs around each of its launches during R
        steps run right after the timed region from the host (the same
        kernels and split plans the graph replays).
Under torchrun (N > 1) the default is the disaggregated step
(fluidgpu_b200.disagg): the first N/2 GPUs hold attention for 64 requests
each (2 ping-pong micro-batches of 32), the other N/2 hold the FFN
tensor-parallel over the intermediate dimension (one GPU at N = 2), every
FFN GPU merging all attention GPUs' rows of a micro-batch into one GEMM per
layer. Attention -> FFN: the O-proj GEMM keeps its rows in the attention
GPU's memory and signals, the FFN GPUs' RMSNorm reads them over NVLink;
FFN -> attention: the down GEMM's epilogue stores into the attention GPUs'
memory and signals (weak scaling in the attention GPUs). On 8 GPUs the
prompts follow config 4's mix (uniform in [128, 4096]) unless --prompt-mix
says otherwise. --mode replicas runs N independent co-located engines
instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tokens/s"
CONFIG = {"workload": "llama-3-8b decode step, batch 64, prompt 4096, paged KV block 16 (BASELINE configs[1])",
          "model": "llama-3-8b (random init)", "batch_per_gpu": 64, "context": 4096,
          "block_size": 16, "l2": "inputs larger than L2 (KV ~35 GB, weights ~16 GB per GPU)"}
CONFIG_GPTOSS = {"workload": "gpt-oss-20b decode step, batch 128, prompt 4096, paged KV block 16, "
                             "MXFP4 experts (BASELINE configs[2] on one GPU)",
                 "model": "gpt-oss-20b (random init, MXFP4 experts)", "batch_per_gpu": 128,
                 "context": 4096, "block_size": 16,
                 "l2": "inputs larger than L2 (KV ~26 GB, experts ~10 GB per GPU)"}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {}


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of this process's
    GPU, sampled through NVML every 10 ms from a thread while the timed region
    runs, plus one sample at its start and one at its end (a region of a few
    hundred milliseconds still gets a record). The GPU is found by UUID, so the
    sample is of the device this rank runs on whatever CUDA_VISIBLE_DEVICES
    says."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index: int, period_s: float = 0.01) -> None:
        self.period = period_s
        self.rows: list[tuple[float, float, int]] = []
        self.handle = None
        self.max_mhz = None
        self.err = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            self.nv = pynvml
            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(cuda_index).uuid)
                uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            except Exception:  # noqa: BLE001
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
            get = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None)
            self._reasons = get or pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception as e:  # noqa: BLE001
            self.handle = None
            self.err = f"NVML unavailable: {type(e).__name__}"

    def _sample(self) -> None:
        nv, h = self.nv, self.handle
        try:
            self.rows.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                              nv.nvmlDeviceGetPowerUsage(h) / 1000.0, int(self._reasons(h))))
        except Exception as e:  # noqa: BLE001
            self.err = f"NVML query failed: {type(e).__name__}"

    def _run(self) -> None:
        while not self._stop.wait(self.period):
            self._sample()

    def start(self) -> None:
        if self.handle is None:
            return
        self.rows = []
        self._stop.clear()
        self._sample()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def stop(self) -> dict:
        if self.handle is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "NVML unavailable"]}
        self._stop.set()
        self._thread.join(timeout=5)
        self._sample()
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [self.err or "no samples"]}
        reasons = sorted({name for _, _, bits in self.rows for bit, name in self.REASONS.items() if bits & bit})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.max_mhz,
                "power_w": statistics.median(r[1] for r in self.rows), "reasons": reasons,
                "samples": len(self.rows), "source": "NVML, 10 ms"}


def attn_bytes(meta: dict, lens_sum: int) -> float:
    """Algorithmic HBM bytes of one paged attention launch: K and V of every
    attended token + Q + O (bf16)."""
    B, nq, nkv, hd = meta["B"], meta["nq"], meta["nkv"], meta["hd"]
    return 2.0 * nkv * hd * 2 * lens_sum + 2.0 * B * nq * hd * 2


def prompt_lengths(batch: int, context: int, mix: str, seed: int = 0) -> list[int]:
    """Prompt length of each sequence: all `context` ("fixed"), or seeded
    uniform in [128, context] ("uniform", config 4's request mix)."""
    if mix == "fixed":
        return [context] * batch
    assert mix == "uniform", f"unknown prompt mix {mix!r}"
    lo = min(128, context)
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, context + 1, (batch,), generator=g).tolist()


def cpu_baseline_sample(batch: int, context: int) -> dict:
    """The oracle port timed on the host cores: one decoder layer plus the
    norm/lm_head/argmax tail at the full batch and context, fp32. The layer
    count it stands for is stated in its own keys."""
    from oracle.cpu_baseline import LayerSample, host_threads, time_sample
    from fluidgpu_b200.model import LLAMA3_8B as S

    threads = host_threads()
    torch.set_num_threads(threads)
    sample = LayerSample(S.hidden, S.n_q, S.n_kv, S.head_dim, S.intermediate, S.vocab, S.rope_theta,
                         batch, context)
    sample.layer()  # warm-up
    r = time_sample(sample, S.num_layers, reps=2)
    return {"value": r["tokens_per_s"], "unit": "tokens/s", "cores": threads, "kind": "port",
            "sampled_layers": 1, "layers": S.num_layers,
            "sampled_ms": {"layer": r["t_layer_s"] * 1e3, "head": r["t_head_s"] * 1e3},
            "sample": (f"oracle (CPU restatement, fp32) of 1 Llama-3-8B decoder layer + norm/lm_head/argmax"
                       f" at batch {batch}, context {context}, timed; the value stands for "
                       f"{S.num_layers} x layer + head = {r['step_s']:.2f} s per step")}


REF_DIR = ROOT / "baseline" / "_ref"


class ReferenceRunner:
    """The reference's own decode path on the host cores: fluidgpu_torch's
    CausalLMRunner + LayerExecutor (installed from the reference's source into
    baseline/_ref), with every task of a Llama-3-8B-architecture model on rank
    0, bf16 (EngineConfig's dtype), its LayerKVCache seeded with `context`
    synthetic tokens. The reference runner decodes one sequence at a time
    (it asserts a [1, 1] token, runner.py:120), so one step here is one token
    of one sequence through embed, 32 x (attention, MLP), norm and lm_head,
    and a batch of B sequences costs B such steps per token."""

    def __init__(self, context: int, seed: int = 0) -> None:
        import tempfile

        sys.path.insert(0, str(REF_DIR))
        from fluidgpu_torch.config import EngineConfig
        from fluidgpu_torch.executor import LayerExecutor
        from fluidgpu_torch.profile import load_profile, make_ranked_task_profile, owned_layer_ids
        from fluidgpu_torch.runner import CausalLMRunner
        from transformers.models.llama import LlamaConfig, LlamaForCausalLM
        from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

        from fluidgpu_b200.model import LLAMA3_8B as S

        cfg = LlamaConfig(num_hidden_layers=S.num_layers, vocab_size=S.vocab, hidden_size=S.hidden,
                          intermediate_size=S.intermediate, num_attention_heads=S.n_q,
                          num_key_value_heads=S.n_kv, head_dim=S.head_dim, rope_theta=S.rope_theta,
                          max_position_embeddings=max(8192, context + 64))
        with torch.device("meta"):
            model = LlamaForCausalLM(cfg).to(torch.bfloat16)
        model.to_empty(device="cpu")
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            # N(0, 0.02) values: one seeded block of 2^20 tiled over each
            # parameter (the step's work does not depend on the values)
            block = (torch.randn(1 << 20, generator=g) * 0.02).to(torch.bfloat16)
            for p in model.parameters():
                flat = p.view(-1)
                n, b = flat.numel(), block.numel()
                q = n // b
                if q:
                    flat[: q * b].view(q, b).copy_(block.unsqueeze(0).expand(q, b))
                if n > q * b:
                    flat[q * b:].copy_(block[: n - q * b])
            for m in model.modules():
                if hasattr(m, "variance_epsilon"):
                    m.weight.fill_(1.0)
        model.model.rotary_emb = LlamaRotaryEmbedding(cfg)  # its buffers were left empty on meta
        model.eval()
        assign = []
        for i in range(S.num_layers):
            assign += [(f"layer_{i}_attn", 0), (f"layer_{i}_mlp", 0)]
        max_len = context + 64
        raw = make_ranked_task_profile(model=S.name, task_assignments=assign, hidden_size=S.hidden,
                                       num_kv_heads=S.n_kv, head_dim=S.head_dim, max_seq_len=max_len)
        self._tmp = tempfile.TemporaryDirectory()
        path = Path(self._tmp.name) / "profile.json"
        path.write_text(json.dumps(raw))
        profile = load_profile(path, model_name=S.name, hf_config=cfg)
        ecfg = EngineConfig(model_name=S.name, profiling_json=path, max_seq_len=max_len, device="cpu",
                            strict_transformers_version=False)

        class _OneRank:  # every task is on rank 0: nothing is ever sent
            def get_rank(self):
                return 0

            def send_tensor(self, t, dst):
                raise AssertionError("co-located plan sent a tensor")

            def recv_tensor(self, t, src):
                raise AssertionError("co-located plan received a tensor")

            def broadcast_tensor(self, t, src=0):
                return None

        self.runner = CausalLMRunner(model, None, LayerExecutor(profile, ecfg, comm_backend=_OneRank()), ecfg,
                                     owned_layer_ids(profile, 0))
        kv = self.runner.kv_cache
        with torch.no_grad():
            kb = torch.randn(S.n_kv, context, S.head_dim, generator=g).to(torch.bfloat16)
            for layer in range(S.num_layers):
                kv.key_cache[layer][0, :, :context].copy_(kb)
                kv.value_cache[layer][0, :, :context].copy_(kb)
        kv.advance(context)
        self.token = torch.tensor([[17]])

    def step(self) -> float:
        """One greedy decode step of the sequence; returns its seconds."""
        t0 = time.perf_counter()
        logits = self.runner.decode_step(self.token)
        self.token = logits.reshape(1, -1).argmax(-1).view(1, 1)
        return time.perf_counter() - t0


def run_reference(args) -> None:
    """The reference arm: the reference's own CPU decode path on the host
    cores (ReferenceRunner) when its package is installed in baseline/_ref,
    else the oracle port (cpu_baseline_sample), each step a bounded sample of
    the workload that the line's keys state."""
    world, rank, local = dist_env()
    if rank != 0:
        return
    from oracle.cpu_baseline import host_threads

    threads = host_threads()
    torch.set_num_threads(threads)
    ctx = args.context
    config = CONFIG
    if world > 1 and args.mode == "disagg":
        # the workload the other arm measures at this N; with config 4's prompt
        # mix the sample runs at its mean prompt length
        config = {**CONFIG, "workload": disagg_workload(world // 2, world // 2, args.batch or 64, ctx,
                                                        args.prompt_mix)}
        if args.prompt_mix == "uniform":
            lens = prompt_lengths(256, ctx, "uniform", seed=0)
            ctx = int(round(sum(lens) / len(lens)))
            config["reference_sample_context"] = ctx
    common = {"impl": "reference", "metric": METRIC, "unit": "tokens/s", "n_gpus": args.gpus,
              "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
              "vs_baseline": None, "data": "synthetic", "config": config}
    if (REF_DIR / "fluidgpu_torch").is_dir():
        t0 = time.perf_counter()
        ref = ReferenceRunner(ctx)
        setup_s = time.perf_counter() - t0
        with torch.inference_mode():
            for _ in range(max(args.warmup, 0)):
                ref.step()
            times = [ref.step() for _ in range(args.steps)]
        step_s = statistics.mean(times)
        value = 1.0 / step_s  # one token of one sequence per step
        sample = (f"fluidgpu_torch CausalLMRunner + LayerExecutor (the reference, installed from its source), "
                  f"every task on one rank, bf16, Llama-3-8B architecture, context {ctx}: each step is one "
                  f"decode step of one sequence (the runner's batch is 1; a batch of 64 takes 64 such steps "
                  f"per token), all 32 layers + norm + lm_head + argmax, {threads} threads")
        line = {**common, "value": value, "ms_per_step": step_s * 1e3, "dtype": "bf16",
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                                 "sample": sample},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "tokens_per_step": 1, "setup_s": setup_s,
                "cpu_port": cpu_baseline_sample(64, ctx)}
    else:
        from fluidgpu_b200.model import LLAMA3_8B as S
        from oracle.cpu_baseline import LayerSample, time_sample

        sample = LayerSample(S.hidden, S.n_q, S.n_kv, S.head_dim, S.intermediate, S.vocab, S.rope_theta,
                             64, ctx)
        with torch.inference_mode():
            for _ in range(max(args.warmup, 0)):
                sample.layer()
        layer_s, head_s = [], []
        for _ in range(args.steps):
            r = time_sample(sample, S.num_layers, reps=1)
            layer_s.append(r["t_layer_s"])
            head_s.append(r["t_head_s"])
        t_layer, t_head = statistics.mean(layer_s), statistics.mean(head_s)
        full_step_s = S.num_layers * t_layer + t_head
        value = 64 / full_step_s
        line = {**common, "value": value, "ms_per_step": (t_layer + t_head) * 1e3, "dtype": "f32",
                "sampled_layers": 1, "layers": S.num_layers, "scale": full_step_s / (t_layer + t_head),
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                                 "sample": f"each timed step: 1 Llama-3-8B decoder layer + norm/lm_head/argmax "
                                           f"at batch 64, context {ctx} (the oracle's restatement, fp32); "
                                           f"value = 64 tokens / (32 x layer + head); the reference package "
                                           f"is not installed in baseline/_ref"},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_fgb200(args) -> None:
    world, rank, local = dist_env()
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))

    from fluidgpu_b200 import build, kernels
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import GPT_OSS_20B, LLAMA3_8B, ModelWeights

    build.build()
    spec = GPT_OSS_20B if args.model == "gpt-oss-20b" else LLAMA3_8B
    config = CONFIG_GPTOSS if args.model == "gpt-oss-20b" else CONFIG
    B, ctx = (args.batch or config["batch_per_gpu"]), args.context
    W, K = args.warmup, args.steps
    R = 3  # replays of the attention-timed graph
    total = ctx + W + 2 * K + R + 8
    cfg = EngineConfig(model_name=spec.name, max_seq_len=total, world_size=1, device=f"cuda:{local}",
                       max_batch=B, cuda_graph_decode=not args.eager)
    weights = ModelWeights.random(spec, seed=0, device=dev)
    eng = DecodeEngine(weights, cfg)
    eng.start(B, prompt_lens=prompt_lengths(B, ctx, args.prompt_mix, seed=rank), reserve_tokens=total)
    g = torch.Generator(device=dev).manual_seed(1 + rank)
    eng.kv_cache.pool.normal_(0.0, 1.0, generator=g)
    eng._tok_dev.copy_(torch.randint(0, spec.vocab, (B,), generator=g, device=dev))

    def barrier():
        if world > 1:
            dist.barrier()

    def one_step():
        if args.eager:
            eng._tok_dev.copy_(eng.step_device(eng._tok_dev))
        else:
            eng.replay()

    # launches one step issues (graph capture counts them; eager counts directly)
    n0 = kernels.launch_count()
    one_step()  # first warm-up step (captures the graph)
    launches_per_step = kernels.launch_count() - n0
    for _ in range(W - 1):
        one_step()
    torch.cuda.synchronize()
    kernels.check_device("bench warm-up")

    # ---- timed: device-resident inputs ----
    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    h0 = time.perf_counter()
    for _ in range(K):
        one_step()
    host_ms = (time.perf_counter() - h0) * 1e3 / K  # enqueue cost per step (diagnostic)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    kernels.check_device("bench timed region")

    # ---- dominant kernel: paged attention durations from event pairs captured
    # around each of its launches (same kernels, same stream, R replays) ----
    lens0 = eng.kv_cache.seq_lengths()
    kernels.KernelTimer.enable("attn")
    for _ in range(R):  # eager steps: the same kernels and split plans the graph replays
        eng._tok_dev.copy_(eng.step_device(eng._tok_dev))
    torch.cuda.synchronize()
    attn = kernels.KernelTimer.durations_ms("attn")
    kernels.KernelTimer.disable()
    tot_bytes, tot_ms = 0.0, 0.0
    for i, (d, meta) in enumerate(attn):
        step = i // spec.num_layers
        win = meta["window"]
        lens_sum = sum(min(l + 1 + step, win) if win else l + 1 + step for l in lens0[:B])
        tot_bytes += attn_bytes(meta, lens_sum)
        tot_ms += d
    attn_launch_ms = tot_ms / max(len(attn), 1)
    attn_launch_bytes = tot_bytes / max(len(attn), 1)
    kernels.check_device("bench roofline region")

    # ---- e2e through the public API: host tokens in, host tokens out ----
    host_tok = eng._tok_dev.cpu().pin_memory()
    torch.cuda.synchronize()
    barrier()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(K):
        host_tok = eng.step(host_tok)
    f1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = f0.elapsed_time(f1)

    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])

    if rank == 0:
        peaks = measured_peaks()
        hbm = peaks.get("hbm_gbs")
        peak_src = "measured" if hbm else "fallback"
        hbm = hbm or 6650.0
        achieved = attn_launch_bytes / (attn_launch_ms * 1e-3) / 1e9
        traffic = None
        tp = ROOT / "profiles" / "attn_traffic.json"
        if tp.exists():
            try:
                tj = json.loads(tp.read_text())
                # ncu dram bytes per token attended, scaled to this launch's tokens
                traffic = tj["dram_bytes_per_kv_token"] * (attn_launch_bytes / (2 * spec.n_kv * spec.head_dim * 2))
            except Exception:
                traffic = None
        value = world * B * K / (ms * 1e-3)
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {**config, "batch_per_gpu": B,
                       "parallelism": f"dp{world} (attention data-parallel by request, FFN co-located)",
                       **({"prompt_lens": f"uniform [128, {ctx}], seeded per rank"}
                          if args.prompt_mix == "uniform" else {})},
            "e2e": {"value": world * B * K / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": B * 8, "d2h_bytes_per_step": B * 8},
            "roofline": {"bound": "hbm", "kernel": "fg_paged_decode_attn", "achieved": achieved,
                         "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_source": f"{peak_src} (hbm_gbs)", "traffic": traffic,
                         "algorithmic_bytes_per_launch": attn_launch_bytes,
                         "launch_ms": attn_launch_ms, "launches": len(attn)},
            "gpu_launches": int(launches_per_step * K),
            "launches_per_step": int(launches_per_step),
            "cuda_graph": not args.eager,
            "host_enqueue_ms_per_step": host_ms,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline and spec is LLAMA3_8B:
            line["cpu_baseline"] = cpu_baseline_sample(B, ctx)
        if world == 1 and spec is LLAMA3_8B and not args.no_extra_models:
            # config 3's model on the same GPU, after the headline's memory is released
            del eng, weights
            kernels.Workspace.clear()
            torch.cuda.empty_cache()
            line["gpt_oss_20b"] = gptoss_step(dev, ctx, W, max(K // 2, 5))
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def gptoss_step(dev: torch.device, ctx: int, W: int, K: int) -> dict:
    """gpt-oss-20b decode step (BASELINE configs[2]'s model on one GPU: batch
    128, context 4096, MXFP4 experts, alternating 128-token windows, sinks),
    CUDA-graph replays, device-timed: an extra line item of the N=1 run."""
    from fluidgpu_b200 import kernels
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import GPT_OSS_20B as spec
    from fluidgpu_b200.model import ModelWeights

    B = CONFIG_GPTOSS["batch_per_gpu"]
    total = ctx + W + K + 8
    eng = DecodeEngine(ModelWeights.random(spec, seed=0, device=dev),
                       EngineConfig(model_name=spec.name, max_seq_len=total, world_size=1, device=str(dev),
                                    max_batch=B, cuda_graph_decode=True))
    eng.start(B, prompt_lens=[ctx] * B, reserve_tokens=total)
    g = torch.Generator(device=dev).manual_seed(7)
    eng.kv_cache.pool.normal_(0.0, 1.0, generator=g)
    eng._tok_dev.copy_(torch.randint(0, spec.vocab, (B,), generator=g, device=dev))
    for _ in range(W):
        eng.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        eng.replay()
    e1.record()
    torch.cuda.synchronize()
    kernels.check_device("gpt-oss-20b step")
    ms = e0.elapsed_time(e1) / K
    out = {"workload": CONFIG_GPTOSS["workload"], "value": B / (ms * 1e-3), "unit": "tokens/s",
           "ms_per_step": ms, "steps": K, "warmup": W, "dtype": "bf16 (experts MXFP4)"}
    eng._graphs.clear()
    del eng
    torch.cuda.empty_cache()
    return out


def disagg_workload(A: int, S: int, batch: int, ctx: int, mix: str) -> str:
    """The workload a disaggregated bench line measures, with the BASELINE
    config it is quoted on (configs[1]: 1 + 1 GPUs; configs[3]: 4 + 4)."""
    prompts = f"prompts uniform in [128, {ctx}]" if mix == "uniform" else f"prompt {ctx}"
    which = {(1, 1): " (BASELINE configs[1])", (4, 4): " (BASELINE configs[3])"}.get((A, S), "")
    return (f"llama-3-8b disaggregated decode step, {A} attention + {S} FFN GPUs, batch {A * batch} "
            f"({batch} per attention GPU), {prompts}, paged KV block 16{which}")


def run_disagg_fused(args) -> None:
    """The disaggregated decode step of fluidgpu_b200.disagg on N GPUs: N/2
    attention GPUs with `batch` sequences each in M micro-batches, N/2 FFN
    GPUs (tensor-parallel, merged batches), fused NVLink hand-offs; every
    rank replays its CUDA graphs."""
    world, rank, local = dist_env()
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    from fluidgpu_b200 import build, kernels
    from fluidgpu_b200.disagg import AttentionRank, DisaggLayout, Fabric, FFNRank, nvlink_bytes_per_step
    from fluidgpu_b200.model import LLAMA3_8B as spec
    from fluidgpu_b200.model import ModelWeights

    build.build()
    M = args.micro_batches
    B = args.batch or 64
    assert B % M == 0, f"--batch {B} must split into {M} micro-batches"
    b = B // M
    lay = DisaggLayout.split(world, M, b, args.handoff)
    role, idx = lay.role(rank)
    ctx, W, K, R = args.context, args.warmup, args.steps, 3
    total = ctx + W + 2 * K + 3 * R + 8
    weights = ModelWeights.random(spec, seed=0, device=dev,
                                  ffn_shard=(idx, lay.S) if role == "ffn" and lay.S > 1 else None)
    if role == "attn":
        r = AttentionRank(lay, rank, weights, total, device=dev, schedule=args.schedule)
        lens = [prompt_lengths(b, ctx, args.prompt_mix, seed=rank * M + m) for m in range(M)]
        r.start(lens, reserve_tokens=total)
        g = torch.Generator(device=dev).manual_seed(1 + rank)
        for m, mb in enumerate(r.mbs):
            mb["kv"].pool.normal_(0.0, 1.0, generator=g)
            r.set_tokens(m, torch.randint(0, spec.vocab, (b,), generator=g, device=dev))
    else:
        r = FFNRank(lay, rank, weights, device=dev)
    t_start = time.perf_counter()

    def trace(what):
        if args.verbose:
            print(f"[rank {rank} {role} {time.perf_counter() - t_start:8.2f}s] {what}", file=sys.stderr, flush=True)

    trace("weights and caches ready")
    imports = Fabric.ipc(r)
    trace("mailboxes mapped")

    def step(graphs=True):
        r.step(graphs=graphs)

    n0 = kernels.launch_count()
    step(graphs=False)  # one eager step: the launches a step issues
    launches = kernels.launch_count() - n0
    torch.cuda.synchronize()
    trace("eager step done")
    kernels.check_device("disagg eager step")
    for _ in range(max(W - 1, 1)):
        step()
    torch.cuda.synchronize()
    trace("warm-up done")
    kernels.check_device("disagg warm-up")

    sampler = ClockSampler(local)
    dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        step()
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    trace(f"timed region done: {ms / K:.3f} ms/step")
    kernels.check_device("disagg timed region")

    # ---- end to end: host tokens in, host tokens out, every step ----
    host_in = [torch.zeros(b, dtype=torch.int64).pin_memory() for _ in range(M)]
    host_out = [torch.zeros(b, dtype=torch.int64).pin_memory() for _ in range(M)]
    if role == "attn":
        for m, mb in enumerate(r.mbs):
            host_in[m].copy_(mb["tok"])
    dist.barrier()
    torch.cuda.synchronize()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(K):
        if role == "attn":
            for m in range(M):
                r.set_tokens(m, host_in[m].to(dev, non_blocking=True))
            outs = r.step(graphs=True)
            for m in range(M):
                host_out[m].copy_(outs[m], non_blocking=True)
            torch.cuda.current_stream().synchronize()
            host_in, host_out = host_out, host_in
        else:
            r.step(graphs=True)
    f1.record()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_ms = f0.elapsed_time(f1)

    # ---- per-role kernel times from event pairs on the launching stream ----
    # R eager steps of every rank (the launches the graphs replay, from the host)
    for _ in range(R):
        step(graphs=False)
    torch.cuda.synchronize()
    kernels.check_device("disagg eager steps")
    dist.barrier()
    role_stats = {}
    if role == "attn":
        # attention GPUs: the attention-side kernels alone (FFN left out), one
        # micro-batch after another on one stream, so launches do not overlap
        lens0 = [mb["kv"].seq_lengths() for mb in r.mbs]
        kernels.KernelTimer.enable("attn")
        for _ in range(R):
            r.step_serial_standalone()
        torch.cuda.synchronize()
        timed = kernels.KernelTimer.durations_ms("attn")
        kernels.KernelTimer.disable()
        tot_b, tot_ms = 0.0, 0.0
        for i, (d, meta) in enumerate(timed):
            st, m = i // (M * spec.num_layers), (i // spec.num_layers) % M
            tot_b += attn_bytes(meta, sum(l + 1 + st for l in lens0[m]))
            tot_ms += d
        role_stats = {"attn_bytes": tot_b, "attn_ms": tot_ms, "attn_launches": len(timed)}
        # the same attention-side work with the FFN left out, on the step's
        # streams: what the hand-offs and the remote FFN add to the step
        for _ in range(R):
            r.step(graphs=True, standalone=True)
        torch.cuda.synchronize()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(R):
            r.step(graphs=True, standalone=True)
        a1.record()
        torch.cuda.synchronize()
        role_stats["alone_ms_per_step"] = a0.elapsed_time(a1) / R
    else:
        # FFN GPUs: their own kernels for one (layer, micro-batch) with no
        # waits, graph-replayed: RMSNorm + gate/up (SwiGLU) + down
        pair_ms = r.time_standalone(R)
        T, H, I = lay.A * b, spec.hidden, r.w.layers[0]["w_down"].K
        role_stats = {"ffn_bytes": 3.0 * H * I * 2 + T * H * 2 * 2, "ffn_flops": 2.0 * T * 3 * H * I,
                      "ffn_ms": pair_ms, "T": T, "I": I}
    kernels.check_device("disagg stand-alone region")
    t = torch.tensor([ms, e2e_ms, float(launches)], device=dev)
    dist.all_reduce(t[:2], op=dist.ReduceOp.MAX)
    dist.all_reduce(t[2:], op=dist.ReduceOp.SUM)
    ms, e2e_ms, launches_all = float(t[0]), float(t[1]), int(t[2])
    stats: list = [None] * world
    dist.all_gather_object(stats, (role, role_stats))
    if rank == 0:
        peaks = measured_peaks()
        hbm = peaks.get("hbm_gbs") or 6650.0
        peak_src = "measured" if peaks.get("hbm_gbs") else "fallback"
        tflops = peaks.get("bf16_tflops_sustained") or 1400.0
        a_stats = [s for ro, s in stats if ro == "attn"]
        f_stats = [s for ro, s in stats if ro == "ffn"]
        attn_gbs = sum(s["attn_bytes"] for s in a_stats) / (sum(s["attn_ms"] for s in a_stats) * 1e-3) / 1e9
        ffn_ms = max(s["ffn_ms"] for s in f_stats)  # per (layer, micro-batch), slowest FFN GPU
        ffn_gbs = f_stats[0]["ffn_bytes"] / (ffn_ms * 1e-3) / 1e9
        ffn_tf = f_stats[0]["ffn_flops"] / (ffn_ms * 1e-3) / 1e12
        step_ms = ms / K
        alone = max(s["alone_ms_per_step"] for s in a_stats)
        nv = nvlink_bytes_per_step(lay, spec.hidden, spec.num_layers)
        tokens = lay.A * M * b * K
        line = {
            "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {**CONFIG, "workload": disagg_workload(lay.A, lay.S, B, ctx, args.prompt_mix),
                       "batch_per_gpu": B, "attention_gpus": lay.A, "ffn_gpus": lay.S,
                       "micro_batches": M, "sequences_per_micro_batch": b, "schedule": args.schedule,
                       "handoff": args.handoff,
                       "parallelism": (f"disaggregated: attention dp{lay.A} / FFN tp{lay.S}, {M} ping-pong micro-"
                                       f"batches of {b} per attention GPU, FFN batches merged over the attention "
                                       f"GPUs ({lay.A * b} tokens), hand-offs stored by the producing GEMM over NVLink"),
                       **({"prompt_lens": f"uniform [128, {ctx}], seeded per micro-batch"}
                          if args.prompt_mix == "uniform" else {})},
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": lay.A * M * b * 8, "d2h_bytes_per_step": lay.A * M * b * 8},
            "roofline": {"bound": "hbm", "kernel": "fg_paged_decode_attn (attention GPUs)", "achieved": attn_gbs,
                         "peak": hbm, "unit": "GB/s", "frac": attn_gbs / hbm, "peak_source": f"{peak_src} (hbm_gbs)",
                         "traffic": None},
            "ffn_roofline": {"kernel": "RMSNorm + gate_up (SwiGLU) + down GEMMs per FFN GPU, one (layer, "
                                       "micro-batch), graph-replayed without waits",
                             "tokens_per_gemm": f_stats[0]["T"], "intermediate_per_gpu": f_stats[0]["I"],
                             "us_per_layer_micro_batch": ffn_ms * 1e3,
                             "achieved_gbs": ffn_gbs, "hbm_frac": ffn_gbs / hbm, "achieved_tflops": ffn_tf,
                             "tensor_frac": ffn_tf / tflops, "tensor_peak_source": "measured (bf16_tflops_sustained)",
                             "note": "decode-size GEMMs are weight-streaming: hbm_frac is their roofline, "
                                     "tensor_frac what the tokens make of the tensor pipe"},
            "handoff": {"nvlink_bytes_per_step": nv, "nvlink_us_per_step_at_770GBs": nv / 770e9 * 1e6,
                        "attention_alone_ms_per_step": alone,
                        "exposed_frac": max(0.0, 1.0 - alone / step_ms),
                        "handoff_frac": max(0.0, 1.0 - alone / step_ms),
                        "handoff_kernels": 0,
                        "note": "exposed_frac = 1 - (attention GPU's own kernels, FFN left out) / step: what the "
                                "hand-offs and the remote FFN add to the attention GPUs' step; there are no "
                                "hand-off kernels (the producing GEMM stores and signals, the consuming "
                                "RMSNorm waits), so handoff_frac is that same exposed share"},
            "gpu_launches": launches_all * K,
            "cuda_graph": True,
            "clocks": clocks,
            "mode": "disagg",
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    r.release_graphs()
    torch.cuda.synchronize()
    dist.barrier()
    imports.close()
    dist.destroy_process_group()


def run_disagg(args) -> None:
    """Disaggregated decode over NVLink (P2PComm hand-offs, no NCCL on the data
    path) driven by a placement plan through the executor, every rank replaying
    captured graphs, M ping-pong micro-batches of `batch` sequences per
    attention rank:
      pipeline : attention (+ embed, head) on GPU 0, the FFN on GPU 1 (config 2)
      tp     : attention data-parallel on the first half of the GPUs, each
               layer's dense FFN tensor-parallel over the second half (config 4)
      ep     : gpt-oss, attention data-parallel on the first half, the experts
               split over the second half (config 3)
    Each attention rank is one pipeline through the FFN ranks; an FFN rank
    serves every pipeline (its own engines and mailboxes per pipeline and
    micro-batch)."""
    world, rank, local = dist_env()
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    from fluidgpu_b200 import build, kernels
    from fluidgpu_b200.comm import P2PComm
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.model import GPT_OSS_20B, LLAMA3_8B, ModelWeights
    from fluidgpu_b200.pingpong import PingPongEngine
    from fluidgpu_b200.profile import attn_ffn_profile, ffn_shard_of, profile_from_dict, sharded_ffn_profile

    build.build()
    mode = args.mode
    if mode == "pipeline":
        assert world == 2, "--mode pipeline runs on two GPUs (attention rank 0, FFN rank 1)"
        attn_ranks, ffn_ranks = [0], [1]
    else:
        assert world >= 2 and world % 2 == 0, f"--mode {mode} needs an even number of GPUs"
        attn_ranks, ffn_ranks = list(range(world // 2)), list(range(world // 2, world))
    spec = GPT_OSS_20B if mode == "ep" else LLAMA3_8B
    base_cfg = CONFIG_GPTOSS if mode == "ep" else CONFIG
    B = args.batch or 64
    ctx, W, K, M = args.context, args.warmup, args.steps, args.micro_batches
    total = ctx + W + K + 8

    # one process group per pipeline: its attention rank is the plan's rank 0
    # (embed and head there), the FFN ranks follow in order
    if mode == "pipeline":
        raw = attn_ffn_profile(spec.name, spec.num_layers, spec.hidden, spec.n_kv, spec.head_dim, total)
    else:
        raw = sharded_ffn_profile(spec.name, spec.num_layers, spec.hidden, spec.n_kv, spec.head_dim, total,
                                  shard_ranks=list(range(1, 1 + len(ffn_ranks))), moe=spec.moe)
    prof = profile_from_dict(raw)
    groups = {a: dist.new_group([a] + ffn_ranks) for a in attn_ranks}  # collective: every rank, same order
    mine = [a for a in attn_ranks if rank == a or rank in ffn_ranks]
    group_rank = 0 if rank in attn_ranks else 1 + ffn_ranks.index(rank)
    weights = ModelWeights.random(spec, seed=0, device=dev, ffn_shard=ffn_shard_of(prof, group_rank))
    cfg = EngineConfig(model_name=spec.name, max_seq_len=total, world_size=prof.rank_count,
                       device=f"cuda:{local}", max_batch=B, cuda_graph_decode=True)
    slot = max(B * spec.hidden * 4, B * spec.qkv_width * 2)
    # zero-copy main-path hand-offs where the plan allows them (disagg)
    comms = {(a, m): P2PComm(slot_bytes=slot, nslot=2, group=groups[a], tag=m, timeout_ms=10000,
                             direct=mode == "pipeline")
             for a in mine for m in range(M)}
    pps = [PingPongEngine(weights, cfg, prof, lambda m, a=a: comms[(a, m)], micro_batches=M) for a in mine]
    g = torch.Generator(device=dev).manual_seed(1)
    for a, pp in zip(mine, pps):
        pp.start(B, prompt_lens=prompt_lengths(B, ctx, args.prompt_mix, seed=a), reserve_tokens=total)
        for eng in pp.engines:
            if eng.kv_cache.pool is not None:
                eng.kv_cache.pool.normal_(0.0, 1.0, generator=g)
            eng._tok_dev.copy_(torch.randint(0, spec.vocab, (B,), generator=g, device=dev))

    for pp in pps:
        pp.capture()
    torch.cuda.synchronize()
    dist.barrier()

    def step():
        for pp in pps:
            pp.step()

    for _ in range(W):
        step()
    torch.cuda.synchronize()
    kernels.check_device(f"{mode} warm-up")
    dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    kernels.check_device(f"{mode} timed region")
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    tokens = len(attn_ranks) * M * B * K
    if rank == 0:
        par = {"pipeline": "attention GPU0 / FFN GPU1",
               "tp": f"attention dp{len(attn_ranks)} / FFN tp{len(ffn_ranks)} (reduce-by-consumer)",
               "ep": f"attention dp{len(attn_ranks)} / experts ep{len(ffn_ranks)} (reduce-by-consumer)"}[mode]
        line = {
            "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {**base_cfg, "batch_per_micro_batch": B, "micro_batches": M,
                       "attention_ranks": len(attn_ranks), "ffn_ranks": len(ffn_ranks),
                       "parallelism": par + ", NVLink hand-offs, ping-pong",
                       **({"prompt_lens": f"uniform [128, {ctx}], seeded per attention rank"}
                          if args.prompt_mix == "uniform" else {})},
            "mode": mode,
        }
        print(json.dumps(line), flush=True)
    for pp in pps:
        for eng in pp.engines:
            eng._graphs.clear()
    torch.cuda.synchronize()
    dist.barrier()
    for c in comms.values():
        c.close()
    dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="fgb200", choices=["fgb200", "reference"])
    ap.add_argument("--batch", type=int, default=0, help="sequences per GPU (default: the model's config)")
    ap.add_argument("--model", default="llama-3-8b", choices=["llama-3-8b", "gpt-oss-20b"])
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra-models", action="store_true", help="N=1: skip the gpt-oss-20b line item")
    ap.add_argument("--handoff", default="pull", choices=["pull", "push"],
                    help="disagg: FFN GPUs read the O-proj rows from the attention GPUs (pull), or the O-proj "
                         "epilogue stores them into every FFN GPU (push)")
    ap.add_argument("--schedule", default="interleaved", choices=["interleaved", "streams"],
                    help="disagg attention GPUs: micro-batches alternating layer by layer on one stream, or each "
                         "on a stream of its own")
    ap.add_argument("--eager", action="store_true", help="launch every kernel from the host (no CUDA graph)")
    ap.add_argument("--mode", default="auto", choices=["auto", "replicas", "disagg", "pipeline", "tp", "ep"],
                    help="auto: co-located at N=1, disagg at N>1. disagg: attention / merged-batch FFN GPUs with "
                         "fused hand-offs (fluidgpu_b200.disagg); replicas: N independent co-located engines; "
                         "pipeline / tp / ep: placement plans through the executor with P2PComm (pipeline: "
                         "2 GPUs; tp: dense FFN tensor-parallel; ep: gpt-oss experts split)")
    ap.add_argument("--micro-batches", type=int, default=2,
                    help="ping-pong micro-batches per attention GPU (disagg, pipeline, tp, ep)")
    ap.add_argument("--verbose", action="store_true", help="phase trace on stderr (disagg)")
    ap.add_argument("--prompt-mix", default=None, choices=["fixed", "uniform"],
                    help="prompt lengths: all --context, or seeded uniform in [128, --context] per sequence "
                         "(config 4's request mix; the default for the disaggregated step on 8 GPUs, fixed "
                         "otherwise)")
    args = ap.parse_args()
    assert args.warmup >= 0 and args.steps > 0
    world = dist_env()[0]
    mode = args.mode if args.mode != "auto" else ("disagg" if world > 1 else "replicas")
    args.mode = mode
    if args.prompt_mix is None:
        args.prompt_mix = "uniform" if (mode == "disagg" and world == 8) else "fixed"
    if args.impl == "reference":
        run_reference(args)
    elif mode == "disagg":
        assert args.model == "llama-3-8b", "the disaggregated step serves the dense model (gpt-oss: --mode ep)"
        run_disagg_fused(args)
    elif mode in ("pipeline", "tp", "ep"):
        run_disagg(args)
    else:
        run_fgb200(args)


if __name__ == "__main__":
    main()
