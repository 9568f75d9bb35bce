"""Kernel microbenchmarks (benchmark config 5 and per-kernel roofline checks).

  python -m fluidgpu_b200.microbench attn  [--batch B] [--context L] [--window W]
  python -m fluidgpu_b200.microbench gemm  [--T T] [--N N] [--K K] [--epilogue store|residual|swiglu]
  python -m fluidgpu_b200.microbench sweep-attn      # B in {1,32,256} x ctx in {512,4096,32768}
  python -m fluidgpu_b200.microbench moe   [--T T]  # gpt-oss MXFP4 expert GEMMs, 32 experts top-4
  python -m fluidgpu_b200.microbench prefill-attn [--batch B] [--S S] [--context L]  # causal prefill attention
  python -m fluidgpu_b200.microbench prefill [--model M] [--batch B] [--S S] [--chunk C]  # whole-model prefill
  python -m fluidgpu_b200.microbench vllm-moe [--expert-device cuda:1]  # vLLM MoE forward_impl, gpt-oss-20b layer
  torchrun --nproc-per-node 2 -m fluidgpu_b200.microbench handoff
      # [T,H] bf16 hand-off GPU0 -> GPU1, T in {1,8,64,256,1024,8192}, H in {2880,4096}:
      # NVLink mailbox put/recv (P2PComm) against NCCL send/recv, one-way time

Each prints one JSON line per case: device time per launch (CUDA events,
median of --iters after --warmup), algorithmic bytes and GB/s, and the
fraction of the measured HBM peak (MEASURED_PEAKS.json when present).
Inputs are seeded N(0,1) (attention) / N(0,0.02) (weights); the KV pool of
each case is sized to the case, so small cases stay small under a profiler.
"""
from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

import torch

from . import _lib, build, kernels

ROOT = Path(__file__).resolve().parent.parent


def _peak_hbm() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


GRAPH = True  # time launches replayed from a CUDA graph (no host overhead inside the window)


def _time(fn, iters: int, warmup: int) -> float:
    """Device milliseconds per call. With GRAPH, `iters` calls are captured in
    one CUDA graph and replayed back to back between two events (the kernels'
    own time plus the inter-kernel gaps a captured decode step also has);
    otherwise each call is bracketed by events (host launch cost included)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if GRAPH:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            fn()  # workspace allocation happens outside the capture
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s):
                for _ in range(iters):
                    fn()
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(3):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) / iters)
        return statistics.median(ts)
    ts = []
    for _ in range(iters):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def bench_attn(B: int, ctx: int, nq: int = 32, nkv: int = 8, hd: int = 128, window: int = 0,
               iters: int = 20, warmup: int = 5, seed: int = 1, plan_len: int = 0) -> dict:
    """plan_len > 0: the length the split plan is made for (at most ctx; the
    plan's slice count is capped by plan_len / 128 pages, so a sweep over
    plan_len visits the smaller slice counts), else ctx."""
    plan = plan_len if 0 < plan_len <= ctx else ctx
    g = torch.Generator(device="cuda").manual_seed(seed)
    pages = (ctx + 15) // 16
    num_blocks = B * pages
    kc = torch.empty((num_blocks, nkv, 16, hd), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
    vc = torch.empty_like(kc).normal_(generator=g)
    perm = torch.randperm(num_blocks, generator=g, device="cuda").to(torch.int32)
    table = perm.view(B, pages).contiguous()
    q = torch.empty((B, nq, hd), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
    lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    out = torch.empty((B, nq * hd), dtype=torch.bfloat16, device="cuda")
    fn = lambda: kernels.paged_decode_attn(q, kc, vc, table, lens, plan, window=window, out=out)  # noqa: E731
    ms = _time(fn, iters, warmup)
    eff = min(ctx, window) if window else ctx
    nbytes = 2.0 * B * nkv * hd * 2 * eff + 2.0 * B * nq * hd * 2
    peak, src = _peak_hbm()
    gbs = nbytes / (ms * 1e-3) / 1e9
    kernels.check_device("attn microbench")
    return {"kernel": "fg_paged_decode_attn", "B": B, "context": ctx, "nq": nq, "nkv": nkv, "hd": hd,
            "window": window, "splits": _lib.lib().fg_attn_splits(B, nkv, hd, plan, window),
            "ms": ms, "bytes": nbytes, "GBps": gbs, "frac_hbm": gbs / peak,
            "peak": f"{src} {peak} GB/s", "timing": "graph" if GRAPH else "eager"}


def bench_gemm(T: int, N: int, K: int, epilogue: str = "store", iters: int = 20, warmup: int = 5,
               seed: int = 2, splits: int = 0, packed: bool = True) -> dict:
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.empty((T, K), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
    w = torch.empty((N, K), dtype=torch.bfloat16, device="cuda").normal_(0, 0.02, generator=g)
    epi = {"store": _lib.FG_EPI_STORE, "residual": _lib.FG_EPI_RESIDUAL, "swiglu": _lib.FG_EPI_SWIGLU}[epilogue]
    n_out = N // 2 if epi == _lib.FG_EPI_SWIGLU else N
    res = torch.empty((T, n_out), dtype=torch.bfloat16, device="cuda").normal_(generator=g) \
        if epi == _lib.FG_EPI_RESIDUAL else None
    out = torch.empty((T, n_out), dtype=torch.bfloat16, device="cuda")
    wk = kernels.PackedWeight(w) if packed else w
    fn = lambda: kernels.gemm(x, wk, epilogue=epi, residual=res, out=out, splits=splits)  # noqa: E731
    ms = _time(fn, iters, warmup)
    nbytes = 2.0 * (N * K + T * K + T * n_out * (2 if res is not None else 1))
    flops = 2.0 * T * N * K
    peak, src = _peak_hbm()
    gbs = nbytes / (ms * 1e-3) / 1e9
    kernels.check_device("gemm microbench")
    used = _lib.lib().fg_gemm_grid(T, N, K, splits) * _lib.lib().fg_gemm_split(T, N, K, splits)
    return {"kernel": "fg_gemm_bf16", "T": T, "N": N, "K": K, "epilogue": epilogue, "grid": used, "packed": packed,
            "ms": ms, "bytes": nbytes, "GBps": gbs, "TFLOPs": flops / (ms * 1e-3) / 1e12,
            "frac_hbm": gbs / peak, "peak": f"{src} {peak} GB/s", "timing": "graph" if GRAPH else "eager"}


def bench_moe(T: int = 128, E: int = 32, k: int = 4, H: int = 2880, I: int = 2880, iters: int = 20,
              warmup: int = 5, seed: int = 3) -> list[dict]:
    """gpt-oss expert GEMMs: MXFP4 gate_up (+bias, SwiGLU-OAI) and down (+bias)
    over T tokens routed top-k among E experts (uniform random routing)."""
    from . import moe

    g = torch.Generator(device="cuda").manual_seed(seed)
    w1 = torch.empty((E, 2 * I, H), device="cuda").normal_(0, 0.02, generator=g)
    w2 = torch.empty((E, H, I), device="cuda").normal_(0, 0.02, generator=g)
    v1, s1 = moe.quantize_mxfp4(w1)
    v2, s2 = moe.quantize_mxfp4(w2)
    del w1, w2
    p1, p2 = moe.pack_mxfp4(v1.contiguous(), s1.contiguous()), moe.pack_mxfp4(v2.contiguous(), s2.contiguous())
    b1 = torch.zeros((E, 2 * I), dtype=torch.bfloat16, device="cuda")
    b2 = torch.zeros((E, H), dtype=torch.bfloat16, device="cuda")
    idx = torch.stack([torch.randperm(E, device="cuda", generator=g)[:k] for _ in range(T)]).to(torch.int32)
    r = moe.Routing(idx, E)
    x = torch.empty((T * k, H), dtype=torch.float16, device="cuda").normal_(generator=g)
    act = torch.empty((T * k, I), dtype=torch.float16, device="cuda").normal_(generator=g)
    touched = int((torch.bincount(idx.reshape(-1).long(), minlength=E) > 0).sum())
    peak, src = _peak_hbm()
    out = []
    for name, xin, wp, bias, N, K, epi in (
            ("gate_up", x, p1, b1, 2 * I, H, _lib.FG_EPI_SWIGLU_OAI),
            ("down", act, p2, b2, H, I, _lib.FG_EPI_STORE)):
        fn = lambda: moe.grouped_gemm(xin, wp, bias, r, N, K, epi)  # noqa: E731
        ms = _time(fn, iters, warmup)
        wbytes = touched * ((N + 127) // 128) * (K // 64) * 4352
        n_out = N // 2 if epi == _lib.FG_EPI_SWIGLU_OAI else N
        nbytes = wbytes + T * k * (K + n_out) * 2
        gbs = nbytes / (ms * 1e-3) / 1e9
        out.append({"kernel": "fg_moe_gemm_mxfp4", "gemm": name, "T": T, "E": E, "k": k, "N": N, "K": K,
                    "experts_touched": touched, "BN": r.BN, "items": int(r.item_count.item()),
                    "ms": ms, "bytes": nbytes, "GBps": gbs, "frac_hbm": gbs / peak,
                    "TFLOPs": 2.0 * T * k * N * K / (ms * 1e-3) / 1e12,
                    "peak": f"{src} {peak} GB/s", "timing": "graph" if GRAPH else "eager"})
    # the small kernels around the expert GEMMs
    xr = torch.empty((T, H), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
    rw = torch.empty((E, H), dtype=torch.bfloat16, device="cuda").normal_(0, 0.02, generator=g)
    wts = torch.softmax(torch.randn(T, k, device="cuda", generator=g), -1).to(torch.bfloat16)
    y = torch.empty((T * k, H), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
    res = torch.empty((T, H), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
    o = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    xp = torch.empty((T * k, H), dtype=torch.float16, device="cuda")
    st = lambda: kernels._stream(xr.device)  # noqa: E731
    small = {
        "router_topk": lambda: moe.router_topk(xr, rw, None, k),
        "permute": lambda: moe.Routing(idx, E),
        "gather": lambda: _lib.call("fg_moe_gather", xr.data_ptr(), r.perm_pair.data_ptr(), T, k, H,
                                    xp.data_ptr(), st()),
        "unpermute": lambda: _lib.call("fg_moe_unpermute", y.data_ptr(), r.inv.data_ptr(), idx.data_ptr(),
                                       wts.data_ptr(), res.data_ptr(), o.data_ptr(), T, k, H, 0, E, 0, st()),
    }
    for name, fn in small.items():
        out.append({"kernel": name, "gemm": name, "T": T, "BN": r.BN, "items": int(r.item_count.item()),
                    "ms": _time(fn, iters, warmup), "GBps": 0.0, "frac_hbm": 0.0})
    kernels.check_device("moe microbench")
    return out


def bench_handoff(iters: int = 50, warmup: int = 10) -> None:
    """Ping-pong [T,H] between ranks 0 and 1; one-way time = round trip / 2."""
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from .comm import P2PComm

    rank = int(os.environ["RANK"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    comm = P2PComm(slot_bytes=8192 * 4096 * 2, nslot=2)
    peer = 1 - rank
    for H in (2880, 4096):
        for T in (1, 8, 64, 256, 1024, 8192):
            x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
            y = torch.empty_like(x)

            def p2p():
                if rank == 0:
                    comm.send_tensor(x, peer)
                    comm.recv_tensor(y, peer)
                else:
                    comm.recv_tensor(y, peer)
                    comm.send_tensor(y, peer)

            def nccl():
                if rank == 0:
                    dist.send(x, peer)
                    dist.recv(y, peer)
                else:
                    dist.recv(y, peer)
                    dist.send(y, peer)

            def timed(fn, n):
                torch.cuda.synchronize()
                dist.barrier()
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record()
                fn(n)
                b.record()
                torch.cuda.synchronize()
                return a.elapsed_time(b) / n / 2 * 1e3  # us, one way

            res = {}
            for name, fn in (("nvlink_put", p2p), ("nccl_sendrecv", nccl)):
                for _ in range(warmup):
                    fn()
                res[name] = timed(lambda n: [fn() for _ in range(n)], iters)
            # the same NVLink ping-pong captured in one graph per rank: device
            # time without host launch overhead (as in the graphed decode step)
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
                for _ in range(iters):
                    p2p()
            torch.cuda.current_stream().wait_stream(s)
            g.replay()
            res["nvlink_graph"] = timed(lambda n: g.replay(), iters)
            del g
            if rank == 0:
                nbytes = T * H * 2
                print(json.dumps({"kernel": "fg_handoff_put/recv", "T": T, "H": H, "bytes": nbytes,
                                  "nvlink_graph_us": res["nvlink_graph"], "nvlink_eager_us": res["nvlink_put"],
                                  "nccl_eager_us": res["nccl_sendrecv"],
                                  "nvlink_graph_GBps": nbytes / res["nvlink_graph"] / 1e3,
                                  "nccl_GBps": nbytes / res["nccl_sendrecv"] / 1e3,
                                  "link_peak_GBps": 770.0}), flush=True)
    kernels.check_device("handoff microbench")
    comm.close()
    dist.destroy_process_group()


def bench_prefill_attn(B: int, S: int, ctx: int = 0, nq: int = 32, nkv: int = 8, hd: int = 128,
                       window: int = 0, iters: int = 10, warmup: int = 3, seed: int = 4) -> dict:
    """fg_prefill_attn: S causal query positions per sequence after `ctx`
    cached ones. FLOPs = 4 * hd * nq * (attended keys summed over queries)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    L = ctx + S
    pages = (L + 15) // 16
    num_blocks = B * pages
    kc = torch.empty((num_blocks, nkv, 16, hd), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
    vc = torch.empty_like(kc).normal_(generator=g)
    table = torch.randperm(num_blocks, generator=g, device="cuda").to(torch.int32).view(B, pages).contiguous()
    q = torch.empty((B * S, nq, hd), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
    first = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    fn = lambda: kernels.prefill_attn(q, kc, vc, table, first, S, window=window, out=out)  # noqa: E731
    ms = _time(fn, iters, warmup)
    keys = sum(min(ctx + j + 1, window) if window else ctx + j + 1 for j in range(S))
    flops = 4.0 * hd * nq * B * keys
    nbytes = 2.0 * (2 * B * S * nq * hd + 2 * B * nkv * hd * L)
    kernels.check_device("prefill attn microbench")
    return {"kernel": "fg_prefill_attn", "B": B, "S": S, "context": ctx, "nq": nq, "nkv": nkv, "hd": hd,
            "window": window, "ms": ms, "TFLOPs": flops / (ms * 1e-3) / 1e12,
            "GBps": nbytes / (ms * 1e-3) / 1e9, "timing": "graph" if GRAPH else "eager"}


def bench_prefill(model: str, B: int, S: int, chunk: int, iters: int = 3, warmup: int = 1) -> dict:
    """Whole-model prefill throughput (random weights): FluidRunner.prefill of
    B prompts of S tokens in chunks of `chunk` positions, eager launches,
    CUDA events around each prefill."""
    from .config import EngineConfig
    from .engine import DecodeEngine
    from .model import SPECS, ModelWeights

    spec = SPECS[model]
    w = ModelWeights.random(spec, seed=0, device=torch.device("cuda:0"))
    eng = DecodeEngine(w, EngineConfig(model_name=spec.name, max_seq_len=S + 8, world_size=1,
                                       device="cuda:0", max_batch=B))
    ids = torch.randint(0, spec.vocab, (B, S), device="cuda")
    ts = []
    for i in range(warmup + iters):
        eng.start(B, reserve_tokens=S + 2)
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        eng.runner.prefill(ids, chunk=chunk)
        b.record()
        torch.cuda.synchronize()
        if i >= warmup:
            ts.append(a.elapsed_time(b))
    ms = statistics.median(ts)
    kernels.check_device("prefill microbench")
    return {"bench": "prefill", "model": model, "B": B, "S": S, "chunk": chunk, "ms": ms,
            "tokens_per_s": B * S / (ms * 1e-3), "timing": "eager, events around the prefill"}


def bench_vllm_moe(T: int, expert_device: str = "cuda:0", E: int = 32, H: int = 2880, I: int = 2880, k: int = 4,
                   iters: int = 20, warmup: int = 5, seed: int = 6) -> dict:
    """The vLLM MoE forward_impl (vllm_ops.make_forward_impl) at gpt-oss-20b
    layer shapes: router logits in, experts on expert_device, the result in
    the home GPU's graph-stable buffer; random MXFP4 codes and scales in the
    checkpoint's format. Eager calls bracketed by events on the home stream
    (the cross-device copies order the expert device's work into it)."""
    from .vllm_ops import ExpertsOnDevice, StableOutput, make_forward_impl

    g = torch.Generator(device="cuda:0").manual_seed(seed)
    gu_b = torch.randint(0, 256, (E, 2 * I, H // 32, 16), generator=g, device="cuda:0", dtype=torch.uint8)
    gu_s = torch.randint(119, 123, (E, 2 * I, H // 32), generator=g, device="cuda:0", dtype=torch.uint8)
    d_b = torch.randint(0, 256, (E, H, I // 32, 16), generator=g, device="cuda:0", dtype=torch.uint8)
    d_s = torch.randint(119, 123, (E, H, I // 32), generator=g, device="cuda:0", dtype=torch.uint8)
    gu_bias = torch.empty(E, 2 * I, device="cuda:0").normal_(0, 0.02, generator=g).to(torch.bfloat16)
    d_bias = torch.empty(E, H, device="cuda:0").normal_(0, 0.02, generator=g).to(torch.bfloat16)
    remote = ExpertsOnDevice(gu_b, gu_s, gu_bias, d_b, d_s, d_bias, expert_device, top_k=k)
    stable = StableOutput(max(T, 1), H, torch.bfloat16, "cuda:0")
    impl = make_forward_impl(remote, "cuda:0", stable)
    x = torch.empty(T, H, device="cuda:0").normal_(generator=g).to(torch.bfloat16)
    lg = torch.empty(T, E, device="cuda:0").normal_(0, 2, generator=g).to(torch.bfloat16)
    global GRAPH
    graph, GRAPH = GRAPH, False
    try:
        ms = _time(lambda: impl(None, x, lg, None), iters, warmup)
    finally:
        GRAPH = graph
    touched = int(torch.unique(torch.topk(lg.float(), k, dim=-1).indices).numel())
    nbytes = touched * 3 * H * I * (0.5 + 1 / 32) + 2.0 * T * H * 2
    kernels.check_device("vllm moe microbench")
    return {"op": "vllm forward_impl (MoE)", "T": T, "E": E, "H": H, "I": I, "k": k,
            "expert_device": expert_device, "experts_touched": touched, "ms": ms,
            "weight_GBps": nbytes / (ms * 1e-3) / 1e9, "timing": "eager, events on the home stream"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["attn", "gemm", "sweep-attn", "llama-gemms", "handoff", "moe",
                                     "prefill-attn", "prefill", "vllm-moe"])
    ap.add_argument("--expert-device", default="cuda:0")
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--S", type=int, default=2048)
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--window", type=int, default=0)
    ap.add_argument("--plan-len", type=int, default=0,
                    help="attn: length the split plan is made for (caps the slice count; default --context)")
    ap.add_argument("--nq", type=int, default=32)
    ap.add_argument("--nkv", type=int, default=8)
    ap.add_argument("--hd", type=int, default=128)
    ap.add_argument("--T", type=int, default=64)
    ap.add_argument("--N", type=int, default=28672)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--epilogue", default="store")
    ap.add_argument("--rowmajor", action="store_true", help="row-major weights (2-D TMA) instead of packed")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--eager", action="store_true", help="event-bracket each call instead of graph replay")
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args()
    global GRAPH
    GRAPH = not a.eager
    build.build()
    if a.what == "handoff":
        bench_handoff()
        return
    torch.cuda.set_device(0)
    if a.what == "attn":
        print(json.dumps(bench_attn(a.batch, a.context, a.nq, a.nkv, a.hd, a.window, a.iters, a.warmup,
                                    plan_len=a.plan_len)))
    elif a.what == "gemm":
        print(json.dumps(bench_gemm(a.T, a.N, a.K, a.epilogue, a.iters, a.warmup, splits=a.splits,
                                    packed=not a.rowmajor)))
    elif a.what == "prefill-attn":
        print(json.dumps(bench_prefill_attn(a.batch, a.S, a.context, a.nq, a.nkv, a.hd, a.window,
                                            a.iters, a.warmup)))
    elif a.what == "prefill":
        print(json.dumps(bench_prefill(a.model, a.batch, a.S, a.chunk)))
    elif a.what == "vllm-moe":
        for T in ([a.T] if a.T != 64 else [1, 64, 128, 512, 2048]):
            print(json.dumps(bench_vllm_moe(T, a.expert_device, iters=a.iters, warmup=a.warmup)), flush=True)
    elif a.what == "moe":
        for line in bench_moe(a.T, iters=a.iters, warmup=a.warmup):
            print(json.dumps(line), flush=True)
    elif a.what == "sweep-attn":
        for B in (1, 32, 256):
            for ctx in (512, 4096, 32768):
                if B * ctx * 8 * 128 * 4 > 40e9:  # keep each case's pool under ~40 GB
                    continue
                print(json.dumps(bench_attn(B, ctx, iters=a.iters, warmup=a.warmup)), flush=True)
                torch.cuda.empty_cache()
    elif a.what == "llama-gemms":
        T = a.T
        for N, K, epi in ((6144, 4096, "store"), (4096, 4096, "residual"), (28672, 4096, "swiglu"),
                          (4096, 14336, "residual"), (128256, 4096, "store")):
            for splits in ([a.splits] if a.splits else [0, 1, 2, 4, 8]):
                print(json.dumps(bench_gemm(T, N, K, epi, a.iters, a.warmup, splits=splits,
                                            packed=not a.rowmajor)), flush=True)


if __name__ == "__main__":
    main()
