"""Two ranks as processes over gloo on CPU: the executor's hand-off protocol
through ProcessGroupComm (torch.distributed send / recv, the reference's own
backend, fluidgpu_torch/comm.py:14-61), and a rank that leaves early being
detected on the host within the process group's timeout.

Mirrors the reference's two-rank runtime tests (test_fine_dense_runtime.py:
103-141, test_executor_boundary.py:27-56) with processes instead of threads.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

LAYERS, B, H = 3, 2, 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, q):
    import torch.distributed as dist

    from fluidgpu_b200.comm import ProcessGroupComm
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.executor import LayerExecutor
    from fluidgpu_b200.profile import attn_ffn_profile, profile_from_dict

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        prof = profile_from_dict(attn_ffn_profile("m", LAYERS, H, 2, 2, 8))
        cfg = EngineConfig(model_name="m", device="cpu", max_seq_len=8, dtype=torch.bfloat16, max_batch=B)
        ex = LayerExecutor(prof, cfg, ProcessGroupComm())
        if case == "leave" and rank == 1:
            # the FFN rank leaves before its first hand-off, between steps
            q.put((rank, "left", None))
            return
        h = torch.zeros(B, 1, H, dtype=torch.bfloat16)
        h = ex.run_stage("embed", lambda x: x, h, mode="decode", seq_len=1)
        ran = []
        for i in range(LAYERS):
            for suffix in ("attn", "mlp"):
                name = f"layer_{i}_{suffix}"

                def fn(x, name=name):
                    ran.append(name)
                    return x + (1 if suffix == "attn" else 2)

                out = ex.run_kernel_group(name, fn, h, mode="decode", seq_len=1, batch=B)
                h = out if out is not None else h
        res = ex.run_stage("norm_lm_head", lambda x: x, h, mode="decode", seq_len=1, batch=B)
        q.put((rank, ran, None if res is None else res.float().tolist()))
        dist.barrier()
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, "error", f"{type(exc).__name__}: {exc}"))
    finally:
        if dist.is_initialized() and not (case == "leave" and rank == 1):
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def _run(case, world=2, join_s=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, a, b = q.get(timeout=join_s)
            results[rank] = (a, b)
    finally:
        for p in procs:
            p.join(timeout=join_s)
            if p.is_alive():
                p.kill()
                p.join()
    return results


def test_attention_ffn_ranks_over_gloo():
    """Attention on rank 0, FFN on rank 1: each layer's hidden state goes
    0 -> 1 -> 0 through torch.distributed; rank 0 ends with the full sum."""
    res = _run("af")
    ran0, out0 = res[0]
    ran1, out1 = res[1]
    assert ran0 == [f"layer_{i}_attn" for i in range(LAYERS)], res
    assert ran1 == [f"layer_{i}_mlp" for i in range(LAYERS)], res
    assert out1 is None
    assert torch.equal(torch.tensor(out0), torch.full((B, 1, H), 3.0 * LAYERS))


def test_rank_that_leaves_is_detected_on_the_host():
    """The FFN rank exits before its first hand-off: the attention rank's
    receive ends with an error (closed peer or the 10 s group timeout)
    instead of waiting for good."""
    res = _run("leave")
    assert res[1][0] == "left"
    status, msg = res[0]
    assert status == "error", res
    assert msg
