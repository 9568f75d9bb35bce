"""The drop-in at the Python seam: the reference's own, unmodified
fluidgpu_torch objects drive FluidRunner on the B200 kernels.

- fluidgpu_torch.profile.make_ranked_task_profile writes the plan and
  load_profile reads it (with the HF config check), fluidgpu_torch.config.
  EngineConfig configures the run, and fluidgpu_torch.executor.LayerExecutor
  walks the tasks, receiving and sending the hidden state where ranks switch.
  FluidRunner supplies the kernel groups.
- One rank (every task on rank 0): prefill and decode logits equal this
  package's own engine bit for bit, and greedy tokens follow the CPU oracle.
- Two ranks as threads on one GPU (attention on rank 0, MLP on rank 1), the
  reference executor on each, hand-offs through P2PComm's same-device
  mailboxes ordered by the host: logits equal the co-located run.
- Two ranks as processes on two GPUs with the reference's own
  fluidgpu_torch.comm.ProcessGroupComm over NCCL (skipped with fewer GPUs).

The reference package is imported from baseline/_ref (installed there from
its source with pip --target); the tests skip, saying so, when it is absent.
Its runner decodes one sequence at a time (its receive buffers are
[1, 1, H]), so these runs use batch 1."""
import os
import socket
import sys
import tempfile
import traceback
from datetime import timedelta
from pathlib import Path

import pytest
import torch

from oracle import decode_ref as oracle

pytestmark = pytest.mark.gpu
REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
if not (REF / "fluidgpu_torch").is_dir():
    pytest.skip("the reference package is not installed in baseline/_ref", allow_module_level=True)
if str(REF) not in sys.path:
    sys.path.insert(0, str(REF))

PROMPT = [[5, 99, 1024, 7, 7, 300, 1999, 42, 8, 640, 11]]
STEPS = 8


def _model():
    from transformers.models.llama import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(num_hidden_layers=3, vocab_size=2048, hidden_size=512, intermediate_size=1024,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=256)
    return LlamaForCausalLM(cfg).to(torch.bfloat16).eval()


def _reference_plan(model, assignments, tmp: Path, max_seq_len=64):
    """(profile, EngineConfig factory) from the reference's own writer and loader."""
    import json

    from fluidgpu_torch.profile import load_profile, make_ranked_task_profile

    c = model.config
    raw = make_ranked_task_profile(model="dropin", task_assignments=assignments, hidden_size=c.hidden_size,
                                   num_kv_heads=c.num_key_value_heads, head_dim=c.hidden_size // c.num_attention_heads,
                                   max_seq_len=max_seq_len)
    path = tmp / "dropin.json"
    path.write_text(json.dumps(raw))
    profile = load_profile(path, model_name="dropin", hf_config=c)

    def cfg(device):
        from fluidgpu_torch.config import EngineConfig

        return EngineConfig(model_name="dropin", profiling_json=path, max_seq_len=max_seq_len, device=device,
                            strict_transformers_version=False)

    return profile, cfg


def _colocated_assignments(layers):
    out = []
    for i in range(layers):
        out += [(f"layer_{i}_attn", 0), (f"layer_{i}_mlp", 0)]
    return out


def _split_assignments(layers):
    out = []
    for i in range(layers):
        out += [(f"layer_{i}_attn", 0), (f"layer_{i}_mlp", 1)]
    return out


def _drive(runner, device):
    """Prefill the prompt, then STEPS greedy decode steps; logits per step on
    the head rank (None elsewhere)."""
    out = runner.prefill(torch.tensor(PROMPT, device=device))
    logits = []
    tok = torch.zeros(1, dtype=torch.int64)
    for _ in range(STEPS):
        if out is not None:
            logits.append(out.reshape(1, -1).float().cpu())
            tok = logits[-1].argmax(-1)
        out = runner.decode_step(tok.to(device).view(1, 1))
    torch.cuda.current_stream().synchronize()
    return logits


def _native_logits(model):
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import ModelWeights

    eng = DecodeEngine(ModelWeights.from_hf(model, "cuda:0"),
                       EngineConfig(model_name="native", max_seq_len=64, world_size=1, device="cuda:0", max_batch=1))
    eng.start(1, reserve_tokens=len(PROMPT[0]) + STEPS + 2)
    return _drive(eng.runner, "cuda:0")


class _OneRank:
    def get_rank(self):
        return 0

    def send_tensor(self, t, dst):
        raise AssertionError("a co-located plan sent a tensor")

    def recv_tensor(self, t, src):
        raise AssertionError("a co-located plan received a tensor")

    def broadcast_tensor(self, t, src=0):
        return None


def test_reference_executor_and_plan_drive_fluid_runner():
    from fluidgpu_torch.executor import LayerExecutor as RefExecutor
    from fluidgpu_torch.profile import owned_layer_ids

    from fluidgpu_b200 import build, kernels
    from fluidgpu_b200.model import ModelWeights
    from fluidgpu_b200.runner import FluidRunner

    build.build()
    model = _model()
    with tempfile.TemporaryDirectory() as d:
        profile, cfg = _reference_plan(model, _colocated_assignments(3), Path(d))
        ecfg = cfg("cuda:0")
        runner = FluidRunner(ModelWeights.from_hf(model, "cuda:0"), None, RefExecutor(profile, ecfg, _OneRank()),
                             ecfg, owned_layer_ids(profile, 0))
        got = _drive(runner, "cuda:0")
    want = _native_logits(model)
    for s in range(STEPS):
        assert torch.equal(got[s], want[s]), f"step {s}: reference-driven logits differ from the native engine"
    # and the tokens follow the exact model wherever its decision is clear
    truth = oracle.OracleModel(oracle.spec_from_hf(model.config),
                               {k: v.float() for k, v in oracle.weights_from_hf(model).items()}, torch.float32)
    lt = truth.prefill(torch.tensor(PROMPT))
    for s in range(STEPS):
        top2 = lt.float().topk(2, dim=-1).values[0]
        if (top2[0] - top2[1]).item() > 2 * (2e-2 + 1e-2 * top2[0].abs().item()):
            assert int(got[s].argmax()) == int(oracle.argmax_lowest(lt.float())[0]), f"step {s}"
        assert ((got[s] - lt.float()).abs() <= 2e-2 + 1e-2 * lt.float().abs()).all(), f"step {s}"
        lt = truth.step(got[s].argmax(-1))
    kernels.check_device("reference-driven runner")


def test_reference_executor_two_ranks_on_one_gpu():
    from fluidgpu_torch.executor import LayerExecutor as RefExecutor
    from fluidgpu_torch.profile import owned_layer_ids

    from fluidgpu_b200.model import ModelWeights
    from fluidgpu_b200.runner import FluidRunner
    from tests.test_handoff_gpu import _one_gpu_group, _run_threads

    model = _model()
    comms = _one_gpu_group(2)[0]
    result = {}
    with tempfile.TemporaryDirectory() as d:
        profile, cfg = _reference_plan(model, _split_assignments(3), Path(d))

        def body(rank):
            ecfg = cfg("cuda:0")
            runner = FluidRunner(ModelWeights.from_hf(model, "cuda:0"), None,
                                 RefExecutor(profile, ecfg, comms[rank]), ecfg, owned_layer_ids(profile, rank))
            result[rank] = _drive(runner, "cuda:0")

        _run_threads(2, body)
    assert result[1] == []
    want = _native_logits(model)
    for s in range(STEPS):
        assert torch.equal(result[0][s], want[s]), f"step {s}: two-rank logits differ from co-located"


# ---------------------------------------------------------------------------
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, port, plan_dir, q):
    try:
        import torch.distributed as dist

        sys.path.insert(0, str(REF))
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev, timeout=timedelta(seconds=60))
        from fluidgpu_torch.comm import ProcessGroupComm
        from fluidgpu_torch.executor import LayerExecutor as RefExecutor
        from fluidgpu_torch.profile import owned_layer_ids

        from fluidgpu_b200 import build
        from fluidgpu_b200.model import ModelWeights
        from fluidgpu_b200.runner import FluidRunner

        build.build()
        model = _model()
        profile, cfg = _reference_plan(model, _split_assignments(3), Path(plan_dir))
        ecfg = cfg(f"cuda:{rank}")
        runner = FluidRunner(ModelWeights.from_hf(model, dev), None, RefExecutor(profile, ecfg, ProcessGroupComm()),
                             ecfg, owned_layer_ids(profile, rank))
        got = _drive(runner, dev)
        dist.barrier()
        dist.destroy_process_group()
        # plain lists: tensors would travel as shared-memory handles that die with this process
        q.put((rank, True, [t.tolist() for t in got] if rank == 0 else None, ""))
    except BaseException:  # noqa: BLE001
        q.put((rank, False, None, traceback.format_exc()))


def test_reference_process_group_comm_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=_nccl_worker, args=(r, port, d, q)) for r in range(2)]
        for p in procs:
            p.start()
        results = sorted(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=60)
    for rank, ok, _, msg in results:
        assert ok, f"rank {rank} failed:\n{msg}"
    from fluidgpu_b200 import build

    build.build()
    want = _native_logits(_model())
    got = [torch.tensor(x, dtype=torch.float32) for x in results[0][2]]
    for s in range(STEPS):
        assert torch.equal(got[s], want[s]), f"step {s}: NCCL two-rank logits differ from co-located"
