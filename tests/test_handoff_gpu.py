"""NVLink hand-off (fg_handoff_put / fg_handoff_recv, fg_handoff_signal /
fg_handoff_wait, P2PComm) and the ping-pong micro-batch schedule.

- A receive whose flag nobody sets gives up after its bound, records the
  peer-flag-timeout status and leaves the context usable (single GPU).
- Ranks as threads on ONE GPU (P2PComm.same_device_group: every rank's
  mailbox in that GPU's memory, the same kernels, slots, flags and sequence
  numbers as across GPUs). The host orders the ranks: each receive or wait is
  enqueued behind a CUDA event recorded after the matching send or signal
  (and each send behind the receive that freed its slot), so no hand-off
  kernel ever waits on a launch that has not completed. Cases: round trips
  of 16 B .. 1 MiB messages through two slots, the same four kernels
  replayed from one captured graph, disaggregated decodes (copying and
  zero-copy) and a fine-grained split plan whose logits equal a co-located
  run bit for bit, a tensor-parallel FFN over two ranks, and the ping-pong
  engine (co-located with graph replays, and disaggregated) whose tokens
  equal one engine per micro-batch.
- Two and three ranks as processes on as many GPUs: the same cases over
  NVLink with the ranks running concurrently (skipped on a box with fewer
  GPUs)."""
import os
import queue
import socket
import threading
import traceback
from collections import defaultdict
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_recv_times_out_cleanly():
    from fluidgpu_b200 import _lib, build, kernels

    build.build()
    lib = _lib.lib()
    slot = 4096
    mb = torch.zeros(lib.fg_mailbox_bytes(2, 2, slot), dtype=torch.uint8, device="cuda")
    out = torch.empty(slot, dtype=torch.uint8, device="cuda")
    kernels.device_status(reset=True)
    # rank 0 waits for a message from rank 1 that is never sent (its own
    # mailbox stands in for the peer's: only the final ack lands there)
    _lib.call("fg_handoff_recv", out.data_ptr(), slot, mb.data_ptr(), mb.data_ptr(), 2, 0, 1, 2, slot,
              200, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    st = kernels.device_status(reset=True)
    assert st & 0xFF == 2, f"expected a peer flag timeout, got status {st:#x}"
    # the context is still usable
    x = torch.arange(10, device="cuda")
    assert int(x.sum().item()) == 45


# ---------------------------------------------------------------------------
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _roundtrip(rank, comm):
    sizes = [16, 4096, 65536, 128 * 1024, 16, 100 * 16, 1 << 20]
    for it in range(24):
        n = sizes[it % len(sizes)] // 2
        if rank == 0:
            x = (torch.arange(n, device="cuda", dtype=torch.float32) + it).to(torch.bfloat16)
            comm.send_tensor(x, 1)
            y = torch.empty_like(x)
            comm.recv_tensor(y, 1)
            torch.cuda.synchronize()
            assert torch.equal(y.float(), x.float() * 2), f"iteration {it}"
        else:
            z = torch.empty(n, dtype=torch.bfloat16, device="cuda")
            comm.recv_tensor(z, 0)
            comm.send_tensor(z * 2, 0)
            torch.cuda.synchronize()


def _graphed(rank, comm):
    n = 8192
    x = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros_like(x)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            if rank == 0:
                comm.send_tensor(x, 1)
                comm.recv_tensor(y, 1)
            else:
                comm.recv_tensor(y, 0)
                x.copy_(y + 1)
                comm.send_tensor(x, 0)
    torch.cuda.current_stream().wait_stream(s)
    for it in range(10):
        if rank == 0:
            x.fill_(float(it))
        g.replay()
        torch.cuda.synchronize()
        if rank == 0:
            assert torch.equal(y, torch.full_like(y, float(it + 1))), f"replay {it}"
    del g


def _attn_ffn_plan():
    from fluidgpu_b200.profile import attn_ffn_profile

    return attn_ffn_profile("disagg", 3, 512, 2, 64, 64)


def _fine_plan():
    from fluidgpu_b200.profile import make_ranked_task_profile

    return make_ranked_task_profile(model="disagg", task_assignments=[
        ("layer_0_qkv", 0), ("layer_0_sdpa", 1), ("layer_0_o_proj", 0),
        ("layer_0_mlp_gate_up", 1), ("layer_0_mlp_down_proj", 0),
        ("layer_1_qkv", 1), ("layer_1_sdpa", 0), ("layer_1_o_proj", 1), ("layer_1_mlp", 0),
        ("layer_2_attn", 1), ("layer_2_mlp_gate_up", 0), ("layer_2_mlp_down_proj", 1),
    ], hidden_size=512, num_kv_heads=2, head_dim=64, max_seq_len=64, rank_count=2)


def _llama():
    from transformers.models.llama import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(num_hidden_layers=3, vocab_size=2048, hidden_size=512, intermediate_size=1024,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=256)
    return LlamaForCausalLM(cfg).to(torch.bfloat16).eval()


def _disaggregated(rank, comm, plan=_attn_ffn_plan, device=None, model=None):
    """`model`: the HF model (built here when None; ranks that are threads of
    one process share one, since the global RNG is shared between threads)."""
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import ModelWeights
    from fluidgpu_b200.profile import has_fine_groups, profile_from_dict

    model = model if model is not None else _llama()
    B, prompt, steps = 4, 10, 6
    dev = device or f"cuda:{rank}"
    ecfg = EngineConfig(model_name="disagg", max_seq_len=64, world_size=2, device=dev, max_batch=B)
    prof = profile_from_dict(plan())
    eng = DecodeEngine(ModelWeights.from_hf(model, dev), ecfg, profile=prof, comm=comm)
    if getattr(comm, "direct", False):
        assert eng.executor._direct == (plan is _attn_ffn_plan)
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, 2048, (B, prompt), generator=g)
    eng.start(B, reserve_tokens=prompt + steps + 2)
    logits = []
    out = eng.runner.prefill(prompts.to(dev))
    tok = torch.zeros(B, dtype=torch.int64)
    for _ in range(steps):
        if rank == 0:
            logits.append(out.reshape(B, -1).float().cpu())
            tok = logits[-1].argmax(-1)
        out = eng.runner.decode_step(tok.to(dev))
    torch.cuda.current_stream().synchronize()
    if rank == 1:
        assert out is None
        return
    # co-located reference on the same GPU, same kernels
    ref = DecodeEngine(ModelWeights.from_hf(model, "cuda:0"),
                       EngineConfig(model_name="colo", max_seq_len=64, world_size=1, device="cuda:0",
                                    max_batch=B))
    ref.start(B, reserve_tokens=prompt + steps + 2)
    out = ref.runner.prefill(prompts.cuda(), chunk=1 if has_fine_groups(prof) else None)
    for s in range(steps):
        lg = out.reshape(B, -1).float().cpu()
        assert torch.equal(lg, logits[s]), f"step {s}: disaggregated logits differ"
        out = ref.runner.decode_step(lg.argmax(-1).cuda())


def _sharded(rank, comm, device=None, model=None):
    """Attention on rank 0, every layer's FFN tensor-parallel over ranks 1 and 2
    (fp32 partials over NVLink, added up on rank 0): logits within the bf16
    tolerance of a co-located run."""
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import ModelWeights
    from fluidgpu_b200.profile import ffn_shard_of, profile_from_dict, sharded_ffn_profile

    model = model if model is not None else _llama()
    B, prompt, steps = 4, 10, 6
    dev = device or f"cuda:{rank}"
    prof = profile_from_dict(sharded_ffn_profile("tp", 3, 512, 2, 64, 64, shard_ranks=[1, 2]))
    eng = DecodeEngine(ModelWeights.from_hf(model, dev, ffn_shard=ffn_shard_of(prof, rank)),
                       EngineConfig(model_name="tp", max_seq_len=64, world_size=3, device=dev,
                                    max_batch=B), profile=prof, comm=comm)
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, 2048, (B, prompt), generator=g)
    eng.start(B, reserve_tokens=prompt + steps + 2)
    logits = []
    out = eng.runner.prefill(prompts.to(dev))
    tok = torch.zeros(B, dtype=torch.int64)
    for _ in range(steps):
        if rank == 0:
            logits.append(out.reshape(B, -1).float().cpu())
            tok = logits[-1].argmax(-1)
        out = eng.runner.decode_step(tok.to(dev))
    torch.cuda.current_stream().synchronize()
    if rank != 0:
        assert out is None
        return
    ref = DecodeEngine(ModelWeights.from_hf(model, "cuda:0"),
                       EngineConfig(model_name="colo", max_seq_len=64, world_size=1, device="cuda:0",
                                    max_batch=B))
    ref.start(B, reserve_tokens=prompt + steps + 2)
    out = ref.runner.prefill(prompts.cuda())
    for s in range(steps):
        lg = out.reshape(B, -1).float().cpu()
        assert ((logits[s] - lg).abs() <= 2e-2 + 1e-2 * lg.abs()).all(), f"step {s}"
        out = ref.runner.decode_step(logits[s].argmax(-1).cuda())


def _direct_graphed(rank, comm):
    """Zero-copy hand-offs (the o_proj / down GEMM writes the peer's slot, the
    peer reads it in place), replayed from per-rank CUDA graphs: greedy tokens
    and logits equal a co-located run bit for bit."""
    from transformers.models.llama import LlamaConfig, LlamaForCausalLM

    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import ModelWeights
    from fluidgpu_b200.profile import profile_from_dict

    assert comm.direct
    torch.manual_seed(0)
    cfg = LlamaConfig(num_hidden_layers=3, vocab_size=2048, hidden_size=512, intermediate_size=1024,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=256)
    model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    B, prompt, steps = 4, 10, 8
    ecfg = EngineConfig(model_name="disagg", max_seq_len=64, world_size=2, device=f"cuda:{rank}",
                        max_batch=B, cuda_graph_decode=True)
    eng = DecodeEngine(ModelWeights.from_hf(model, f"cuda:{rank}"), ecfg, profile=profile_from_dict(_attn_ffn_plan()),
                       comm=comm)
    assert eng.executor._direct
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, 2048, (B, prompt), generator=g)
    eng.start(B, reserve_tokens=prompt + steps + 2)
    out = eng.runner.prefill(prompts.cuda())  # eager steps through the direct channel
    tok = out.reshape(B, -1).float().argmax(-1).cpu() if rank == 0 else torch.zeros(B, dtype=torch.int64)
    toks = []
    for _ in range(steps):  # graphed steps
        nxt = eng.step(tok)
        if rank == 0:
            toks.append(nxt)
            tok = nxt
    torch.cuda.synchronize()
    if rank != 0:
        return
    ref = DecodeEngine(ModelWeights.from_hf(model, "cuda:0"),
                       EngineConfig(model_name="colo", max_seq_len=64, world_size=1, device="cuda:0",
                                    max_batch=B, cuda_graph_decode=True))
    ref.start(B, reserve_tokens=prompt + steps + 2)
    out = ref.runner.prefill(prompts.cuda())
    tok = out.reshape(B, -1).float().argmax(-1).cpu()
    for s in range(steps):
        tok = ref.step(tok)
        assert torch.equal(tok, toks[s]), f"step {s}: direct hand-off tokens differ"


CASES = {"roundtrip": _roundtrip, "graphed": _graphed, "disaggregated": _disaggregated,
         "fine_split": lambda rank, comm: _disaggregated(rank, comm, _fine_plan), "sharded": _sharded,
         "direct": _disaggregated, "direct_graphed": _direct_graphed}


def _worker(rank, world, port, case, q):
    try:
        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        from fluidgpu_b200 import build, kernels
        from fluidgpu_b200.comm import P2PComm

        build.build()
        comm = P2PComm(slot_bytes=1 << 20, nslot=2, timeout_ms=5000, direct=case.startswith("direct"))
        CASES[case](rank, comm)
        torch.cuda.synchronize()
        kernels.check_device(f"{case} rank {rank}")
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, True, ""))
    except BaseException:  # noqa: BLE001
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.parametrize("case", [c for c in CASES if c != "sharded"])
def test_two_ranks(case):
    _spawn(case, 2)


def test_three_ranks_tensor_parallel_ffn():
    _spawn("sharded", 3)


def _spawn(case, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for _ in procs:
        results.append(q.get(timeout=300))
    for p in procs:
        p.join(timeout=60)
    for rank, ok, msg in sorted(results):
        assert ok, f"rank {rank} failed:\n{msg}"


# ---------------------------------------------------------------------------
# ranks as threads on one GPU
# ---------------------------------------------------------------------------
class _HostOrdered:
    """One rank's P2PComm for ranks that share a GPU, ordered by the host.

    Every hand-off kernel is enqueued only behind the kernel it depends on,
    through a CUDA event that the other rank recorded after enqueueing it: a
    receive behind its send, a send behind the receive that drained its slot
    (message n - nslot), a wait behind its signal. Every device-side flag a
    kernel tests is therefore already set when it starts: none waits on a
    launch that has not run."""

    def __init__(self, comm, board):
        self.c = comm
        self.board = board
        self.rank = comm.rank
        self.direct = comm.direct
        self.slot_bytes = comm.slot_bytes
        self.sent = defaultdict(int)

    def get_rank(self):
        return self.rank

    def _post(self, key):
        ev = torch.cuda.Event()
        ev.record()
        self.board[key].put(ev)

    def _take(self, key):
        ev = self.board[key].get(timeout=60)
        torch.cuda.current_stream().wait_event(ev)

    def send_tensor(self, t, dst):
        if self.sent[dst] >= self.c.nslot:
            self._take(("ack", dst, self.rank))
        self.c.send_tensor(t, dst)
        self.sent[dst] += 1
        self._post(("msg", self.rank, dst))

    def recv_tensor(self, out, src):
        self._take(("msg", src, self.rank))
        self.c.recv_tensor(out, src)
        self._post(("ack", self.rank, src))

    def direct_out(self, dst, shape, dtype):
        return self.c.direct_out(dst, shape, dtype)

    def direct_signal(self, dst):
        self.c.direct_signal(dst)
        self._post(("dmsg", self.rank, dst))

    def direct_wait(self, src):
        self._take(("dmsg", src, self.rank))
        self.c.direct_wait(src)

    def direct_in(self, src, shape, dtype):
        return self.c.direct_in(src, shape, dtype)

    def broadcast_tensor(self, t, src=0):
        return None


def _one_gpu_group(world, *, direct=False, channels=1, slot=1 << 20):
    """[channel][rank] host-ordered comms of `world` ranks on cuda:0."""
    from fluidgpu_b200.comm import P2PComm

    board = defaultdict(queue.Queue)
    out = []
    for _ in range(channels):
        comms = P2PComm.same_device_group(world, slot, nslot=2, timeout_ms=5000,
                                          device=torch.device("cuda", 0), direct=direct)
        out.append([_HostOrdered(c, board) for c in comms])
    return out


def _run_threads(world, body):
    """body(rank) in one thread per rank, each on its own stream of cuda:0."""
    from fluidgpu_b200 import build, kernels

    build.build()
    errors = []

    def run(rank):
        try:
            torch.cuda.set_device(0)
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                body(rank)
            s.synchronize()
        except BaseException:  # noqa: BLE001
            errors.append((rank, traceback.format_exc()))

    kernels.device_status(reset=True)
    threads = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=600)
    assert not any(t.is_alive() for t in threads), "a rank thread did not finish"
    assert not errors, "\n".join(f"rank {r}:\n{m}" for r, m in errors)
    torch.cuda.synchronize()
    kernels.check_device("one-GPU ranks")


ONE_GPU_CASES = {
    "roundtrip": (2, False, lambda r, c, m: _roundtrip(r, c)),
    "disaggregated": (2, False, lambda r, c, m: _disaggregated(r, c, device="cuda:0", model=m)),
    "fine_split": (2, False, lambda r, c, m: _disaggregated(r, c, _fine_plan, device="cuda:0", model=m)),
    "direct": (2, True, lambda r, c, m: _disaggregated(r, c, device="cuda:0", model=m)),
    "sharded": (3, False, lambda r, c, m: _sharded(r, c, device="cuda:0", model=m)),
}


@pytest.mark.parametrize("case", list(ONE_GPU_CASES))
def test_ranks_on_one_gpu(case):
    world, direct, fn = ONE_GPU_CASES[case]
    comms = _one_gpu_group(world, direct=direct)[0]
    model = _llama()  # one model for all rank threads (the RNG is process-wide)
    _run_threads(world, lambda r: fn(r, comms[r], model))


def test_handoff_kernels_replayed_from_one_graph():
    """Rank 0's put, rank 1's receive, rank 1's put and rank 0's receive in
    stream order inside one captured graph, replayed 24 times: the device
    sequence numbers advance on every replay and the two slots alternate."""
    from fluidgpu_b200 import build, kernels
    from fluidgpu_b200.comm import P2PComm

    build.build()
    c0, c1 = P2PComm.same_device_group(2, 1 << 16, nslot=2, timeout_ms=5000, device=torch.device("cuda", 0))
    n = 12288  # 24 KiB of bf16
    x = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    mid = torch.zeros_like(x)
    back = torch.zeros_like(x)
    y = torch.zeros_like(x)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    kernels.device_status(reset=True)
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            c0.send_tensor(x, 1)
            c1.recv_tensor(mid, 0)
            torch.add(mid, 1, out=back)
            c1.send_tensor(back, 0)
            c0.recv_tensor(y, 1)
    torch.cuda.current_stream().wait_stream(s)
    base = torch.arange(n, device="cuda", dtype=torch.float32) % 97
    for it in range(24):
        x.copy_((base + it).to(torch.bfloat16))
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, (x.float() + 1).to(torch.bfloat16)), f"replay {it}"
    del g
    kernels.check_device("graphed hand-off")


def _pp_reference(model, prompts, steps):
    """Greedy tokens of each micro-batch's sequences from a co-located engine
    of their own: [M][steps] tensors [B]."""
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import ModelWeights

    out = []
    for p in prompts:
        B, S = p.shape
        eng = DecodeEngine(ModelWeights.from_hf(model, "cuda:0"),
                           EngineConfig(model_name="colo", max_seq_len=64, world_size=1, device="cuda:0",
                                        max_batch=B))
        eng.start(B, reserve_tokens=S + steps + 2)
        lg = eng.runner.prefill(p.cuda())
        tok = lg.reshape(B, -1).float().argmax(-1)
        toks = [tok.cpu()]
        for _ in range(steps - 1):
            tok = eng.runner.decode_step(tok).reshape(B, -1).float().argmax(-1)
            toks.append(tok.cpu())
        out.append(toks)
    return out


def _pp_run(rank, comm_of, model, prompts, steps, plan, world, graphs):
    """A PingPongEngine on this rank: prefill each micro-batch, then `steps`
    interleaved greedy steps; returns [M][steps] token tensors on the head
    rank."""
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.model import ModelWeights
    from fluidgpu_b200.pingpong import PingPongEngine
    from fluidgpu_b200.profile import profile_from_dict

    M = len(prompts)
    B, S = prompts[0].shape
    cfg = EngineConfig(model_name="pp", max_seq_len=64, world_size=world, device="cuda:0", max_batch=B,
                       cuda_graph_decode=graphs)
    pp = PingPongEngine(ModelWeights.from_hf(model, "cuda:0"), cfg, profile_from_dict(plan), comm_of,
                        micro_batches=M)
    pp.start(B, reserve_tokens=S + steps + 2)
    toks = [[] for _ in range(M)]
    for m, eng in enumerate(pp.engines):
        lg = eng.runner.prefill(prompts[m].cuda())
        if lg is not None:
            first = lg.reshape(B, -1).float().argmax(-1)
            eng.set_tokens(first)
            toks[m].append(first.cpu())
    if graphs:
        pp.capture()
    for _ in range(steps - 1):
        outs = pp.step()
        for m, o in enumerate(outs):
            if o is not None:
                toks[m].append(o.cpu())
    torch.cuda.current_stream().synchronize()
    return toks


@pytest.mark.parametrize("M", [2, 3])
def test_pingpong_colocated_graphs(M):
    """The ping-pong engine on one rank: M micro-batches, each its own runner,
    KV slice and captured graph, replayed interleaved on staggered-priority
    streams; every micro-batch's greedy tokens equal an engine of its own."""
    from fluidgpu_b200 import build, kernels
    from fluidgpu_b200.comm import LocalComm
    from fluidgpu_b200.profile import colocated_profile

    build.build()
    model = _llama()
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 2048, (4, 9 + 3 * m), generator=g) for m in range(M)]
    steps = 10
    plan = colocated_profile("pp", 3, 512, 2, 64, 64)
    got = _pp_run(0, lambda m: LocalComm(), model, prompts, steps, plan, 1, graphs=True)
    want = _pp_reference(model, prompts, steps)
    for m in range(M):
        for s in range(steps):
            assert torch.equal(got[m][s], want[m][s]), f"micro-batch {m} step {s}"
    kernels.check_device("ping-pong co-located")


def test_pingpong_disaggregated_one_gpu():
    """Two micro-batches ping-ponging between an attention rank and an FFN
    rank (threads on one GPU, host-ordered zero-copy hand-offs, one mailbox
    set per micro-batch): tokens equal an engine per micro-batch."""
    from fluidgpu_b200.profile import attn_ffn_profile

    model = _llama()
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 2048, (4, 10), generator=g) for _ in range(2)]
    steps = 8
    plan = attn_ffn_profile("pp", 3, 512, 2, 64, 64)
    chans = _one_gpu_group(2, direct=True, channels=2)
    result = {}

    def body(rank):
        result[rank] = _pp_run(rank, lambda m: chans[m][rank], model, prompts, steps, plan, 2, graphs=False)

    _run_threads(2, body)
    want = _pp_reference(model, prompts, steps)
    for m in range(2):
        assert len(result[0][m]) == steps
        for s in range(steps):
            assert torch.equal(result[0][m][s], want[m][s]), f"micro-batch {m} step {s}"
