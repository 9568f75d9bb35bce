"""CUDA-graph decode: replaying the captured step must reproduce the eager
kernel path bit for bit (same kernels, same launch plans), across a length
bucket boundary (a new capture), with the host mirror in step."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _engine(graph: bool, batch=4, max_len=600):
    from fluidgpu_b200 import build
    from fluidgpu_b200.config import EngineConfig
    from fluidgpu_b200.engine import DecodeEngine
    from fluidgpu_b200.model import ModelSpec, ModelWeights

    build.build()
    spec = ModelSpec(name="graph-test", family="llama", num_layers=2, hidden=512, n_q=8, n_kv=2,
                     head_dim=64, intermediate=1024, vocab=1000, rope_theta=10000.0)
    w = ModelWeights.random(spec, seed=3, device="cuda")
    cfg = EngineConfig(model_name="g", max_seq_len=max_len, world_size=1, device="cuda:0",
                       max_batch=batch, cuda_graph_decode=graph)
    return DecodeEngine(w, cfg)


def test_graph_replay_matches_eager_tokens():
    from fluidgpu_b200 import kernels

    batch, start = 4, 250  # bucket 256 -> 512 boundary crossed during the run
    toks = {}
    for graph in (False, True):
        eng = _engine(graph, batch)
        eng.start(batch, prompt_lens=[start] * batch, reserve_tokens=300)
        g = torch.Generator(device="cuda").manual_seed(0)
        eng.kv_cache.pool.normal_(0.0, 1.0, generator=g)
        host = torch.arange(batch, dtype=torch.int64) + 7
        seq = []
        for _ in range(20):
            host = eng.step(host.pin_memory())
            seq.append(host.clone())
        toks[graph] = torch.stack(seq)
        assert eng.kv_cache.seq_lengths() == [start + 20] * batch
        if graph:
            assert set(eng._graphs) == {256, 512}
        kernels.check_device("graph test")
    assert torch.equal(toks[False], toks[True])
