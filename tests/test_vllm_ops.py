"""vLLM op boundary, host side (no GPU): the weight format and activation the
drop-in assumes, pinned against the libraries the reference's vLLM path
calls, and the op / proxy / runner plumbing.

  * MXFP4 checkpoint tensors (`*_blocks` [E, R, K/32, 16], `*_scales`
    [E, R, K/32]) decode as transformers' convert_moe_packed_tensors
    decodes them (the reference's bf16 expert path,
    vllm_integration.py:500-513): low nibble first, e8m0 bias 127;
  * SwiGLU-OAI on interleaved gate/up rows equals vLLM's own
    SwiGLUOAIAndMul.forward_native (the activation fused_marlin_moe applies,
    vllm_integration.py:473-482);
  * `vllm::fluidgpu_remote_mlp` is registered with a fake impl (what vLLM's
    tracer sees) and FluidRemoteMLP emits it; install_moe_forward sets the
    attribute the `vllm::moe_forward` op calls in this vLLM (`_forward_impl`)
    and in the reference's (`forward_impl`)."""
from types import SimpleNamespace

import pytest
import torch

from oracle import decode_ref as ref


def test_checkpoint_mxfp4_layout_matches_transformers():
    from transformers.integrations.mxfp4 import convert_moe_packed_tensors

    g = torch.Generator().manual_seed(0)
    E, R, K = 3, 16, 96
    blocks = torch.randint(0, 256, (E, R, K // 32, 16), generator=g, dtype=torch.uint8)
    scales = torch.randint(118, 134, (E, R, K // 32), generator=g, dtype=torch.uint8)
    hf = convert_moe_packed_tensors(blocks, scales, dtype=torch.float32)  # [E, K, R]: x @ W layout
    ours = ref.mxfp4_dequantize(blocks.reshape(E, R, K // 2), scales, torch.float32)
    assert torch.equal(ours, hf.transpose(1, 2))


def test_swiglu_oai_matches_vllm_native():
    import inspect

    act_mod = pytest.importorskip("vllm.model_executor.layers.activation")
    cls = act_mod.SwigluOAIAndMul
    # the module's defaults (alpha, limit) without building a CustomOp, which
    # needs a device-bound vLLM config
    params = inspect.signature(cls.__init__).parameters
    self_ = SimpleNamespace(alpha=params["alpha"].default, limit=params["limit"].default)
    assert (self_.alpha, self_.limit) == (1.702, 7.0)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(5, 2 * 64, generator=g) * 6  # beyond the clamp limit on both sides
    want = cls.forward_native(self_, x)
    got = ref.swiglu_oai(x[:, 0::2], x[:, 1::2])
    torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-6)


def test_remote_mlp_op_fake_and_proxy():
    from torch._subclasses.fake_tensor import FakeTensorMode

    from fluidgpu_b200 import vllm_ops

    assert hasattr(torch.ops.vllm, "fluidgpu_remote_mlp")
    with FakeTensorMode():
        x = torch.empty(7, 64, dtype=torch.bfloat16)
        y = torch.ops.vllm.fluidgpu_remote_mlp(x, "layers.0.mlp")
        assert y.shape == x.shape and y.dtype == x.dtype
    calls = []

    class Probe:
        def __call__(self, h):
            calls.append(h.shape)
            return h * 2

    vllm_ops.register_remote_mlp("probe", Probe())
    mod = vllm_ops.FluidRemoteMLP("probe")
    # the CUDA impl needs a CUDA tensor; on the host only the dispatch to the
    # registry is checked through the Python entry the op wraps
    assert vllm_ops._remote_mlp(torch.ones(2, 3), "probe").sum().item() == 12.0
    assert calls == [torch.Size([2, 3])]
    assert mod.layer_key == "probe"


@pytest.mark.parametrize("attr", ["_forward_impl", "forward_impl"])
def test_install_moe_forward_sets_the_runner_entry(attr):
    from fluidgpu_b200 import vllm_ops

    runner = SimpleNamespace(**{attr: None})
    layer = SimpleNamespace(runner=runner)

    def impl(*a, **k):
        return "ours"

    vllm_ops.install_moe_forward(layer, impl)
    assert getattr(runner, attr) is impl


def test_oracle_decode_split_adds_up():
    """The oracle's expert-range partials over [0, n) and [n, E) sum to the
    full expert output (the reference's decode split, vllm_integration.py:
    1052-1093)."""
    g = torch.Generator().manual_seed(2)
    T, E, H, I, k = 9, 8, 64, 32, 2
    x = torch.randn(T, H, generator=g)
    lg = torch.randn(T, E, generator=g)
    w1, b1 = torch.randn(E, 2 * I, H, generator=g) * 0.1, torch.randn(E, 2 * I, generator=g) * 0.1
    w2, b2 = torch.randn(E, H, I, generator=g) * 0.1, torch.randn(E, H, generator=g) * 0.1
    full = ref.vllm_moe_experts(x, lg, w1, b1, w2, b2, k)
    parts = ref.vllm_moe_experts(x, lg, w1, b1, w2, b2, k, (0, 3)) + \
        ref.vllm_moe_experts(x, lg, w1, b1, w2, b2, k, (3, E))
    torch.testing.assert_close(parts, full, rtol=1e-5, atol=1e-5)


def _fake_worker(tp=1, eager=False, mode="PIECEWISE", splitting=None, max_seqs=48, model="/nonexistent"):
    from fluidgpu_b200 import vllm_ops

    class Mode:
        name = mode

        def has_full_cudagraphs(self):
            return mode.startswith("FULL")

    comp = SimpleNamespace(cudagraph_mode=Mode(), max_cudagraph_capture_size=256,
                           splitting_ops=splitting if splitting is not None
                           else [vllm_ops.MOE_FORWARD_OP, vllm_ops.REMOTE_MLP_OP])
    cfg = SimpleNamespace(
        parallel_config=SimpleNamespace(tensor_parallel_size=tp, pipeline_parallel_size=1),
        compilation_config=comp,
        model_config=SimpleNamespace(enforce_eager=eager, model=model, dtype=torch.bfloat16,
                                     hf_config=SimpleNamespace(num_experts_per_tok=4)),
        scheduler_config=SimpleNamespace(max_num_seqs=max_seqs))
    return SimpleNamespace(vllm_config=cfg, model_runner=SimpleNamespace(model="MODEL"), device="cuda:0")


def test_apply_fluid_placement_environment(monkeypatch):
    """The worker hook reads the reference's environment variables and checks
    vLLM's configuration the way the reference does (TP=1/PP=1, piecewise
    graphs split at the ops) before installing anything."""
    from fluidgpu_b200 import vllm_ops

    seen = {}
    monkeypatch.setattr(vllm_ops, "install", lambda model, **kw: seen.update(model=model, **kw) or {"moe": 1})
    monkeypatch.delenv("FLUIDGPU_VLLM_PLACEMENT", raising=False)
    assert vllm_ops.apply_fluid_placement(_fake_worker()) is None  # default: off
    monkeypatch.setenv("FLUIDGPU_VLLM_PLACEMENT", "sideways")
    with pytest.raises(AssertionError, match="unknown placement"):
        vllm_ops.apply_fluid_placement(_fake_worker())
    monkeypatch.setenv("FLUIDGPU_VLLM_PLACEMENT", "af")
    with pytest.raises(AssertionError, match="TP=1/PP=1"):
        vllm_ops.apply_fluid_placement(_fake_worker(tp=2))
    with pytest.raises(AssertionError, match="PIECEWISE"):
        vllm_ops.apply_fluid_placement(_fake_worker(mode="FULL_AND_PIECEWISE"))
    with pytest.raises(AssertionError, match="splitting_ops"):
        vllm_ops.apply_fluid_placement(_fake_worker(splitting=[]))
    # eager mode needs no graph split
    assert vllm_ops.apply_fluid_placement(_fake_worker(eager=True, splitting=[])) == {"moe": 1}
    assert seen["expert_device"] == "cuda:1" and seen["decode_split"] == 0.0
    assert seen["phase_aware"] is False and seen["decode_threshold"] == 96  # max(64, 2 x 48)
    assert seen["home"] == "cuda:0" and seen["max_tokens"] == 256 and seen["top_k"] == 4
    assert seen["reader"] is None and seen["model"] == "MODEL"
    monkeypatch.setenv("FLUIDGPU_EXPERT_DEVICE", "cuda:3")
    monkeypatch.setenv("FLUIDGPU_DECODE_SPLIT", "0.5")
    monkeypatch.setenv("FLUIDGPU_PHASE_AWARE", "1")
    monkeypatch.setenv("FLUIDGPU_DECODE_LOCAL_THRESHOLD", "17")
    vllm_ops.apply_fluid_placement(_fake_worker())
    assert seen["expert_device"] == "cuda:3" and seen["decode_split"] == 0.5
    assert seen["phase_aware"] is True and seen["decode_threshold"] == 17


def test_fluid_compilation_config_splits_at_the_ops():
    pytest.importorskip("vllm.config.compilation")
    from fluidgpu_b200 import vllm_ops

    cc = vllm_ops.fluid_compilation_config()
    assert cc["cudagraph_mode"] == "PIECEWISE"
    assert vllm_ops.MOE_FORWARD_OP in cc["splitting_ops"] and vllm_ops.REMOTE_MLP_OP in cc["splitting_ops"]
    assert len(cc["splitting_ops"]) == len(set(cc["splitting_ops"]))
