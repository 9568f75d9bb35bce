"""vLLM op boundary on the B200 kernels: the drop-in for the reference's
vLLM integration (fluidgpu_torch/vllm_integration.py), where FluidGPU puts a
model's feed-forward groups on an "expert device" next to vLLM's own engine.

The seams are the reference's, unchanged:
  * gpt-oss / MoE: the function behind vLLM's opaque `vllm::moe_forward` op,
    `forward_impl(layer, hidden_states [T,H], router_logits [T,E],
    shared_experts_input=None) -> [T,H]` (vllm_integration.py:1419-1615),
    installed on each FusedMoE layer's runner (`forward_impl` in vLLM 0.18,
    `_forward_impl` in 0.22, which adds `input_ids`);
  * dense MLP: the custom op `vllm::fluidgpu_remote_mlp(hidden_states,
    layer_key) -> Tensor` with a fake impl for tracing (:1375-1399) and the
    proxy module whose class-level forward emits it (:1403-1416);
  * graph-stable outputs (:227-287): for token counts up to the largest
    piecewise-graph capture size, results land in one persistent buffer on
    the home GPU, so every replay sees the same address;
  * the worker hook `apply_fluid_placement(worker)` (:1668-1866) and the
    `fluid_compilation_config()` that splits vLLM's FX graph at the ops
    (:2042-2073), configured by the same environment variables.

What runs behind them is this package's: expert weights stay MXFP4 in the
fg_pack_mxfp4 tile records (no marlin repack, no bf16 dequantisation) and run
through fg_moe_topk_softmax -> fg_moe_permute -> fg_moe_gather ->
fg_moe_gemm_mxfp4 (gate_up, SwiGLU-OAI) -> fg_moe_gemm_mxfp4 (down) ->
fg_moe_unpermute; the dense MLP's [gate; up] weight is regrouped into 64-row
blocks so one tcgen05 GEMM applies SiLU(gate) * up in its epilogue, and the
down GEMM stores. Hops between the home GPU and the expert device are peer
copies over NVLink (the reference stages through host memory or RDMA: its
A100 / L40S pair has no peer access).

MoE semantics (vllm_integration.py:452-485, MarlinExpertsOnDevice): top-k of
the router logits, softmax over the k selected, experts with biases and
SwiGLU-OAI on interleaved gate/up rows (alpha 1.702, limit 7), weighted sum.
`expert_range` loads experts [lo, hi) only and returns the fp32 partial over
them (the reference's expert_map split, :371-390); two partials add up to the
full output (the decode split, :1052-1093).
"""
from __future__ import annotations

import glob
import json
import os
from pathlib import Path
from types import SimpleNamespace
from typing import Any

import torch

from . import _lib, kernels, moe
from ._lib import call
from .model import interleave_gate_up

REMOTE_MLP_OP = "vllm::fluidgpu_remote_mlp"
MOE_FORWARD_OP = "vllm::moe_forward"


def _env(name: str, default: str) -> str:
    return os.environ.get(name, default)


# ---------------------------------------------------------------------------
# hops and graph-stable outputs
# ---------------------------------------------------------------------------
def hop_tensor(tensor: torch.Tensor, dst_device: str | torch.device) -> torch.Tensor:
    """The tensor on dst_device: itself when it is there already, else a peer
    copy over NVLink ordered after the producer's stream (hop_tensor,
    vllm_integration.py:169-188)."""
    dst = torch.device(dst_device)
    if tensor.device == dst:
        return tensor
    return tensor.to(dst, non_blocking=True)


class StableOutput:
    """Persistent [max_tokens, width] output buffer on the home GPU: results
    of up to max_tokens rows are returned as views of it (the address a
    piecewise CUDA graph captured), larger ones as fresh tensors
    (_StableOutput, vllm_integration.py:227-287). One buffer per micro-batch
    id, so concurrent micro-batch streams never share rows."""

    def __init__(self, max_tokens: int, width: int, dtype: torch.dtype, device: str | torch.device) -> None:
        self.max_tokens = int(max_tokens)
        self.width = int(width)
        self.dtype = dtype
        self.device = torch.device(device)
        self._bufs: dict[int, torch.Tensor] = {}
        if self.max_tokens > 0:
            self._bufs[0] = torch.zeros((self.max_tokens, self.width), dtype=dtype, device=self.device)

    def view(self, num_tokens: int, ubatch: int = 0) -> torch.Tensor | None:
        """The rows a result of num_tokens rows lands in, or None (too large)."""
        if num_tokens > self.max_tokens:
            return None
        buf = self._bufs.get(ubatch)
        if buf is None:
            buf = torch.zeros((self.max_tokens, self.width), dtype=self.dtype, device=self.device)
            self._bufs[ubatch] = buf
        return buf[:num_tokens]

    def stage(self, result: torch.Tensor, ubatch: int = 0) -> torch.Tensor:
        dst = self.view(result.shape[0], ubatch)
        if dst is None:
            return hop_tensor(result, self.device)
        if dst.data_ptr() != result.data_ptr():
            dst.copy_(result, non_blocking=True)
        return dst


def _ubatch_id() -> int:
    """vLLM's dual-batch-overlap micro-batch id (0 when it is off or vLLM is
    not loaded)."""
    try:
        from vllm.v1.worker.ubatching import dbo_current_ubatch_id
    except Exception:  # noqa: BLE001 - vLLM absent: one micro-batch
        return 0
    try:
        return int(dbo_current_ubatch_id())
    except Exception:  # noqa: BLE001
        return 0


# ---------------------------------------------------------------------------
# checkpoint access
# ---------------------------------------------------------------------------
class CheckpointReader:
    """Random access to safetensors shards by tensor name (CheckpointReader,
    vllm_integration.py:290-312)."""

    def __init__(self, model_dir: str | Path) -> None:
        from safetensors import safe_open

        self._open = safe_open
        model_dir = Path(model_dir)
        index = model_dir / "model.safetensors.index.json"
        if index.exists():
            weight_map = json.loads(index.read_text())["weight_map"]
            self._shard_of = {k: model_dir / v for k, v in weight_map.items()}
        else:
            self._shard_of = {}
            for shard in sorted(glob.glob(str(model_dir / "*.safetensors"))):
                with safe_open(shard, framework="pt") as f:
                    for key in f.keys():
                        self._shard_of[key] = Path(shard)
        assert self._shard_of, f"no safetensors under {model_dir}"

    def get(self, name: str) -> torch.Tensor:
        with self._open(str(self._shard_of[name]), framework="pt") as f:
            return f.get_tensor(name)


# ---------------------------------------------------------------------------
# experts and dense MLP on a device
# ---------------------------------------------------------------------------
def topk_softmax(router_logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """router_logits [T, E] -> (bf16 weights [T, k], int32 expert ids [T, k])."""
    lg = router_logits if router_logits.dtype == torch.bfloat16 else router_logits.to(torch.bfloat16)
    lg = lg.contiguous()
    T, E = lg.shape
    w = torch.empty((T, k), dtype=torch.bfloat16, device=lg.device)
    idx = torch.empty((T, k), dtype=torch.int32, device=lg.device)
    call("fg_moe_topk_softmax", lg.data_ptr(), T, E, k, w.data_ptr(), idx.data_ptr(), kernels._stream(lg.device))
    return w, idx


class ExpertsOnDevice:
    """One layer's gpt-oss experts on `device` in the MXFP4 tile records
    (counterpart of MarlinExpertsOnDevice, vllm_integration.py:315-495).

    Inputs are the checkpoint's tensors: gate_up_blocks [E, 2I, H/32, 16]
    (or [E, 2I, H/2]) uint8 e2m1 pairs (low nibble first), gate_up_scales
    [E, 2I, H/32] uint8 e8m0, gate_up_bias [E, 2I] with gate/up rows
    alternating one by one; down_* likewise [E, H, I/32, 16], [E, H, I/32],
    [E, H]. The values are used as they are (no requantisation)."""

    def __init__(self, gate_up_blocks: torch.Tensor, gate_up_scales: torch.Tensor, gate_up_bias: torch.Tensor,
                 down_blocks: torch.Tensor, down_scales: torch.Tensor, down_bias: torch.Tensor,
                 device: str | torch.device, *, top_k: int = 4,
                 expert_range: tuple[int, int] | None = None) -> None:
        dev = torch.device(device)
        E = int(gate_up_blocks.shape[0])
        N1 = int(gate_up_blocks.shape[1])
        gu_v = gate_up_blocks.reshape(E, N1, -1)
        H = int(gu_v.shape[2]) * 2
        I = N1 // 2
        d_v = down_blocks.reshape(E, H, -1)
        assert d_v.shape[2] * 2 == I, f"down blocks {tuple(down_blocks.shape)} do not match I={I}"
        lo, hi = expert_range if expert_range is not None else (0, E)
        assert 0 <= lo < hi <= E, f"bad expert range [{lo}, {hi}) of {E}"
        self.device, self.top_k = dev, int(top_k)
        self.num_experts, self.hidden_size, self.intermediate_size = E, H, I
        self.expert_range = (lo, hi)
        sl = slice(lo, hi)
        with torch.cuda.device(dev):
            gu_s = gate_up_scales.reshape(E, N1, H // 32)[sl].to(dev)
            v1 = moe.interleave64(gu_v[sl].to(dev)).contiguous()
            s1 = moe.interleave64(gu_s).contiguous()
            b1 = moe.interleave64(gate_up_bias[sl].to(dev).float().unsqueeze(-1)).squeeze(-1)
            v2 = d_v[sl].to(dev).contiguous()
            s2 = down_scales.reshape(E, H, I // 32)[sl].to(dev).contiguous()
            self.W = {
                "moe_w1": moe.pack_mxfp4(v1, s1),
                "moe_b1": b1.to(torch.bfloat16).contiguous(),
                "moe_w2": moe.pack_mxfp4(v2, s2),
                "moe_b2": down_bias[sl].to(device=dev, dtype=torch.bfloat16).contiguous(),
                "moe_shape": (hi - lo, H, I),
                "moe_expert_range": (lo, hi),
            }
        self._spec = SimpleNamespace(num_experts=E)

    @classmethod
    def from_checkpoint(cls, reader: CheckpointReader, layer_idx: int, device: str | torch.device, *,
                        top_k: int = 4, expert_range: tuple[int, int] | None = None) -> "ExpertsOnDevice":
        p = f"model.layers.{layer_idx}.mlp.experts"
        return cls(reader.get(f"{p}.gate_up_proj_blocks"), reader.get(f"{p}.gate_up_proj_scales"),
                   reader.get(f"{p}.gate_up_proj_bias"), reader.get(f"{p}.down_proj_blocks"),
                   reader.get(f"{p}.down_proj_scales"), reader.get(f"{p}.down_proj_bias"), device,
                   top_k=top_k, expert_range=expert_range)

    @property
    def partial(self) -> bool:
        return self.expert_range != (0, self.num_experts)

    def forward_on_device(self, x: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        """Route + run the experts on self.device: x [T, H] bf16, router_logits
        [T, E] -> bf16 [T, H], or the fp32 partial [T, H] over expert_range."""
        assert x.device == self.device and router_logits.device == self.device, "inputs must be on the expert device"
        assert x.shape[-1] == self.hidden_size, f"hidden {x.shape[-1]} != {self.hidden_size}"
        assert router_logits.shape[-1] == self.num_experts, "router logits must cover every expert"
        x = x.reshape(-1, self.hidden_size)
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        with torch.cuda.device(self.device):
            weights, idx = topk_softmax(router_logits.reshape(-1, self.num_experts), self.top_k)
            return moe.experts_forward(x.contiguous(), idx, weights, self.W, self._spec)


class DenseMLPOnDevice:
    """A dense gated MLP, down(SiLU(gate x) * up x), on `device`
    (RemoteDenseMLP's compute, vllm_integration.py:1249-1372). w_gate_up is
    vLLM's merged [gate; up] weight [2I, H]; w_down [H, I]; no biases."""

    def __init__(self, w_gate_up: torch.Tensor, w_down: torch.Tensor, device: str | torch.device) -> None:
        dev = torch.device(device)
        N2, H = w_gate_up.shape
        I = N2 // 2
        assert tuple(w_down.shape) == (H, I), f"down {tuple(w_down.shape)} != ({H}, {I})"
        self.device, self.hidden_size, self.intermediate_size = dev, int(H), int(I)
        with torch.cuda.device(dev):
            gu = w_gate_up.to(device=dev, dtype=torch.bfloat16)
            self.gate_up = kernels.PackedWeight(interleave_gate_up(gu[:I], gu[I:]).contiguous())
            self.down = kernels.PackedWeight(w_down.to(device=dev, dtype=torch.bfloat16).contiguous())

    def forward_on_device(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        assert x.device == self.device, "input must be on the MLP's device"
        x = x.reshape(-1, self.hidden_size)
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        with torch.cuda.device(self.device):
            act = kernels.gemm(x.contiguous(), self.gate_up, epilogue=_lib.FG_EPI_SWIGLU, slot="vllm.mlp")
            return kernels.gemm(act, self.down, out=out, slot="vllm.mlp")


# ---------------------------------------------------------------------------
# the two op boundaries
# ---------------------------------------------------------------------------
def _sum_partials(parts: list[torch.Tensor], home: torch.device, out: torch.Tensor | None) -> torch.Tensor:
    stacked = torch.stack([hop_tensor(p, home) for p in parts])
    return kernels.sum_partials(stacked, out=out)


def make_forward_impl(remote: ExpertsOnDevice, home: str | torch.device, stable_out: StableOutput | None, *,
                      local: ExpertsOnDevice | None = None, decode_local: ExpertsOnDevice | None = None,
                      decode_threshold: int = 0):
    """Replacement for the FusedMoE runner's forward_impl (vllm_integration.py:
    1419-1615). `remote` holds the experts on the expert device. With
    `local` (experts [0, n) on the home GPU, remote holding [n, E)), both
    halves run at once and their fp32 partials add up (the decode split).
    With `decode_local` (all experts on the home GPU), batches of up to
    decode_threshold tokens stay home (phase-aware placement)."""
    home = torch.device(home)
    if local is not None:
        assert local.partial and remote.partial and local.expert_range[1] == remote.expert_range[0], (
            "a split needs local experts [0, n) and remote experts [n, E)")
        assert local.expert_range[0] == 0 and remote.expert_range[1] == remote.num_experts, (
            "the two halves of a split must cover every expert")
    else:
        assert not remote.partial, "experts of a sub-range need the home half (local=) to make the full output"

    def forward_impl(layer: Any, hidden_states: torch.Tensor, router_logits: torch.Tensor,
                     shared_experts_input: torch.Tensor | None = None,
                     input_ids: torch.Tensor | None = None) -> torch.Tensor:
        assert shared_experts_input is None, "shared-experts MoE is not supported"
        T = hidden_states.shape[0]
        ub = _ubatch_id()
        dst = stable_out.view(T, ub) if stable_out is not None else None
        if decode_local is not None and T <= decode_threshold:
            out = decode_local.forward_on_device(hidden_states, router_logits)
            return stable_out.stage(out, ub) if stable_out is not None else out
        x = hop_tensor(hidden_states, remote.device)
        lg = hop_tensor(router_logits, remote.device)
        if local is not None:
            part_remote = remote.forward_on_device(x, lg)
            part_local = local.forward_on_device(hidden_states, router_logits)
            with torch.cuda.device(home):
                return _sum_partials([part_local, part_remote], home, dst)
        out = remote.forward_on_device(x, lg)
        if stable_out is None:
            return hop_tensor(out, home)
        return stable_out.stage(out, ub)

    return forward_impl


class RemoteDenseMLP:
    """A dense MLP relocated to the expert device, with boundary hops
    (RemoteDenseMLP, vllm_integration.py:1249-1372). With keep_local, a
    home-GPU copy computes batches of up to decode_threshold tokens in place
    (phase-aware placement)."""

    def __init__(self, w_gate_up: torch.Tensor, w_down: torch.Tensor, device: str | torch.device,
                 home: str | torch.device, stable_out: StableOutput | None, *, keep_local: bool = False,
                 decode_threshold: int = 0) -> None:
        self.home = torch.device(home)
        self.remote = DenseMLPOnDevice(w_gate_up, w_down, device)
        self.local = DenseMLPOnDevice(w_gate_up, w_down, self.home) if keep_local else None
        self.decode_threshold = int(decode_threshold)
        self.stable_out = stable_out

    def __call__(self, hidden_states: torch.Tensor) -> torch.Tensor:
        T = hidden_states.shape[0]
        ub = _ubatch_id()
        dst = self.stable_out.view(T, ub) if self.stable_out is not None else None
        if self.local is not None and T <= self.decode_threshold:
            return self.local.forward_on_device(hidden_states, out=dst)
        if self.remote.device == self.home:
            return self.remote.forward_on_device(hidden_states, out=dst)
        out = self.remote.forward_on_device(hop_tensor(hidden_states, self.remote.device))
        return self.stable_out.stage(out, ub) if self.stable_out is not None else hop_tensor(out, self.home)


_REMOTE_MLPS: dict[str, RemoteDenseMLP] = {}


def register_remote_mlp(layer_key: str, mlp: RemoteDenseMLP) -> None:
    _REMOTE_MLPS[layer_key] = mlp


def _remote_mlp(hidden_states: torch.Tensor, layer_key: str) -> torch.Tensor:
    return _REMOTE_MLPS[layer_key](hidden_states)


def _remote_mlp_fake(hidden_states: torch.Tensor, layer_key: str) -> torch.Tensor:
    return torch.empty_like(hidden_states)


_OP_LIB: torch.library.Library | None = None


def register_remote_mlp_op() -> None:
    """Define `vllm::fluidgpu_remote_mlp(Tensor hidden_states, str layer_key)
    -> Tensor` (CUDA impl + fake impl, fixed stride order), once per
    process; a definition made by the reference's module is kept."""
    global _OP_LIB
    if _OP_LIB is not None or hasattr(torch.ops.vllm, "fluidgpu_remote_mlp"):
        return
    lib = torch.library.Library("vllm", "FRAGMENT")
    lib.define("fluidgpu_remote_mlp(Tensor hidden_states, str layer_key) -> Tensor",
               tags=(torch.Tag.needs_fixed_stride_order,))
    lib.impl("fluidgpu_remote_mlp", _remote_mlp, "CUDA")
    torch.library.register_fake("vllm::fluidgpu_remote_mlp", _remote_mlp_fake, lib=lib)
    _OP_LIB = lib


register_remote_mlp_op()


class FluidRemoteMLP(torch.nn.Module):
    """Stands in for a relocated dense MLP: its class-level forward emits one
    opaque custom-op node carrying the registry key (FluidRemoteMLP,
    vllm_integration.py:1403-1416)."""

    def __init__(self, layer_key: str) -> None:
        super().__init__()
        self.layer_key = layer_key

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        return torch.ops.vllm.fluidgpu_remote_mlp(hidden_states, self.layer_key)


# ---------------------------------------------------------------------------
# installation into a loaded vLLM model
# ---------------------------------------------------------------------------
def _model_layers(model: torch.nn.Module) -> list[torch.nn.Module]:
    inner = getattr(model, "model", None)
    layers = getattr(inner, "layers", None)
    assert layers is not None, f"no model.layers on {type(model).__name__}"
    return list(layers)


def install_moe_forward(moe_layer: Any, forward_impl: Any) -> None:
    """Point a FusedMoE layer's runner at forward_impl: the attribute the
    opaque `vllm::moe_forward` op calls (`_forward_impl` in vLLM 0.22,
    `forward_impl` in 0.18)."""
    runner = getattr(moe_layer, "runner", None)
    assert runner is not None, f"{type(moe_layer).__name__} has no MoE runner"
    name = "_forward_impl" if hasattr(runner, "_forward_impl") else "forward_impl"
    setattr(runner, name, forward_impl)


def install(model: torch.nn.Module, *, expert_device: str, home: str, max_tokens: int,
            reader: CheckpointReader | None = None, dtype: torch.dtype = torch.bfloat16,
            top_k: int = 4, decode_split: float = 0.0, phase_aware: bool = False,
            decode_threshold: int = 0) -> dict[str, int]:
    """Move every layer's feed-forward group of a loaded vLLM model to
    expert_device behind the op boundaries (the placement part of
    apply_fluid_placement, vllm_integration.py:1668-1866): FusedMoE layers
    (`layer.mlp.experts` with a runner) get a forward_impl over experts read
    from the checkpoint; dense MLPs (gate_up_proj / down_proj) are replaced
    by FluidRemoteMLP proxies. decode_split = fraction of experts kept on the
    home GPU (0: all remote); phase_aware keeps decode-size batches home."""
    layers = _model_layers(model)
    counts = {"moe": 0, "dense": 0}
    stable: StableOutput | None = None
    for i, layer in enumerate(layers):
        mlp = layer.mlp
        experts = getattr(mlp, "experts", None)
        if experts is not None and hasattr(experts, "runner"):
            assert reader is not None, "MoE placement reads the experts from the checkpoint"
            if stable is None:
                stable = StableOutput(max_tokens, int(experts.hidden_size), dtype, home)
            E = int(getattr(experts, "global_num_experts", 0) or experts.num_experts)
            if decode_split > 0:
                n = max(1, min(E - 1, int(round(decode_split * E))))
                local = ExpertsOnDevice.from_checkpoint(reader, i, home, top_k=top_k, expert_range=(0, n))
                remote = ExpertsOnDevice.from_checkpoint(reader, i, expert_device, top_k=top_k,
                                                         expert_range=(n, E))
                impl = make_forward_impl(remote, home, stable, local=local)
            else:
                remote = ExpertsOnDevice.from_checkpoint(reader, i, expert_device, top_k=top_k)
                dl = ExpertsOnDevice.from_checkpoint(reader, i, home, top_k=top_k) if phase_aware else None
                impl = make_forward_impl(remote, home, stable, decode_local=dl, decode_threshold=decode_threshold)
            install_moe_forward(experts, impl)
            counts["moe"] += 1
        elif hasattr(mlp, "gate_up_proj") and hasattr(mlp, "down_proj"):
            gu, dn = mlp.gate_up_proj, mlp.down_proj
            assert getattr(gu, "bias", None) is None and getattr(dn, "bias", None) is None, (
                "biased dense MLP is not supported")
            if stable is None:
                stable = StableOutput(max_tokens, int(dn.weight.shape[0]), dtype, home)
            key = f"layers.{i}.mlp"
            register_remote_mlp(key, RemoteDenseMLP(gu.weight.data, dn.weight.data, expert_device, home, stable,
                                                    keep_local=phase_aware, decode_threshold=decode_threshold))
            layer.mlp = FluidRemoteMLP(key)
            counts["dense"] += 1
    return counts


def apply_fluid_placement(worker: Any) -> dict[str, int] | None:
    """The worker hook (vllm_integration.py:1668-1866): after vLLM loads the
    weights, before the first traced forward. Environment, as the
    reference's: FLUIDGPU_VLLM_PLACEMENT none | af | af-bf16 (both place the
    feed-forward groups on the expert device; experts stay MXFP4 either
    way), FLUIDGPU_EXPERT_DEVICE (default cuda:1), FLUIDGPU_DECODE_SPLIT,
    FLUIDGPU_PHASE_AWARE, FLUIDGPU_DECODE_LOCAL_THRESHOLD."""
    placement = _env("FLUIDGPU_VLLM_PLACEMENT", "none")
    if placement == "none":
        return None
    assert placement in ("af", "af-bf16"), f"unknown placement {placement!r}"
    cfg = worker.vllm_config
    par = cfg.parallel_config
    assert par.tensor_parallel_size == 1 and par.pipeline_parallel_size == 1, (
        "FLUIDGPU placement supports TP=1/PP=1 (the second GPU is the expert side)")
    comp = cfg.compilation_config
    graphs = not cfg.model_config.enforce_eager and getattr(comp.cudagraph_mode, "name", "NONE") != "NONE"
    if graphs:
        assert not comp.cudagraph_mode.has_full_cudagraphs(), (
            "FLUIDGPU placement requires cudagraph_mode=PIECEWISE; pass compilation_config=fluid_compilation_config()")
        assert MOE_FORWARD_OP in comp.splitting_ops or REMOTE_MLP_OP in comp.splitting_ops, (
            "FLUIDGPU ops missing from splitting_ops; pass compilation_config=fluid_compilation_config()")
    max_seqs = int(getattr(cfg.scheduler_config, "max_num_seqs", 32) or 32)
    model_dir = Path(cfg.model_config.model)
    reader = CheckpointReader(model_dir) if model_dir.exists() else None
    hf = cfg.model_config.hf_config
    return install(worker.model_runner.model, expert_device=_env("FLUIDGPU_EXPERT_DEVICE", "cuda:1"),
                   home=str(worker.device), max_tokens=int(getattr(comp, "max_cudagraph_capture_size", 0) or 0),
                   reader=reader, dtype=cfg.model_config.dtype,
                   top_k=int(getattr(hf, "num_experts_per_tok", 4) or 4),
                   decode_split=float(_env("FLUIDGPU_DECODE_SPLIT", "0")),
                   phase_aware=_env("FLUIDGPU_PHASE_AWARE", "0") == "1",
                   decode_threshold=int(_env("FLUIDGPU_DECODE_LOCAL_THRESHOLD", str(max(64, 2 * max_seqs)))))


def fluid_compilation_config() -> dict[str, Any]:
    """compilation_config for piecewise CUDA graphs around the ops: vLLM
    splits its FX graph at them (with its own attention / KV-cache ops, the
    list replaces vLLM's), so they run eagerly between graph replays
    (fluid_compilation_config, vllm_integration.py:2042-2073)."""
    from vllm.config.compilation import CompilationConfig

    return {
        "cudagraph_mode": "PIECEWISE",
        "splitting_ops": [*CompilationConfig._attention_ops, "vllm::unified_kv_cache_update",
                          "vllm::unified_mla_kv_cache_update", MOE_FORWARD_OP, REMOTE_MLP_OP],
    }
