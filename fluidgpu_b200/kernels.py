"""Torch-facing wrappers over the C ABI (include/fgb200.h).

Each wrapper checks its tensors (CUDA, dtype, contiguity), allocates outputs
through the torch caching allocator, hands raw pointers and the current
CUDA stream to libfgb200.so and raises on a nonzero status. The C entry
points never allocate; scratch space comes from `Workspace`, one buffer per
(device, stream) so calls that may overlap on the GPU never share one.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import call

_BF16 = torch.bfloat16


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check(t: torch.Tensor, name: str, dtype: torch.dtype | None = None) -> None:
    assert t.is_cuda, f"{name} must be a CUDA tensor, got {t.device}"
    assert t.is_contiguous(), f"{name} must be contiguous"
    if dtype is not None:
        assert t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}"


class KernelTimer:
    """CUDA-event brackets around selected entry points, on the launching
    stream. Off unless a name is enabled; bench.py turns on the dominant
    kernel inside its timed region to measure that kernel's live duration."""

    enabled: set[str] = set()
    events: dict[str, list[tuple[torch.cuda.Event, torch.cuda.Event, dict]]] = {}

    @classmethod
    def enable(cls, *names: str) -> None:
        cls.enabled = set(names)
        cls.events = {n: [] for n in names}

    @classmethod
    def disable(cls) -> None:
        cls.enabled = set()

    @classmethod
    def start(cls, name: str):
        if name not in cls.enabled:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    @classmethod
    def stop(cls, name: str, ev0, **meta) -> None:
        if ev0 is None:
            return
        ev1 = torch.cuda.Event(enable_timing=True)
        ev1.record()
        cls.events[name].append((ev0, ev1, meta))

    @classmethod
    def durations_ms(cls, name: str) -> list[tuple[float, dict]]:
        return [(a.elapsed_time(b), m) for a, b, m in cls.events.get(name, [])]


class Workspace:
    """Zero-initialised scratch buffers keyed by (device, slot).

    Kernels that share a slot run in stream order; callers that may overlap
    on the GPU (several runners, several streams) use distinct slot names.
    The GEMM stream-K tickets must start at zero and the kernels leave them at
    zero again, so a buffer is zeroed once, when it is (re)allocated.
    Buffers persist (and may be captured into CUDA graphs).
    """

    _bufs: dict[tuple[int, str], torch.Tensor] = {}

    @classmethod
    def get(cls, nbytes: int, device: torch.device, slot: str) -> torch.Tensor | None:
        if nbytes <= 0:
            return None
        key = (device.index if device.index is not None else torch.cuda.current_device(), slot)
        buf = cls._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            buf = torch.zeros(size + 256, dtype=torch.uint8, device=device)
            off = (-buf.data_ptr()) % 256
            buf = buf[off : off + size]
            cls._bufs[key] = buf
        return buf

    @classmethod
    def clear(cls) -> None:
        cls._bufs.clear()


def launch_count() -> int:
    """Kernels libfgb200.so has launched in this process."""
    return int(_lib.lib().fg_launch_count())


def device_status(reset: bool = True) -> int:
    """Device status word (0 = no device-side failure). Synchronises."""
    v = _lib.ctypes.c_uint(0)
    call("fg_device_status", _lib.ctypes.byref(v), int(reset), _stream())
    return int(v.value)


def check_device(what: str = "fgb200") -> None:
    st = device_status(reset=True)
    if st:
        kind = st & 0xFF
        site = st >> 8
        names = {1: "pipeline wait timeout", 2: "peer flag timeout", 3: "index out of range",
                 4: "MXFP4 block scale outside the row's exact range"}
        raise RuntimeError(f"{what}: device-side failure '{names.get(kind, kind)}' at site {site:#x}")


# ---------------------------------------------------------------------------
# ops
# ---------------------------------------------------------------------------
def embed(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _check(ids, "ids", torch.int64)
    _check(table, "table", _BF16)
    T = ids.numel()
    V, H = table.shape
    if out is None:
        out = torch.empty((T, H), dtype=_BF16, device=table.device)
    call("fg_embed", _ptr(ids), _ptr(table), _ptr(out), T, H, V, _stream(table.device))
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, mode: int = _lib.FG_NORM_LLAMA,
            out: torch.Tensor | None = None) -> torch.Tensor:
    _check(x, "x", _BF16)
    _check(weight, "weight", _BF16)
    H = x.shape[-1]
    T = x.numel() // H
    if out is None:
        out = torch.empty_like(x)
    call("fg_rmsnorm", _ptr(x), _ptr(weight), _ptr(out), T, H, float(eps), mode, _stream(x.device))
    return out


class PackedWeight:
    """A [N, K] bf16 weight in the tile layout of fg_pack_weight_bf16
    (contiguous 16 KB swizzled 128x64 tiles), ready for fg_gemm_bf16_packed."""

    def __init__(self, w: torch.Tensor) -> None:
        _check(w, "w", _BF16)
        assert w.ndim == 2, "weight must be [N, K]"
        self.N, self.K = int(w.shape[0]), int(w.shape[1])
        self.device = w.device
        nbytes = _lib.lib().fg_packed_weight_bytes(self.N, self.K)
        self.data = torch.empty(nbytes, dtype=torch.uint8, device=w.device)
        call("fg_pack_weight_bf16", _ptr(w), _ptr(self.data), self.N, self.K, _stream(w.device))

    @property
    def shape(self) -> tuple[int, int]:
        return (self.N, self.K)

    def nbytes(self) -> int:
        return self.data.numel()


def gemm(x: torch.Tensor, w: "torch.Tensor | PackedWeight", *, epilogue: int = _lib.FG_EPI_STORE,
         residual: torch.Tensor | None = None, bias: torch.Tensor | None = None,
         out: torch.Tensor | None = None, splits: int = 0, slot: str = "gemm") -> torch.Tensor:
    """acc = x @ w.T on tcgen05 with the given epilogue (see fg_gemm_bf16)."""
    _check(x, "x", _BF16)
    packed = isinstance(w, PackedWeight)
    if not packed:
        _check(w, "w", _BF16)
    K = x.shape[-1]
    T = x.numel() // K
    N, Kw = w.shape
    assert Kw == K, f"gemm: x has K={K}, w has K={Kw}"
    n_out = N // 2 if epilogue == _lib.FG_EPI_SWIGLU else N
    out_dtype = torch.float32 if epilogue == _lib.FG_EPI_F32 else _BF16
    if out is None:
        out = torch.empty((*x.shape[:-1], n_out), dtype=out_dtype, device=x.device)
    assert out.dtype == out_dtype, f"gemm: epilogue {epilogue} writes {out_dtype}, out is {out.dtype}"
    if residual is not None:
        _check(residual, "residual", _BF16)
        assert residual.numel() == T * n_out, "residual shape mismatch"
    if bias is not None:
        _check(bias, "bias", _BF16)
    lib = _lib.lib()
    ws_bytes = lib.fg_gemm_workspace_bytes(T, N, K, splits)
    ws = Workspace.get(ws_bytes, x.device, slot)
    ev = KernelTimer.start("gemm")
    call("fg_gemm_bf16_packed" if packed else "fg_gemm_bf16", _ptr(x),
         _ptr(w.data) if packed else _ptr(w), _ptr(out), _ptr(residual), _ptr(bias), T, N, K,
         epilogue, splits, _ptr(ws), ws_bytes, _stream(x.device))
    KernelTimer.stop("gemm", ev, T=T, N=N, K=K)
    return out


def sum_partials(partials: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """[S, ...] fp32 partial sums -> bf16 [...] = sum over S in order (fg_sum_partials)."""
    _check(partials, "partials", torch.float32)
    S = partials.shape[0]
    n = partials[0].numel()
    if out is None:
        out = torch.empty(partials.shape[1:], dtype=_BF16, device=partials.device)
    _check(out, "out", _BF16)
    assert out.numel() == n, "sum_partials: out size mismatch"
    call("fg_sum_partials", _ptr(partials), S, n, _ptr(out), _stream(partials.device))
    return out


def rope_kv_append(qkv: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor,
                   attention_scaling: float, block_table: torch.Tensor, k_cache: torch.Tensor,
                   v_cache: torch.Tensor, nq: int, nkv: int, hd: int,
                   q_out: torch.Tensor | None = None) -> torch.Tensor:
    _check(qkv, "qkv", _BF16)
    _check(positions, "positions", torch.int32)
    _check(inv_freq, "inv_freq", torch.float32)
    _check(block_table, "block_table", torch.int32)
    _check(k_cache, "k_cache", _BF16)
    _check(v_cache, "v_cache", _BF16)
    B = positions.numel()
    assert qkv.numel() == B * (nq + 2 * nkv) * hd, "qkv shape mismatch"
    num_blocks, _, block_size, _ = k_cache.shape
    if q_out is None:
        q_out = torch.empty((B, nq, hd), dtype=_BF16, device=qkv.device)
    call("fg_rope_kv_append", _ptr(qkv), _ptr(positions), _ptr(inv_freq), float(attention_scaling),
         _ptr(block_table), block_table.shape[1], num_blocks, _ptr(q_out), _ptr(k_cache),
         _ptr(v_cache), B, nq, nkv, hd, block_size, _stream(qkv.device))
    return q_out


def rope_kv_append_tokens(qkv: torch.Tensor, seq_ids: torch.Tensor, positions: torch.Tensor,
                          inv_freq: torch.Tensor, attention_scaling: float, block_table: torch.Tensor,
                          k_cache: torch.Tensor, v_cache: torch.Tensor, nq: int, nkv: int, hd: int,
                          q_out: torch.Tensor | None = None) -> torch.Tensor:
    """rope_kv_append for T tokens: token t of sequence seq_ids[t] at positions[t]."""
    _check(qkv, "qkv", _BF16)
    _check(seq_ids, "seq_ids", torch.int32)
    _check(positions, "positions", torch.int32)
    _check(inv_freq, "inv_freq", torch.float32)
    _check(block_table, "block_table", torch.int32)
    T = positions.numel()
    assert seq_ids.numel() == T and qkv.numel() == T * (nq + 2 * nkv) * hd, "qkv / token shape mismatch"
    num_blocks, _, block_size, _ = k_cache.shape
    if q_out is None:
        q_out = torch.empty((T, nq, hd), dtype=_BF16, device=qkv.device)
    call("fg_rope_kv_append_tokens", _ptr(qkv), _ptr(seq_ids), _ptr(positions), _ptr(inv_freq),
         float(attention_scaling), _ptr(block_table), block_table.shape[1], num_blocks, _ptr(q_out),
         _ptr(k_cache), _ptr(v_cache), T, nq, nkv, hd, block_size, _stream(qkv.device))
    return q_out


def prefill_attn(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                 first_pos: torch.Tensor, S: int, *, window: int = 0, sinks: torch.Tensor | None = None,
                 scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal attention of S query positions per sequence (q [B*S, nq, hd],
    sequence b's queries at first_pos[b] ..) over the paged cache."""
    _check(q, "q", _BF16)
    _check(first_pos, "first_pos", torch.int32)
    T, nq, hd = q.shape
    B = first_pos.numel()
    assert T == B * S, f"prefill q has {T} rows, expected {B} x {S}"
    num_blocks, nkv, block_size, _ = k_cache.shape
    if out is None:
        out = torch.empty((T, nq, hd), dtype=_BF16, device=q.device)
    if sinks is not None:
        _check(sinks, "sinks", torch.float32)
    call("fg_prefill_attn", _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(block_table), _ptr(first_pos),
         _ptr(sinks), _ptr(out), B, S, nq, nkv, hd, block_size, num_blocks, block_table.shape[1], window,
         float(scale if scale is not None else hd ** -0.5), _stream(q.device))
    return out


def kv_append(k: torch.Tensor, v: torch.Tensor, seq_ids: torch.Tensor, positions: torch.Tensor,
              block_table: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
    """Write rotated k / raw v [T, nkv, hd] into their paged slots."""
    _check(k, "k", _BF16)
    _check(v, "v", _BF16)
    _check(seq_ids, "seq_ids", torch.int32)
    _check(positions, "positions", torch.int32)
    _check(block_table, "block_table", torch.int32)
    T, nkv, hd = k.shape
    num_blocks, nkv2, block_size, hd2 = k_cache.shape
    assert (nkv2, hd2) == (nkv, hd), "cache heads/head_dim mismatch"
    call("fg_kv_append", _ptr(k), _ptr(v), _ptr(seq_ids), _ptr(positions), _ptr(block_table),
         block_table.shape[1], num_blocks, _ptr(k_cache), _ptr(v_cache), T, nkv, hd, block_size,
         _stream(k.device))


def paged_decode_attn(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      block_table: torch.Tensor, seq_lens: torch.Tensor, max_seq_len: int, *,
                      window: int = 0, sinks: torch.Tensor | None = None,
                      scale: float | None = None, out: torch.Tensor | None = None,
                      slot: str = "attn") -> torch.Tensor:
    _check(q, "q", _BF16)
    _check(k_cache, "k_cache", _BF16)
    _check(v_cache, "v_cache", _BF16)
    _check(block_table, "block_table", torch.int32)
    _check(seq_lens, "seq_lens", torch.int32)
    B, nq, hd = q.shape
    num_blocks, nkv, block_size, hd2 = k_cache.shape
    assert hd2 == hd, "head_dim mismatch between q and cache"
    if sinks is not None:
        _check(sinks, "sinks", torch.float32)
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if out is None:
        out = torch.empty((B, nq * hd), dtype=_BF16, device=q.device)
    lib = _lib.lib()
    ws_bytes = lib.fg_attn_workspace_bytes(B, nq, nkv, hd, max_seq_len, window)
    ws = Workspace.get(ws_bytes, q.device, slot)
    ev = KernelTimer.start("attn")
    call("fg_paged_decode_attn", _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(block_table),
         _ptr(seq_lens), _ptr(sinks), _ptr(out), _ptr(ws), ws_bytes, B, nq, nkv, hd, block_size,
         num_blocks, block_table.shape[1], int(max_seq_len), int(window), float(scale),
         _stream(q.device))
    KernelTimer.stop("attn", ev, B=B, nq=nq, nkv=nkv, hd=hd, window=int(window),
                     max_seq_len=int(max_seq_len))
    return out


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _check(logits, "logits", _BF16)
    V = logits.shape[-1]
    T = logits.numel() // V
    if out is None:
        out = torch.empty((T,), dtype=torch.int64, device=logits.device)
    call("fg_argmax", _ptr(logits), _ptr(out), T, V, _stream(logits.device))
    return out


def advance(positions: torch.Tensor | None, seq_lens: torch.Tensor | None) -> None:
    ref = positions if positions is not None else seq_lens
    if ref is None:
        return
    call("fg_advance", _ptr(positions), _ptr(seq_lens), ref.numel(), _stream(ref.device))
