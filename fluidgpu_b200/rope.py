"""Rotary-embedding frequency tables for the decode kernels.

fg_rope_kv_append takes inv_freq[hd/2] and one attention scaling factor and
evaluates cos/sin on the device. These functions produce those two values
for the RoPE variants the supported families use:
  default : inv_freq[i] = theta^(-2i/d)                      (Llama-3, Qwen)
  llama3  : Llama-3.1 frequency-dependent wavelength rescale (low/high
            frequency factors, smooth blend in between)
  yarn    : YaRN (Peng et al., 2023) interpolation/extrapolation ramp with
            attention scaling 0.1*ln(factor)+1                 (gpt-oss)
They follow the published definitions that transformers' rope init
functions implement, which the reference's HF modules call.
"""
from __future__ import annotations

import math

import torch


def default(head_dim: int, theta: float) -> tuple[torch.Tensor, float]:
    i = torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float32)
    return 1.0 / (theta ** (i / head_dim)), 1.0


def llama3(head_dim: int, theta: float, factor: float, low_freq_factor: float,
           high_freq_factor: float, original_max: int) -> tuple[torch.Tensor, float]:
    inv, _ = default(head_dim, theta)
    low_wavelen = original_max / low_freq_factor
    high_wavelen = original_max / high_freq_factor
    wavelen = 2 * math.pi / inv
    scaled = torch.where(wavelen > low_wavelen, inv / factor, inv)
    smooth = (original_max / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor)
    blended = (1 - smooth) * scaled / factor + smooth * scaled
    medium = (wavelen >= high_wavelen) & (wavelen <= low_wavelen)
    return torch.where(medium, blended, scaled), 1.0


def yarn(head_dim: int, theta: float, factor: float, original_max: int, beta_fast: float = 32.0,
         beta_slow: float = 1.0, truncate: bool = True,
         attention_factor: float | None = None) -> tuple[torch.Tensor, float]:
    half = head_dim // 2
    base_freq = theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim)
    extrapolated = 1.0 / base_freq
    interpolated = 1.0 / (factor * base_freq)

    def dim_for_rotations(rotations: float) -> float:
        # dimension index whose wavelength fits `rotations` turns in original_max
        return head_dim * math.log(original_max / (rotations * 2 * math.pi)) / (2 * math.log(theta))

    lo, hi = dim_for_rotations(beta_fast), dim_for_rotations(beta_slow)
    if truncate:
        lo, hi = math.floor(lo), math.ceil(hi)
    lo, hi = max(lo, 0), min(hi, head_dim - 1)
    if lo == hi:
        hi += 0.001
    ramp = ((torch.arange(half, dtype=torch.float32) - lo) / (hi - lo)).clamp(0, 1)
    keep_extrapolated = 1 - ramp
    inv = interpolated * (1 - keep_extrapolated) + extrapolated * keep_extrapolated
    scale = attention_factor if attention_factor is not None else 0.1 * math.log(factor) + 1.0
    return inv, float(scale)
