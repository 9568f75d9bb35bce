"""The router kernel's fp64 shortcut, modelled on the CPU: an fp64 sum of the
exact bf16 x bf16 products in the kernel's order (each lane's elements in
sequence, then a butterfly over 32 lanes, lane 0's result), an error bound
E = 2 (n 2^-52) sum|p|, and acceptance only when s - E and s + E round to
the same finite nonzero bf16. Whenever the model accepts, its answer must be
the exactly rounded logit (the oracle's, itself checked against rational
arithmetic); where it declines, the kernel takes the exact accumulation.
Inputs: random rows, rows built to land on or next to bf16 rounding
midpoints, heavy cancellation, and wide exponent spreads."""
import numpy as np
import torch

from oracle import decode_ref as ref


def _bf16_round_f64(v: float) -> int:
    """bf16 bits nearest to the float64 v (ties to even)."""
    r = float(ref.round_bf16_f64(np.array([v]))[0][0])
    return int(torch.tensor([r], dtype=torch.float32).to(torch.bfloat16).view(torch.int16).item()) & 0xFFFF


def _model(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None):
    """(accepted, bf16 bits) of the kernel's shortcut for one x row, one w row."""
    H = x.numel()
    p = x.double().numpy() * w.double().numpy()  # exact
    lanes_s = np.zeros(32)
    lanes_a = np.zeros(32)
    for i in range(0, H // 8):  # uint4 i (8 elements) belongs to lane i % 32
        lane = i % 32
        for j in range(8 * i, 8 * i + 8):
            lanes_s[lane] = lanes_s[lane] + p[j]
            lanes_a[lane] = lanes_a[lane] + abs(p[j])
    idx = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        lanes_s = lanes_s + lanes_s[idx ^ o]
        lanes_a = lanes_a + lanes_a[idx ^ o]
    s, a = float(lanes_s[0]), float(lanes_a[0])
    if b is not None:
        bv = float(b.double())
        s, a = s + bv, a + abs(bv)
    if not (np.isfinite(s) and np.isfinite(a)):
        return False, None
    n = 8.0 * (H // 8) + 1.0
    e2 = 2.0 * (a * (n * 2.0 ** -52))
    lo, hi = _bf16_round_f64(s - e2), _bf16_round_f64(s + e2)
    if lo != hi or (lo & 0x7FFF) == 0 or (lo & 0x7F80) == 0x7F80:
        return False, None
    return True, lo


def _bits(t: torch.Tensor) -> list[int]:
    return [int(v) & 0xFFFF for v in t.view(torch.int16).reshape(-1).tolist()]


def _check(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> tuple[int, int]:
    exact = _bits(ref.exact_linear_bf16(x, w, b))
    accepted = 0
    for t in range(x.shape[0]):
        for e in range(w.shape[0]):
            ok, bits = _model(x[t], w[e], None if b is None else b[e])
            if ok:
                accepted += 1
                assert bits == exact[t * w.shape[0] + e], (t, e, hex(bits), hex(exact[t * w.shape[0] + e]))
    return accepted, x.shape[0] * w.shape[0]


def test_filter_agrees_with_exact_rounding_on_random_rows():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(6, 2880, generator=g).to(torch.bfloat16)
    w = (torch.randn(8, 2880, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(8, generator=g) * 0.1).to(torch.bfloat16)
    acc, total = _check(x, w, b)
    assert acc == total  # random rows never come within the bound of a midpoint


def test_filter_declines_near_midpoints_and_cancellation():
    g = torch.Generator().manual_seed(1)
    H = 256
    rows_x, rows_w = [], []
    for t in range(12):
        x = torch.randn(H, generator=g).to(torch.bfloat16)
        w = (torch.randn(H, generator=g) * 0.05).to(torch.bfloat16)
        # move the sum onto a bf16 midpoint (or one product away from it):
        # the last element takes the rest
        w[-1] = 0
        s = (x.double() * w.double()).sum().item()
        r = float(torch.tensor([s]).to(torch.bfloat16).double())
        q = 2.0 ** (np.frexp(r)[1] - 8)
        target = r + q / 2 + (0 if t % 3 == 0 else (q * 2.0 ** -40 if t % 3 == 1 else -q * 2.0 ** -40))
        x[-1] = 1.0
        w[-1] = torch.tensor([target - s], dtype=torch.float64).to(torch.bfloat16)
        rows_x.append(x)
        rows_w.append(w)
    # heavy cancellation: a row and its negation, plus a tiny remainder
    x = torch.randn(H, generator=g).to(torch.bfloat16)
    rows_x.append(x)
    w = torch.cat([torch.ones(H // 2), -torch.ones(H // 2)]).to(torch.bfloat16)
    x2 = torch.cat([x[: H // 2], x[: H // 2]])
    x2[0] = x2[0] + 2.0 ** -20
    rows_x[-1] = x2.to(torch.bfloat16)
    rows_w.append(w)
    # a spread of exponents far wider than the fixed-point window
    wide = torch.tensor([2.0 ** 100, 1.0, 2.0 ** -100, -(2.0 ** 100)] * (H // 4)).to(torch.bfloat16)
    rows_x.append(wide)
    rows_w.append(torch.ones(H).to(torch.bfloat16))
    X = torch.stack(rows_x)
    W = torch.stack(rows_w)
    acc, total = _check(X, W, None)
    assert acc < total  # the midpoint rows are left to the exact accumulation
