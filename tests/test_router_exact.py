"""The oracle's exactly rounded router logits against rational arithmetic
(CPU). The router's bf16 logit is defined as the bf16 nearest (ties to even)
to the exact value x . w + b; the B200 kernel computes that number, so the
oracle's restatement (float64 products, math.fsum, a rational tie check) is
checked here against an independent computation in fractions, on inputs
chosen to hit the hard cases: exact ties, subnormal results and inputs,
heavy cancellation, and exponent spreads far wider than any fixed-point
window."""
from fractions import Fraction

import torch

from oracle import decode_ref as ref


def _bf16_value(bits: int) -> Fraction:
    sign = -1 if bits & 0x8000 else 1
    e = (bits >> 7) & 0xFF
    m = bits & 0x7F
    if e == 0:
        return sign * Fraction(m, 2 ** 133)
    return sign * Fraction(128 + m, 128) * Fraction(2) ** (e - 127)


def _round_bf16_exact(v: Fraction) -> int:
    """bf16 bits nearest to v, ties to even, by exhaustive search of the
    two neighbours (independent of the oracle's float64 route)."""
    if v == 0:
        return 0
    sign = 0x8000 if v < 0 else 0
    a = abs(v)
    lo, hi = 0, 0x7F80  # magnitudes are monotone in the bit pattern
    while hi - lo > 1:
        mid = (lo + hi) // 2
        if _bf16_value(mid) <= a:
            lo = mid
        else:
            hi = mid
    dl, dh = a - _bf16_value(lo), _bf16_value(hi) - a
    pick = lo if dl < dh or (dl == dh and lo % 2 == 0) else hi
    return sign | pick


def _bits(t: torch.Tensor) -> list[int]:
    return [int(b) & 0xFFFF for b in t.view(torch.int16).reshape(-1).tolist()]


def _exact_logits(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> list[int]:
    xb, wb, bb = _bits(x), _bits(w), _bits(b)
    T, H = x.shape
    E = w.shape[0]
    out = []
    for t in range(T):
        for e in range(E):
            s = sum(_bf16_value(xb[t * H + h]) * _bf16_value(wb[e * H + h]) for h in range(H))
            out.append(_round_bf16_exact(s + _bf16_value(bb[e])))
    return out


def _from_bits(bits: list[int], shape) -> torch.Tensor:
    return torch.tensor([b - 0x10000 if b >= 0x8000 else b for b in bits], dtype=torch.int16).view(
        torch.bfloat16).reshape(shape)


def test_exact_router_logits_random():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(5, 96, generator=g).to(torch.bfloat16)
    w = (torch.randn(6, 96, generator=g) * 0.05).to(torch.bfloat16)
    b = (torch.randn(6, generator=g) * 0.1).to(torch.bfloat16)
    got = ref.exact_linear_bf16(x, w, b)
    assert _bits(got) == _exact_logits(x, w, b)


def test_exact_router_logits_hard_cases():
    # ties: 1 + 2^-8 lies exactly between two bf16 values (1 and 1 + 2^-7)
    x = _from_bits([0x3F80, 0x3B80, 0, 0], (1, 4))          # 1, 2^-8
    w = _from_bits([0x3F80, 0x3F80, 0, 0,                    # -> 1 + 2^-8: tie, to even (1)
                    0x3F80, 0x3F80, 0x0001, 0x0001,          # + 2^-133 * ... tiny: breaks the tie up
                    0xBF80, 0x3F80, 0, 0], (3, 4))           # -1 + 2^-8: cancellation
    x2 = _from_bits([0x3F80, 0x3B80, 0x3F80, 0x3F80], (1, 4))
    b = _from_bits([0, 0, 0], (3,))
    for xx in (x, x2):
        assert _bits(ref.exact_linear_bf16(xx, w, b)) == _exact_logits(xx, w, b)
    # subnormal inputs and results, a spread of ~250 binades, exact cancellation
    vals = [0x0001, 0x0081, 0x7F00, 0xFF00, 0x3F80, 0x0300, 0x8003, 0x4000]
    x3 = _from_bits(vals, (1, 8))
    w3 = _from_bits([0x0001, 0x0001, 0x0080, 0x0080, 0x0001, 0x3F80, 0x3F80, 0x0001,
                     0x3F80, 0x0000, 0x0000, 0x0000, 0x0000, 0x0000, 0x0000, 0x0000], (2, 8))
    b3 = _from_bits([0x8001, 0x0002], (2,))
    assert _bits(ref.exact_linear_bf16(x3, w3, b3)) == _exact_logits(x3, w3, b3)


def test_softmax_topk_weights_round_once():
    v = torch.tensor([[2.0, 1.0, 0.5, -3.0], [1.0, 1.0, 1.0, 1.0]]).to(torch.bfloat16).float()
    w = ref.softmax_topk_bf16(v)
    p = torch.exp(v.double() - v.double()[:, :1])
    exp = (p / p.sum(-1, keepdim=True))
    for got, e in zip(_bits(w), exp.reshape(-1).tolist()):
        assert got == _round_bf16_exact(Fraction(e))
    assert torch.equal(w[1], torch.full((4,), 0.25, dtype=torch.bfloat16))
