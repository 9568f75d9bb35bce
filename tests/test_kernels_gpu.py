"""Per-kernel parity on the GPU: each C-ABI entry point against the CPU oracle
(oracle/decode_ref.py) or a plain fp32 torch reference, on seeded inputs."""
import math

import pytest
import torch

from oracle import decode_ref as ref

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from fluidgpu_b200 import build

    build.build()
    yield
    from fluidgpu_b200 import kernels

    kernels.check_device("kernel tests")


def _gen(seed):
    g = torch.Generator().manual_seed(seed)
    return g


def _randn(shape, g, scale=1.0, dtype=torch.bfloat16):
    return (torch.randn(shape, generator=g) * scale).to(dtype)


# ---------------------------------------------------------------------------
def test_embed_and_bad_index():
    from fluidgpu_b200 import kernels

    g = _gen(0)
    table = _randn((1000, 256), g)
    ids = torch.randint(0, 1000, (37,), generator=g)
    out = kernels.embed(ids.to(DEV), table.to(DEV))
    assert torch.equal(out.cpu(), table[ids])
    kernels.check_device("embed")
    bad = torch.tensor([5, 1000, -1], dtype=torch.int64)
    out = kernels.embed(bad.to(DEV), table.to(DEV)).cpu()
    assert torch.equal(out[0], table[5]) and out[1:].abs().sum() == 0
    assert kernels.device_status(reset=True) & 0xFF == 3


@pytest.mark.parametrize("H,T", [(1024, 8), (4096, 64), (2880, 5), (64, 1)])
@pytest.mark.parametrize("fp32mul", [False, True])
def test_rmsnorm(H, T, fp32mul):
    from fluidgpu_b200 import kernels

    g = _gen(1)
    x = _randn((T, H), g)
    w = _randn((H,), g, 0.5) + 1.0
    mode = 1 if fp32mul else 0
    out = kernels.rmsnorm(x.to(DEV), w.to(DEV).to(torch.bfloat16), 1e-5, mode).cpu()
    exp = ref.rms_norm(x, w.to(torch.bfloat16), 1e-5, fp32mul)
    diff = (out.float() - exp.float()).abs()
    # identical up to one bf16 ulp from the fp32 reduction order
    assert (diff <= exp.float().abs() * 2 ** -7 + 1e-6).all()
    assert (diff == 0).float().mean() > 0.9


def _gemm_ref(x, w, bias=None):
    y = x.float() @ w.float().T
    if bias is not None:
        y = y + bias.float()
    return y


@pytest.mark.parametrize(
    "T,N,K,splits",
    [
        (1, 128, 64, 1),
        (8, 256, 1024, 0),
        (13, 384, 640, 2),
        (64, 6144, 4096, 0),
        (64, 4096, 4096, 0),
        (33, 2880, 2880, 0),     # N not a multiple of 128
        (100, 512, 1024, 3),
        (256, 1024, 512, 1),
        (300, 640, 256, 0),      # two token tiles
        (64, 1000, 200, 0),      # K tail inside one 64-wide stage
        (64, 4096, 4096, 8),     # cluster of 8 CTAs per tile, DSMEM reduction
        (40, 896, 1024, -7),     # persistent stream-K, 7 CTAs: uneven tile splits
        (64, 128256 // 8, 4096, 0),  # many tiles: automatic stream-K
        (200, 640, 512, -5),     # stream-K with two token tiles
    ],
)
@pytest.mark.parametrize("packed", [True, False])
def test_gemm_store(T, N, K, splits, packed):
    from fluidgpu_b200 import kernels

    g = _gen(2)
    x = _randn((T, K), g)
    w = _randn((N, K), g, 0.05)
    wd = kernels.PackedWeight(w.to(DEV)) if packed else w.to(DEV)
    out = kernels.gemm(x.to(DEV), wd, splits=splits).cpu()
    exp = _gemm_ref(x, w)
    err = (out.float() - exp).abs().max().item()
    assert err <= 1e-2 * exp.abs().max().item() + 1e-3, err


def test_gemm_bias_residual():
    from fluidgpu_b200 import kernels

    g = _gen(3)
    T, N, K = 64, 4096, 4096
    x = _randn((T, K), g)
    w = _randn((N, K), g, 0.02)
    b = _randn((N,), g, 0.1)
    r = _randn((T, N), g)
    for splits, wd in ((1, w.to(DEV)), (4, w.to(DEV)), (0, kernels.PackedWeight(w.to(DEV))),
                       (3, kernels.PackedWeight(w.to(DEV))), (-11, kernels.PackedWeight(w.to(DEV)))):
        out = kernels.gemm(x.to(DEV), wd, epilogue=1, residual=r.to(DEV), bias=b.to(DEV),
                           splits=splits).cpu()
        exp = r.float() + _gemm_ref(x, w, b).to(torch.bfloat16).float()
        err = (out.float() - exp).abs().max().item()
        assert err <= 2e-2 * exp.abs().max().item(), (splits, err)


@pytest.mark.parametrize("T,I,K,splits", [(64, 14336, 4096, 0), (8, 2816, 1024, 0), (5, 128, 64, 1),
                                           (64, 512, 4096, 4), (64, 512, 4096, -9), (64, 2816, 1024, 6)])
def test_gemm_swiglu(T, I, K, splits):
    from fluidgpu_b200 import kernels

    g = _gen(4)
    x = _randn((T, K), g)
    wg = _randn((I, K), g, 0.02)
    wu = _randn((I, K), g, 0.02)
    # gate/up interleaved in blocks of 64 rows
    w = torch.stack([wg.view(I // 64, 64, K), wu.view(I // 64, 64, K)], dim=1).reshape(2 * I, K)
    out = kernels.gemm(x.to(DEV), kernels.PackedWeight(w.to(DEV)), epilogue=2, splits=splits).cpu()
    out2 = kernels.gemm(x.to(DEV), w.to(DEV), epilogue=2, splits=splits).cpu()
    assert torch.equal(out, out2)  # same tiles, same order: packed == row-major bit for bit
    gate = _gemm_ref(x, wg).to(torch.bfloat16)
    up = _gemm_ref(x, wu).to(torch.bfloat16)
    exp = ref.silu_mul(gate, up).float()
    err = (out.float() - exp).abs().max().item()
    assert err <= 2e-2 * exp.abs().max().item() + 1e-4, err


@pytest.mark.parametrize("T,N,K,epi", [(512, 36864, 128, 0),   # 576 tiles: 144 persistent CTAs x 4
                                        (520, 25600, 192, 1),   # residual + bias, ragged last token tile
                                        (512, 19200, 128, 2)])  # SwiGLU, 300 tiles: 100 CTAs x 3
@pytest.mark.parametrize("packed", [True, False])
def test_gemm_many_tokens_persistent(T, N, K, epi, packed):
    """Many tokens (prefill): the automatic plan takes the persistent kernel
    over whole tiles (a grid dividing the tile count, no workspace); per tile
    its MMAs run over K in the same order as the one-tile-per-CTA kernel
    (splits=1), so both give the same bits, and both match fp32."""
    from fluidgpu_b200 import _lib, kernels

    g = _gen(9)
    x = _randn((T, K), g)
    w = _randn((N, K), g, 0.05)
    b = _randn((N,), g, 0.1) if epi == 1 else None
    r = _randn((T, N), g) if epi == 1 else None
    wd = kernels.PackedWeight(w.to(DEV)) if packed else w.to(DEV)
    kw = dict(epilogue=epi, residual=None if r is None else r.to(DEV), bias=None if b is None else b.to(DEV))
    lib = _lib.lib()
    tiles = (N + 127) // 128 * ((T + 255) // 256)
    grid = lib.fg_gemm_grid(T, N, K, 0)
    assert grid <= 148 and tiles % grid == 0 and lib.fg_gemm_workspace_bytes(T, N, K, 0) == 0, (grid, tiles)
    many = kernels.gemm(x.to(DEV), wd, splits=0, **kw).cpu()
    one = kernels.gemm(x.to(DEV), wd, splits=1, **kw).cpu()
    assert torch.equal(many, one)
    acc = _gemm_ref(x, w, b)
    if epi == 0:
        exp = acc
    elif epi == 1:
        exp = r.float() + acc.to(torch.bfloat16).float()
    else:
        gu = acc.to(torch.bfloat16).view(T, N // 128, 2, 64)
        exp = ref.silu_mul(gu[:, :, 0].reshape(T, -1), gu[:, :, 1].reshape(T, -1)).float()
    err = (many.float() - exp).abs().max().item()
    assert err <= 2e-2 * exp.abs().max().item() + 1e-3, err


def test_pack_weight_layout():
    """Packed tile (nt, kb): 16-byte chunk c of row r sits at chunk c ^ (r % 8)."""
    from fluidgpu_b200 import kernels

    g = _gen(9)
    N, K = 200, 136  # ragged in both dimensions
    w = _randn((N, K), g)
    pw = kernels.PackedWeight(w.to(DEV))
    data = pw.data.cpu().view(torch.bfloat16).view(2, 3, 128, 8, 8)  # [nt][kb][row][slot][8]
    for nt in range(2):
        for kb in range(3):
            for r in (0, 5, 71, 127):
                for c in range(8):
                    n, k = nt * 128 + r, kb * 64 + c * 8
                    got = data[nt, kb, r, c ^ (r % 8)]
                    exp = w[n, k:k + 8] if (n < N and k < K) else torch.zeros(8, dtype=torch.bfloat16)
                    assert torch.equal(got, exp), (nt, kb, r, c)


def test_gemm_chain_with_pdl():
    """Back-to-back dependent GEMMs and norms (programmatic dependent launch):
    each result feeds the next call; compare the whole chain to torch."""
    from fluidgpu_b200 import kernels

    g = _gen(10)
    T, H, I = 64, 1024, 2048
    x = _randn((T, H), g)
    ws = [_randn((I, H), g, 0.03), _randn((H, I), g, 0.03), _randn((I, H), g, 0.03)]
    pw = [kernels.PackedWeight(w.to(DEV)) for w in ws]
    h = x.to(DEV)
    ref_h = x.float()
    for it in range(3):
        a = kernels.gemm(h, pw[0])
        h = kernels.gemm(a, pw[1], epilogue=1, residual=h)
        ref_a = (ref_h.to(torch.bfloat16).float() @ ws[0].float().T).to(torch.bfloat16).float()
        ref_h = (ref_h + (ref_a @ ws[1].float().T).to(torch.bfloat16).float()).to(torch.bfloat16).float()
    err = (h.cpu().float() - ref_h).abs().max().item()
    assert err <= 3e-2 * ref_h.abs().max().item(), err


# ---------------------------------------------------------------------------
def _paged_setup(B, nkv, hd, lens, num_blocks, g):
    max_blocks = max((l + 15) // 16 for l in lens)
    perm = torch.randperm(num_blocks, generator=g)
    table = torch.full((B, max_blocks), -1, dtype=torch.int32)
    used = 0
    for b, l in enumerate(lens):
        nb = (l + 15) // 16
        table[b, :nb] = perm[used : used + nb].to(torch.int32)
        used += nb
    assert used <= num_blocks
    kc = _randn((num_blocks, nkv, 16, hd), g)
    vc = _randn((num_blocks, nkv, 16, hd), g)
    return table, kc, vc


def _gather(cache, table, b, L):
    nb = (L + 15) // 16
    pages = cache[table[b, :nb].long()]  # [nb, nkv, 16, hd]
    return pages.permute(0, 2, 1, 3).reshape(nb * 16, pages.shape[1], pages.shape[3])[:L]


@pytest.mark.parametrize(
    "B,nq,nkv,hd,lens,window,sinks",
    [
        (3, 32, 8, 128, [1, 17, 300], 0, False),
        (4, 16, 4, 64, [16, 33, 250, 5], 0, False),
        (2, 64, 8, 64, [300, 129], 128, True),
        (2, 64, 8, 64, [1000, 7], 0, True),
        (5, 32, 8, 128, [4096, 4000, 2048, 17, 4097], 0, False),
        (1, 32, 8, 128, [32768], 0, False),
        (1, 64, 8, 64, [30000], 0, True),
        (8, 4, 2, 64, [20, 21, 22, 23, 24, 25, 26, 27], 2, False),
    ],
)
def test_paged_attention(B, nq, nkv, hd, lens, window, sinks):
    from fluidgpu_b200 import kernels

    g = _gen(5)
    num_blocks = sum((l + 15) // 16 for l in lens) + 7
    table, kc, vc = _paged_setup(B, nkv, hd, lens, num_blocks, g)
    q = _randn((B, nq, hd), g)
    sk = (torch.randn(nq, generator=g) * 2.0) if sinks else None
    seq = torch.tensor(lens, dtype=torch.int32)
    out = kernels.paged_decode_attn(
        q.to(DEV), kc.to(DEV), vc.to(DEV), table.to(DEV), seq.to(DEV), max(lens), window=window,
        sinks=None if sk is None else sk.to(DEV),
    ).cpu()
    scale = 1.0 / math.sqrt(hd)
    for b, L in enumerate(lens):
        k = _gather(kc, table, b, L)
        v = _gather(vc, table, b, L)
        exp = ref.attention_one(q[b], k, v, scale, window, sk).reshape(-1)
        err = (out[b].float() - exp).abs().max().item()
        assert err <= 2e-2, (b, L, err)


def test_rope_kv_append():
    from fluidgpu_b200 import kernels

    g = _gen(6)
    B, nq, nkv, hd = 4, 8, 2, 128
    num_blocks = 16
    positions = torch.tensor([0, 15, 16, 40], dtype=torch.int32)
    table = torch.randperm(num_blocks, generator=g)[: B * 4].view(B, 4).to(torch.int32)
    qkv = _randn((B, (nq + 2 * nkv) * hd), g)
    inv_freq = ref.default_inv_freq(hd, 500000.0)
    kc = torch.zeros((num_blocks, nkv, 16, hd), dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kcd, vcd = kc.to(DEV), vc.to(DEV)
    q = kernels.rope_kv_append(qkv.to(DEV), positions.to(DEV), inv_freq.to(DEV), 1.0,
                               table.to(DEV), kcd, vcd, nq, nkv, hd).cpu()
    cos, sin = ref.rope_cos_sin(positions.long(), inv_freq, 1.0, torch.bfloat16)
    x = qkv.view(B, nq + 2 * nkv, hd)
    eq = ref.apply_rope(x[:, :nq], cos, sin)
    ek = ref.apply_rope(x[:, nq : nq + nkv], cos, sin)
    ev = x[:, nq + nkv :]
    assert (q.float() - eq.float()).abs().max() <= 2 ** -6 * eq.float().abs().max()
    kcd, vcd = kcd.cpu(), vcd.cpu()
    written = torch.zeros(num_blocks, 16, dtype=torch.bool)
    for b in range(B):
        p = int(positions[b])
        blk = int(table[b, p // 16])
        written[blk, p % 16] = True
        assert (kcd[blk, :, p % 16].float() - ek[b].float()).abs().max() <= 2 ** -6 * ek.float().abs().max()
        assert torch.equal(vcd[blk, :, p % 16], ev[b])
    # nothing else touched
    assert kcd.permute(0, 2, 1, 3)[~written].abs().sum() == 0
    assert vcd.permute(0, 2, 1, 3)[~written].abs().sum() == 0


def test_argmax_ties_lowest_index():
    from fluidgpu_b200 import kernels

    g = _gen(7)
    T, V = 6, 128256
    logits = _randn((T, V), g)
    logits[1, 100] = 50.0
    logits[1, 7] = 50.0
    logits[2, V - 1] = 60.0
    logits[3, :] = 1.0
    out = kernels.argmax(logits.to(DEV)).cpu()
    exp = ref.argmax_lowest(logits.float())
    assert torch.equal(out, exp)
    assert out[1] == 7 and out[2] == V - 1 and out[3] == 0


def test_advance():
    from fluidgpu_b200 import kernels

    pos = torch.arange(5, dtype=torch.int32, device=DEV)
    lens = pos + 1
    kernels.advance(pos, lens)
    assert pos.cpu().tolist() == [1, 2, 3, 4, 5]
    assert lens.cpu().tolist() == [2, 3, 4, 5, 6]


@pytest.mark.parametrize(
    "B,nq,nkv,hd,S,ctx,window,sinks",
    [
        (2, 32, 8, 128, 37, [0, 20], 0, False),     # Llama-style GQA 4, context before the chunk
        (3, 16, 4, 64, 64, [0, 0, 5], 0, False),
        (2, 64, 8, 64, 50, [0, 100], 16, True),     # gpt-oss-style GQA 8, window, sinks
        (1, 8, 8, 128, 130, [3], 0, False),         # MHA (64 positions per CTA)
        (2, 32, 2, 64, 33, [0, 0], 0, True),        # GQA 16
    ],
)
def test_prefill_attention(B, nq, nkv, hd, S, ctx, window, sinks):
    """Causal prefill attention over the pages: query j of sequence b sits at
    position ctx[b] + j and attends keys 0 .. ctx[b] + j (and the window)."""
    from fluidgpu_b200 import kernels

    g = _gen(9)
    lens = [c + S for c in ctx]
    num_blocks = sum((l + 15) // 16 for l in lens) + 5
    table, kc, vc = _paged_setup(B, nkv, hd, lens, num_blocks, g)
    q = _randn((B * S, nq, hd), g)
    sk = (torch.randn(nq, generator=g) * 2.0) if sinks else None
    first = torch.tensor(ctx, dtype=torch.int32)
    out = kernels.prefill_attn(q.to(DEV), kc.to(DEV), vc.to(DEV), table.to(DEV), first.to(DEV), S,
                               window=window, sinks=None if sk is None else sk.to(DEV)).cpu()
    scale = 1.0 / math.sqrt(hd)
    worst = 0.0
    for b in range(B):
        k = _gather(kc, table, b, lens[b])
        v = _gather(vc, table, b, lens[b])
        for j in range(S):
            L = ctx[b] + j + 1
            exp = ref.attention_one(q[b * S + j], k[:L], v[:L], scale, window, sk)
            worst = max(worst, (out[b * S + j].float() - exp.reshape(nq, hd)).abs().max().item())
    assert worst <= 2e-2, worst


def test_rope_kv_append_tokens_matches_per_sequence():
    """The token-wise form equals the per-sequence one bit for bit."""
    from fluidgpu_b200 import kernels

    g = _gen(10)
    B, S, nq, nkv, hd = 3, 5, 8, 2, 64
    num_blocks = 12
    table = torch.randperm(num_blocks, generator=g)[: B * 4].view(B, 4).to(torch.int32)
    qkv = _randn((B * S, (nq + 2 * nkv) * hd), g)
    inv_freq = ref.default_inv_freq(hd, 10000.0).to(DEV)
    seq = torch.arange(B, dtype=torch.int32).repeat_interleave(S)
    start = torch.tensor([0, 14, 30], dtype=torch.int32)
    pos = (start[:, None] + torch.arange(S, dtype=torch.int32)[None, :]).reshape(-1)
    kc1 = torch.zeros((num_blocks, nkv, 16, hd), dtype=torch.bfloat16, device=DEV)
    vc1, kc2, vc2 = kc1.clone(), kc1.clone(), kc1.clone()
    qkvd, td = qkv.to(DEV), table.to(DEV)
    q1 = kernels.rope_kv_append_tokens(qkvd, seq.to(DEV), pos.to(DEV), inv_freq, 1.0, td, kc1, vc1, nq, nkv, hd)
    q2 = torch.empty_like(q1)
    for j in range(S):  # one position of every sequence at a time, as decode does
        rows = torch.arange(B) * S + j
        x = qkvd[rows.to(DEV)].contiguous()
        q2[rows.to(DEV)] = kernels.rope_kv_append(x, (start + j).to(DEV), inv_freq, 1.0, td, kc2, vc2, nq, nkv, hd)
    assert torch.equal(q1, q2) and torch.equal(kc1, kc2) and torch.equal(vc1, vc2)


# ---------------------------------------------------------------------------
# hand-off kernels of the disaggregated step, one GPU (local destinations)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("T,N,K,epi,route", [
    (32, 4096, 14336, "f32", "split"),        # down projection, split-K over 8 CTAs per tile
    (32, 4096, 4096, "residual", "broadcast"),  # O-proj, split-K over 4 CTAs per tile
    (64, 4096, 14336, "residual", "split"),
    (4, 512, 512, "residual", "broadcast"),     # one CTA per tile
])
def test_routed_gemm_matches_plain_and_signals(T, N, K, epi, route):
    from fluidgpu_b200 import _lib, kernels
    from fluidgpu_b200._lib import call, ptr_array

    g = _gen(21)
    x = _randn((T, K), g).to(DEV)
    w = kernels.PackedWeight(_randn((N, K), g, 0.02).to(DEV))
    res = _randn((T, N), g).to(DEV)
    code = _lib.FG_EPI_F32 if epi == "f32" else _lib.FG_EPI_RESIDUAL
    dt = torch.float32 if epi == "f32" else torch.bfloat16
    want = kernels.gemm(x, w, epilogue=code, residual=res)
    n_dst = 2
    if route == "split":
        rows = (T + n_dst - 1) // n_dst
        dst = [torch.full((rows, N), float("nan"), dtype=dt, device=DEV) for _ in range(n_dst)]
        r_code, row0 = _lib.FG_ROUTE_SPLIT, 0
    else:
        rows, row0 = 3 * T, T  # a row block in the middle of each destination
        dst = [torch.full((rows, N), float("nan"), dtype=dt, device=DEV) for _ in range(n_dst)]
        r_code = _lib.FG_ROUTE_BROADCAST
    flags = torch.zeros(n_dst * 32, dtype=torch.int32, device=DEV)  # 128 bytes apart
    epoch = torch.tensor([5], dtype=torch.int32, device=DEV)
    ticket = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels.device_status(reset=True)
    for rep in range(2):  # the ticket rearms for the next call
        call("fg_gemm_bf16_packed_routed", x.data_ptr(), w.data.data_ptr(), res.data_ptr(), None, T, N, K, code,
             r_code, ptr_array([d.data_ptr() for d in dst]), n_dst, rows if route == "split" else 0, row0,
             ptr_array([flags[32 * i:32 * i + 1].data_ptr() for i in range(n_dst)]), n_dst, epoch.data_ptr(),
             32, 7 + rep, ticket.data_ptr(), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert int(ticket.item()) == 0, "ticket not rearmed"
        assert flags[::32].tolist() == [5 * 32 + 7 + rep] * n_dst, flags[::32].tolist()
    kernels.check_device("routed gemm")
    if route == "split":
        got = torch.cat(dst)[:T]
    else:
        for d in dst[1:]:
            assert torch.equal(d[row0:row0 + T], dst[0][row0:row0 + T])
        assert torch.isnan(dst[0][:row0].float()).all() and torch.isnan(dst[0][row0 + T:].float()).all()
        got = dst[0][row0:row0 + T]
    assert torch.equal(got, want), "routed result differs from fg_gemm_bf16_packed"


def test_waiting_norms_match_rmsnorm():
    """fg_rmsnorm_wait / fg_sum_rmsnorm_wait / fg_rmsnorm_gather_wait with
    their flags already at the awaited value: the results of fg_rmsnorm (and
    of fg_sum_partials then fg_rmsnorm) bit for bit, and the gathered rows
    equal to their sources."""
    from fluidgpu_b200 import _lib, kernels
    from fluidgpu_b200._lib import call, ptr_array

    g = _gen(22)
    T, H, S = 64, 4096, 3
    x = _randn((T, H), g).to(DEV)
    w = (1.0 + _randn((H,), g, 0.1)).to(DEV)
    parts = torch.randn(S, T, H, generator=g).float().to(DEV)
    epoch = torch.tensor([3], dtype=torch.int32, device=DEV)
    flags = torch.full((4 * 32,), 3 * 10 + 4, dtype=torch.int32, device=DEV)  # epoch * 10 + 4 reached
    fptr = ptr_array([flags[32 * i:32 * i + 1].data_ptr() for i in range(4)])
    stream = torch.cuda.current_stream().cuda_stream
    for mode in (_lib.FG_NORM_LLAMA, _lib.FG_NORM_FP32MUL):
        out = torch.empty_like(x)
        call("fg_rmsnorm_wait", x.data_ptr(), w.data_ptr(), out.data_ptr(), T, H, 1e-5, mode, fptr, 4, 16,
             epoch.data_ptr(), 10, 4, 1000, stream)
        assert torch.equal(out, kernels.rmsnorm(x, w, 1e-5, mode))
        h = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
        xo = torch.empty_like(h)
        call("fg_sum_rmsnorm_wait", parts.data_ptr(), S, h.data_ptr(), w.data_ptr(), xo.data_ptr(), T, H, 1e-5,
             mode, fptr, 4, epoch.data_ptr(), 10, 4, 1000, stream)
        hs = kernels.sum_partials(parts)
        assert torch.equal(h, hs)
        assert torch.equal(xo, kernels.rmsnorm(hs, w, 1e-5, mode))
        # gathering form: the rows of x live in four separate buffers of 16
        # rows (stand-ins for four attention GPUs' send buffers)
        srcs = [x[16 * i:16 * (i + 1)].clone() for i in range(4)]
        gathered = torch.full_like(x, float("nan"))
        out2 = torch.empty_like(x)
        call("fg_rmsnorm_gather_wait", ptr_array([t.data_ptr() for t in srcs]), 4, 16, gathered.data_ptr(),
             w.data_ptr(), out2.data_ptr(), T, H, 1e-5, mode, fptr, 4, 16, epoch.data_ptr(), 10, 4, 1000, stream)
        assert torch.equal(gathered, x)
        assert torch.equal(out2, out)
    kernels.check_device("waiting norms")


def test_waiting_norm_times_out_cleanly():
    """A flag that never reaches its value: the wait gives up after its bound,
    the device status records a peer flag timeout (site 0x501) and the
    context stays usable."""
    from fluidgpu_b200 import kernels
    from fluidgpu_b200._lib import call, ptr_array

    x = torch.zeros(4, 512, dtype=torch.bfloat16, device=DEV)
    w = torch.ones(512, dtype=torch.bfloat16, device=DEV)
    flags = torch.zeros(32, dtype=torch.int32, device=DEV)
    epoch = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels.device_status(reset=True)
    call("fg_rmsnorm_wait", x.data_ptr(), w.data_ptr(), torch.empty_like(x).data_ptr(), 4, 512, 1e-5, 0,
         ptr_array([flags.data_ptr()]), 1, 4, epoch.data_ptr(), 1, 1, 100, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    st = kernels.device_status(reset=True)
    assert st & 0xFF == 2 and (st >> 8) == 0x501, f"status {st:#x}"
    assert int(torch.arange(10, device=DEV).sum().item()) == 45
