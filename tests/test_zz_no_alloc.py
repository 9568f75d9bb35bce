"""fg_paged_decode_attn_noalloc, the attention entry point for callers that
cannot allocate device memory (a runtime that owns all device memory through
its own pool, an FFI binding without a device allocator): it must give the
results of fg_paged_decode_attn with a caller workspace, call after call,
while the split scratch lives in the library's built-in device array.

Kept in a file of its own that pytest collects last, so a failure here cannot
stop the rest of a `-x` run; it passes alone in a fresh process and after the
other tests (the first call on the device resolves the array's address)."""
import math

import pytest
import torch

from oracle import decode_ref as oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _inputs(seed, B, nq, nkv, hd, lens):
    g = torch.Generator().manual_seed(seed)
    num_blocks = sum((l + 15) // 16 for l in lens) + 3
    max_blocks = max((l + 15) // 16 for l in lens)
    perm = torch.randperm(num_blocks, generator=g)
    table = torch.full((B, max_blocks), -1, dtype=torch.int32)
    used = 0
    for b, l in enumerate(lens):
        nb = (l + 15) // 16
        table[b, :nb] = perm[used:used + nb].to(torch.int32)
        used += nb
    kc = torch.randn(num_blocks, nkv, 16, hd, generator=g).to(torch.bfloat16)
    vc = torch.randn(num_blocks, nkv, 16, hd, generator=g).to(torch.bfloat16)
    q = torch.randn(B, nq, hd, generator=g).to(torch.bfloat16)
    seq = torch.tensor(lens, dtype=torch.int32)
    return [t.to(DEV) for t in (q, kc, vc, table, seq)]


def _noalloc(lib, q, kc, vc, table, seq, out, max_len, window=0, sinks=None):
    B, nq, hd = q.shape
    num_blocks, nkv, bs, _ = kc.shape
    return lib.fg_paged_decode_attn_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), table.data_ptr(), seq.data_ptr(),
        None if sinks is None else sinks.data_ptr(), out.data_ptr(), B, nq, nkv, hd, bs,
        num_blocks, table.shape[1], max_len, window, 1.0 / math.sqrt(hd),
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point_two_calls_in_a_row():
    from fluidgpu_b200 import _lib, build, kernels

    build.build()
    lib = _lib.lib()
    cases = [
        # (seed, B, nq, nkv, hd, lens, window, sinks): both split their pages,
        # so the built-in scratch carries partials between the two kernels
        (11, 6, 32, 8, 128, [4000, 17, 2500, 1, 3333, 4096], 0, False),
        (12, 4, 64, 8, 64, [700, 129, 2048, 5], 1024, True),
    ]
    for seed, B, nq, nkv, hd, lens, window, use_sinks in cases:
        q, kc, vc, table, seq = _inputs(seed, B, nq, nkv, hd, lens)
        sinks = torch.randn(nq, generator=torch.Generator().manual_seed(seed)).float().to(DEV) \
            if use_sinks else None
        max_len = max(lens)
        need = lib.fg_attn_workspace_bytes(B, nq, nkv, hd, max_len, window)
        assert need > 0, "the case must exercise the split scratch"
        ref = kernels.paged_decode_attn(q, kc, vc, table, seq, max_len, window=window, sinks=sinks)
        # the oracle's fp32 attention over the same pages (what both entry
        # points approximate): within the attention tolerance
        qc, kcc, vcc, tc = q.cpu(), kc.cpu(), vc.cpu(), table.cpu().long()
        exp = torch.stack([oracle.attention_one(
            qc[b], kcc[tc[b, :(lens[b] + 15) // 16]].transpose(1, 2).reshape(-1, nkv, hd)[:lens[b]],
            vcc[tc[b, :(lens[b] + 15) // 16]].transpose(1, 2).reshape(-1, nkv, hd)[:lens[b]],
            1.0 / math.sqrt(hd), window, None if sinks is None else sinks.cpu()).reshape(-1)
            for b in range(B)])
        for call in range(2):  # two calls in a row share (and reuse) the built-in scratch
            out = torch.full_like(ref, float("nan"))
            rc = _noalloc(lib, q, kc, vc, table, seq, out, max_len, window, sinks)
            assert rc == 0, lib.fg_last_error()
            torch.cuda.synchronize()
            assert torch.equal(out, ref), f"call {call}: differs from fg_paged_decode_attn"
            err = (out.float().cpu().reshape(B, -1) - exp).abs().max().item()
            assert err <= 2e-2, f"call {call}: {err} from the oracle"
    kernels.check_device("no-alloc attention")


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from fluidgpu_b200 import _lib, build

    build.build()
    lib = _lib.lib()
    # a shape whose split plan on this GPU needs more than the 8 MiB built in
    # (the plan depends on the SM count and the kernel's occupancy)
    shapes = [(B, nq, nkv, ctx) for nq, nkv in ((128, 8), (256, 16), (512, 32))
              for B in (8, 16, 32, 64, 128) for ctx in (32768, 131072)]
    big = [sh for sh in shapes if lib.fg_attn_workspace_bytes(sh[0], sh[1], sh[2], 128, sh[3], 0) > (8 << 20)]
    assert big, "no candidate shape needs more than the built-in scratch"
    B, nq, nkv, ctx = big[0]
    dummy = torch.zeros(16, dtype=torch.bfloat16, device=DEV)
    rc = lib.fg_paged_decode_attn_noalloc(
        dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
        None, dummy.data_ptr(), B, nq, nkv, 128, 16, 1, ctx // 16, ctx, 0, 0.1,
        torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.FG_ERR_ARG
    assert b"built-in" in lib.fg_last_error()
