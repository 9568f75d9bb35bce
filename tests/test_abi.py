"""The C ABI: libfgb200.so builds for sm_100a here (nvcc cross-compiles), loads
without a GPU, and exports exactly what include/fgb200.h declares."""
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared() -> set[str]:
    text = (ROOT / "include" / "fgb200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"^\s*(?:const\s+)?[\w ]+?\**\s*\b(fg_\w+)\s*\(", text, flags=re.M))


@pytest.fixture(scope="module")
def lib_path():
    from fluidgpu_b200 import build

    return build.build()


def test_header_declares_entry_points():
    names = _declared()
    for must in ("fg_gemm_bf16", "fg_paged_decode_attn", "fg_rope_kv_append", "fg_last_error",
                 "fg_device_status", "fg_kv_append", "fg_argmax", "fg_embed", "fg_rmsnorm"):
        assert must in names


def test_library_exports_every_declared_symbol(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = _declared() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_binding_covers_header(lib_path):
    from fluidgpu_b200 import _lib

    assert set(_lib.SIGNATURES) == _declared()
    handle = _lib.lib()
    for name in _lib.SIGNATURES:
        assert getattr(handle, name) is not None
    assert handle.fg_version() >= 1


def test_argument_errors_need_no_gpu(lib_path):
    """Shape/pointer validation happens on the host before any CUDA call."""
    from fluidgpu_b200 import _lib

    h = _lib.lib()
    rc = h.fg_gemm_bf16(None, None, None, None, None, 4, 128, 64, 0, 1, None, 0, None)
    assert rc == _lib.FG_ERR_ARG
    assert b"null pointer" in h.fg_last_error()
    rc = h.fg_paged_decode_attn(1, 1, 1, 1, 1, None, 1, None, 0, 1, 32, 8, 96, 16, 1, 1, 16, 0,
                                1.0, None)
    assert rc == _lib.FG_ERR_ARG and b"hd must be 64 or 128" in h.fg_last_error()
    assert h.fg_gemm_workspace_bytes(64, 4096, 4096, -7) > 0   # stream-K reduces through it
    assert h.fg_gemm_workspace_bytes(64, 4096, 4096, 4) == 0   # cluster split-K: on chip
    assert h.fg_gemm_workspace_bytes(64, 4096, 4096, 1) == 0


def test_no_cluster_multicast_anywhere():
    """Multi-GPU safety rule: no bulk/TMA load with cluster multicast in any source."""
    pat = "multi" + "cast::cluster"
    for p in list((ROOT / "fluidgpu_b200" / "csrc").rglob("*")) + [ROOT / "include" / "fgb200.h"]:
        if p.is_file():
            assert pat not in p.read_text(), p


@pytest.mark.parametrize("T,N,K", [(64, 6144, 4096), (64, 4096, 4096), (64, 28672, 4096), (64, 4096, 14336),
                                   (128, 5760, 2880), (1, 128256, 4096)])
def test_gemm_plan_decode_sizes(lib_path, T, N, K):
    """Decode sizes (one token tile): one CTA per tile or split-K clusters,
    never a workspace (planning queries run without a GPU; 148 SMs assumed)."""
    from fluidgpu_b200 import _lib

    lib = _lib.lib()
    tiles = (N + 127) // 128
    assert lib.fg_gemm_grid(T, N, K, 0) == tiles
    assert 1 <= lib.fg_gemm_split(T, N, K, 0) <= 8
    assert lib.fg_gemm_workspace_bytes(T, N, K, 0) == 0


@pytest.mark.parametrize("T,N,K,grid", [(2048, 28672, 4096, 128), (4096, 4096, 14336, 128),
                                        (512, 28672, 4096, 112), (2048, 4096, 4096, 128),
                                        (512, 19200, 128, 100)])
def test_gemm_plan_prefill_sizes(lib_path, T, N, K, grid):
    """Many tokens: a persistent grid that divides the tile count (whole tiles
    per CTA, no split tile, so no workspace)."""
    from fluidgpu_b200 import _lib

    lib = _lib.lib()
    tiles = (N + 127) // 128 * ((T + 255) // 256)
    g = lib.fg_gemm_grid(T, N, K, 0)
    assert g == grid and tiles % g == 0
    assert lib.fg_gemm_workspace_bytes(T, N, K, 0) == 0


@pytest.mark.parametrize("hd", [64, 128])
def test_attn_split_plan_bounds(lib_path, hd):
    """Attention split plan (planning queries run without a GPU): 1..128 slices
    per (sequence, kv head), at least 8 pages of 16 tokens per slice, a window
    bounding the span, and split scratch exactly when there is more than one
    slice (the merge kernel holds one factor per slice for up to 128)."""
    from fluidgpu_b200 import _lib

    lib = _lib.lib()
    nq, nkv = (64, 8) if hd == 64 else (32, 8)
    for B in (1, 2, 7, 32, 64, 128, 256):
        for ctx in (1, 16, 129, 512, 4096, 32768, 131072):
            for window in (0, 128):
                s = lib.fg_attn_splits(B, nkv, hd, ctx, window)
                span = min(ctx, window + 16) if window else ctx
                pages = (span + 15) // 16
                assert 1 <= s <= 128, (B, ctx, window, s)
                assert s == 1 or s <= pages // 8, (B, ctx, window, s)
                ws = lib.fg_attn_workspace_bytes(B, nq, nkv, hd, ctx, window)
                if s == 1:
                    assert ws == 0
                else:
                    rows = B * nq * s
                    assert ws == ((rows * hd * 4 + 255) // 256) * 256 + rows * 2 * 4
    # batch 1 at long context spreads one sequence over many slices
    assert lib.fg_attn_splits(1, nkv, hd, 32768, 0) > 8
    assert lib.fg_attn_splits(1, nkv, hd, 32768, 128) <= 2


def test_missing_library_fails_loudly(tmp_path):
    """No fallback: without the CUDA library every entry point raises (here
    in a fresh interpreter pointed at a path with no library)."""
    import os
    import sys

    code = ("from fluidgpu_b200 import _lib\n"
            "try:\n    _lib.call('fg_last_error')\nexcept RuntimeError as e:\n    print('RAISED', e)\n")
    env = {**os.environ, "FGB200_LIB": str(tmp_path / "absent" / "libfgb200.so")}
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    assert "RAISED" in r.stdout and "not found" in r.stdout


def test_product_never_imports_the_oracle():
    """The oracle is test infrastructure: no module of the package imports it."""
    for p in (ROOT / "fluidgpu_b200").rglob("*.py"):
        src = p.read_text()
        assert not re.search(r"^\s*(from|import)\s+oracle\b", src, re.M), p
        assert "decode_ref" not in src and "cpu_baseline" not in src, p


@pytest.mark.parametrize("T,k,E,BN", [(1, 4, 32, 16), (32, 4, 32, 16), (64, 4, 32, 16), (65, 4, 32, 32),
                                      (128, 4, 32, 32), (129, 4, 32, 64), (512, 4, 32, 64), (4096, 4, 32, 64)])
def test_moe_tile_plan(lib_path, T, k, E, BN):
    """Token tile of the expert GEMM: room for about twice the mean rows per
    expert (16 / 32 / 64), so most experts stream their weights once; the
    work-item bound covers one partial tile per expert plus the full ones."""
    from fluidgpu_b200 import _lib

    lib = _lib.lib()
    assert lib.fg_moe_tile_tokens(T, k, E) == BN
    assert lib.fg_moe_max_items(T, k, E, BN) == E + (T * k + BN - 1) // BN
    assert lib.fg_moe_max_items(0, k, E, BN) == 0
