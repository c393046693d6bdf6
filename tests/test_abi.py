"""The C-ABI library: it loads, exports every entry point include/*.h declares, and rejects bad
arguments on the host before any device work. CPU only (no compute calls)."""
import ctypes as C
import subprocess

import pytest

import msgl
from msgl._lib import LIB_PATH, SIGNATURES


def test_library_loads_and_versions():
    L = msgl.lib()
    assert b"sm_100a" in L.msgl_version()


def test_exports_every_header_symbol():
    names = msgl.header_symbols()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    # every declared entry point has a ctypes signature in the binding
    assert not [n for n in names if n not in SIGNATURES]


def test_host_side_validation():
    L = msgl.lib()
    # hidden not a multiple of 8 -> UNSUPPORTED_SHAPE, no launch
    rc = L.msgl_launch_rmsnorm(None, None, None, 4, 7, 1e-6, 1, None)
    assert rc == 2 and b"multiple of 8" in L.msgl_last_error()
    # head_dim != 128 for the fused QK-norm kernel
    assert L.msgl_qknorm_rope_store_kv(None, None, None, None, 16, None, None, None, None, None,
                                       1, 8, 2, 64, 1e-6, None) == 2
    # attention: unsupported page size / head ratio
    assert L.msgl_paged_attention_decode(None, None, None, 16, None, 1, None, 1, 16, 8, 2, 128, 8,
                                         1.0, None, None, 0, None) == 2
    assert L.msgl_paged_attention_decode(None, None, None, 16, None, 1, None, 1, 16, 6, 4, 128, 16,
                                         1.0, None, None, 0, None) == 1
    # GEMM: K not a multiple of 8
    assert L.msgl_gemm_bf16(None, None, None, 4, 128, 100, 1, None, 0, None) == 2
    # MoE: router partials count outside [1, 64]; combine with top_k above 32
    assert L.msgl_moe_route_topk_partials(None, 0, 4, 128, 8, 1, None, None, None) == 1
    assert L.msgl_moe_route_topk_partials(None, 65, 4, 128, 8, 1, None, None, None) == 1
    assert L.msgl_moe_combine(None, None, None, 4, 33, 2048, None, None) == 2
    # split-K partials: more than 256 tokens (rejected before any pointer is used)
    fake = 256  # an address that is never dereferenced
    assert L.msgl_gemm_bf16_partials(fake, fake, fake, 300, 128, 256, 1, None) == 2
    assert L.msgl_gemm_bf16_partials(None, None, None, 16, 128, 256, 1, None) == 1
    # combine + add + RMSNorm: null pointers, top_k above 32, hidden above 8192, rows not
    # 16-byte aligned (all rejected before any pointer is used)
    assert L.msgl_moe_combine_add_rmsnorm(None, None, None, 4, 8, 2048, None, None, 1e-6, None, None) == 1
    assert L.msgl_moe_combine_add_rmsnorm(fake, fake, fake, 4, 33, 2048, fake, fake, 1e-6, fake, None) == 2
    assert L.msgl_moe_combine_add_rmsnorm(fake, fake, fake, 4, 8, 8200, fake, fake, 1e-6, fake, None) == 2
    assert L.msgl_moe_combine_add_rmsnorm(fake, fake, fake, 4, 8, 2048, fake, fake, 1e-6, fake + 8, None) == 1
    # zero-size work is a no-op
    assert L.msgl_launch_rmsnorm(None, None, None, 0, 64, 1e-6, 1, None) == 0
    assert L.msgl_moe_combine_add_rmsnorm(fake, fake, fake, 0, 8, 2048, fake, fake, 1e-6, fake, None) == 0


def test_workspace_sizes():
    L = msgl.lib()
    # decode GEMMs split K and need a workspace; the large-M prefill GEMM does not
    assert L.msgl_gemm_workspace_size(128, 6144, 4096) > 0
    assert L.msgl_gemm_workspace_size(2048, 151936, 4096) == 0
    # 128 requests x 8 kv heads x 2048 tokens: split-KV workspace present
    assert L.msgl_paged_attention_workspace_size(128, 2048, 32, 8, 128) > 0


def test_partials_split_plan_host():
    """Split-K partials plan (host only, 148 SMs without a device): one 128-token tile up to 128
    tokens, two tiles up to 256 (the split count then fills the GPU with both tiles), none above;
    the workspace of msgl_gemm_bf16 covers its 129..256-token partials."""
    L = msgl.lib()
    # Qwen3-30B-A3B qkv 5120 x 2048: 20 tiles of 256 rows -> 7 splits at one token tile, 3 at two
    assert L.msgl_gemm_partials_splits(128, 5120, 2048) == 7
    assert L.msgl_gemm_partials_splits(256, 5120, 2048) == 3
    assert L.msgl_gemm_partials_splits(200, 5120, 2048) == 3
    assert L.msgl_gemm_partials_splits(257, 5120, 2048) == 0
    # router 128 x 2048: one tile, split count capped by K / (4 x 64)
    assert L.msgl_gemm_partials_splits(256, 128, 2048) == 8
    for M, N, K in [(256, 5120, 2048), (200, 2048, 4096), (256, 128, 2048)]:
        S = L.msgl_gemm_partials_splits(M, N, K)
        assert L.msgl_gemm_workspace_size(M, N, K) >= S * M * N * 4
