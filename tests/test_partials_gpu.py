"""Split-K partials path on a B200, through the C ABI: the partials GEMM and the two kernels that
consume its output (fused add + RMSNorm, QK-norm + RoPE + KV store).

msgl_gemm_bf16_partials writes parts[s] = x[:, Ks] W[:, Ks]^T (fp32) for the s-th of S equal
k-block ranges (64-wide k-blocks); each split is checked against a float64 product over the same
columns (relative L2 <= 1e-5: fp32 accumulation of bf16 products), and the sum over splits
against x W^T. The consumers add the partials in split order, so the residual they write is
bit-exact against the same fp32 additions done on the host, and V rows (a pure copy of the
summed row, rounded to bf16) are bit-exact too.
"""
import numpy as np
import pytest
import torch

from oracle import bf16_round

pytestmark = pytest.mark.gpu

EPS = 1e-6
ERR_INVALID_ARG, ERR_UNSUPPORTED_SHAPE = 1, 2


def dev(a, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dtype).contiguous()


def host(t):
    return t.float().cpu().numpy()


def rn(rng, *shape, std=1.0):
    return bf16_round(rng.standard_normal(shape).astype(np.float32) * std)


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def split_sum(parts):
    """fp32 sum over the leading axis in index order (the consumers' order)."""
    s = parts[0].astype(np.float32).copy()
    for p in parts[1:]:
        s += p.astype(np.float32)
    return s


@pytest.mark.parametrize("M,N,K,S", [
    (1, 128, 64, 1), (7, 256, 128, 2), (16, 384, 1024, None), (100, 1000, 200, 3),
    (128, 6144, 4096, None), (128, 4096, 12288, None), (64, 4096, 4096, 5), (128, 768, 4096, 16),
    (33, 200, 1000, 16),
    # 129..256 tokens: a second 128-token tile in the grid (the last one partly filled)
    (256, 5120, 2048, None), (200, 2048, 4096, None), (129, 128, 2048, 4), (256, 1000, 200, 3),
])
def test_gemm_partials(cuda, M, N, K, S):
    from msgl import ops
    rng = np.random.default_rng(M + 3 * N + 7 * K)
    x, w = rn(rng, M, K), rn(rng, N, K, std=0.05)
    if S is None:
        S = ops.gemm_partials_splits(M, N, K)
        assert S >= 1
    parts = host(ops.linear_partials(dev(x), dev(w), S))
    assert parts.shape == (S, M, N)
    KB = (K + 63) // 64
    xd, wd = x.astype(np.float64), w.astype(np.float64)
    for s in range(S):
        k0, k1 = s * KB // S * 64, min((s + 1) * KB // S * 64, K)
        ref = xd[:, k0:k1] @ wd[:, k0:k1].T
        assert rel_l2(parts[s], ref) < 1e-5, (s, rel_l2(parts[s], ref))
    assert rel_l2(parts.sum(0), xd @ wd.T) < 1e-5
    again = host(ops.linear_partials(dev(x), dev(w), S))
    assert np.array_equal(parts, again)  # no cross-CTA order: deterministic
    assert ops.device_error() == (0, 0)


def test_gemm_partials_rejects_bad_sizes(cuda):
    from msgl import lib, ops
    x = torch.zeros(300, 256, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(128, 256, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(8, 300, 128, dtype=torch.float32, device="cuda")
    L = lib()
    p = lambda t: t.data_ptr()
    assert L.msgl_gemm_bf16_partials(p(x), p(w), p(out), 300, 128, 256, 1, None) == ERR_UNSUPPORTED_SHAPE
    assert L.msgl_gemm_bf16_partials(p(x), p(w), p(out), 16, 128, 256, 5, None) == ERR_INVALID_ARG
    assert L.msgl_gemm_bf16_partials(p(x), p(w), p(out), 16, 128, 256, 0, None) == ERR_INVALID_ARG
    assert L.msgl_gemm_bf16_partials(p(x), p(w), p(out), 0, 128, 256, 2, None) == 0
    assert L.msgl_gemm_partials_splits(300, 128, 256) == 0
    torch.cuda.synchronize()
    assert ops.device_error() == (0, 0)


# hidden <= 4096 with <= 16 partials: the one-thread-per-4-elements kernel (one or two load
# batches); (2, 3, 5120) and (20, 4, 1024): the 8-elements-per-thread kernel
@pytest.mark.parametrize("P,T,H", [(1, 5, 1024), (4, 128, 4096), (3, 17, 2048), (16, 2, 4096),
                                   (9, 128, 4096), (2, 3, 5120), (20, 4, 1024)])
def test_add_partials_rmsnorm(cuda, oracle, P, T, H):
    from msgl import ops
    rng = np.random.default_rng(P * 100 + T)
    parts = (rng.standard_normal((P, T, H)) * 0.5).astype(np.float32)
    r = rng.standard_normal((T, H)).astype(np.float32)
    w = rn(rng, H)
    x = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    rd = dev(r, torch.float32)
    ops.add_partials_rmsnorm_(dev(parts, torch.float32), x, rd, dev(w), EPS)
    s = split_sum(parts)
    ex, er = oracle.add_rmsnorm(s, r, w, EPS)
    assert np.array_equal(host(rd), s + r)  # same fp32 additions, same order
    np.testing.assert_allclose(host(rd), er, rtol=1e-6, atol=1e-6)
    assert rel_l2(host(x), ex) < 5e-3
    assert ops.device_error() == (0, 0)


@pytest.mark.parametrize("hq,hkv,P", [(32, 8, 3), (16, 4, 6), (8, 1, 16)])
def test_qknorm_rope_store_kv_partials(cuda, oracle, hq, hkv, P):
    from msgl import ops
    rng = np.random.default_rng(hq * 10 + P)
    T, D = 11, 128
    table = oracle.rope_table(D, 4096, 1e6)
    parts = (rng.standard_normal((P, T, (hq + 2 * hkv) * D)) * 0.6).astype(np.float32)
    qkv = split_sum(parts)
    qn, kn = bf16_round(1 + 0.1 * rng.standard_normal(D).astype(np.float32)), rn(rng, D)
    pos = rng.integers(0, 4096, T).astype(np.int32)
    num_slots = 48
    slots = rng.permutation(num_slots)[:T].astype(np.int32)
    slots[5] = -1  # padding token: no store
    kp = torch.zeros(num_slots, hkv * D, dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros_like(kp)
    qo = ops.qknorm_rope_store_kv_partials(dev(parts, torch.float32), kp, vp, dev(pos, torch.int32),
                                           dev(slots, torch.int32), dev(table, torch.float32),
                                           dev(qn), dev(kn), hq, hkv, EPS)
    qd, kd = hq * D, hkv * D
    q = oracle.rope(oracle.rmsnorm(qkv[:, :qd], qn, EPS), pos, hq, D, table)
    k = oracle.rope(oracle.rmsnorm(qkv[:, qd:qd + kd], kn, EPS), pos, hkv, D, table)
    v = bf16_round(qkv[:, qd + kd:])
    assert rel_l2(host(qo).reshape(T, -1), q) < 5e-3
    ek, ev = np.zeros((num_slots, kd), np.float32), np.zeros((num_slots, kd), np.float32)
    keep = slots >= 0
    oracle.store_kv_slots(k[keep], v[keep], ek, ev, slots[keep])
    assert rel_l2(host(kp), ek) < 5e-3
    assert np.array_equal(host(vp), ev)  # V: the summed row rounded to bf16
    assert ops.device_error() == (0, 0)


def test_partials_chain_matches_bf16_path(cuda, oracle):
    """o_proj as partials + fused add/norm vs o_proj (bf16) + add/norm: same result within the
    bf16 rounding of the projection output, which the partials path skips."""
    from msgl import ops
    rng = np.random.default_rng(11)
    T, H, K = 128, 4096, 4096
    a, w = rn(rng, T, K), rn(rng, H, K, std=0.02)
    r = rng.standard_normal((T, H)).astype(np.float32)
    nw = rn(rng, H)
    parts = ops.linear_partials(dev(a), dev(w))
    x1, r1 = torch.empty(T, H, dtype=torch.bfloat16, device="cuda"), dev(r, torch.float32)
    ops.add_partials_rmsnorm_(parts, x1, r1, dev(nw), EPS)
    x2, r2 = ops.linear(dev(a), dev(w)), dev(r, torch.float32)
    ops.add_rmsnorm_(x2, r2, dev(nw), EPS)
    ex, er = oracle.add_rmsnorm(a.astype(np.float64) @ w.astype(np.float64).T, r, nw, EPS)
    assert rel_l2(host(r1), er) < 1e-5
    assert rel_l2(host(r2), er) < 5e-3
    assert rel_l2(host(x1), ex) < 5e-3 and rel_l2(host(x2), ex) < 5e-3
    assert ops.device_error() == (0, 0)
