"""Parity of every libmsgl kernel against the oracle, through the C ABI, on a B200.

Inputs are seeded bf16-representable values; the oracle computes in fp32 on the same values.
Tolerances (bf16 outputs vs fp32 oracle): relative L2 <= 1e-2 and max-abs bounds stated per
test; integer / copy outputs are bit-exact.
"""
import numpy as np
import pytest
import torch

from oracle import bf16_round

pytestmark = pytest.mark.gpu

EPS = 1e-6


def dev(a, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dtype).contiguous()


def host(t):
    return t.float().cpu().numpy()


def rn(rng, *shape, std=1.0):
    return bf16_round(rng.standard_normal(shape).astype(np.float32) * std)


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


# ------------------------------------------------------------------ norms
@pytest.mark.parametrize("H", [64, 1024, 2048, 4096, 5120])
def test_rmsnorm(cuda, oracle, H):
    from msgl import ops
    rng = np.random.default_rng(H)
    x, w = rn(rng, 7, H), rn(rng, H)
    ref = oracle.rmsnorm(x, w, EPS)
    out = host(ops.rmsnorm(dev(x), dev(w), EPS))
    assert rel_l2(out, ref) < 5e-3
    out32 = host(ops.rmsnorm(dev(x, torch.float32), dev(w, torch.float32), EPS))
    np.testing.assert_allclose(out32, ref, rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("H", [1024, 4096])
def test_add_rmsnorm(cuda, oracle, H):
    from msgl import ops
    rng = np.random.default_rng(3)
    x, r, w = rn(rng, 9, H), rng.standard_normal((9, H)).astype(np.float32), rn(rng, H)
    xd, rd = dev(x), dev(r, torch.float32)
    ops.add_rmsnorm_(xd, rd, dev(w), EPS)
    ex, er = oracle.add_rmsnorm(x, r, w, EPS)
    np.testing.assert_allclose(host(rd), er, rtol=1e-6, atol=1e-6)
    assert rel_l2(host(xd), ex) < 5e-3
    xd = dev(x)
    rd = torch.empty(9, H, dtype=torch.float32, device="cuda")
    ops.add_rmsnorm_(xd, rd, dev(w), EPS, first=True)
    ex, er = oracle.add_rmsnorm(x, None, w, EPS, first=True)
    assert np.array_equal(host(rd), er)
    assert rel_l2(host(xd), ex) < 5e-3


def test_embed_rmsnorm_and_gather(cuda, oracle):
    from msgl import ops
    rng = np.random.default_rng(4)
    V, H = 1000, 1024
    E, w = rn(rng, V, H), rn(rng, H)
    ids = np.array([5, -1, 999, 1000, 0, 42], np.int32)
    x, r = ops.embed_rmsnorm(dev(E), dev(ids, torch.int32), dev(w), EPS)
    emb = oracle.embedding(E, ids)
    assert np.array_equal(host(r), emb)
    ex, _ = oracle.add_rmsnorm(emb, None, w, EPS, first=True)
    assert rel_l2(host(x), ex) < 5e-3
    g = ops.index_gather(dev(E), dev(ids, torch.int32))
    assert np.array_equal(host(g), emb)


# ------------------------------------------------------------------ RoPE / KV store
def test_rope_and_store_kv_page(cuda, oracle):
    from msgl import ops
    rng = np.random.default_rng(5)
    T, hq, hkv, D, P = 11, 4, 2, 128, 16
    table = oracle.rope_table(D, 4096, 1e6)
    pos = rng.integers(0, 4096, T).astype(np.int32)
    q, k = rn(rng, T, hq * D), rn(rng, T, hkv * D)
    qd, kd = dev(q, torch.float32), dev(k, torch.float32)
    ops.rope_(qd, kd, dev(pos, torch.int32), dev(table, torch.float32), hq, hkv, D)
    np.testing.assert_allclose(host(qd), oracle.rope(q, pos, hq, D, table), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(kd), oracle.rope(k, pos, hkv, D, table), rtol=1e-5, atol=1e-5)
    # store_kv_page: copy semantics, bit-exact
    pt = np.array([3, 0], np.int32)
    kc = torch.zeros(4 * P, hkv * D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    v = rn(rng, T, hkv * D)
    ops.store_kv_page(dev(k), dev(v), kc, vc, dev(pt, torch.int32), P, hkv, D)
    ek, ev = np.zeros((4 * P, hkv * D), np.float32), np.zeros((4 * P, hkv * D), np.float32)
    oracle.store_kv_page(k, v, ek, ev, pt, P, hkv, D)
    assert np.array_equal(host(kc), ek) and np.array_equal(host(vc), ev)


@pytest.mark.parametrize("hq,hkv", [(16, 8), (32, 8), (32, 4)])
def test_qknorm_rope_store_kv(cuda, oracle, hq, hkv):
    from msgl import ops
    rng = np.random.default_rng(hq + hkv)
    T, D = 13, 128
    table = oracle.rope_table(D, 8192, 1e6)
    qkv = rn(rng, T, (hq + 2 * hkv) * D)
    qn, kn = bf16_round(1 + 0.1 * rng.standard_normal(D).astype(np.float32)), rn(rng, D)
    pos = rng.integers(0, 8192, T).astype(np.int32)
    num_slots = 64
    slots = rng.permutation(num_slots)[:T].astype(np.int32)
    slots[3] = -1  # padding token: no store
    kp = torch.zeros(num_slots, hkv * D, dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros_like(kp)
    qo = ops.qknorm_rope_store_kv(dev(qkv), kp, vp, dev(pos, torch.int32), dev(slots, torch.int32),
                                  dev(table, torch.float32), dev(qn), dev(kn), hq, hkv, EPS)
    qd, kd = hq * D, hkv * D
    q = oracle.rope(oracle.rmsnorm(qkv[:, :qd], qn, EPS), pos, hq, D, table)
    k = oracle.rope(oracle.rmsnorm(qkv[:, qd:qd + kd], kn, EPS), pos, hkv, D, table)
    v = qkv[:, qd + kd:]
    assert rel_l2(host(qo).reshape(T, -1), q) < 5e-3
    ek, ev = np.zeros((num_slots, kd), np.float32), np.zeros((num_slots, kd), np.float32)
    keep = slots >= 0
    oracle.store_kv_slots(k[keep], v[keep], ek, ev, slots[keep])
    assert rel_l2(host(kp), ek) < 5e-3
    assert np.array_equal(host(vp), ev)  # V is a pure copy
    assert np.count_nonzero(host(kp).any(axis=1)) == keep.sum()


# ------------------------------------------------------------------ paged attention
def make_paged(rng, seq_lens, hkv, num_pages, P=16, D=128):
    """Random KV pool and page tables: each request's pages drawn from a random permutation."""
    pages_per = [(s + P - 1) // P for s in seq_lens]
    max_pages = max(max(pages_per), 1)
    perm = rng.permutation(num_pages).astype(np.int32)
    pt = np.zeros((len(seq_lens), max_pages), np.int32)
    off = 0
    for r, n in enumerate(pages_per):
        pt[r, :n] = perm[off:off + n]
        off += n
    assert off <= num_pages
    kp = rn(rng, num_pages * P, hkv * D)
    vp = rn(rng, num_pages * P, hkv * D)
    return kp, vp, pt


@pytest.mark.parametrize("hq,hkv,seq_lens", [
    (16, 8, [1, 15, 16, 17, 100, 513]),
    (32, 8, [2048, 1, 777, 4096]),
    (32, 4, [300, 33, 2500]),
    (8, 8, [64, 5]),
    (16, 2, [1000]),
    (4, 1, [200, 17, 1]),     # one kv head: four pages per stage
    (12, 6, [100, 260]),      # head groups of two
    (32, 16, [300, 40]),      # four head groups per request
])
def test_paged_decode(cuda, oracle, hq, hkv, seq_lens):
    from msgl import ops
    rng = np.random.default_rng(sum(seq_lens) + hq)
    B = len(seq_lens)
    num_pages = sum((s + 15) // 16 for s in seq_lens) + 3
    kp, vp, pt = make_paged(rng, seq_lens, hkv, num_pages)
    q = rn(rng, B, hq * 128)
    seq = np.array(seq_lens, np.int32)
    ref = oracle.paged_attention(q, kp, vp, pt, seq, np.arange(B + 1, dtype=np.int32), hq, hkv, 128, 16)
    ws = ops.attention_workspace(B, max(seq_lens), hq, hkv)
    args = (dev(q), dev(kp), dev(vp), dev(pt, torch.int32), dev(seq, torch.int32), max(seq_lens), hq, hkv)
    out = host(ops.paged_attention_decode(*args, workspace=ws)).reshape(B, -1)
    assert rel_l2(out, ref) < 1e-2, rel_l2(out, ref)
    assert np.abs(out - ref).max() < 3e-2
    # the split-KV arrival counters reset themselves: reusing the workspace gives identical bits
    out2 = host(ops.paged_attention_decode(*args, workspace=ws)).reshape(B, -1)
    assert np.array_equal(out, out2)
    assert ops.device_error() == (0, 0)


@pytest.mark.parametrize("hq,hkv,qlens,ctx", [
    (16, 8, [128, 128, 128, 128], [128, 128, 128, 128]),   # prefill from an empty cache
    (32, 8, [1, 17, 64, 5], [40, 17, 200, 1029]),          # extend after a cached prefix
    (32, 4, [33, 100], [33, 300]),
    (8, 8, [70], [70]),
])
def test_paged_extend(cuda, oracle, hq, hkv, qlens, ctx):
    from msgl import ops
    rng = np.random.default_rng(sum(ctx) + hq)
    B = len(qlens)
    num_pages = sum((s + 15) // 16 for s in ctx) + 2
    kp, vp, pt = make_paged(rng, ctx, hkv, num_pages)
    indptr = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    q = rn(rng, int(indptr[-1]), hq * 128)
    seq = np.array(ctx, np.int32)
    ref = oracle.paged_attention(q, kp, vp, pt, seq, indptr, hq, hkv, 128, 16)
    out = ops.paged_attention_extend(dev(q), dev(kp), dev(vp), dev(pt, torch.int32),
                                     dev(seq, torch.int32), dev(indptr, torch.int32), max(qlens),
                                     hq, hkv)
    out = host(out).reshape(q.shape[0], -1)
    assert rel_l2(out, ref) < 1e-2, rel_l2(out, ref)
    assert ops.device_error() == (0, 0)


@pytest.mark.parametrize("hq,hkv,qlens,ctx", [
    (16, 2, [300, 512], [1500, 512]),        # group 8: 16 tokens per tile, cached prefix
    (32, 8, [257, 64, 1], [900, 64, 700]),   # group 4, ragged, a one-token request
    (8, 4, [200], [1000]),                   # group 2
    (4, 4, [129, 128], [129, 640]),          # group 1: 128 tokens per tile
])
def test_paged_extend_tc(cuda, oracle, monkeypatch, hq, hkv, qlens, ctx):
    """The tcgen05 extend kernel (128-row tiles, S and O in TMEM) against the oracle over longer
    prefills, every group size; the warp-MMA kernel (MSGL_EXTEND_TC=0) on the same inputs too."""
    from msgl import ops
    rng = np.random.default_rng(sum(ctx) + 7 * hq)
    num_pages = sum((c + 15) // 16 for c in ctx) + 3
    kp, vp, pt = make_paged(rng, ctx, hkv, num_pages)
    indptr = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    q = rn(rng, int(indptr[-1]), hq * 128)
    seq = np.array(ctx, np.int32)
    ref = oracle.paged_attention(q, kp, vp, pt, seq, indptr, hq, hkv, 128, 16)
    args = (dev(q), dev(kp), dev(vp), dev(pt, torch.int32), dev(seq, torch.int32),
            dev(indptr, torch.int32), max(qlens), hq, hkv)
    out = host(ops.paged_attention_extend(*args)).reshape(q.shape[0], -1)
    assert rel_l2(out, ref) < 1e-2, rel_l2(out, ref)
    monkeypatch.setenv("MSGL_EXTEND_TC", "0")
    legacy = host(ops.paged_attention_extend(*args)).reshape(q.shape[0], -1)
    assert rel_l2(legacy, ref) < 1e-2
    assert ops.device_error() == (0, 0)


def test_paged_extend_tc_chunk_shape(cuda, monkeypatch):
    """The 32B chunked prefill at a TP8 rank (8 q heads, 1 kv head): the last 2048-token chunk of
    an 8192-token prompt, causal, pages scattered; tcgen05 kernel vs warp-MMA kernel (the fp32
    oracle would take minutes at this size), and run-to-run bit equality."""
    from msgl import ops
    rng = np.random.default_rng(21)
    CH, PL = 2048, 8192
    kp, vp, pt = make_paged(rng, [PL], 1, PL // 16 + 5)
    q = rn(rng, CH, 8 * 128)
    args = (dev(q), dev(kp), dev(vp), dev(pt, torch.int32),
            dev(np.array([PL], np.int32), torch.int32), dev(np.array([0, CH], np.int32), torch.int32),
            CH, 8, 1)
    a = host(ops.paged_attention_extend(*args))
    b = host(ops.paged_attention_extend(*args))
    assert np.array_equal(a, b)
    monkeypatch.setenv("MSGL_EXTEND_TC", "0")
    c = host(ops.paged_attention_extend(*args))
    assert rel_l2(a.reshape(CH, -1), c.reshape(CH, -1)) < 1e-2
    assert ops.device_error() == (0, 0)


def make_shared_prefix(rng, S, suffix_lens, hkv, extra=4, P=16, D=128):
    """Page tables whose first S columns are the same pages for every request (a shared prefix),
    then each request's own pages; contexts S * 16 + suffix_len."""
    own = [(n + P - 1) // P for n in suffix_lens]
    num_pages = S + sum(own) + extra
    perm = rng.permutation(num_pages).astype(np.int32)
    width = S + max(max(own), 1)
    pt = np.zeros((len(suffix_lens), width), np.int32)
    pt[:, :S] = perm[:S]
    off = S
    for r, n in enumerate(own):
        pt[r, S:S + n] = perm[off:off + n]
        off += n
    kp = rn(rng, num_pages * P, hkv * D)
    vp = rn(rng, num_pages * P, hkv * D)
    seq = np.array([S * P + n for n in suffix_lens], np.int32)
    return kp, vp, pt, seq


@pytest.mark.parametrize("hq,hkv,S,suffix", [
    (32, 8, 8, [1, 17, 300, 16, 0, 255]),     # empty suffix, partial / full last pages
    (16, 2, 5, [40, 1, 99]),
    (8, 1, 3, [5, 70]),                        # one kv head, group 8
    (32, 16, 4, [33, 2]),                      # four head groups
    (32, 8, 64, [1024] * 4 + [7, 900]),        # long shared prefix (bench-like)
    (32, 8, 6, list(range(1, 41))),            # 40 requests: 3 row tiles of 64 (request, head) rows
    (4, 1, 5, [3, 60, 17] * 8),                # one TP8 rank of Qwen3-8B: 4 q heads on 1 kv head
])
def test_paged_decode_cascade(cuda, oracle, hq, hkv, S, suffix):
    from msgl import ops
    rng = np.random.default_rng(S * 31 + hq + len(suffix))
    kp, vp, pt, seq = make_shared_prefix(rng, S, suffix, hkv)
    B = len(suffix)
    q = rn(rng, B, hq * 128)
    ref = oracle.paged_attention(q, kp, vp, pt, seq, np.arange(B + 1, dtype=np.int32), hq, hkv, 128, 16)
    L = int(seq.max())
    args = (dev(q), dev(kp), dev(vp), dev(pt, torch.int32), dev(seq, torch.int32), L)
    n = ops.lib().msgl_paged_attention_cascade_workspace_size(B, L, S, hq, hkv, 128)
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    out = host(ops.paged_attention_decode_cascade(*args, S, hq, hkv, workspace=ws)).reshape(B, -1)
    assert rel_l2(out, ref) < 1e-2, rel_l2(out, ref)
    plain = host(ops.paged_attention_decode(*args, hq, hkv)).reshape(B, -1)
    assert rel_l2(out, plain) < 5e-3
    # counters reset themselves: a second call on the same workspace gives the same bits
    out2 = host(ops.paged_attention_decode_cascade(*args, S, hq, hkv, workspace=ws)).reshape(B, -1)
    assert np.array_equal(out, out2)
    assert ops.device_error() == (0, 0)


def test_paged_decode_cascade_detects_unshared_prefix(cuda):
    """A row whose 'shared' columns differ is reported in the error word (no fault)."""
    from msgl import ops
    rng = np.random.default_rng(5)
    kp, vp, pt, seq = make_shared_prefix(rng, 4, [20, 30], 8)
    pt[1, 2] = pt[1, 4]  # request 1 does not share column 2
    q = rn(rng, 2, 32 * 128)
    ops.device_error(reset=True)
    ops.paged_attention_decode_cascade(dev(q), dev(kp), dev(vp), dev(pt, torch.int32),
                                       dev(seq, torch.int32), int(seq.max()), 4, 32, 8)
    torch.cuda.synchronize()
    assert ops.device_error() == (6, 205)  # MSGL_ERR_BOUNDS at the sharing check


def test_decode_equals_extend_single_token(cuda):
    """Decode and extend agree on one-token-per-request batches."""
    from msgl import ops
    rng = np.random.default_rng(9)
    seq_lens = [100, 2000, 16]
    kp, vp, pt = make_paged(rng, seq_lens, 8, 200)
    q = rn(rng, 3, 32 * 128)
    seq = dev(np.array(seq_lens, np.int32), torch.int32)
    a = ops.paged_attention_decode(dev(q), dev(kp), dev(vp), dev(pt, torch.int32), seq, 2000, 32, 8)
    b = ops.paged_attention_extend(dev(q), dev(kp), dev(vp), dev(pt, torch.int32), seq,
                                   dev(np.arange(4, dtype=np.int32), torch.int32), 1, 32, 8)
    assert rel_l2(host(a).reshape(3, -1), host(b).reshape(3, -1)) < 5e-3


# ------------------------------------------------------------------ GEMMs
@pytest.mark.parametrize("M,N,K", [
    (1, 128, 64), (7, 256, 128), (16, 384, 1024), (64, 1024, 1024), (128, 6144, 4096),
    (128, 1000, 200), (200, 512, 4096), (300, 640, 576), (96, 4096, 12288),
    # row-range schedule: 148 tiles of 176 rows; 136 tiles of 192 rows, the last one partial
    (77, 26048, 320), (128, 26088, 256),
    # 129..256 tokens: split-K partials over both token tiles (Qwen3-30B-A3B qkv / router at
    # b256), or two passes of 128
    (256, 5120, 2048), (256, 128, 2048), (129, 4096, 4096),
    # short K (a TP8 / TP4 rank's o_proj, a TP8 rank's down): narrow row tiles over the whole K
    (128, 4096, 512), (100, 4096, 1024), (128, 4096, 1536), (5, 4096, 512),
])
def test_gemm_bf16(cuda, M, N, K):
    from msgl import ops
    rng = np.random.default_rng(M * 7 + N + K)
    x, w = rn(rng, M, K), rn(rng, N, K, std=0.05)
    ref = (torch.from_numpy(x).double() @ torch.from_numpy(w).double().T).numpy()
    y = host(ops.linear(dev(x), dev(w)))
    assert rel_l2(y, ref) < 8e-3, rel_l2(y, ref)
    y32 = host(ops.linear(dev(x), dev(w), out_dtype=torch.float32))
    assert rel_l2(y32, ref) < 1e-5, rel_l2(y32, ref)
    # deterministic (split-K sums in a fixed order)
    y32b = host(ops.linear(dev(x), dev(w), out_dtype=torch.float32))
    assert np.array_equal(y32, y32b)
    assert ops.device_error() == (0, 0)


def test_gemm_workspace_shared_across_shapes(cuda):
    """One workspace reused, in stream order, by split-K GEMMs of different shapes (as the
    executor does across a layer): decode shapes as partials + reduce, (200, 512, 4096) as
    stream-K, whose flags share the workspace's zero-filled head; every result stays correct."""
    from msgl import ops
    rng = np.random.default_rng(12)
    shapes = [(128, 6144, 4096), (128, 4096, 4096), (200, 512, 4096), (300, 512, 4096),
              (128, 4096, 12288), (4, 1000, 512)]
    ws = torch.zeros(max(ops.gemm_workspace(*s).numel() for s in shapes), dtype=torch.uint8,
                     device="cuda")
    data = [(rn(rng, M, K), rn(rng, N, K, std=0.02)) for M, N, K in shapes]
    for rep in range(2):
        for (x, w) in data:
            ref = (torch.from_numpy(x).double() @ torch.from_numpy(w).double().T).numpy()
            y = host(ops.linear(dev(x), dev(w), out_dtype=torch.float32, workspace=ws))
            assert rel_l2(y, ref) < 1e-5, (rep, x.shape, w.shape)
    assert ops.device_error() == (0, 0)


def test_decode_workspace_shared_across_shapes(cuda, oracle):
    from msgl import ops
    rng = np.random.default_rng(13)
    cases = [[2048, 1000, 77, 3000], [513, 4096], [100] * 9]
    ws = torch.zeros(max(ops.attention_workspace(len(c), max(c), 32, 8).numel() for c in cases),
                     dtype=torch.uint8, device="cuda")
    for rep in range(2):
        for seq_lens in cases:
            B = len(seq_lens)
            kp, vp, pt = make_paged(rng, seq_lens, 8, sum((s + 15) // 16 for s in seq_lens) + 1)
            q = rn(rng, B, 32 * 128)
            seq = np.array(seq_lens, np.int32)
            ref = oracle.paged_attention(q, kp, vp, pt, seq, np.arange(B + 1, dtype=np.int32),
                                         32, 8, 128, 16)
            out = ops.paged_attention_decode(dev(q), dev(kp), dev(vp), dev(pt, torch.int32),
                                             dev(seq, torch.int32), max(seq_lens), 32, 8,
                                             workspace=ws)
            assert rel_l2(host(out).reshape(B, -1), ref) < 1e-2, (rep, seq_lens)
    assert ops.device_error() == (0, 0)


def test_gemm_matches_oracle_linear(cuda, oracle):
    from msgl import ops
    rng = np.random.default_rng(1)
    x, w = rn(rng, 4, 512), rn(rng, 256, 512, std=0.05)
    ref = oracle.linear(x, w)
    y = host(ops.linear(dev(x), dev(w), out_dtype=torch.float32))
    np.testing.assert_allclose(y, ref, rtol=1e-4, atol=1e-4)


# (128, 12288, 1024) and (5, 12288, 256): 24576 weight rows take the row-range schedule (whole
# 176-row tiles per CTA); (4, 3072, 1024), (128, 1536, 4096) (a TP8 rank of Qwen3-8B) and
# (96, 6144, 512): small gate_up (2I x K <= 16M elements) on the cluster kernel, or split-K
# partials summed by the SwiGLU reduce kernel where the cluster plan does not balance;
# (37, 96, 256) the cluster kernel, (300, 768, 512) stream-K, (256, 768, 2048) two passes of
# 128 tokens
@pytest.mark.parametrize("M,I,K", [(4, 3072, 1024), (128, 1536, 4096), (37, 96, 256), (300, 768, 512),
                                   (128, 12288, 1024), (5, 12288, 256), (96, 6144, 512),
                                   (256, 768, 2048),
                                   # short K at 64 / 128 tokens: narrow row tiles (Qwen3-0.6B)
                                   (64, 3072, 1024), (128, 3072, 1024)])
def test_gate_up_silu(cuda, oracle, M, I, K):
    from msgl import ops
    rng = np.random.default_rng(M + I)
    x, wgu = rn(rng, M, K), rn(rng, 2 * I, K, std=0.05)
    gu = oracle.linear(x, wgu)
    ref = oracle.swiglu(gu[:, :I], gu[:, I:])
    wp = ops.pack_gate_up(dev(wgu))
    y = host(ops.gate_up_silu(dev(x), wp))
    assert rel_l2(y, ref) < 8e-3, rel_l2(y, ref)


@pytest.mark.parametrize("M,V,K", [(4, 1024, 256), (64, 151936, 1024), (130, 4096, 512),
                                   (128, 37984, 512), (128, 18992, 512),  # TP4 / TP8 shards
                                   (256, 37984, 1024)])
def test_lm_head_argmax(cuda, oracle, M, V, K):
    from msgl import ops
    rng = np.random.default_rng(M + V)
    x, w = rn(rng, M, K), rn(rng, V, K, std=0.05)
    w[V // 2] = w[V // 3]  # exact duplicate rows -> ties resolved to the lower id
    ids = host(ops.lm_head_argmax(dev(x), dev(w))).astype(np.int64)
    logits = host(ops.linear(dev(x), dev(w), out_dtype=torch.float32))
    assert np.array_equal(ids, oracle.argmax(logits))
    ref = oracle.linear(x, w)
    top2 = np.sort(ref, axis=1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 1e-3
    assert np.array_equal(ids[clear], oracle.argmax(ref)[clear])


def test_argmax_ties(cuda, oracle):
    from msgl import ops
    rng = np.random.default_rng(2)
    lg = rng.standard_normal((5, 151936)).astype(np.float32)
    lg[1, [7, 90000]] = 100.0
    lg[2, :] = 0.0
    out = host(ops.argmax(dev(lg, torch.float32))).astype(np.int64)
    assert np.array_equal(out, oracle.argmax(lg))
    assert out[1] == 7 and out[2] == 0


def test_fill_normal(cuda):
    from msgl import ops
    t = torch.empty(1 << 20, dtype=torch.bfloat16, device="cuda")
    ops.fill_normal_(t, seed=0, std=0.02)
    a = t.float()
    assert abs(a.mean().item()) < 1e-3 and abs(a.std().item() - 0.02) < 1e-3
    t2 = ops.fill_normal_(torch.empty_like(t), seed=0, std=0.02)
    assert torch.equal(t, t2)
