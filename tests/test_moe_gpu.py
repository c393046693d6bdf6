"""MoE path on the GPU against the oracle: router top-k (ids bit-exact on identical fp32 logits,
ties to the larger expert id), permute (bit-exact stable counting sort), grouped tcgen05 GEMMs
(dense and gate_up+SwiGLU), combine, and the whole expert block vs the reference expert loop."""
import numpy as np
import pytest
import torch

from oracle import bf16_round

pytestmark = pytest.mark.gpu


def dev(a, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dtype).contiguous()


def host(t):
    return t.float().cpu().numpy() if t.dtype != torch.int32 else t.cpu().numpy()


def rn(rng, *shape, std=1.0):
    return bf16_round(rng.standard_normal(shape).astype(np.float32) * std)


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def route(logits, k, norm=True):
    import msgl
    T, E = logits.shape
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    w = torch.empty(T, k, dtype=torch.float32, device="cuda")
    msgl.check(msgl.lib().msgl_moe_route_topk(logits.data_ptr(), T, E, k, int(norm), ids.data_ptr(),
                                              w.data_ptr(), torch.cuda.current_stream().cuda_stream))
    return ids, w


def permute(ids, E):
    import msgl
    T, k = ids.shape
    off = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    tok = torch.empty(T * k, dtype=torch.int32, device="cuda")
    pos = torch.empty(T * k, dtype=torch.int32, device="cuda")
    msgl.check(msgl.lib().msgl_moe_permute(ids.data_ptr(), T, k, E, off.data_ptr(), tok.data_ptr(),
                                           pos.data_ptr(), torch.cuda.current_stream().cuda_stream))
    return off, tok, pos


@pytest.mark.parametrize("T,E,k", [(1, 8, 2), (37, 128, 8), (256, 128, 8), (5, 60, 4)])
def test_route_topk(cuda, oracle, T, E, k):
    rng = np.random.default_rng(T + E)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    logits[0, [3, E - 1]] = 10.0            # exact tie at the top: larger id first
    if T > 1:
        logits[-1, :] = 0.5                 # all equal: ids E-1, E-2, ...
    for norm in (True, False):
        ids, w = route(dev(logits, torch.float32), k, norm)
        eid, ew = oracle.router_topk(logits, k, norm)
        assert np.array_equal(host(ids), eid)
        np.testing.assert_allclose(host(w), ew, rtol=2e-6, atol=1e-7)
    assert list(host(ids)[0][:2]) == [E - 1, 3]


def test_router_logits_gemm_then_topk(cuda, oracle):
    """Full router: fp32-output GEMM then top-k; ids equal the oracle's wherever the oracle's
    k-th / (k+1)-th logit margin exceeds the logit error."""
    from msgl import ops
    rng = np.random.default_rng(7)
    T, H, E, k = 64, 2048, 128, 8
    x, wr = rn(rng, T, H), rn(rng, E, H, std=0.02)
    lg = ops.linear(dev(x), dev(wr), out_dtype=torch.float32)
    ids, _ = route(lg, k)
    ref = oracle.linear(x, wr)
    eid, _ = oracle.router_topk(ref, k)
    srt = -np.sort(-ref, axis=1)
    margin = np.minimum(srt[:, k - 1] - srt[:, k], np.min(-np.diff(srt[:, :k], axis=1), axis=1))
    err = np.abs(host(lg) - ref).max()
    clear = margin > 4 * err
    assert clear.mean() > 0.5
    assert np.array_equal(host(ids)[clear], eid[clear])


@pytest.mark.parametrize("T,H,E,k", [(256, 2048, 128, 8), (200, 2048, 128, 8), (64, 512, 60, 4)])
def test_route_topk_partials(cuda, oracle, T, H, E, k):
    """Router logits as split-K partials summed by the top-k kernel in part order: the same ids
    and weights as the top-k of the partials' in-order fp32 sum (bit-exact), and the oracle's ids
    where the logit margin is clear."""
    import msgl
    from msgl import ops
    rng = np.random.default_rng(T + E)
    x, wr = rn(rng, T, H), rn(rng, E, H, std=0.02)
    S = ops.gemm_partials_splits(T, E, H)
    assert S >= 2
    parts = ops.linear_partials(dev(x), dev(wr), S)
    summed = parts[0].clone()
    for p in range(1, S):
        summed += parts[p]
    ids_ref, w_ref = route(summed, k)
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    w = torch.empty(T, k, dtype=torch.float32, device="cuda")
    msgl.check(msgl.lib().msgl_moe_route_topk_partials(
        parts.data_ptr(), S, T, E, k, 1, ids.data_ptr(), w.data_ptr(),
        torch.cuda.current_stream().cuda_stream))
    assert np.array_equal(host(ids), host(ids_ref))
    assert np.array_equal(host(w), host(w_ref))
    ref = oracle.linear(x, wr)
    eid, _ = oracle.router_topk(ref, k)
    srt = -np.sort(-ref, axis=1)
    margin = np.minimum(srt[:, k - 1] - srt[:, k], np.min(-np.diff(srt[:, :k], axis=1), axis=1))
    clear = margin > 4 * np.abs(host(summed) - ref).max()
    assert clear.mean() > 0.5
    assert np.array_equal(host(ids)[clear], eid[clear])


@pytest.mark.parametrize("T,E,k", [(3, 8, 2), (256, 128, 8), (4096, 128, 8)])
def test_permute(cuda, T, E, k):
    rng = np.random.default_rng(T)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    off, tok, pos = permute(dev(ids, torch.int32), E)
    flat = ids.reshape(-1)
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=E)
    assert np.array_equal(host(off), np.concatenate([[0], np.cumsum(counts)]))
    assert np.array_equal(host(tok), order // k)
    inv = np.empty_like(order)
    inv[order] = np.arange(order.size)
    assert np.array_equal(host(pos), inv)


# the last two cases have tiles of 128 / 256 rows (the persistent grouped kernel's sizes)
@pytest.mark.parametrize("T,E,k,H,I", [(16, 8, 2, 256, 96), (256, 128, 8, 2048, 768), (2048, 32, 4, 512, 256),
                                       (2048, 64, 8, 512, 256)])
def test_expert_block(cuda, oracle, monkeypatch, T, E, k, H, I):
    """permute -> gather -> grouped gate_up+SwiGLU -> grouped down -> combine, vs the reference
    expert loop (qwen3_moe.cpp:74-108) restated in the oracle."""
    import msgl
    from msgl import ops
    rng = np.random.default_rng(T + E + H)
    x = rn(rng, T, H)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    wts = rng.random((T, k)).astype(np.float32)
    wts /= wts.sum(1, keepdims=True)
    gu = [rn(rng, 2 * I, H, std=0.05) for _ in range(E)]
    dn = [rn(rng, H, I, std=0.05) for _ in range(E)]
    ref = oracle.moe_experts(x, ids, wts, gu, dn)

    s = torch.cuda.current_stream().cuda_stream
    L = msgl.lib()
    off, tok, pos = permute(dev(ids, torch.int32), E)
    xs = ops.index_gather(dev(x), tok)
    gu_packed = torch.stack([ops.pack_gate_up(dev(w)) for w in gu]).contiguous()
    dn_d = dev(np.stack(dn))
    R = T * k
    ws = torch.zeros(L.msgl_grouped_gemm_workspace_size(R, E), dtype=torch.uint8, device="cuda")
    act = torch.empty(R, I, dtype=torch.bfloat16, device="cuda")
    msgl.check(L.msgl_grouped_gemm_gate_up_silu(xs.data_ptr(), gu_packed.data_ptr(), act.data_ptr(),
                                                off.data_ptr(), E, I, H, R, ws.data_ptr(), ws.numel(), s))
    ys = torch.empty(R, H, dtype=torch.bfloat16, device="cuda")
    msgl.check(L.msgl_grouped_gemm_bf16(act.data_ptr(), dn_d.data_ptr(), ys.data_ptr(), off.data_ptr(),
                                        E, H, I, R, ws.data_ptr(), ws.numel(), s))
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    msgl.check(L.msgl_moe_combine(ys.data_ptr(), pos.data_ptr(), dev(wts, torch.float32).data_ptr(),
                                  T, k, H, out.data_ptr(), s))
    assert rel_l2(host(out), ref) < 1e-2, rel_l2(host(out), ref)
    assert ops.device_error() == (0, 0)
    # both grouped schedules forced (persistent, one CTA per tile) give the default's bits: the
    # same k order in all of them
    for force in ("0", "1"):
        monkeypatch.setenv("MSGL_GROUPED_PERSISTENT", force)
        act2, ys2 = torch.empty_like(act), torch.empty_like(ys)
        msgl.check(L.msgl_grouped_gemm_gate_up_silu(xs.data_ptr(), gu_packed.data_ptr(), act2.data_ptr(),
                                                    off.data_ptr(), E, I, H, R, ws.data_ptr(), ws.numel(), s))
        msgl.check(L.msgl_grouped_gemm_bf16(act2.data_ptr(), dn_d.data_ptr(), ys2.data_ptr(),
                                            off.data_ptr(), E, H, I, R, ws.data_ptr(), ws.numel(), s))
        assert torch.equal(act, act2) and torch.equal(ys, ys2), force
    assert ops.device_error() == (0, 0)
    # the down projection over the tile list that gate_up left in the workspace (the engine's
    # sequence): the same bits under the default schedule and both forced ones
    for force in (None, "0", "1"):
        if force is None:
            monkeypatch.delenv("MSGL_GROUPED_PERSISTENT", raising=False)
        else:
            monkeypatch.setenv("MSGL_GROUPED_PERSISTENT", force)
        ws.zero_()
        act2, ys2 = torch.empty_like(act), torch.empty_like(ys)
        msgl.check(L.msgl_grouped_gemm_gate_up_silu(xs.data_ptr(), gu_packed.data_ptr(), act2.data_ptr(),
                                                    off.data_ptr(), E, I, H, R, ws.data_ptr(), ws.numel(), s))
        msgl.check(L.msgl_grouped_gemm_bf16_reuse_tiles(act2.data_ptr(), dn_d.data_ptr(), ys2.data_ptr(),
                                                        off.data_ptr(), E, H, I, R, ws.data_ptr(),
                                                        ws.numel(), s))
        assert torch.equal(act, act2) and torch.equal(ys, ys2), force
    assert ops.device_error() == (0, 0)


@pytest.mark.parametrize("T,k,H", [(1, 8, 2048), (256, 8, 2048), (37, 4, 1032), (64, 2, 4096), (3, 32, 8192)])
def test_combine_add_rmsnorm(cuda, T, k, H):
    """The combine fused with the residual add and the next RMSNorm equals msgl_moe_combine
    followed by msgl_add_rmsnorm bit for bit (dropped pairs, pos = -1, included), and both match
    an fp32 torch restatement."""
    import msgl
    from msgl import ops
    rng = np.random.default_rng(T * 31 + H)
    R = T * k
    ys = dev(rn(rng, R, H))
    pos = rng.permutation(R).astype(np.int32)
    pos[rng.random(R) < 0.05] = -1
    wts = rng.random((T, k)).astype(np.float32)
    resid0 = rn(rng, T, H).astype(np.float32)
    g = dev(1.0 + 0.1 * rn(rng, H))
    eps = 1e-6
    s = torch.cuda.current_stream().cuda_stream
    L = msgl.lib()
    pos_d, w_d = dev(pos, torch.int32), dev(wts, torch.float32)

    x1 = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    r1 = dev(resid0, torch.float32)
    msgl.check(L.msgl_moe_combine(ys.data_ptr(), pos_d.data_ptr(), w_d.data_ptr(), T, k, H, x1.data_ptr(), s))
    msgl.check(L.msgl_add_rmsnorm(x1.data_ptr(), r1.data_ptr(), g.data_ptr(), T, H, eps, 0, s))

    x2 = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    r2 = dev(resid0, torch.float32)
    msgl.check(L.msgl_moe_combine_add_rmsnorm(ys.data_ptr(), pos_d.data_ptr(), w_d.data_ptr(), T, k, H,
                                              r2.data_ptr(), g.data_ptr(), eps, x2.data_ptr(), s))
    torch.cuda.synchronize()
    assert torch.equal(r1, r2) and torch.equal(x1, x2)
    assert ops.device_error() == (0, 0)

    # fp32 restatement: m = bf16(sum_j w y[pos]); r += m; x = r * rsqrt(mean(r^2) + eps) * g
    yf = ys.float()
    pt = torch.from_numpy(pos).long().cuda().view(T, k)
    gathered = yf[pt.clamp(min=0)] * (pt >= 0).unsqueeze(-1)
    m = (gathered * w_d.view(T, k, 1)).sum(1).bfloat16().float()
    r = torch.from_numpy(resid0).cuda() + m
    xr = r * torch.rsqrt(r.pow(2).mean(-1, keepdim=True) + eps) * g.float()
    # (torch sums the k products in another order, so its bf16 rounding of m may land one bf16
    # ulp, 2^-8 relative, away from the kernel's)
    assert bool(((r2 - r).abs() <= m.abs() * 2.0 ** -7 + 1e-5).all())
    assert rel_l2(host(x2), xr.cpu().numpy()) < 1e-2
