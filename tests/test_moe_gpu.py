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
