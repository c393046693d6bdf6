"""The oracle (C restatement) against the reference: golden fixtures and, when oracle/_ref is
built, live comparisons on fresh seeded inputs. CPU only."""
import numpy as np
import pytest

from oracle import OracleModel, bf16_round

EPS = 1e-6


def test_rmsnorm_golden(oracle, golden):
    out = oracle.rmsnorm(golden["rmsnorm_x"], golden["rmsnorm_w"], EPS)
    assert np.array_equal(out, golden["ref_rmsnorm"])


def test_add_rmsnorm_golden(oracle, golden):
    x, r = oracle.add_rmsnorm(golden["add_x"], golden["add_res"], golden["rmsnorm_w"], EPS)
    assert np.array_equal(x, golden["ref_add_x"]) and np.array_equal(r, golden["ref_add_res"])
    x, r = oracle.add_rmsnorm(golden["add_x"], None, golden["rmsnorm_w"], EPS, first=True)
    assert np.array_equal(x, golden["ref_add_first_x"])
    assert np.array_equal(r, golden["ref_add_first_res"])


def test_linear_golden(oracle, golden):
    assert np.array_equal(oracle.linear(golden["linear_x"], golden["linear_w"]), golden["ref_linear"])


def test_swiglu_golden(oracle, golden):
    assert np.array_equal(oracle.swiglu(golden["swiglu_g"], golden["swiglu_u"]), golden["ref_swiglu"])


def test_rope_golden(oracle, golden):
    t128 = oracle.rope_table(128, 64, 1e6)
    assert np.array_equal(t128, golden["ref_rope_table_128"])
    assert np.array_equal(oracle.rope_table(16, 32, 10000.0), golden["ref_rope_table_16"])
    out = oracle.rope(golden["rope_x"], golden["rope_pos"], 2, 128, t128)
    assert np.array_equal(out, golden["ref_rope"])


def test_attention_golden_mha(oracle, golden):
    """The paged restatement reproduces Attention::forward bit for bit in its defined (MHA,
    single-sequence) configuration, with the sequence scattered over permuted pages."""
    q, k, v = golden["attn_q"], golden["attn_k"], golden["attn_v"]
    T, H, D, P = q.shape[0], 4, 16, 4
    pt = np.array([[5, 0, 2]], np.int32)
    kp = np.zeros((8 * P, H * D), np.float32)
    vp = np.zeros_like(kp)
    oracle.store_kv_page(k, v, kp, vp, pt[0], P, H, D)
    out = oracle.paged_attention(q, kp, vp, pt, [T], [0, T], H, H, D, P)
    assert np.array_equal(out, golden["ref_attn_mha"])


def test_router_golden_with_tie(oracle, golden):
    logits = oracle.linear(golden["router_x"], golden["router_w"])
    for sfx, norm in (("", True), ("_nonorm", False)):
        ids, w = oracle.router_topk(logits, 4, norm)
        assert np.array_equal(ids, golden["ref_router_ids" + sfx])
        assert np.array_equal(w, golden["ref_router_w" + sfx])
    # rows 3 and 10 of the router weight are identical: the larger index must come first
    ids = golden["ref_router_ids"]
    for row in ids:
        if 3 in row and 10 in row:
            assert list(row).index(10) < list(row).index(3)


def test_embedding_golden(oracle, golden):
    assert np.array_equal(oracle.embedding(golden["embed_w"], golden["embed_ids"]), golden["ref_embed"])


def test_argmax_first_max(oracle):
    logits = np.array([[0, 3, 1, 3], [-1, -1, -1, -1], [2, 1, 0, 5]], np.float32)
    assert list(oracle.argmax(logits)) == [1, 0, 3]


@pytest.mark.parametrize("kind", ["dense", "moe"])
def test_model_forward_golden(oracle, golden, kind):
    """Oracle composition (qwen3.cpp:16-83 with the fixes) vs the reference's whole-model forward
    for one token, where the reference path is defined."""
    import importlib.util, os
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(os.path.dirname(__file__), "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    extra = {} if kind == "dense" else {"num_experts": 4, "top_k": 2, "moe_inter": 32}
    cfg = dict(num_layers=2, hidden=64, num_q_heads=4, num_kv_heads=4, head_dim=16, inter=128,
               vocab=1000, eps=1e-6, rope_base=1e6, max_position=64, norm_topk=True,
               page_size=16, **extra)
    _, named = mg.tiny_model_weights(np.random.default_rng(7 if kind == "dense" else 8), cfg)
    m = OracleModel(oracle, cfg, named, num_slots=32)
    logits = m.forward([417], [5], [0], np.array([[0]], np.int32), [1], [0, 1])
    np.testing.assert_array_equal(logits, golden[f"ref_model_{kind}_logits"])


def test_paged_restatement_regression(oracle, golden):
    g = golden
    out = oracle.paged_attention(g["paged_q"], g["paged_k"], g["paged_v"], g["paged_pt"],
                                 g["paged_seq"], g["paged_indptr"], 8, 2, 128, 16)
    assert np.array_equal(out, g["oracle_paged"])


def test_paged_gqa_equals_mha_expansion(oracle):
    """GQA restatement == MHA restatement with each kv head repeated for its query group."""
    rng = np.random.default_rng(5)
    hq, hkv, D, P = 8, 2, 16, 4
    T = 11
    q = bf16_round(rng.standard_normal((T, hq * D)).astype(np.float32))
    k = bf16_round(rng.standard_normal((T, hkv * D)).astype(np.float32))
    v = bf16_round(rng.standard_normal((T, hkv * D)).astype(np.float32))
    pt = np.array([[2, 0, 1]], np.int32)
    kp = np.zeros((3 * P, hkv * D), np.float32); vp = np.zeros_like(kp)
    oracle.store_kv_page(k, v, kp, vp, pt[0], P, hkv, D)
    gqa = oracle.paged_attention(q, kp, vp, pt, [T], [0, T], hq, hkv, D, P)
    rep = lambda a: np.repeat(a.reshape(-1, hkv, D), hq // hkv, axis=1).reshape(a.shape[0], -1)
    kp2, vp2 = np.zeros((3 * P, hq * D), np.float32), np.zeros((3 * P, hq * D), np.float32)
    oracle.store_kv_page(rep(k), rep(v), kp2, vp2, pt[0], P, hq, D)
    mha = oracle.paged_attention(q, kp2, vp2, pt, [T], [0, T], hq, hq, D, P)
    assert np.array_equal(gqa, mha)


# ---------------------------------------------------------------- live, against oracle/_ref
def test_live_ops_vs_reference(oracle, reflib):
    rng = np.random.default_rng(11)
    for H in (8, 96, 1024):
        x = rng.standard_normal((3, H)).astype(np.float32)
        w = rng.standard_normal(H).astype(np.float32)
        assert np.array_equal(oracle.rmsnorm(x, w, EPS), reflib.rmsnorm(x, w, EPS))
        r = rng.standard_normal((3, H)).astype(np.float32)
        a, b = oracle.add_rmsnorm(x, r, w, EPS), reflib.add_rmsnorm(x, r, w, EPS)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    x = rng.standard_normal((5, 200)).astype(np.float32)
    W = rng.standard_normal((33, 200)).astype(np.float32)
    assert np.array_equal(oracle.linear(x, W), reflib.linear(x, W))
    T, H, D = 13, 2, 128
    q, k, v = (rng.standard_normal((T, H * D)).astype(np.float32) for _ in range(3))
    ref = reflib.attention_mha(q, k, v, H, D)
    P = 16
    pt = np.array([[1, 0]], np.int32)
    kp = np.zeros((2 * P, H * D), np.float32); vp = np.zeros_like(kp)
    oracle.store_kv_page(k, v, kp, vp, pt[0], P, H, D)
    assert np.array_equal(oracle.paged_attention(q, kp, vp, pt, [T], [0, T], H, H, D, P), ref)
    pos = rng.integers(0, 4096, 9).astype(np.int32)
    xr = rng.standard_normal((9, 4 * 128)).astype(np.float32)
    tab = oracle.rope_table(128, 4096, 1e6)
    assert np.array_equal(oracle.rope(xr, pos, 4, 128, tab), reflib.rope(xr, pos, 4, 128, 4096, 1e6))
