"""Generate tests/golden/*.npz from the reference's own compiled CPU code.

    make -C oracle ref && python tests/golden/make_golden.py

Every array under a `ref_` key is an output of the reference sources (oracle/_ref, built from
the mini-sglang-cpp sources by oracle/Makefile): RMSNorm, fused add+RMSNorm, Linear, SwiGLU,
RotaryEmbedding (table and apply), Attention (multi-head; the only defined case), MoERouter
(including an exact tie), Embedding, KVCachePool / RadixCache page ids, and the whole-model
forward of Qwen3ForCausalLM / Qwen3MoEForCausalLM for one token (a configuration in which the
reference path is defined: one key, so RoPE on K and QK-norm do not enter).

Keys under `oracle_` are outputs of the C restatement for cases the reference cannot run (GQA,
paged, multi-request): regression pins of the restatement, not reference pins.
Inputs are seeded (numpy PCG64); weights are bf16-representable values.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from oracle import Oracle, RefLib, bf16_round  # noqa: E402


def rn(rng, *shape, std=1.0):
    return bf16_round(rng.standard_normal(shape).astype(np.float32) * std)


def tiny_model_weights(rng, cfg):
    """Weights in ref_model_forward order, plus the same weights keyed by oracle names."""
    H, V, D = cfg["hidden"], cfg["vocab"], cfg["head_dim"]
    hq, hkv, I = cfg["num_q_heads"], cfg["num_kv_heads"], cfg["inter"]
    E, Im = cfg.get("num_experts", 0), cfg.get("moe_inter", 0)
    order, named = [], {}

    def add(name, arr):
        order.append(arr)
        named[name] = arr

    add("embed", rn(rng, V, H, std=0.5))
    for l in range(cfg["num_layers"]):
        p = f"layers.{l}."
        add(p + "input_ln", bf16_round(1.0 + 0.1 * rng.standard_normal(H).astype(np.float32)))
        add(p + "qkv", rn(rng, (hq + 2 * hkv) * D, H, std=0.1))
        add(p + "o", rn(rng, H, hq * D, std=0.1))
        add(p + "post_ln", bf16_round(1.0 + 0.1 * rng.standard_normal(H).astype(np.float32)))
        if E:
            add(p + "router", rn(rng, E, H, std=0.1))
            for e in range(E):
                add(p + f"experts.{e}.gate_up", rn(rng, 2 * Im, H, std=0.1))
                add(p + f"experts.{e}.down", rn(rng, H, Im, std=0.1))
        else:
            add(p + "gate_up", rn(rng, 2 * I, H, std=0.1))
            add(p + "down", rn(rng, H, I, std=0.1))
        named[p + "q_norm"] = np.ones(D, np.float32)
        named[p + "k_norm"] = np.ones(D, np.float32)
    add("norm", bf16_round(1.0 + 0.1 * rng.standard_normal(H).astype(np.float32)))
    add("lm_head", rn(rng, V, H, std=0.1))
    return order, named


def main():
    ref, orc = RefLib(), Oracle()
    rng = np.random.default_rng(20240601)
    g = {}
    eps = 1e-6

    x = rn(rng, 5, 64); w = rn(rng, 64); res = rn(rng, 5, 64)
    g["rmsnorm_x"], g["rmsnorm_w"] = x, w
    g["ref_rmsnorm"] = ref.rmsnorm(x, w, eps)
    g["add_x"], g["add_res"] = x, res
    g["ref_add_x"], g["ref_add_res"] = ref.add_rmsnorm(x, res, w, eps)
    g["ref_add_first_x"], g["ref_add_first_res"] = ref.add_rmsnorm(x, None, w, eps, first=True)

    lx, lw = rn(rng, 3, 96), rn(rng, 40, 96)
    g["linear_x"], g["linear_w"], g["ref_linear"] = lx, lw, ref.linear(lx, lw)

    sg, su = rn(rng, 50, std=3.0), rn(rng, 50)
    g["swiglu_g"], g["swiglu_u"], g["ref_swiglu"] = sg, su, ref.swiglu(sg, su)

    g["ref_rope_table_128"] = ref.rope_table(128, 64, 1e6)
    g["ref_rope_table_16"] = ref.rope_table(16, 32, 10000.0)
    rq = rn(rng, 4, 2 * 128)
    rpos = np.array([0, 3, 63, 17], np.int32)
    g["rope_x"], g["rope_pos"] = rq, rpos
    g["ref_rope"] = ref.rope(rq, rpos, 2, 128, 64, 1e6)

    T, Hh, D = 9, 4, 16
    aq, ak, av = rn(rng, T, Hh * D), rn(rng, T, Hh * D), rn(rng, T, Hh * D)
    g["attn_q"], g["attn_k"], g["attn_v"] = aq, ak, av
    g["ref_attn_mha"] = ref.attention_mha(aq, ak, av, Hh, D)

    rx, rw = rn(rng, 7, 32), rn(rng, 16, 32)
    rw[10] = rw[3]  # identical expert rows -> exactly tied logits (tie order pin)
    g["router_x"], g["router_w"] = rx, rw
    g["ref_router_ids"], g["ref_router_w"] = ref.router(rx, rw, 4, True)
    g["ref_router_ids_nonorm"], g["ref_router_w_nonorm"] = ref.router(rx, rw, 4, False)

    ew = rn(rng, 10, 8)
    eids = np.array([3, -1, 10, 0, 9], np.int32)
    g["embed_w"], g["embed_ids"], g["ref_embed"] = ew, eids, ref.embedding(ew, eids)

    # KVCachePool LIFO order and RadixCache matches (tests/unit/test_scheduler.cpp:9-39 cases)
    L = ref.lib
    pool = L.ref_pool_create(100, 1)
    allocs = [L.ref_pool_allocate(pool) for _ in range(5)]
    L.ref_pool_free(pool, allocs[1]); L.ref_pool_free(pool, allocs[3])
    allocs += [L.ref_pool_allocate(pool) for _ in range(3)]
    g["ref_pool_allocs"] = np.array(allocs, np.int32)
    g["ref_pool_free_after"] = np.array([L.ref_pool_num_free(pool)], np.int32)
    rad = L.ref_radix_create(pool)
    seq1 = np.array([1, 2, 3, 4, 5], np.int32)
    L.ref_radix_insert(rad, seq1, 5, np.array([10, 11, 12, 13, 14], np.int32), 5)
    import ctypes as C
    for name, seq in (("full", seq1), ("partial", np.array([1, 2, 3, 9, 10], np.int32)),
                      ("miss", np.array([7, 8], np.int32))):
        pages = np.zeros(16, np.int32)
        npg = C.c_int(0)
        matched = L.ref_radix_match(rad, seq, seq.size, pages, 16, C.byref(npg))
        g[f"ref_radix_{name}_matched"] = np.array([matched], np.int32)
        g[f"ref_radix_{name}_pages"] = pages[: npg.value].copy()
    L.ref_radix_destroy(rad); L.ref_pool_destroy(pool)

    # whole model, one token (dense and MoE, multi-head)
    for kind, extra in (("dense", {}), ("moe", {"num_experts": 4, "top_k": 2, "moe_inter": 32})):
        cfg = dict(num_layers=2, hidden=64, num_q_heads=4, num_kv_heads=4, head_dim=16, inter=128,
                   vocab=1000, eps=1e-6, rope_base=1e6, max_position=64, norm_topk=True, **extra)
        order, _ = tiny_model_weights(np.random.default_rng(7 if kind == "dense" else 8), cfg)
        ids, pos = np.array([417], np.int32), np.array([5], np.int32)
        g[f"ref_model_{kind}_logits"] = ref.model_forward(cfg, order, ids, pos)

    # restatement regression pins (GQA, paged, ragged): decode + extend over one pool
    hq, hkv, D, P = 8, 2, 128, 16
    seq_lens = np.array([1, 17, 40], np.int32)
    qlens = np.array([1, 1, 5], np.int32)
    q_indptr = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    pages_per = (seq_lens + P - 1) // P
    perm = np.random.default_rng(3).permutation(16).astype(np.int32)
    pt = np.zeros((3, 4), np.int32)
    off = 0
    for r in range(3):
        pt[r, : pages_per[r]] = perm[off: off + pages_per[r]]
        off += pages_per[r]
    kp, vp = rn(rng, 16 * P, hkv * D), rn(rng, 16 * P, hkv * D)
    qq = rn(rng, int(q_indptr[-1]), hq * D)
    g.update(paged_q=qq, paged_k=kp, paged_v=vp, paged_pt=pt, paged_seq=seq_lens,
             paged_indptr=q_indptr)
    g["oracle_paged"] = orc.paged_attention(qq, kp, vp, pt, seq_lens, q_indptr, hq, hkv, D, P)

    out = os.path.join(HERE, "golden_ops.npz")
    np.savez_compressed(out, **g)
    print("wrote", out, os.path.getsize(out), "bytes,", len(g), "arrays")


if __name__ == "__main__":
    main()
