/*
 * msgl_oracle.c -- CPU restatement of the mini-sglang-cpp per-layer Qwen3 forward path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker). Never linked into or called by the product library.
 * Each function cites the reference file:line it follows; see msgl_oracle.h for the contract.
 * Build: oracle/Makefile -> oracle/liboracle.so (plain C11, -O3, no fast-math, so the fp32
 * arithmetic keeps the reference's operation order and rounding).
 */
#include "msgl_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* layer.cpp:15-42 */
void oracle_embedding(const float* w, int64_t num_rows, int64_t hidden, const int32_t* ids,
                      int64_t num_ids, float* out) {
    for (int64_t i = 0; i < num_ids; ++i) {
        int32_t id = ids[i];
        if (id >= 0 && id < num_rows) {
            memcpy(out + i * hidden, w + (int64_t)id * hidden, (size_t)hidden * sizeof(float));
        } else {
            memset(out + i * hidden, 0, (size_t)hidden * sizeof(float));
        }
    }
}

/* layer.cpp:57-69 (per-row body shared by forward and the aliasing first fused call) */
static void rmsnorm_row(const float* in, const float* w, int64_t hidden, float eps, float* out) {
    float sum_sq = 0.0f;
    for (int64_t j = 0; j < hidden; ++j) sum_sq += in[j] * in[j];
    float inv_rms = 1.0f / sqrtf(sum_sq / (float)hidden + eps);
    for (int64_t j = 0; j < hidden; ++j) out[j] = in[j] * inv_rms * w[j];
}

/* layer.cpp:48-77 */
void oracle_rmsnorm(const float* x, const float* w, int64_t num_tokens, int64_t hidden, float eps,
                    float* out) {
#pragma omp parallel for schedule(static) if (num_tokens * hidden > (1 << 16))
    for (int64_t i = 0; i < num_tokens; ++i) rmsnorm_row(x + i * hidden, w, hidden, eps, out + i * hidden);
}

/* layer.cpp:79-112 */
void oracle_add_rmsnorm(float* x, float* residual, const float* w, int64_t num_tokens,
                        int64_t hidden, float eps, int first) {
    if (first) {
        /* residual = x; x = forward(x)  (layer.cpp:80-84) */
        memcpy(residual, x, (size_t)(num_tokens * hidden) * sizeof(float));
        for (int64_t i = 0; i < num_tokens; ++i)
            rmsnorm_row(residual + i * hidden, w, hidden, eps, x + i * hidden);
        return;
    }
    for (int64_t i = 0; i < num_tokens; ++i) {
        float* tx = x + i * hidden;
        float* tr = residual + i * hidden;
        float sum_sq = 0.0f;
        for (int64_t j = 0; j < hidden; ++j) {
            tr[j] += tx[j];
            sum_sq += tr[j] * tr[j];
        }
        float inv_rms = 1.0f / sqrtf(sum_sq / (float)hidden + eps);
        for (int64_t j = 0; j < hidden; ++j) tx[j] = tr[j] * inv_rms * w[j];
    }
}

/* layer.cpp:132-140. Each output keeps the reference's sequential accumulation over `in`
 * (so results are bit-identical to Linear::forward); eight outputs are carried side by side
 * only to give the CPU independent dependency chains. */
void oracle_linear(const float* x, const float* w, const float* bias, int64_t num_tokens,
                   int64_t in_features, int64_t out_features, float* out) {
    const int64_t OB = 8;
    int64_t nob = (out_features + OB - 1) / OB;
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
    for (int64_t i = 0; i < num_tokens; ++i) {
        for (int64_t ob = 0; ob < nob; ++ob) {
            const float* xr = x + i * in_features;
            int64_t o0 = ob * OB;
            int64_t cnt = out_features - o0 < OB ? out_features - o0 : OB;
            float acc[8];
            const float* wr[8];
            for (int u = 0; u < OB; ++u) {
                int64_t o = o0 + (u < cnt ? u : 0);
                acc[u] = bias ? bias[o] : 0.0f;
                wr[u] = w + o * in_features;
            }
            for (int64_t k = 0; k < in_features; ++k) {
                float xv = xr[k];
                acc[0] += xv * wr[0][k];
                acc[1] += xv * wr[1][k];
                acc[2] += xv * wr[2][k];
                acc[3] += xv * wr[3][k];
                acc[4] += xv * wr[4][k];
                acc[5] += xv * wr[5][k];
                acc[6] += xv * wr[6][k];
                acc[7] += xv * wr[7][k];
            }
            for (int u = 0; u < cnt; ++u) out[i * out_features + o0 + u] = acc[u];
        }
    }
}

/* layer.cpp:155-158 */
void oracle_swiglu(const float* gate, const float* up, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) {
        float silu_g = gate[i] / (1.0f + expf(-gate[i]));
        out[i] = silu_g * up[i];
    }
}

/* layer.cpp:168-175 */
void oracle_rope_table(int head_dim, int max_position, float base, float* table) {
    for (int p = 0; p < max_position; ++p) {
        for (int i = 0; i < head_dim / 2; ++i) {
            float freq = 1.0f / powf(base, (2.0f * (float)i) / (float)head_dim);
            float val = (float)p * freq;
            table[(int64_t)p * head_dim + i] = cosf(val);
            table[(int64_t)p * head_dim + head_dim / 2 + i] = sinf(val);
        }
    }
}

/* layer.cpp:186-198, one (token, head) vector per iteration with the token's own position */
void oracle_rope(float* x, const int32_t* positions, int64_t num_tokens, int num_heads,
                 int head_dim, const float* table) {
    int half = head_dim / 2;
    for (int64_t t = 0; t < num_tokens; ++t) {
        const float* cs = table + (int64_t)positions[t] * head_dim;
        for (int h = 0; h < num_heads; ++h) {
            float* q = x + (t * num_heads + h) * head_dim;
            for (int d = 0; d < half; ++d) {
                float c = cs[d], s = cs[half + d];
                float q0 = q[d], q1 = q[half + d];
                q[d] = q0 * c - q1 * s;
                q[half + d] = q0 * s + q1 * c;
            }
        }
    }
}

/* kernels/cuda/radix.cu:19-22 */
void oracle_store_kv_page(const float* k, const float* v, float* k_pool, float* v_pool,
                          const int32_t* page_table, int page_size, int num_heads, int head_dim,
                          int64_t num_tokens) {
    int64_t stride = (int64_t)num_heads * head_dim;
    for (int64_t t = 0; t < num_tokens; ++t) {
        int64_t slot = (int64_t)page_table[t / page_size] * page_size + t % page_size;
        memcpy(k_pool + slot * stride, k + t * stride, (size_t)stride * sizeof(float));
        memcpy(v_pool + slot * stride, v + t * stride, (size_t)stride * sizeof(float));
    }
}

void oracle_store_kv_slots(const float* k, const float* v, float* k_pool, float* v_pool,
                           const int32_t* slot_mapping, int64_t num_tokens, int64_t row_elems) {
    for (int64_t t = 0; t < num_tokens; ++t) {
        int64_t slot = slot_mapping[t];
        memcpy(k_pool + slot * row_elems, k + t * row_elems, (size_t)row_elems * sizeof(float));
        memcpy(v_pool + slot * row_elems, v + t * row_elems, (size_t)row_elems * sizeof(float));
    }
}

/* layer.cpp:226-257 per request over the paged pool (see header). Requests are independent and
 * run in parallel; the value sum keeps the reference's order (j ascending for every output d),
 * with the j loop outside so that each V row is read once, contiguously. */
void oracle_paged_attention(const float* q, const float* k_pool, const float* v_pool,
                            const int32_t* page_table, int max_pages, const int32_t* seq_lens,
                            const int32_t* q_indptr, int num_reqs, int num_q_heads,
                            int num_kv_heads, int head_dim, int page_size, float scale,
                            float* out) {
    int group = num_q_heads / num_kv_heads;
    int64_t kv_stride = (int64_t)num_kv_heads * head_dim;
#pragma omp parallel for schedule(dynamic, 1) if (num_reqs > 1)
    for (int r = 0; r < num_reqs; ++r) {
        int ctx = seq_lens[r];
        int n = q_indptr[r + 1] - q_indptr[r];
        const int32_t* pt = page_table + (int64_t)r * max_pages;
        float* scores = (float*)malloc(sizeof(float) * (size_t)(ctx > 0 ? ctx : 1));
        int64_t* slots = (int64_t*)malloc(sizeof(int64_t) * (size_t)(ctx > 0 ? ctx : 1));
        float* val = (float*)malloc(sizeof(float) * (size_t)head_dim);
        for (int j = 0; j < ctx; ++j)
            slots[j] = (int64_t)pt[j / page_size] * page_size + j % page_size;
        for (int i = 0; i < n; ++i) {
            int64_t t = q_indptr[r] + i;
            int qpos = ctx - n + i;
            for (int h = 0; h < num_q_heads; ++h) {
                int kvh = h / group;
                const float* qv = q + (t * num_q_heads + h) * head_dim;
                float max_score = -1e9f;
                for (int j = 0; j <= qpos; ++j) {
                    const float* kv = k_pool + slots[j] * kv_stride + (int64_t)kvh * head_dim;
                    float dot = 0.0f;
                    for (int d = 0; d < head_dim; ++d) dot += qv[d] * kv[d];
                    scores[j] = dot * scale;
                    if (scores[j] > max_score) max_score = scores[j];
                }
                float sum_exp = 0.0f;
                for (int j = 0; j <= qpos; ++j) {
                    scores[j] = expf(scores[j] - max_score);
                    sum_exp += scores[j];
                }
                for (int d = 0; d < head_dim; ++d) val[d] = 0.0f;
                for (int j = 0; j <= qpos; ++j) {
                    float prob = scores[j] / sum_exp;
                    const float* vv = v_pool + slots[j] * kv_stride + (int64_t)kvh * head_dim;
                    for (int d = 0; d < head_dim; ++d) val[d] += prob * vv[d];
                }
                float* o = out + (t * num_q_heads + h) * head_dim;
                for (int d = 0; d < head_dim; ++d) o[d] = val[d];
            }
        }
        free(val);
        free(scores);
        free(slots);
    }
}

/* std::greater<std::pair<float,int>>: larger logit first; equal logits -> larger index first */
static int pair_greater(float va, int ia, float vb, int ib) {
    return va > vb || (!(vb > va) && ia > ib);
}

/* layer.cpp:283-305 on given logits */
void oracle_router_topk(const float* logits, int64_t num_tokens, int num_experts, int top_k,
                        int norm_topk, int32_t* ids, float* weights) {
    float* val = (float*)malloc(sizeof(float) * (size_t)num_experts);
    int* idx = (int*)malloc(sizeof(int) * (size_t)num_experts);
    for (int64_t t = 0; t < num_tokens; ++t) {
        for (int e = 0; e < num_experts; ++e) {
            val[e] = logits[t * num_experts + e];
            idx[e] = e;
        }
        /* selection: after step k, positions [0,k] hold the k+1 greatest in order */
        for (int k = 0; k < top_k; ++k) {
            int best = k;
            for (int e = k + 1; e < num_experts; ++e)
                if (pair_greater(val[e], idx[e], val[best], idx[best])) best = e;
            float tv = val[k]; val[k] = val[best]; val[best] = tv;
            int ti = idx[k]; idx[k] = idx[best]; idx[best] = ti;
        }
        float sum_exp = 0.0f;
        for (int k = 0; k < top_k; ++k) {
            ids[t * top_k + k] = idx[k];
            float prob = expf(val[k]);
            weights[t * top_k + k] = prob;
            sum_exp += prob;
        }
        if (norm_topk)
            for (int k = 0; k < top_k; ++k) weights[t * top_k + k] /= sum_exp;
    }
    free(val);
    free(idx);
}

/* qwen3_moe.cpp:74-108 */
void oracle_moe_experts(const float* x, const int32_t* ids, const float* weights,
                        int64_t num_tokens, int top_k, int hidden, int inter,
                        const float* const* gate_up_w, const float* const* down_w, float* out) {
    float* gu = (float*)malloc(sizeof(float) * 2 * (size_t)inter);
    float* act = (float*)malloc(sizeof(float) * (size_t)inter);
    float* y = (float*)malloc(sizeof(float) * (size_t)hidden);
    memset(out, 0, sizeof(float) * (size_t)(num_tokens * hidden));
    for (int64_t t = 0; t < num_tokens; ++t) {
        for (int k = 0; k < top_k; ++k) {
            int e = ids[t * top_k + k];
            float wgt = weights[t * top_k + k];
            oracle_linear(x + t * hidden, gate_up_w[e], NULL, 1, hidden, 2 * (int64_t)inter, gu);
            oracle_swiglu(gu, gu + inter, inter, act);
            oracle_linear(act, down_w[e], NULL, 1, inter, hidden, y);
            float* dst = out + t * hidden;
            for (int h = 0; h < hidden; ++h) dst[h] += wgt * y[h];
        }
    }
    free(gu);
    free(act);
    free(y);
}

/* scheduler.cpp:117-124 */
void oracle_argmax(const float* logits, int64_t num_rows, int64_t vocab, int32_t* out) {
    for (int64_t i = 0; i < num_rows; ++i) {
        const float* r = logits + i * vocab;
        int32_t best = 0;
        float max_val = r[0];
        for (int64_t v = 1; v < vocab; ++v) {
            if (r[v] > max_val) {
                max_val = r[v];
                best = (int32_t)v;
            }
        }
        out[i] = best;
    }
}

/* qwen3.cpp:16-83 (dense) and qwen3_moe.cpp:23-112 (MoE), with QK-norm between the split
 * (qwen3.cpp:45) and RoPE (qwen3.cpp:48), KV stored to the pool before attention. */
void oracle_decoder_layer(const oracle_config_t* cfg, const oracle_layer_t* L,
                          const oracle_batch_t* b, const float* rope_table, float* x,
                          float* residual, int first) {
    int64_t T = b->num_tokens;
    int H = cfg->hidden, D = cfg->head_dim, Hq = cfg->num_q_heads, Hkv = cfg->num_kv_heads;
    int64_t qd = (int64_t)Hq * D, kd = (int64_t)Hkv * D, tot = qd + 2 * kd;

    oracle_add_rmsnorm(x, residual, L->input_ln, T, H, cfg->eps, first);

    float* qkv = (float*)malloc(sizeof(float) * (size_t)(T * tot));
    oracle_linear(x, L->w_qkv, NULL, T, H, tot, qkv);
    float* q = (float*)malloc(sizeof(float) * (size_t)(T * qd));
    float* k = (float*)malloc(sizeof(float) * (size_t)(T * kd));
    float* v = (float*)malloc(sizeof(float) * (size_t)(T * kd));
    for (int64_t i = 0; i < T; ++i) {  /* qwen3.cpp:39-44 */
        memcpy(q + i * qd, qkv + i * tot, sizeof(float) * (size_t)qd);
        memcpy(k + i * kd, qkv + i * tot + qd, sizeof(float) * (size_t)kd);
        memcpy(v + i * kd, qkv + i * tot + qd + kd, sizeof(float) * (size_t)kd);
    }
    free(qkv);

    /* QK-norm: per-head RMSNorm(D, eps) over [T*heads, D] (layer.cpp:48-77 with size D) */
    float* tmp = (float*)malloc(sizeof(float) * (size_t)(T * qd));
    oracle_rmsnorm(q, L->q_norm, T * Hq, D, cfg->eps, tmp);
    memcpy(q, tmp, sizeof(float) * (size_t)(T * qd));
    oracle_rmsnorm(k, L->k_norm, T * Hkv, D, cfg->eps, tmp);
    memcpy(k, tmp, sizeof(float) * (size_t)(T * kd));
    free(tmp);

    oracle_rope(q, b->positions, T, Hq, D, rope_table);
    oracle_rope(k, b->positions, T, Hkv, D, rope_table);
    oracle_store_kv_slots(k, v, L->k_pool, L->v_pool, b->slot_mapping, T, kd);

    float* attn = (float*)malloc(sizeof(float) * (size_t)(T * qd));
    oracle_paged_attention(q, L->k_pool, L->v_pool, b->page_table, b->max_pages, b->seq_lens,
                           b->q_indptr, b->num_reqs, Hq, Hkv, D, cfg->page_size,
                           1.0f / sqrtf((float)D), attn);
    free(q);
    free(k);
    free(v);

    float* attn_out = (float*)malloc(sizeof(float) * (size_t)(T * H));
    oracle_linear(attn, L->w_o, NULL, T, qd, H, attn_out);
    free(attn);

    oracle_add_rmsnorm(attn_out, residual, L->post_ln, T, H, cfg->eps, 0);

    if (cfg->num_experts > 0) {
        float* logits = (float*)malloc(sizeof(float) * (size_t)(T * cfg->num_experts));
        oracle_linear(attn_out, L->w_router, NULL, T, H, cfg->num_experts, logits);
        int32_t* ids = (int32_t*)malloc(sizeof(int32_t) * (size_t)(T * cfg->top_k));
        float* wts = (float*)malloc(sizeof(float) * (size_t)(T * cfg->top_k));
        oracle_router_topk(logits, T, cfg->num_experts, cfg->top_k, cfg->norm_topk, ids, wts);
        oracle_moe_experts(attn_out, ids, wts, T, cfg->top_k, H, cfg->moe_inter,
                           L->expert_gate_up, L->expert_down, x);
        free(logits);
        free(ids);
        free(wts);
    } else {
        int64_t I = cfg->inter;
        float* gu = (float*)malloc(sizeof(float) * (size_t)(T * 2 * I));
        oracle_linear(attn_out, L->w_gate_up, NULL, T, H, 2 * I, gu);
        float* act = (float*)malloc(sizeof(float) * (size_t)(T * I));
        for (int64_t i = 0; i < T; ++i)  /* qwen3.cpp:71-76 split, then SwiGLU */
            oracle_swiglu(gu + i * 2 * I, gu + i * 2 * I + I, I, act + i * I);
        free(gu);
        oracle_linear(act, L->w_down, NULL, T, I, H, x);
        free(act);
    }
    free(attn_out);
}
