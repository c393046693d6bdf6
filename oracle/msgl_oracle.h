/*
 * msgl_oracle.h -- CPU restatement of the mini-sglang-cpp per-layer Qwen3 forward path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker: tests, the smoke check and the
 * CPU-baseline leg of bench.py may call it; the product path (libmsgl) never links or calls it.
 *
 * Every routine is plain fp32 C and follows the cited reference file:line (paths relative to
 * the mini-sglang-cpp project root). Where the reference is defective on the path (GQA indexing,
 * no paging, Q-only RoPE, no QK-norm) the restatement keeps the reference arithmetic and applies
 * the minimal fix, named at each function.
 *
 * Parity is pinned by tests/golden/: fixtures produced by the reference's own compiled sources
 * (oracle/_ref, built by oracle/Makefile) for every op the reference implements correctly.
 */
#ifndef MSGL_ORACLE_H
#define MSGL_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Embedding::forward, src/layer/layer.cpp:15-42. Out-of-range ids give a zero row. */
void oracle_embedding(const float* w, int64_t num_rows, int64_t hidden, const int32_t* ids,
                      int64_t num_ids, float* out);

/* RMSNorm::forward, src/layer/layer.cpp:48-77: y = x * (1/sqrt(sum(x^2)/H + eps)) * w. */
void oracle_rmsnorm(const float* x, const float* w, int64_t num_tokens, int64_t hidden, float eps,
                    float* out);

/* RMSNorm::forward_fused_add, src/layer/layer.cpp:79-112: res += x; x = rmsnorm(res).
 * first != 0 models the aliasing first call (layer.cpp:80-84): res = x; x = rmsnorm(x). */
void oracle_add_rmsnorm(float* x, float* residual, const float* w, int64_t num_tokens,
                        int64_t hidden, float eps, int first);

/* Linear::forward, src/layer/layer.cpp:122-143: y[i,o] = sum_in x[i,in] * W[o,in] (+ b[o]).
 * W is [out, in] row-major. Loop order as the reference; split across OpenMP threads by row. */
void oracle_linear(const float* x, const float* w, const float* bias, int64_t num_tokens,
                   int64_t in_features, int64_t out_features, float* out);

/* SwiGLU::forward, src/layer/layer.cpp:145-161: out = g / (1 + exp(-g)) * u. */
void oracle_swiglu(const float* gate, const float* up, int64_t n, float* out);

/* RotaryEmbedding ctor, src/layer/layer.cpp:163-176: table [max_pos, D]; cos in the first half,
 * sin in the second half, freq_i = 1 / powf(base, 2i/D). */
void oracle_rope_table(int head_dim, int max_position, float base, float* table);

/* RotaryEmbedding::forward rotate-half math (src/layer/layer.cpp:191-198) applied to every
 * (token, head) of x [T, heads, D] with that token's own position (fixes D4: the reference
 * indexes positions by token*heads+head and rotates only q). */
void oracle_rope(float* x, const int32_t* positions, int64_t num_tokens, int num_heads,
                 int head_dim, const float* table);

/* Slot formula of store_kv_page_kernel, kernels/cuda/radix.cu:19-22:
 * slot(t) = page_table[t / P] * P + t % P, pool[slot, h*D + d]. k/v are [T, heads*D]. */
void oracle_store_kv_page(const float* k, const float* v, float* k_pool, float* v_pool,
                          const int32_t* page_table, int page_size, int num_heads, int head_dim,
                          int64_t num_tokens);

/* Store k/v rows at explicit pool slots (slot_mapping[t]); same pool layout as above. */
void oracle_store_kv_slots(const float* k, const float* v, float* k_pool, float* v_pool,
                           const int32_t* slot_mapping, int64_t num_tokens, int64_t row_elems);

/* Attention::forward math, src/layer/layer.cpp:226-257 (scale 1/sqrt(D), max init -1e9,
 * exp(s - max), p = e / sum, fp32), restated per request over the paged pool:
 *  - request r owns query rows [q_indptr[r], q_indptr[r+1]) and a KV context of seq_lens[r]
 *    tokens (its new tokens already stored), read through page_table[r*max_pages + j/P];
 *  - query row i of a request with n rows sits at position seq_len - n + i (causal: j <= it);
 *  - GQA: query head h reads kv head h / (Hq / Hkv) (fixes D1, D2). */
void oracle_paged_attention(const float* q, const float* k_pool, const float* v_pool,
                            const int32_t* page_table, int max_pages, const int32_t* seq_lens,
                            const int32_t* q_indptr, int num_reqs, int num_q_heads,
                            int num_kv_heads, int head_dim, int page_size, float scale, float* out);

/* MoERouter::route top-k + weights, src/layer/layer.cpp:283-305, on precomputed fp32 logits
 * [T, E]: descending by logit, ties to the larger expert index (std::greater on
 * pair<float,int>), w = exp(logit), divided by the top-k sum when norm_topk. */
void oracle_router_topk(const float* logits, int64_t num_tokens, int num_experts, int top_k,
                        int norm_topk, int32_t* ids, float* weights);

/* MoE expert loop, src/model/qwen3_moe.cpp:68-109: out[t] = sum_k w_k * down_e(silu(g) * u)
 * with gate_up_e [2I, H] (gate rows first) and down_e [H, I]; weights indexed by expert. */
void oracle_moe_experts(const float* x, const int32_t* ids, const float* weights,
                        int64_t num_tokens, int top_k, int hidden, int inter,
                        const float* const* gate_up_w, const float* const* down_w, float* out);

/* Greedy sampling, src/scheduler/scheduler.cpp:117-124: strict '>' scan, ties to lowest id. */
void oracle_argmax(const float* logits, int64_t num_rows, int64_t vocab, int32_t* out);

/* ---- Whole decoder layer / model (src/model/qwen3.cpp:16-83, 168-180) ---- */
typedef struct {
    const float* input_ln;   /* [H] */
    const float* w_qkv;      /* [(Hq+2Hkv)D, H], rows q | k | v */
    const float* q_norm;     /* [D] */
    const float* k_norm;     /* [D] */
    const float* w_o;        /* [H, Hq D] */
    const float* post_ln;    /* [H] */
    const float* w_gate_up;  /* [2I, H], rows gate | up  (dense layers) */
    const float* w_down;     /* [H, I]                   (dense layers) */
    const float* w_router;   /* [E, H]                   (MoE layers)   */
    const float* const* expert_gate_up; /* E x [2 Imoe, H] */
    const float* const* expert_down;    /* E x [H, Imoe]   */
    float* k_pool;           /* [slots, Hkv D] */
    float* v_pool;
} oracle_layer_t;

typedef struct {
    int hidden, num_q_heads, num_kv_heads, head_dim, inter;
    int num_experts, top_k, moe_inter, norm_topk;
    float eps;
    int page_size;
} oracle_config_t;

/* Per-step batch metadata (host): T tokens over B requests. */
typedef struct {
    int64_t num_tokens;
    int num_reqs;
    const int32_t* positions;    /* [T] */
    const int32_t* slot_mapping; /* [T] */
    const int32_t* page_table;   /* [B, max_pages] */
    int max_pages;
    const int32_t* seq_lens;     /* [B] context incl. this step's tokens */
    const int32_t* q_indptr;     /* [B+1] */
} oracle_batch_t;

/* One Qwen3DecoderLayer::forward (qwen3.cpp:16-83 / qwen3_moe.cpp:23-112) with QK-norm.
 * x: [T,H] in/out (layer input is the previous layer's mlp_out), residual: [T,H] in/out.
 * first != 0 for layer 0 (residual aliasing). rope_table: [max_pos, D]. */
void oracle_decoder_layer(const oracle_config_t* cfg, const oracle_layer_t* layer,
                          const oracle_batch_t* batch, const float* rope_table, float* x,
                          float* residual, int first);

#ifdef __cplusplus
}
#endif
#endif /* MSGL_ORACLE_H */
