// layers.h -- device-side layer classes of the executor.
//
// Same class and method names as the reference's layer ops (include/minisgl/layer/layer.h:11-96),
// with the bodies dispatching to the libmsgl C ABI. Differences, all deliberate:
//  * the caller owns every buffer (the reference allocates a fresh Tensor per call,
//    src/layer/layer.cpp:17,50,124,147,218,273);
//  * activations are bf16, accumulation fp32, the residual stream fp32;
//  * Attention reads the paged per-layer KV pool (the reference attends over the flattened batch,
//    layer.cpp:226-257) and RotaryEmbedding rotates q and k (layer.cpp:186-199 rotates q only);
//  * gate_up and SwiGLU are one GEMM (GateUpSwiGLU) and QK-norm + RoPE + KV store one kernel.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "msgl_engine.h"

namespace msgl {
namespace engine {

using bf16_t = uint16_t;  // bf16 storage

struct Fail : std::runtime_error {
    int code;
    Fail(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

inline void ck(int rc, const char* what) {
    if (rc != MSGL_OK) throw Fail(rc, std::string(what) + ": " + msgl_last_error());
}
inline void ckc(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw Fail(MSGL_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Device buffer owned by the executor.
struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        if (this != &o) {
            reset();
            p = o.p; bytes = o.bytes;
            o.p = nullptr; o.bytes = 0;
        }
        return *this;
    }
    ~DevBuf() { reset(); }
    void alloc(size_t n) {
        reset();
        if (n == 0) return;
        ckc(cudaMalloc(&p, n), "cudaMalloc");
        bytes = n;
    }
    void reset() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    template <typename T>
    T* as() const { return static_cast<T*>(p); }
};

// Workspace shared by the GEMMs / attention of one executor (they run in stream order).
struct Scratch {
    void* gemm_ws = nullptr;
    size_t gemm_ws_bytes = 0;
    void* attn_ws = nullptr;
    size_t attn_ws_bytes = 0;
};

class RMSNorm {  // layer.h:23-34
  public:
    RMSNorm() = default;
    RMSNorm(int size, float eps) : size_(size), eps_(eps) {}
    void forward_fused_add(bf16_t* x, float* residual, int num_tokens, bool first,
                           cudaStream_t s) const {
        ck(msgl_add_rmsnorm(x, residual, weight.p, num_tokens, size_, eps_, first ? 1 : 0, s),
           "RMSNorm::forward_fused_add");
    }
    // the same with the added input the sum of fp32 split-K partials [nparts][T][size]
    void forward_fused_add_partials(const float* parts, int nparts, bf16_t* x, float* residual,
                                    int num_tokens, cudaStream_t s) const {
        ck(msgl_add_partials_rmsnorm(parts, nparts, x, residual, weight.p, num_tokens, size_, eps_, s),
           "RMSNorm::forward_fused_add(partials)");
    }
    DevBuf weight;  // bf16 [size]
    int size() const { return size_; }
    float eps() const { return eps_; }

  private:
    int size_ = 0;
    float eps_ = 1e-6f;
};

class Linear {  // layer.h:36-48; y = x W^T, W [out, in]
  public:
    Linear() = default;
    Linear(int in_features, int out_features) : in_(in_features), out_(out_features) {}
    void forward(const bf16_t* x, bf16_t* y, int num_tokens, const Scratch& ws,
                 cudaStream_t s) const {
        ck(msgl_gemm_bf16(x, weight.p, y, num_tokens, out_, in_, MSGL_BF16, ws.gemm_ws,
                          ws.gemm_ws_bytes, s),
           "Linear::forward");
    }
    // Decode-sized batches whose next kernel adds the K split: fp32 partials [S][T][out];
    // returns S (0: not available for this size, use forward).
    int partial_splits(int num_tokens) const { return msgl_gemm_partials_splits(num_tokens, out_, in_); }
    // partials apply at this step size (up to 256 tokens: two 128-token tiles)
    bool partials_fit(int num_tokens) const { return num_tokens <= 256; }
    int forward_partials(const bf16_t* x, float* parts, int num_tokens, cudaStream_t s) const {
        const int S = partial_splits(num_tokens);
        ck(msgl_gemm_bf16_partials(x, weight.p, parts, num_tokens, out_, in_, S, s),
           "Linear::forward(partials)");
        return S;
    }
    size_t workspace(int max_tokens) const { return msgl_gemm_workspace_size(max_tokens, out_, in_); }
    DevBuf weight;  // bf16 [out, in]
    int in_features() const { return in_; }
    int out_features() const { return out_; }

  private:
    int in_ = 0, out_ = 0;
};

// gate_up_proj + split + SwiGLU (qwen3.cpp:60-79) as one GEMM on the packed gate/up weight.
class GateUpSwiGLU {
  public:
    GateUpSwiGLU() = default;
    GateUpSwiGLU(int in_features, int inter) : in_(in_features), inter_(inter) {}
    void forward(const bf16_t* x, bf16_t* act, int num_tokens, const Scratch& ws,
                 cudaStream_t s) const {
        ck(msgl_gemm_gate_up_silu(x, weight_packed.p, act, num_tokens, inter_, in_, ws.gemm_ws,
                                  ws.gemm_ws_bytes, s),
           "GateUpSwiGLU::forward");
    }
    size_t workspace(int max_tokens) const {
        return msgl_gemm_workspace_size(max_tokens, 2 * inter_, in_);
    }
    DevBuf weight_packed;  // bf16 [2 * inter, in], rows packed by msgl_pack_gate_up
    int inter() const { return inter_; }
    int in_features() const { return in_; }

  private:
    int in_ = 0, inter_ = 0;
};

// RotaryEmbedding (layer.h:57-68): one fp32 [max_position, D] table for all layers (the
// reference builds one per layer, D18), computed on the host with the reference formula
// (layer.cpp:168-175) and uploaded.
class RotaryEmbedding {
  public:
    void init(int head_dim, int max_position, float base, cudaStream_t s);
    DevBuf cos_sin_cache;
    int head_dim = 128, max_position = 0;
};

// QK-norm + RoPE + KV-page store, then paged attention (replaces Attention, layer.h:70-81).
class Attention {
  public:
    Attention() = default;
    Attention(int hq, int hkv, int head_dim, float eps)
        : hq_(hq), hkv_(hkv), head_dim_(head_dim), eps_(eps) {}
    // qkv [T, (hq + 2 hkv) D] -> q [T, hq, D] (normed, rotated); k / v stored in the pools.
    void prepare(const bf16_t* qkv, bf16_t* q, void* k_pool, void* v_pool, int64_t num_slots,
                 const int* positions, const int* slot_mapping, const RotaryEmbedding& rope,
                 const void* q_norm_w, const void* k_norm_w, int num_tokens, cudaStream_t s) const {
        ck(msgl_qknorm_rope_store_kv(qkv, q, k_pool, v_pool, num_slots, positions, slot_mapping,
                                     rope.cos_sin_cache.as<float>(), q_norm_w, k_norm_w,
                                     num_tokens, hq_, hkv_, head_dim_, eps_, s),
           "Attention::prepare");
    }
    // the same from the QKV projection's fp32 split-K partials [nparts][T][(hq + 2 hkv) D]
    void prepare_partials(const float* parts, int nparts, bf16_t* q, void* k_pool, void* v_pool,
                          int64_t num_slots, const int* positions, const int* slot_mapping,
                          const RotaryEmbedding& rope, const void* q_norm_w, const void* k_norm_w,
                          int num_tokens, cudaStream_t s) const {
        ck(msgl_qknorm_rope_store_kv_partials(parts, nparts, q, k_pool, v_pool, num_slots,
                                              positions, slot_mapping,
                                              rope.cos_sin_cache.as<float>(), q_norm_w, k_norm_w,
                                              num_tokens, hq_, hkv_, head_dim_, eps_, s),
           "Attention::prepare(partials)");
    }
    void forward(const bf16_t* q, const void* k_pool, const void* v_pool, int64_t num_slots,
                 const msgl_batch& b, bf16_t* out, const Scratch& ws, cudaStream_t s) const {
        const float scale = 1.0f / sqrtf(static_cast<float>(head_dim_));  // layer.cpp:212
        // decode over a prefix that every request shares (radix-cache hit): the cascade kernel
        // attends the shared pages once per kv head for the whole batch -- when a CTA holds four
        // kv heads. With one or two (ranks of wide tensor parallelism) the plain kernel is faster
        // (128 x 2048 with a 1024-token prefix: 18.0 vs 21.9 us at one kv head, 30.0 vs 32.9 us
        // at two).
        const int sp = b.shared_prefix_pages;
        if (b.is_decode && b.num_reqs >= 2 && hkv_ % 4 == 0 && sp >= kMinCascadePages && sp <= b.max_pages &&
            sp * 16 <= b.max_seq_len &&
            msgl_paged_attention_cascade_workspace_size(b.num_reqs, b.max_seq_len, sp, hq_, hkv_,
                                                        head_dim_) <= ws.attn_ws_bytes)
            ck(msgl_paged_attention_decode_cascade(q, k_pool, v_pool, num_slots, b.page_table,
                                                   b.max_pages, b.seq_lens, b.num_reqs,
                                                   b.max_seq_len, sp, hq_, hkv_, head_dim_, 16,
                                                   scale, out, ws.attn_ws, ws.attn_ws_bytes, s),
               "Attention::forward(cascade decode)");
        else if (b.is_decode)
            ck(msgl_paged_attention_decode(q, k_pool, v_pool, num_slots, b.page_table, b.max_pages,
                                           b.seq_lens, b.num_reqs, b.max_seq_len, hq_, hkv_,
                                           head_dim_, 16, scale, out, ws.attn_ws, ws.attn_ws_bytes,
                                           s),
               "Attention::forward(decode)");
        else if (b.decode_tail > 0 && b.decode_tail < b.num_reqs && b.decode_tail < b.num_tokens &&
                 msgl_paged_attention_workspace_size(b.decode_tail, b.max_seq_len, hq_, hkv_,
                                                     head_dim_) <= ws.attn_ws_bytes) {
            // chunked prefill mixed with decodes: the prefill requests through extend, the decode
            // tail (one row each, the last rows of the step) through the split-KV decode kernel
            const int nd = b.decode_tail, np_ = b.num_reqs - nd, t0 = b.num_tokens - nd;
            const size_t row = static_cast<size_t>(hq_) * head_dim_;
            ck(msgl_paged_attention_extend(q, k_pool, v_pool, num_slots, b.page_table, b.max_pages,
                                           b.seq_lens, b.q_indptr, np_, b.max_q_len, hq_, hkv_,
                                           head_dim_, 16, scale, out, s),
               "Attention::forward(extend part)");
            ck(msgl_paged_attention_decode(q + t0 * row, k_pool, v_pool, num_slots,
                                           b.page_table + static_cast<size_t>(np_) * b.max_pages,
                                           b.max_pages, b.seq_lens + np_, nd, b.max_seq_len, hq_,
                                           hkv_, head_dim_, 16, scale, out + t0 * row, ws.attn_ws,
                                           ws.attn_ws_bytes, s),
               "Attention::forward(decode tail)");
        } else {
            ck(msgl_paged_attention_extend(q, k_pool, v_pool, num_slots, b.page_table, b.max_pages,
                                           b.seq_lens, b.q_indptr, b.num_reqs, b.max_q_len, hq_,
                                           hkv_, head_dim_, 16, scale, out, s),
               "Attention::forward(extend)");
        }
    }
    int hq() const { return hq_; }
    int hkv() const { return hkv_; }

    static constexpr int kMinCascadePages = 2;  // shorter shared prefixes: plain decode

  private:
    int hq_ = 0, hkv_ = 0, head_dim_ = 128;
    float eps_ = 1e-6f;
};

// MoERouter (layer.h:83-96) + the expert loop of Qwen3MoEDecoderLayer::forward
// (src/model/qwen3_moe.cpp:62-111): router logits GEMM (fp32 out) -> top-k -> stable
// permutation by expert -> gather -> grouped gate_up+SwiGLU -> grouped down -> weighted combine.
struct MoEScratch {
    float* logits = nullptr;      // [T, E], or the router's split-K partials [S, T, E]
    int* topk_ids = nullptr;      // [T, k]
    float* topk_w = nullptr;      // [T, k]
    int* offsets = nullptr;       // [E + 1]
    int* sorted_token = nullptr;  // [T k]
    int* pair_pos = nullptr;      // [T k]
    bf16_t* xs = nullptr;         // [T k, H]
    bf16_t* act = nullptr;        // [T k, inter]
    bf16_t* ys = nullptr;         // [T k, H]
    void* grouped_ws = nullptr;
    size_t grouped_ws_bytes = 0;
    size_t logits_floats = 0;     // capacity of `logits`
};

class MoEExperts {
  public:
    MoEExperts() = default;
    MoEExperts(int hidden, int num_experts, int top_k, int inter, bool norm_topk)
        : hidden_(hidden), E_(num_experts), k_(top_k), inter_(inter), norm_topk_(norm_topk) {}
    // x [T, H] (post-attention normed) -> out [T, H] (may alias x: x is consumed first).
    // With next_norm: residual += the expert output and out = next_norm(residual), the residual
    // add and RMSNorm that follow the layer (qwen3.cpp:19), in the combine kernel.
    void forward(const bf16_t* x, bf16_t* out, int T, const MoEScratch& ms, const Scratch& ws,
                 cudaStream_t s, const RMSNorm* next_norm = nullptr,
                 float* residual = nullptr) const {
        // router logits (layer.cpp:273-280): as split-K partials summed by the top-k kernel when
        // the step has <= 256 tokens and the scratch holds them, else one fp32 GEMM
        const int S = router_splits(T);
        if (S >= 2 && static_cast<size_t>(S) * T * E_ <= ms.logits_floats) {
            ck(msgl_gemm_bf16_partials(x, router.p, ms.logits, T, E_, hidden_, S, s),
               "MoERouter logits (partials)");
            ck(msgl_moe_route_topk_partials(ms.logits, S, T, E_, k_, norm_topk_ ? 1 : 0,
                                            ms.topk_ids, ms.topk_w, s),
               "MoERouter::route");
        } else {
            ck(msgl_gemm_bf16(x, router.p, ms.logits, T, E_, hidden_, MSGL_F32, ws.gemm_ws,
                              ws.gemm_ws_bytes, s), "MoERouter logits");
            ck(msgl_moe_route_topk(ms.logits, T, E_, k_, norm_topk_ ? 1 : 0, ms.topk_ids,
                                   ms.topk_w, s),
               "MoERouter::route");
        }
        ck(msgl_moe_permute(ms.topk_ids, T, k_, E_, ms.offsets, ms.sorted_token, ms.pair_pos, s),
           "moe permute");
        ck(msgl_launch_index_gather(x, ms.sorted_token, ms.xs, hidden_, T * k_, T, MSGL_BF16, s),
           "moe gather");
        ck(msgl_grouped_gemm_gate_up_silu(ms.xs, gate_up_packed.p, ms.act, ms.offsets, E_, inter_,
                                          hidden_, T * k_, ms.grouped_ws, ms.grouped_ws_bytes, s),
           "experts gate_up");
        // (same offsets, rows and experts as gate_up: its tile list is still in the workspace)
        ck(msgl_grouped_gemm_bf16_reuse_tiles(ms.act, down.p, ms.ys, ms.offsets, E_, hidden_,
                                              inter_, T * k_, ms.grouped_ws, ms.grouped_ws_bytes,
                                              s),
           "experts down");
        if (next_norm)
            ck(msgl_moe_combine_add_rmsnorm(ms.ys, ms.pair_pos, ms.topk_w, T, k_, hidden_, residual,
                                            next_norm->weight.p, next_norm->eps(), out, s),
               "moe combine + add + RMSNorm");
        else
            ck(msgl_moe_combine(ms.ys, ms.pair_pos, ms.topk_w, T, k_, hidden_, out, s), "moe combine");
    }
    DevBuf router;          // bf16 [E, H]
    DevBuf gate_up_packed;  // bf16 [E, 2 inter, H], each expert packed by msgl_pack_gate_up
    DevBuf down;            // bf16 [E, H, inter]
    // split-K partials of the router logits GEMM for a T-token step (0: one fp32 GEMM instead)
    int router_splits(int T) const { return msgl_gemm_partials_splits(T, E_, hidden_); }
    int num_experts() const { return E_; }
    int top_k() const { return k_; }
    int inter() const { return inter_; }

  private:
    int hidden_ = 0, E_ = 0, k_ = 0, inter_ = 0;
    bool norm_topk_ = true;
};

}  // namespace engine
}  // namespace msgl
