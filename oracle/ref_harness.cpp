// ref_harness.cpp -- extern "C" shims over the reference's own compiled sources.
//
// TEST INFRASTRUCTURE ONLY. Built by oracle/Makefile together with the reference sources
// (compiled where they lie, never copied) into oracle/_ref/libref_harness.so. The shims only
// move data in and out of reference `Tensor`s and call reference objects; all arithmetic is the
// reference's. Used to pin the C restatement (oracle/msgl_oracle.c) and as the timed CPU
// reference path of bench.py.
#include <cstring>
#include <memory>
#include <vector>

#include "minisgl/cache/kvcache.h"
#include "minisgl/layer/layer.h"
#include "minisgl/model/config.h"
#include "minisgl/model/qwen3.h"
#include "minisgl/model/qwen3_moe.h"

using namespace minisgl;

namespace {
std::shared_ptr<Tensor> make_f32(std::vector<int64_t> shape, const float* src) {
    auto t = Tensor::create(std::move(shape), DataType::Float32, DeviceType::CPU);
    if (src) std::memcpy(t->data(), src, t->size_in_bytes());
    return t;
}
std::shared_ptr<Tensor> make_i32(std::vector<int64_t> shape, const int32_t* src) {
    auto t = Tensor::create(std::move(shape), DataType::Int32, DeviceType::CPU);
    if (src) std::memcpy(t->data(), src, t->size_in_bytes());
    return t;
}
void copy_out(const std::shared_ptr<Tensor>& t, float* dst) {
    std::memcpy(dst, t->data(), t->size_in_bytes());
}
}  // namespace

extern "C" {

// Embedding::forward (src/layer/layer.cpp:15-42)
void ref_embedding(const float* w, int num_rows, int hidden, const int32_t* ids, int n,
                   float* out) {
    Embedding emb(num_rows, hidden);
    emb.weight = make_f32({num_rows, hidden}, w);
    copy_out(emb.forward(make_i32({n}, ids)), out);
}

// RMSNorm::forward (src/layer/layer.cpp:48-77)
void ref_rmsnorm(const float* x, const float* w, int num_tokens, int hidden, float eps,
                 float* out) {
    RMSNorm norm(hidden, eps);
    norm.weight = make_f32({hidden}, w);
    copy_out(norm.forward(make_f32({num_tokens, hidden}, x)), out);
}

// RMSNorm::forward_fused_add (src/layer/layer.cpp:79-112); first != 0 -> null residual.
void ref_add_rmsnorm(float* x, float* residual, const float* w, int num_tokens, int hidden,
                     float eps, int first) {
    RMSNorm norm(hidden, eps);
    norm.weight = make_f32({hidden}, w);
    auto xt = make_f32({num_tokens, hidden}, x);
    std::shared_ptr<Tensor> rt = first ? nullptr : make_f32({num_tokens, hidden}, residual);
    norm.forward_fused_add(xt, rt);
    copy_out(xt, x);
    copy_out(rt, residual);
}

// Linear::forward (src/layer/layer.cpp:122-143)
void ref_linear(const float* x, const float* w, int num_tokens, int in_f, int out_f, float* out) {
    Linear lin(in_f, out_f);
    lin.weight = make_f32({out_f, in_f}, w);
    copy_out(lin.forward(make_f32({num_tokens, in_f}, x)), out);
}

// A persistent Linear (weights set once, as in a loaded model) for timing Linear::forward.
struct RefLinearHandle {
    Linear lin;
    int in_f;
    RefLinearHandle(int i, int o) : lin(i, o), in_f(i) {}
};
void* ref_linear_create(const float* w, int in_f, int out_f) {
    auto* h = new RefLinearHandle(in_f, out_f);
    h->lin.weight = make_f32({out_f, in_f}, w);
    return h;
}
void ref_linear_run(void* handle, const float* x, int num_tokens, float* out) {
    auto* h = static_cast<RefLinearHandle*>(handle);
    copy_out(h->lin.forward(make_f32({num_tokens, h->in_f}, x)), out);
}
void ref_linear_destroy(void* handle) { delete static_cast<RefLinearHandle*>(handle); }

// SwiGLU::forward (src/layer/layer.cpp:145-161)
void ref_swiglu(const float* g, const float* u, int n, float* out) {
    SwiGLU s;
    copy_out(s.forward(make_f32({n}, g), make_f32({n}, u)), out);
}

// RotaryEmbedding table (src/layer/layer.cpp:163-176), read back through forward():
// q = (1..1 | 0..0) rotates to (cos | sin) for the probed position.
void ref_rope_table(int head_dim, int max_position, float base, float* table) {
    RotaryEmbedding rope(head_dim, max_position, base);
    std::vector<float> probe(head_dim, 0.0f);
    for (int i = 0; i < head_dim / 2; ++i) probe[i] = 1.0f;
    std::shared_ptr<Tensor> none;
    for (int p = 0; p < max_position; ++p) {
        auto q = make_f32({1, head_dim}, probe.data());
        rope.forward(make_i32({1}, &p), q, none);
        copy_out(q, table + static_cast<int64_t>(p) * head_dim);
    }
}

// RotaryEmbedding::forward (src/layer/layer.cpp:178-199) called on one token's [heads, D]
// slice at a time, so its `pos[i % numel]` lookup reads that token's own position.
void ref_rope(float* x, const int32_t* positions, int num_tokens, int num_heads, int head_dim,
              int max_position, float base) {
    RotaryEmbedding rope(head_dim, max_position, base);
    std::shared_ptr<Tensor> none;
    for (int t = 0; t < num_tokens; ++t) {
        float* row = x + static_cast<int64_t>(t) * num_heads * head_dim;
        auto q = make_f32({num_heads, head_dim}, row);
        rope.forward(make_i32({1}, positions + t), q, none);
        copy_out(q, row);
    }
}

// Attention::forward (src/layer/layer.cpp:214-262), multi-head (Hq == Hkv) only: the only
// configuration for which the reference indexing is defined.
void ref_attention_mha(const float* q, const float* k, const float* v, int num_tokens,
                       int num_heads, int head_dim, float* out) {
    Attention attn(num_heads, head_dim);
    std::vector<int64_t> shp{num_tokens, static_cast<int64_t>(num_heads) * head_dim};
    copy_out(attn.forward(make_f32(shp, q), make_f32(shp, k), make_f32(shp, v)), out);
}

// MoERouter::route (src/layer/layer.cpp:270-309)
void ref_router(const float* x, const float* w, int num_tokens, int hidden, int num_experts,
                int top_k, int norm_topk, int32_t* ids, float* weights) {
    MoERouter router(hidden, num_experts, top_k, norm_topk != 0);
    router.weight = make_f32({num_experts, hidden}, w);
    std::shared_ptr<Tensor> rw;
    auto sel = router.route(make_f32({num_tokens, hidden}, x), rw);
    std::memcpy(ids, sel->data(), sel->size_in_bytes());
    copy_out(rw, weights);
}

// ---- KV page pool and radix cache (src/cache/kvcache.cpp) ----
void* ref_pool_create(int num_pages, int page_size) {
    return new std::shared_ptr<KVCachePool>(
        std::make_shared<KVCachePool>(num_pages, page_size, 1, 1, DeviceType::CPU));
}
void ref_pool_destroy(void* p) { delete static_cast<std::shared_ptr<KVCachePool>*>(p); }
int ref_pool_allocate(void* p) { return (*static_cast<std::shared_ptr<KVCachePool>*>(p))->allocate_page(); }
void ref_pool_free(void* p, int page) { (*static_cast<std::shared_ptr<KVCachePool>*>(p))->free_page(page); }
int ref_pool_num_free(void* p) { return (*static_cast<std::shared_ptr<KVCachePool>*>(p))->num_free_pages(); }

void* ref_radix_create(void* pool) {
    return new RadixCache(*static_cast<std::shared_ptr<KVCachePool>*>(pool));
}
void ref_radix_destroy(void* r) { delete static_cast<RadixCache*>(r); }
void ref_radix_insert(void* r, const int32_t* tokens, int n, const int32_t* pages, int np) {
    static_cast<RadixCache*>(r)->insert_prefix(std::vector<int32_t>(tokens, tokens + n),
                                               std::vector<int>(pages, pages + np));
}
// Returns matched token count; writes up to `cap` page ids and their count.
int ref_radix_match(void* r, const int32_t* tokens, int n, int32_t* pages, int cap, int* num_pages) {
    auto m = static_cast<RadixCache*>(r)->match_prefix(std::vector<int32_t>(tokens, tokens + n));
    int c = 0;
    for (int pg : m.page_indices) {
        if (c < cap) pages[c] = pg;
        ++c;
    }
    *num_pages = c;
    return m.matched_tokens;
}

// ---- Whole-model forward (src/model/qwen3.cpp:168-180 / qwen3_moe.cpp:201-213) ----
// Weights are passed in this order: embed [V,H]; per layer: input_ln [H], qkv [(Hq+2Hkv)D,H],
// o [H,HqD], post_ln [H], then dense: gate_up [2I,H], down [H,I]; or MoE: router [E,H], then
// per expert gate_up [2Im,H], down [H,Im]; then final norm [H], lm_head [V,H].
// Defined (no out-of-bounds reads) only for num_q_heads == num_kv_heads.
void ref_model_forward(int num_layers, int hidden, int num_q_heads, int num_kv_heads,
                       int head_dim, int inter, int vocab, float eps, float rope_base,
                       int max_position, int num_experts, int top_k, int moe_inter,
                       int norm_topk, const float* const* weights, const int32_t* ids,
                       const int32_t* positions, int num_tokens, float* logits) {
    ModelConfig cfg;
    cfg.num_layers = num_layers;
    cfg.hidden_size = hidden;
    cfg.num_qo_heads = num_q_heads;
    cfg.num_kv_heads = num_kv_heads;
    cfg.head_dim = head_dim;
    cfg.intermediate_size = inter;
    cfg.vocab_size = vocab;
    cfg.rms_norm_eps = eps;
    cfg.rotary_config.base = rope_base;
    cfg.rotary_config.max_position = max_position;
    cfg.rotary_config.head_dim = head_dim;
    cfg.num_experts = num_experts;
    cfg.num_experts_per_tok = top_k;
    cfg.moe_intermediate_size = moe_inter;
    cfg.norm_topk_prob = norm_topk != 0;
    int64_t qkv_rows = static_cast<int64_t>(num_q_heads + 2 * num_kv_heads) * head_dim;
    int64_t qd = static_cast<int64_t>(num_q_heads) * head_dim;
    int wi = 0;
    auto next = [&](std::vector<int64_t> shape) { return make_f32(std::move(shape), weights[wi++]); };
    std::shared_ptr<Tensor> out;
    auto ids_t = make_i32({num_tokens}, ids);
    auto pos_t = make_i32({num_tokens}, positions);
    if (num_experts > 0) {
        Qwen3MoEForCausalLM m(cfg);
        m.embed_tokens.weight = next({vocab, hidden});
        for (int l = 0; l < num_layers; ++l) {
            auto& L = *m.layers[l];
            L.input_layernorm.weight = next({hidden});
            L.qkv_proj.weight = next({qkv_rows, hidden});
            L.o_proj.weight = next({hidden, qd});
            L.post_attention_layernorm.weight = next({hidden});
            L.router.weight = next({num_experts, hidden});
            for (int e = 0; e < num_experts; ++e) {
                L.expert_gate_up[e]->weight = next({2 * moe_inter, hidden});
                L.expert_down[e]->weight = next({hidden, moe_inter});
            }
        }
        m.norm.weight = next({hidden});
        m.lm_head.weight = next({vocab, hidden});
        out = m.forward(ids_t, pos_t);
    } else {
        Qwen3ForCausalLM m(cfg);
        m.embed_tokens.weight = next({vocab, hidden});
        for (int l = 0; l < num_layers; ++l) {
            auto& L = *m.layers[l];
            L.input_layernorm.weight = next({hidden});
            L.qkv_proj.weight = next({qkv_rows, hidden});
            L.o_proj.weight = next({hidden, qd});
            L.post_attention_layernorm.weight = next({hidden});
            L.gate_up_proj.weight = next({2 * inter, hidden});
            L.down_proj.weight = next({hidden, inter});
        }
        m.norm.weight = next({hidden});
        m.lm_head.weight = next({vocab, hidden});
        out = m.forward(ids_t, pos_t);
    }
    copy_out(out, logits);
}

}  // extern "C"
