// qwen3.cpp -- the device-side Qwen3 executor (Qwen3DecoderLayer / Qwen3ForCausalLM of
// src/model/qwen3.cpp:16-83, 85-92, 168-180) and its C ABI (include/msgl_engine.h).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "layers.h"
#include "msgl_engine.h"

namespace msgl {
namespace engine {

void RotaryEmbedding::init(int d, int max_pos, float base, cudaStream_t s) {
    head_dim = d;
    max_position = max_pos;
    std::vector<float> t(static_cast<size_t>(max_pos) * d);
    for (int p = 0; p < max_pos; ++p)  // layer.cpp:168-175
        for (int i = 0; i < d / 2; ++i) {
            float freq = 1.0f / std::pow(base, (2.0f * i) / d);
            float val = p * freq;
            t[static_cast<size_t>(p) * d + i] = std::cos(val);
            t[static_cast<size_t>(p) * d + d / 2 + i] = std::sin(val);
        }
    cos_sin_cache.alloc(t.size() * sizeof(float));
    ckc(cudaMemcpyAsync(cos_sin_cache.p, t.data(), t.size() * sizeof(float),
                        cudaMemcpyHostToDevice, s),
        "rope table upload");
    ckc(cudaStreamSynchronize(s), "rope table upload");
}

struct Qwen3DecoderLayer {  // qwen3.h:11-30
    RMSNorm input_layernorm, post_attention_layernorm;
    Linear qkv_proj, o_proj, down_proj;
    GateUpSwiGLU gate_up_proj;  // gate_up_proj + swiglu
    Attention attn;
    MoEExperts moe;             // Qwen3MoEDecoderLayer: router + experts (qwen3_moe.h:13-30)
    DevBuf q_norm, k_norm;      // Qwen3 per-head norms (absent in the reference, D14)
    DevBuf k_pool, v_pool;      // [num_slots, hkv * D] bf16
};

struct Model {
    msgl_model_config cfg{};
    int hq = 0, hkv = 0, inter = 0, vocab_l = 0;  // this rank's shard
    int kv_head0 = 0;                              // first global kv head held by this rank
    int vocab0 = 0;                                // first lm_head row (token id) of this rank
    msgl_tp* tp = nullptr;                         // communicator (tp_size > 1), not owned
    bf16_t* tp_part[2] = {nullptr, nullptr};       // its peer-mapped slots: row-parallel outputs
    bf16_t* tp_x = nullptr;                        // two-shot all-reduce: x lives in slot 2
    DevBuf tp_logits_local, tp_logits_all;         // logits under TP: this rank's vocab columns,
                                                   // then every rank's (all-gathered)
    std::vector<Qwen3DecoderLayer> layers;
    DevBuf embed;        // [V, H]
    RMSNorm norm;        // final norm
    Linear lm_head;      // [V_l, H]
    RotaryEmbedding rope;
    int64_t num_slots = 0;
    int page_size = 16;
    int layers_run = -1;  // debug: run only the first n layers

    // workspace (allocated once)
    DevBuf x, residual, qkv, q, attn_out, act, x_last, res_last, packed, gemm_ws, attn_ws;
    // fp32 split-K partials of a decode-sized projection, added by the kernel that follows it
    // (qkv: QK-norm + RoPE; o_proj / down_proj: the fused add + RMSNorm, tensor parallel size 1)
    DevBuf parts;
    Scratch scratch;
    DevBuf moe_logits, moe_ids, moe_w, moe_off, moe_tok, moe_pos, moe_xs, moe_act, moe_ys, moe_ws;
    MoEScratch moe_scratch;
    int moe_inter = 0;  // this rank's expert intermediate size
    // device copies of a host batch (msgl_model_step_host)
    // (two sets, used in turn: an asynchronous host step may be submitted while the previous
    // one runs; `done` marks the completion of the step that last used the set)
    struct Staging {
        DevBuf ids, pos, slots, pt, seq, indptr, last, next;
        cudaEvent_t done = nullptr;
        int num_reqs = 0;
    };
    Staging st[2];
    DevBuf dec_next;            // greedy tokens of msgl_model_decode_steps
    uint64_t st_submitted = 0;  // host steps submitted so far (the next one uses st[n % 2])
    int st_max_pages = 0;
    // captured decode graphs, keyed by every pointer and shape field of the step
    struct GraphEntry {
        std::vector<int64_t> key;
        cudaGraphExec_t exec = nullptr;
    };
    std::vector<GraphEntry> graphs;

    void graphs_reset() {  // captured graphs hold the old communicator / buffers
        for (auto& g : graphs)
            if (g.exec) cudaGraphExecDestroy(g.exec);
        graphs.clear();
    }
    ~Model() {
        graphs_reset();
        for (auto& x : st)
            if (x.done) cudaEventDestroy(x.done);
    }

    int64_t weight_bytes() const {
        int64_t b = embed.bytes + norm.weight.bytes + lm_head.weight.bytes;
        for (auto& L : layers)
            b += L.input_layernorm.weight.bytes + L.post_attention_layernorm.weight.bytes +
                 L.qkv_proj.weight.bytes + L.o_proj.weight.bytes + L.down_proj.weight.bytes +
                 L.gate_up_proj.weight_packed.bytes + L.q_norm.bytes + L.k_norm.bytes +
                 L.moe.router.bytes + L.moe.gate_up_packed.bytes + L.moe.down.bytes;
        return b;
    }
};

static void validate(const msgl_model_config& c) {
    auto bad = [](const char* m) { throw Fail(MSGL_ERR_INVALID_ARG, m); };
    if (c.num_layers <= 0 || c.hidden <= 0 || c.vocab <= 0 || c.max_tokens <= 0 || c.max_reqs <= 0)
        bad("model: non-positive size");
    if (c.head_dim != 128) throw Fail(MSGL_ERR_UNSUPPORTED_SHAPE, "model: head_dim must be 128");
    if (c.num_kv_heads <= 0 || c.num_q_heads % c.num_kv_heads) bad("model: Hq % Hkv");
    if (c.tp_size < 1 || c.tp_rank < 0 || c.tp_rank >= c.tp_size) bad("model: tp rank/size");
    if (c.num_q_heads % c.tp_size) bad("model: Hq % tp");
    if (c.num_experts > 0) {
        if (c.num_experts > 256 || c.top_k <= 0 || c.top_k > 32 || c.top_k > c.num_experts)
            throw Fail(MSGL_ERR_UNSUPPORTED_SHAPE, "model: MoE needs <= 256 experts, top_k <= 32");
        if (c.moe_inter % c.tp_size || (c.moe_inter / c.tp_size) % 16)
            bad("model: moe_inter / tp must be a multiple of 16");
    } else if (c.inter % c.tp_size || (c.inter / c.tp_size) % 16) {
        bad("model: inter / tp must be a multiple of 16");
    }
}

static void create(Model& m, const msgl_model_config& c) {
    validate(c);
    m.cfg = c;
    const int tp = c.tp_size, D = c.head_dim, H = c.hidden;
    int plan[8];
    ck(msgl_tp_shard_plan(c.num_q_heads, c.num_kv_heads,
                          c.num_experts > 0 ? c.moe_inter : c.inter, c.vocab, c.tp_rank, tp, plan),
       "model: tensor-parallel shard");
    m.hq = plan[1];
    m.kv_head0 = plan[2];
    m.hkv = plan[3];
    m.inter = c.num_experts > 0 ? 0 : c.inter / tp;
    m.moe_inter = c.num_experts > 0 ? c.moe_inter / tp : 0;
    m.vocab0 = plan[6];
    m.vocab_l = plan[7];
    if (m.vocab_l <= 0) throw Fail(MSGL_ERR_INVALID_ARG, "model: empty vocab shard");
    m.layers.resize(c.num_layers);
    cudaStream_t s = nullptr;
    for (auto& L : m.layers) {
        L.input_layernorm = RMSNorm(H, c.eps);
        L.post_attention_layernorm = RMSNorm(H, c.eps);
        L.qkv_proj = Linear(H, (m.hq + 2 * m.hkv) * D);
        L.o_proj = Linear(m.hq * D, H);
        L.gate_up_proj = GateUpSwiGLU(H, m.inter);
        L.down_proj = Linear(m.inter, H);
        L.attn = Attention(m.hq, m.hkv, D, c.eps);
        L.input_layernorm.weight.alloc(H * 2);
        L.post_attention_layernorm.weight.alloc(H * 2);
        L.qkv_proj.weight.alloc(static_cast<size_t>(L.qkv_proj.out_features()) * H * 2);
        L.o_proj.weight.alloc(static_cast<size_t>(H) * m.hq * D * 2);
        if (c.num_experts > 0) {
            const size_t E = c.num_experts, Im = m.moe_inter;
            L.moe = MoEExperts(H, c.num_experts, c.top_k, m.moe_inter, c.norm_topk != 0);
            L.moe.router.alloc(E * H * 2);
            L.moe.gate_up_packed.alloc(E * 2 * Im * H * 2);
            L.moe.down.alloc(E * H * Im * 2);
        } else {
            L.gate_up_proj.weight_packed.alloc(static_cast<size_t>(2 * m.inter) * H * 2);
            L.down_proj.weight.alloc(static_cast<size_t>(H) * m.inter * 2);
        }
        L.q_norm.alloc(D * 2);
        L.k_norm.alloc(D * 2);
    }
    m.embed.alloc(static_cast<size_t>(c.vocab) * H * 2);
    m.norm = RMSNorm(H, c.eps);
    m.norm.weight.alloc(H * 2);
    m.lm_head = Linear(H, m.vocab_l);
    m.lm_head.weight.alloc(static_cast<size_t>(m.vocab_l) * H * 2);
    m.rope.init(D, c.max_position, c.rope_base, s);

    // workspace
    const size_t T = c.max_tokens, B = c.max_reqs;
    m.x.alloc(T * H * 2);
    m.residual.alloc(T * H * 4);
    m.qkv.alloc(T * (m.hq + 2 * m.hkv) * D * 2);
    m.q.alloc(T * m.hq * D * 2);
    m.attn_out.alloc(T * m.hq * D * 2);
    m.act.alloc(T * std::max(m.inter, H) * 2);
    m.x_last.alloc(B * H * 2);
    m.res_last.alloc(B * H * 4);
    m.packed.alloc(B * 8);
    // split-K workspaces: the largest any step size up to capacity can ask for
    size_t gws = 0;
    const auto& L0 = m.layers[0];
    for (int t = 1; t <= static_cast<int>(T); ++t) {
        gws = std::max(gws, L0.qkv_proj.workspace(t));
        gws = std::max(gws, L0.o_proj.workspace(t));
        if (c.num_experts > 0) {
            gws = std::max(gws, msgl_gemm_workspace_size(t, c.num_experts, H));
        } else {
            gws = std::max(gws, L0.gate_up_proj.workspace(t));
            gws = std::max(gws, L0.down_proj.workspace(t));
        }
        if (t <= static_cast<int>(B)) gws = std::max(gws, m.lm_head.workspace(t));
    }
    m.gemm_ws.alloc(std::max<size_t>(gws, 256));
    ckc(cudaMemset(m.gemm_ws.p, 0, m.gemm_ws.bytes), "gemm workspace");
    size_t aws = 0;
    for (int b = 1; b <= static_cast<int>(B); ++b)
        aws = std::max(aws, msgl_paged_attention_workspace_size(b, c.max_position, m.hq, m.hkv, D));
    // the cascade decode (shared prefix) needs at most 5x the plain decode's partial storage
    // (at most 4 prefix chunks per suffix chunk)
    aws = aws > 0 ? 5 * aws : 0;
    m.attn_ws.alloc(std::max<size_t>(aws, 256));
    ckc(cudaMemset(m.attn_ws.p, 0, m.attn_ws.bytes), "attention workspace");
    m.scratch = Scratch{m.gemm_ws.p, m.gemm_ws.bytes, m.attn_ws.p, m.attn_ws.bytes};
    // split-K partials (steps of <= 256 tokens; MSGL_SPLITK_PARTIALS=0 turns the path off)
    const char* env_parts = std::getenv("MSGL_SPLITK_PARTIALS");
    if (!(env_parts && env_parts[0] == '0')) {
        // the split count depends on the number of 128-token tiles: the largest buffer is at
        // 128 tokens or at the largest step size up to 256
        auto need = [&](const Linear& l) {
            size_t n = 0;
            for (size_t cap : {size_t(128), size_t(256)}) {
                const int tm = static_cast<int>(std::min<size_t>(T, cap));
                if (l.partials_fit(tm))
                    n = std::max(n, static_cast<size_t>(l.partial_splits(tm)) * tm *
                                        l.out_features() * sizeof(float));
            }
            return n;
        };
        size_t pb = need(L0.qkv_proj);
        if (tp == 1) {
            pb = std::max(pb, need(L0.o_proj));
            if (c.num_experts == 0) pb = std::max(pb, need(L0.down_proj));
        }
        if (pb > 0) m.parts.alloc(pb);
    }
    if (c.num_experts > 0) {
        const size_t E = c.num_experts, k = c.top_k, R = T * k;
        // router logits, or their split-K partials for steps of <= 256 tokens
        size_t lf = T * E;
        for (int t = 1; t <= static_cast<int>(std::min<size_t>(T, 256)); ++t)
            lf = std::max(lf, static_cast<size_t>(std::max(0, m.layers[0].moe.router_splits(t))) *
                                  t * E);
        m.moe_logits.alloc(lf * 4);
        m.moe_ids.alloc(T * k * 4);
        m.moe_w.alloc(T * k * 4);
        m.moe_off.alloc((E + 1) * 4);
        m.moe_tok.alloc(R * 4);
        m.moe_pos.alloc(R * 4);
        m.moe_xs.alloc(R * H * 2);
        m.moe_act.alloc(R * m.moe_inter * 2);
        m.moe_ys.alloc(R * H * 2);
        size_t gw = 0;
        for (size_t r = k; r <= R; r += k)
            gw = std::max(gw, msgl_grouped_gemm_workspace_size(static_cast<int>(r), c.num_experts));
        m.moe_ws.alloc(std::max<size_t>(gw, 256));
        m.moe_scratch = MoEScratch{m.moe_logits.as<float>(), m.moe_ids.as<int>(), m.moe_w.as<float>(),
                                   m.moe_off.as<int>(), m.moe_tok.as<int>(), m.moe_pos.as<int>(),
                                   m.moe_xs.as<bf16_t>(), m.moe_act.as<bf16_t>(), m.moe_ys.as<bf16_t>(),
                                   m.moe_ws.p, m.moe_ws.bytes, lf};
    }
    m.st_max_pages = (c.max_position + 15) / 16;
    for (auto& x : m.st) {
        x.ids.alloc(T * 4);
        x.pos.alloc(T * 4);
        x.slots.alloc(T * 4);
        x.pt.alloc(B * m.st_max_pages * 4);
        x.seq.alloc(B * 4);
        x.indptr.alloc((B + 1) * 4);
        x.last.alloc(B * 4);
        x.next.alloc(B * 4);
        ckc(cudaEventCreateWithFlags(&x.done, cudaEventDisableTiming), "staging event");
    }
    m.dec_next.alloc(B * 4);
}

// ----------------------------------------------------------------------------- weights
static void fill(DevBuf& b, uint64_t seed, uint64_t id, float mean, float std, cudaStream_t s) {
    ck(msgl_fill_normal_bf16(b.p, static_cast<int64_t>(b.bytes / 2), seed, id, mean, std, s),
       "random_init");
}

static void random_init(Model& m, uint64_t seed, float std, cudaStream_t s) {
    uint64_t id = static_cast<uint64_t>(m.cfg.tp_rank) << 40;
    fill(m.embed, seed, id++, 0.f, std, s);
    for (auto& L : m.layers) {
        fill(L.input_layernorm.weight, seed, id++, 1.f, 0.f, s);
        fill(L.qkv_proj.weight, seed, id++, 0.f, std, s);
        fill(L.q_norm, seed, id++, 1.f, 0.f, s);
        fill(L.k_norm, seed, id++, 1.f, 0.f, s);
        fill(L.o_proj.weight, seed, id++, 0.f, std, s);
        fill(L.post_attention_layernorm.weight, seed, id++, 1.f, 0.f, s);
        if (m.cfg.num_experts > 0) {
            fill(L.moe.router, seed, id++, 0.f, std, s);
            fill(L.moe.gate_up_packed, seed, id++, 0.f, std, s);
            fill(L.moe.down, seed, id++, 0.f, std, s);
        } else {
            fill(L.gate_up_proj.weight_packed, seed, id++, 0.f, std, s);  // i.i.d.: packing is moot
            fill(L.down_proj.weight, seed, id++, 0.f, std, s);
        }
    }
    fill(m.norm.weight, seed, id++, 1.f, 0.f, s);
    fill(m.lm_head.weight, seed, id++, 0.f, std, s);
    ckc(cudaStreamSynchronize(s), "random_init");
}

// Copy rows [r0, r0 + nrows) x cols [c0, c0 + ncols) of a host [rows, cols] bf16 matrix.
static void upload_block(void* dst, const bf16_t* src, int64_t cols, int64_t r0, int64_t nrows,
                         int64_t c0, int64_t ncols, cudaStream_t s) {
    ckc(cudaMemcpy2DAsync(dst, ncols * 2, src + r0 * cols + c0, cols * 2, ncols * 2, nrows,
                          cudaMemcpyHostToDevice, s),
        "set_weight upload");
}

static void set_weight(Model& m, const std::string& name, const bf16_t* h, int64_t numel,
                       cudaStream_t s) {
    const auto& c = m.cfg;
    const int64_t H = c.hidden, D = c.head_dim, tp = c.tp_size, r = c.tp_rank;
    auto need = [&](int64_t n) {
        if (numel != n) throw Fail(MSGL_ERR_INVALID_ARG, "set_weight " + name + ": numel mismatch");
    };
    if (name == "embed") { need(c.vocab * H); upload_block(m.embed.p, h, H, 0, c.vocab, 0, H, s); }
    else if (name == "norm") { need(H); upload_block(m.norm.weight.p, h, H, 0, 1, 0, H, s); }
    else if (name == "lm_head") { need(c.vocab * H); upload_block(m.lm_head.weight.p, h, H, m.vocab0, m.vocab_l, 0, H, s); }
    else if (name.rfind("layers.", 0) == 0) {
        size_t dot = name.find('.', 7);
        int l = std::stoi(name.substr(7, dot - 7));
        if (l < 0 || l >= c.num_layers) throw Fail(MSGL_ERR_INVALID_ARG, "set_weight: layer");
        std::string f = name.substr(dot + 1);
        auto& L = m.layers[l];
        const int64_t hq_g = c.num_q_heads, hkv_g = c.num_kv_heads, I = c.inter;
        if (f == "input_ln") { need(H); upload_block(L.input_layernorm.weight.p, h, H, 0, 1, 0, H, s); }
        else if (f == "post_ln") { need(H); upload_block(L.post_attention_layernorm.weight.p, h, H, 0, 1, 0, H, s); }
        else if (f == "q_norm") { need(D); upload_block(L.q_norm.p, h, D, 0, 1, 0, D, s); }
        else if (f == "k_norm") { need(D); upload_block(L.k_norm.p, h, D, 0, 1, 0, D, s); }
        else if (f == "qkv") {  // rows q | k | v; keep this rank's q heads and kv heads
            need((hq_g + 2 * hkv_g) * D * H);
            char* dst = static_cast<char*>(L.qkv_proj.weight.p);
            upload_block(dst, h, H, r * m.hq * D, m.hq * D, 0, H, s);
            dst += m.hq * D * H * 2;
            upload_block(dst, h, H, (hq_g + m.kv_head0) * D, m.hkv * D, 0, H, s);
            dst += m.hkv * D * H * 2;
            upload_block(dst, h, H, (hq_g + hkv_g + m.kv_head0) * D, m.hkv * D, 0, H, s);
        } else if (f == "o") {  // [H, Hq D]: column shard
            need(H * hq_g * D);
            upload_block(L.o_proj.weight.p, h, hq_g * D, 0, H, r * m.hq * D, m.hq * D, s);
        } else if (f == "gate_up") {  // rows gate | up: this rank's I/tp of each, then pack
            need(2 * I * H);
            DevBuf tmp;
            tmp.alloc(static_cast<size_t>(2 * m.inter) * H * 2);
            upload_block(tmp.p, h, H, r * m.inter, m.inter, 0, H, s);
            upload_block(static_cast<char*>(tmp.p) + static_cast<size_t>(m.inter) * H * 2, h, H,
                         I + r * m.inter, m.inter, 0, H, s);
            ck(msgl_pack_gate_up(tmp.p, L.gate_up_proj.weight_packed.p, m.inter, H, s), "pack_gate_up");
            ckc(cudaStreamSynchronize(s), "set_weight");
        } else if (f == "router") {  // [E, H], replicated on every rank
            need(static_cast<int64_t>(c.num_experts) * H);
            upload_block(L.moe.router.p, h, H, 0, c.num_experts, 0, H, s);
        } else if (f.rfind("experts.", 0) == 0) {
            size_t d2 = f.find('.', 8);
            const int e = std::stoi(f.substr(8, d2 - 8));
            const std::string part = f.substr(d2 + 1);
            if (e < 0 || e >= c.num_experts) throw Fail(MSGL_ERR_INVALID_ARG, "set_weight: expert");
            const int64_t Im = c.moe_inter, Iml = m.moe_inter;
            if (part == "gate_up") {  // [2 Im, H] rows gate | up: this rank's Im/tp of each, packed
                need(2 * Im * H);
                DevBuf tmp;
                tmp.alloc(static_cast<size_t>(2 * Iml) * H * 2);
                upload_block(tmp.p, h, H, r * Iml, Iml, 0, H, s);
                upload_block(static_cast<char*>(tmp.p) + static_cast<size_t>(Iml) * H * 2, h, H,
                             Im + r * Iml, Iml, 0, H, s);
                char* dst = static_cast<char*>(L.moe.gate_up_packed.p) +
                            static_cast<size_t>(e) * 2 * Iml * H * 2;
                ck(msgl_pack_gate_up(tmp.p, dst, static_cast<int>(Iml), H, s), "pack_gate_up");
                ckc(cudaStreamSynchronize(s), "set_weight");
            } else if (part == "down") {  // [H, Im]: column shard
                need(H * Im);
                char* dst = static_cast<char*>(L.moe.down.p) + static_cast<size_t>(e) * H * Iml * 2;
                upload_block(dst, h, Im, 0, H, r * Iml, Iml, s);
            } else {
                throw Fail(MSGL_ERR_INVALID_ARG, "set_weight: unknown tensor " + name);
            }
        } else if (f == "down") {  // [H, I]: column shard
            need(H * I);
            upload_block(L.down_proj.weight.p, h, I, 0, H, r * m.inter, m.inter, s);
        } else {
            throw Fail(MSGL_ERR_INVALID_ARG, "set_weight: unknown tensor " + name);
        }
    } else {
        throw Fail(MSGL_ERR_INVALID_ARG, "set_weight: unknown tensor " + name);
    }
    ckc(cudaStreamSynchronize(s), "set_weight");
}

static void alloc_kv(Model& m, int num_pages, int page_size, cudaStream_t s) {
    if (page_size != 16) throw Fail(MSGL_ERR_UNSUPPORTED_SHAPE, "alloc_kv: page_size must be 16");
    if (num_pages <= 0) throw Fail(MSGL_ERR_INVALID_ARG, "alloc_kv: num_pages");
    m.graphs_reset();  // captured graphs hold the old pools' addresses
    m.page_size = page_size;
    m.num_slots = static_cast<int64_t>(num_pages) * page_size;
    const size_t bytes = static_cast<size_t>(m.num_slots) * m.hkv * m.cfg.head_dim * 2;
    for (auto& L : m.layers) {
        L.k_pool.alloc(bytes);
        L.v_pool.alloc(bytes);
        ckc(cudaMemsetAsync(L.k_pool.p, 0, bytes, s), "alloc_kv");
        ckc(cudaMemsetAsync(L.v_pool.p, 0, bytes, s), "alloc_kv");
    }
    ckc(cudaStreamSynchronize(s), "alloc_kv");
}

// ----------------------------------------------------------------------------- forward
// Qwen3ForCausalLM::forward (qwen3.cpp:168-180) with Qwen3DecoderLayer::forward (:16-83) inlined.
static void forward(Model& m, const msgl_batch& b, int* next_tokens, float* logits,
                    cudaStream_t s) {
    const auto& c = m.cfg;
    if (b.num_tokens <= 0 || b.num_tokens > c.max_tokens || b.num_reqs <= 0 ||
        b.num_reqs > c.max_reqs)
        throw Fail(MSGL_ERR_INVALID_ARG, "forward: batch exceeds the executor's capacity");
    if (b.is_decode && b.num_tokens != b.num_reqs)
        throw Fail(MSGL_ERR_INVALID_ARG, "forward: decode needs one token per request");
    if (b.max_seq_len > c.max_position)
        throw Fail(MSGL_ERR_INVALID_ARG, "forward: max_seq_len exceeds max_position");
    if (m.num_slots == 0) throw Fail(MSGL_ERR_INVALID_ARG, "forward: KV pools not allocated");
    if (c.tp_size > 1 && !m.tp) throw Fail(MSGL_ERR_INVALID_ARG, "forward: tp_size > 1 needs msgl_model_set_tp");
    const int T = b.num_tokens, H = c.hidden;
    // tensor parallel with the two-shot all-reduce: x is the peer-mapped slot every rank's
    // all-reduce stores its normed rows into (the residual then stays row-partitioned)
    auto* x = m.tp_x ? m.tp_x : m.x.as<bf16_t>();
    float* res = m.residual.as<float>();
    auto allreduce_norm = [&](bf16_t* part, const void* w, const char* what) {
        if (m.tp_x)
            ck(msgl_tp_fused_allreduce_add_rmsnorm_2shot(m.tp, part, x, res, w, T, H, c.eps, 0, s), what);
        else
            ck(msgl_tp_fused_allreduce_add_rmsnorm(m.tp, part, x, res, w, T, H, c.eps, 0, s), what);
    };
    const int nl = m.layers_run >= 0 ? std::min(m.layers_run, c.num_layers) : c.num_layers;

    // embed_tokens + layer 0's input_layernorm (residual aliasing first call, layer.cpp:80-84)
    ck(msgl_embed_rmsnorm(m.embed.p, b.input_ids, T, c.vocab, H, m.layers[0].input_layernorm.weight.p,
                          c.eps, x, res, s),
       "embed_tokens");
    // Tensor parallel: the row-parallel outputs (o_proj, down_proj / expert combine) go to the
    // communicator's peer-mapped rows, and one kernel all-reduces them over NVLink fused with
    // the residual add and the next RMSNorm (post-attention norm; the next layer's input norm;
    // after the last layer the final norm).
    // (o_proj uses slot 0, down_proj slot 1: consecutive all-reduces alternate slots)
    bf16_t* part_o = m.tp ? m.tp_part[0] : x;
    bf16_t* part_d = m.tp ? m.tp_part[1] : x;
    // Steps of <= 256 tokens: qkv, o_proj and (dense, tensor parallel size 1) down_proj write
    // fp32 split-K partials that the next kernel adds, instead of reducing the K split across
    // CTAs inside the GEMM. `pend` = splits of down_proj partials the next norm has to add.
    float* parts = m.parts.as<float>();
    auto use_parts = [&](const Linear& l) { return parts != nullptr && l.partials_fit(T); };
    int pend = 0;
    bool normed = false;  // the previous layer's MoE combine already ran this layer's input norm
    for (int l = 0; l < nl; ++l) {
        auto& L = m.layers[l];
        if (l > 0 && !m.tp && !normed) {  // qwen3.cpp:19
            if (pend)
                L.input_layernorm.forward_fused_add_partials(parts, pend, x, res, T, s);
            else
                L.input_layernorm.forward_fused_add(x, res, T, false, s);
            pend = 0;
        }
        normed = false;
        if (use_parts(L.qkv_proj)) {  // :22, :28-48
            const int S = L.qkv_proj.forward_partials(x, parts, T, s);
            L.attn.prepare_partials(parts, S, m.q.as<bf16_t>(), L.k_pool.p, L.v_pool.p,
                                    m.num_slots, b.positions, b.slot_mapping, m.rope, L.q_norm.p,
                                    L.k_norm.p, T, s);
        } else {
            L.qkv_proj.forward(x, m.qkv.as<bf16_t>(), T, m.scratch, s);
            L.attn.prepare(m.qkv.as<bf16_t>(), m.q.as<bf16_t>(), L.k_pool.p, L.v_pool.p,
                           m.num_slots, b.positions, b.slot_mapping, m.rope, L.q_norm.p,
                           L.k_norm.p, T, s);
        }
        L.attn.forward(m.q.as<bf16_t>(), L.k_pool.p, L.v_pool.p, m.num_slots, b,
                       m.attn_out.as<bf16_t>(), m.scratch, s);                // :51-52
        if (m.tp) {  // row-parallel o_proj (:55): all-reduce fused with the add + norm of :57
            L.o_proj.forward(m.attn_out.as<bf16_t>(), part_o, T, m.scratch, s);
            allreduce_norm(part_o, L.post_attention_layernorm.weight.p, "o_proj all-reduce");
        } else if (use_parts(L.o_proj)) {
            const int S = L.o_proj.forward_partials(m.attn_out.as<bf16_t>(), parts, T, s);
            L.post_attention_layernorm.forward_fused_add_partials(parts, S, x, res, T, s);
        } else {
            L.o_proj.forward(m.attn_out.as<bf16_t>(), part_o, T, m.scratch, s);
            L.post_attention_layernorm.forward_fused_add(x, res, T, false, s);  // :57
        }
        if (c.num_experts > 0) {  // qwen3_moe.cpp:62-111
            if (!m.tp && l + 1 < nl) {  // + the residual add and the next layer's input norm
                L.moe.forward(x, x, T, m.moe_scratch, m.scratch, s, &m.layers[l + 1].input_layernorm,
                              res);
                normed = true;
            } else {
                L.moe.forward(x, part_d, T, m.moe_scratch, m.scratch, s);
            }
        } else {
            L.gate_up_proj.forward(x, m.act.as<bf16_t>(), T, m.scratch, s);  // :60-79
            // (the last layer's down_proj writes x, the hidden state msgl_model_hidden reads)
            if (use_parts(L.down_proj) && !m.tp && l + 1 < nl)               // :80
                pend = L.down_proj.forward_partials(m.act.as<bf16_t>(), parts, T, s);
            else
                L.down_proj.forward(m.act.as<bf16_t>(), part_d, T, m.scratch, s);
        }
        if (m.tp) {  // row-parallel down_proj / expert combine: all-reduce + add + next norm
            const void* next_w = l + 1 < nl ? m.layers[l + 1].input_layernorm.weight.p : m.norm.weight.p;
            allreduce_norm(part_d, next_w, "mlp all-reduce");
        }
    }
    // final norm on each request's last row (qwen3.cpp:177, sampling row of D10), lm_head +
    // greedy argmax (scheduler.cpp:117-124)
    const int B = b.num_reqs;
    bf16_t* xl = x;
    float* rl = res;
    if (!b.is_decode) {
        ck(msgl_launch_index_gather(x, b.last_idx, m.x_last.p, H, B, T, MSGL_BF16, s), "gather x");
        if (!m.tp)
            ck(msgl_launch_index_gather(res, b.last_idx, m.res_last.p, H, B, T, MSGL_F32, s),
               "gather res");
        xl = m.x_last.as<bf16_t>();
        rl = m.res_last.as<float>();
    }
    if (!m.tp) m.norm.forward_fused_add(xl, rl, B, false, s);  // (TP: done by the last all-reduce)
    if (m.tp) {  // vocab-parallel lm_head: local best (logit, id), max over the ranks
        if (logits) {  // this rank's vocab columns in fp32, all-gathered, placed as columns
            const int world = c.tp_size, vpad = (c.vocab + world - 1) / world;
            const size_t chunk = static_cast<size_t>(B) * vpad * sizeof(float);
            ck(msgl_gemm_bf16(xl, m.lm_head.weight.p, m.tp_logits_local.p, B, m.vocab_l, H, MSGL_F32,
                              m.scratch.gemm_ws, m.scratch.gemm_ws_bytes, s), "lm_head logits shard");
            ck(msgl_tp_all_gather(m.tp, m.tp_logits_local.p, m.tp_logits_all.p, chunk, s),
               "logits all-gather");
            for (int q = 0; q < world; ++q) {  // rank q's [B, rows_q] block -> columns [q vpad, ...)
                const int rows_q = std::min(vpad, c.vocab - q * vpad);
                if (rows_q <= 0) continue;
                ckc(cudaMemcpy2DAsync(logits + static_cast<size_t>(q) * vpad, static_cast<size_t>(c.vocab) * 4,
                                      static_cast<const char*>(m.tp_logits_all.p) + q * chunk,
                                      static_cast<size_t>(rows_q) * 4, static_cast<size_t>(rows_q) * 4, B,
                                      cudaMemcpyDeviceToDevice, s),
                    "logits placement");
            }
        }
        ck(msgl_lm_head_argmax_partial(xl, m.lm_head.weight.p, B, m.vocab_l, H, m.vocab0,
                                       m.packed.as<unsigned long long>(), m.scratch.gemm_ws,
                                       m.scratch.gemm_ws_bytes, s), "lm_head");
        ck(msgl_tp_argmax_combine(m.tp, m.packed.as<unsigned long long>(), next_tokens, B, s),
           "argmax over ranks");
        return;
    }
    ck(msgl_lm_head_argmax(xl, m.lm_head.weight.p, B, m.vocab_l, H,
                           m.packed.as<unsigned long long>(), next_tokens, m.scratch.gemm_ws,
                           m.scratch.gemm_ws_bytes, s),
       "lm_head");
    if (logits)
        ck(msgl_gemm_bf16(xl, m.lm_head.weight.p, logits, B, m.vocab_l, H, MSGL_F32,
                          m.scratch.gemm_ws, m.scratch.gemm_ws_bytes, s),
           "lm_head logits");
}

static std::vector<int64_t> graph_key(const msgl_batch& b, const int* next, const float* logits) {
    return {b.num_tokens, b.num_reqs, b.is_decode, b.max_pages, b.max_seq_len, b.max_q_len,
            b.shared_prefix_pages, b.decode_tail, reinterpret_cast<int64_t>(b.input_ids), reinterpret_cast<int64_t>(b.positions),
            reinterpret_cast<int64_t>(b.slot_mapping), reinterpret_cast<int64_t>(b.page_table),
            reinterpret_cast<int64_t>(b.seq_lens), reinterpret_cast<int64_t>(b.q_indptr),
            reinterpret_cast<int64_t>(b.last_idx), reinterpret_cast<int64_t>(next),
            reinterpret_cast<int64_t>(logits)};
}

static void run(Model& m, const msgl_batch& b, int* next, float* logits, int flags,
                cudaStream_t s) {
    if (!(flags & MSGL_FWD_GRAPH)) {
        forward(m, b, next, logits, s);
        return;
    }
    if (s == nullptr) throw Fail(MSGL_ERR_INVALID_ARG, "graph step needs a non-default stream");
    auto key = graph_key(b, next, logits);
    for (auto& g : m.graphs)
        if (g.key == key) {
            ckc(cudaGraphLaunch(g.exec, s), "cudaGraphLaunch");
            return;
        }
    // one eager pass first: first-use work (module loading, attribute setting) stays out of
    // the capture
    forward(m, b, next, logits, s);
    cudaGraph_t graph = nullptr;
    ckc(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
        forward(m, b, next, logits, s);
    } catch (...) {
        cudaStreamEndCapture(s, &graph);
        if (graph) cudaGraphDestroy(graph);
        throw;
    }
    ckc(cudaStreamEndCapture(s, &graph), "end capture");
    cudaGraphExec_t exec = nullptr;
    cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    ckc(e, "cudaGraphInstantiate");
    m.graphs.push_back({key, exec});
    ckc(cudaGraphLaunch(exec, s), "cudaGraphLaunch");
}

// The scheduler-facing step (Scheduler::step -> forward, scheduler.cpp:83-124) on host arrays:
// H2D into one staging set, the step, D2H of the greedy tokens; with `wait` the host waits for
// it (msgl_model_step_host), otherwise it returns at once (msgl_model_step_host_async: overlap
// scheduling -- the host builds the next batch while this one runs). Returns the step's ticket.
static uint64_t step_host(Model& m, const msgl_batch& hb, int* host_next, int flags,
                          cudaStream_t s, bool wait) {
    const int T = hb.num_tokens, B = hb.num_reqs;
    if (T <= 0 || T > m.cfg.max_tokens || B <= 0 || B > m.cfg.max_reqs)
        throw Fail(MSGL_ERR_INVALID_ARG, "step_host: batch exceeds the executor's capacity");
    if (hb.max_pages <= 0 || hb.max_pages > m.st_max_pages)
        throw Fail(MSGL_ERR_INVALID_ARG, "step_host: page-table width exceeds max_position / 16");
    const bool prev_ids = (flags & MSGL_STEP_TOKENS_FROM_PREV) != 0;
    const uint64_t ticket = m.st_submitted;
    Model::Staging& x = m.st[ticket % 2];
    if (prev_ids) {
        const Model::Staging& p = m.st[(ticket + 1) % 2];
        if (ticket == 0 || !hb.is_decode || T != B || B > p.num_reqs)
            throw Fail(MSGL_ERR_INVALID_ARG,
                       "step_host: tokens from the previous step need a decode step of at most "
                       "its requests, after one");
    }
    auto h2d = [&](DevBuf& d, const int* h, size_t n) {
        if (!h) throw Fail(MSGL_ERR_INVALID_ARG, "step_host: null host array");
        ckc(cudaMemcpyAsync(d.p, h, n * 4, cudaMemcpyHostToDevice, s), "step_host H2D");
    };
    if (prev_ids)  // row r continues request r of the previous step: its greedy token, on device
        ckc(cudaMemcpyAsync(x.ids.p, m.st[(ticket + 1) % 2].next.p, static_cast<size_t>(B) * 4,
                            cudaMemcpyDeviceToDevice, s),
            "step_host tokens from the previous step");
    else
        h2d(x.ids, hb.input_ids, T);
    h2d(x.pos, hb.positions, T);
    h2d(x.slots, hb.slot_mapping, T);
    h2d(x.pt, hb.page_table, static_cast<size_t>(B) * hb.max_pages);
    h2d(x.seq, hb.seq_lens, B);
    h2d(x.indptr, hb.q_indptr, B + 1);
    h2d(x.last, hb.last_idx, B);
    msgl_batch db = hb;
    if (hb.shared_prefix_pages == MSGL_SHARED_PREFIX_DETECT) {
        // leading page-table columns that are the same page in every row, covered by every
        // context (two or more requests)
        int n = 0;
        if (B >= 2) {
            int min_len = hb.seq_lens[0];
            for (int r = 1; r < B; ++r) min_len = std::min(min_len, hb.seq_lens[r]);
            const int cap = std::min(hb.max_pages, min_len / 16);
            for (; n < cap; ++n) {
                const int p = hb.page_table[n];
                bool same = true;
                for (int r = 1; r < B && same; ++r)
                    same = hb.page_table[static_cast<size_t>(r) * hb.max_pages + n] == p;
                if (!same) break;
            }
        }
        db.shared_prefix_pages = n;
    }
    if (hb.decode_tail == MSGL_DECODE_TAIL_DETECT) {  // trailing requests with one query row
        int n = 0;
        if (!hb.is_decode)
            while (n < B - 1 && hb.q_indptr[B - n] - hb.q_indptr[B - n - 1] == 1) ++n;
        db.decode_tail = n;
    }
    if (db.decode_tail < 0 || db.decode_tail >= B) db.decode_tail = 0;
    db.input_ids = x.ids.as<int>();
    db.positions = x.pos.as<int>();
    db.slot_mapping = x.slots.as<int>();
    db.page_table = x.pt.as<int>();
    db.seq_lens = x.seq.as<int>();
    db.q_indptr = x.indptr.as<int>();
    db.last_idx = x.last.as<int>();
    run(m, db, x.next.as<int>(), nullptr, hb.is_decode ? (flags & MSGL_FWD_GRAPH) : 0, s);
    ckc(cudaMemcpyAsync(host_next, x.next.p, B * 4, cudaMemcpyDeviceToHost, s), "step_host D2H");
    ckc(cudaEventRecord(x.done, s), "step_host event");
    x.num_reqs = B;
    m.st_submitted = ticket + 1;
    if (wait) ckc(cudaEventSynchronize(x.done), "step_host sync");
    return ticket;
}

static void step_wait(Model& m, uint64_t ticket) {
    if (ticket >= m.st_submitted || ticket + 2 < m.st_submitted)
        throw Fail(MSGL_ERR_INVALID_ARG, "step_wait: not one of the last two submitted steps");
    ckc(cudaEventSynchronize(m.st[ticket % 2].done), "step_wait");
}

}  // namespace engine
}  // namespace msgl

using namespace msgl::engine;

struct msgl_model {
    Model m;
};

namespace msgl {
int set_error(int code, const char* msg);
}

template <typename F>
static int guarded(F&& f) {
    try {
        f();
        return MSGL_OK;
    } catch (const Fail& e) {
        return msgl::set_error(e.code, e.what());
    } catch (const std::exception& e) {
        return msgl::set_error(MSGL_ERR_INVALID_ARG, e.what());
    }
}

extern "C" {

int msgl_model_create(const msgl_model_config* cfg, msgl_model** out) {
    if (!cfg || !out) return msgl::set_error(MSGL_ERR_INVALID_ARG, "model_create: null");
    *out = nullptr;
    auto* mm = new msgl_model();
    int rc = guarded([&] { create(mm->m, *cfg); });
    if (rc) {
        delete mm;
        return rc;
    }
    *out = mm;
    return MSGL_OK;
}

int msgl_model_destroy(msgl_model* m) {
    delete m;
    return MSGL_OK;
}

int msgl_model_random_init(msgl_model* m, uint64_t seed, float std, msgl_stream_t stream) {
    if (!m) return msgl::set_error(MSGL_ERR_INVALID_ARG, "null model");
    return guarded([&] { random_init(m->m, seed, std, stream); });
}

int msgl_model_set_weight(msgl_model* m, const char* name, const uint16_t* host_bf16,
                          int64_t numel, msgl_stream_t stream) {
    if (!m || !name || !host_bf16) return msgl::set_error(MSGL_ERR_INVALID_ARG, "set_weight: null");
    return guarded([&] { set_weight(m->m, name, host_bf16, numel, stream); });
}

int64_t msgl_model_weight_bytes(const msgl_model* m) { return m ? m->m.weight_bytes() : 0; }

int msgl_model_get_config(const msgl_model* m, msgl_model_config* out) {
    if (!m || !out) return msgl::set_error(MSGL_ERR_INVALID_ARG, "get_config: null");
    *out = m->m.cfg;
    return MSGL_OK;
}

int msgl_model_alloc_kv(msgl_model* m, int num_pages, int page_size, msgl_stream_t stream) {
    if (!m) return msgl::set_error(MSGL_ERR_INVALID_ARG, "null model");
    return guarded([&] { alloc_kv(m->m, num_pages, page_size, stream); });
}

int msgl_model_kv_pool(msgl_model* m, int layer, void** k_pool, void** v_pool, int64_t* num_slots) {
    if (!m || layer < 0 || layer >= m->m.cfg.num_layers)
        return msgl::set_error(MSGL_ERR_INVALID_ARG, "kv_pool: layer");
    if (k_pool) *k_pool = m->m.layers[layer].k_pool.p;
    if (v_pool) *v_pool = m->m.layers[layer].v_pool.p;
    if (num_slots) *num_slots = m->m.num_slots;
    return MSGL_OK;
}

int msgl_model_forward(msgl_model* m, const msgl_batch* batch, int* next_tokens, float* logits,
                       int flags, msgl_stream_t stream) {
    if (!m || !batch || !next_tokens) return msgl::set_error(MSGL_ERR_INVALID_ARG, "forward: null");
    return guarded([&] { run(m->m, *batch, next_tokens, logits, flags, stream); });
}

int msgl_model_step_host(msgl_model* m, const msgl_batch* host_batch, int* host_next_tokens,
                         int flags, msgl_stream_t stream) {
    if (!m || !host_batch || !host_next_tokens)
        return msgl::set_error(MSGL_ERR_INVALID_ARG, "step_host: null");
    return guarded([&] { step_host(m->m, *host_batch, host_next_tokens, flags & ~MSGL_STEP_TOKENS_FROM_PREV,
                                   static_cast<cudaStream_t>(stream), true); });
}

int msgl_model_step_host_async(msgl_model* m, const msgl_batch* host_batch, int* host_next_tokens,
                               int flags, msgl_stream_t stream, uint64_t* ticket) {
    if (!m || !host_batch || !host_next_tokens)
        return msgl::set_error(MSGL_ERR_INVALID_ARG, "step_host_async: null");
    return guarded([&] {
        const uint64_t t = step_host(m->m, *host_batch, host_next_tokens, flags,
                                     static_cast<cudaStream_t>(stream), false);
        if (ticket) *ticket = t;
    });
}

int msgl_model_step_wait(msgl_model* m, uint64_t ticket) {
    if (!m) return msgl::set_error(MSGL_ERR_INVALID_ARG, "step_wait: null");
    return guarded([&] { step_wait(m->m, ticket); });
}

int msgl_model_decode_steps(msgl_model* m, const msgl_batch* batch, int num_steps, int* token_log,
                            const int* free_pages, int* free_top, int flags, msgl_stream_t stream) {
    return msgl_model_decode_steps_stop(m, batch, num_steps, token_log, free_pages, free_top,
                                        nullptr, flags, stream);
}

int msgl_model_decode_steps_stop(msgl_model* m, const msgl_batch* batch, int num_steps,
                                 int* token_log, const int* free_pages, int* free_top,
                                 const msgl_stop_rules* stop, int flags, msgl_stream_t stream) {
    if (!m || !batch || num_steps < 0 || (num_steps > 0 && (!token_log || !free_pages || !free_top)))
        return msgl::set_error(MSGL_ERR_INVALID_ARG, "decode_steps: bad args");
    if (stop && (!stop->max_new_tokens || !stop->finished || !stop->generated ||
                 stop->num_stop_ids < 0 || (stop->num_stop_ids > 0 && !stop->stop_ids)))
        return msgl::set_error(MSGL_ERR_INVALID_ARG, "decode_steps: bad stop rules");
    return guarded([&] {
        Model& md = m->m;
        if (!batch->is_decode || batch->num_tokens != batch->num_reqs)
            throw Fail(MSGL_ERR_INVALID_ARG, "decode_steps: needs a decode batch");
        // every step runs with the same shape fields, so a captured graph serves them all; the
        // context bound is the page-table width (the advance kernel refuses to go past it)
        msgl_batch b = *batch;
        b.max_seq_len = std::min(b.max_pages * md.page_size, md.cfg.max_position);
        const int B = b.num_reqs;
        int* next = md.dec_next.as<int>();
        auto* s = static_cast<cudaStream_t>(stream);
        for (int st = 0; st < num_steps; ++st) {
            run(md, b, next, nullptr, flags & MSGL_FWD_GRAPH, s);
            int* row = token_log + static_cast<int64_t>(st) * B;
            if (stop)  // finish rules: the log gets the token, or -1 once a request finished
                ck(msgl_decode_finish(next, row, stop->max_new_tokens, stop->ignore_eos,
                                      stop->stop_ids, stop->num_stop_ids, stop->finished,
                                      stop->generated, B, stream),
                   "decode_steps: finish");
            else
                ckc(cudaMemcpyAsync(row, next, sizeof(int) * B, cudaMemcpyDeviceToDevice, s),
                    "decode_steps: token log");
            if (st + 1 < num_steps)  // the arrays of *batch are advanced in place
                ck(msgl_decode_advance_masked(next, const_cast<int*>(b.input_ids), const_cast<int*>(b.positions),
                                              const_cast<int*>(b.slot_mapping), const_cast<int*>(b.page_table),
                                              b.max_pages, const_cast<int*>(b.seq_lens), free_pages,
                                              free_top, stop ? stop->finished : nullptr, B,
                                              md.page_size, stream),
                   "decode_steps: advance");
        }
    });
}

int msgl_model_debug_hidden(msgl_model* m, void** x, float** residual) {
    if (!m) return msgl::set_error(MSGL_ERR_INVALID_ARG, "null model");
    if (x) *x = m->m.x.p;
    if (residual) *residual = m->m.residual.as<float>();
    return MSGL_OK;
}

int msgl_model_set_tp(msgl_model* m, msgl_tp* tp) {
    if (!m) return msgl::set_error(MSGL_ERR_INVALID_ARG, "null model");
    const int world = tp ? msgl_tp_world(tp) : 1;
    if (world != m->m.cfg.tp_size || (tp && msgl_tp_rank(tp) != m->m.cfg.tp_rank))
        return msgl::set_error(MSGL_ERR_INVALID_ARG, "set_tp: communicator rank/world differ from the config");
    m->m.tp = nullptr;
    m->m.tp_part[0] = m->m.tp_part[1] = nullptr;
    m->m.tp_x = nullptr;
    if (world > 1) {  // collective: every rank of the communicator calls set_tp
        const size_t need = static_cast<size_t>(m->m.cfg.max_tokens) * m->m.cfg.hidden * 2;
        void* buf[2] = {nullptr, nullptr};
        size_t have = 0;
        if (msgl_tp_p2p_buffer(tp, 0, &buf[0], &have) != MSGL_OK) {
            const int rc = msgl_tp_enable_p2p(tp, need, nullptr);
            if (rc) return rc;
            msgl_tp_p2p_buffer(tp, 0, &buf[0], &have);
        }
        msgl_tp_p2p_buffer(tp, 1, &buf[1], &have);
        if (have < need) return msgl::set_error(MSGL_ERR_WORKSPACE, "set_tp: peer-mapped region too small");
        const int vpad = (m->m.cfg.vocab + world - 1) / world;
        const size_t chunk = static_cast<size_t>(m->m.cfg.max_reqs) * vpad * sizeof(float);
        const int rc = guarded([&] {
            m->m.tp_logits_local.alloc(chunk);
            m->m.tp_logits_all.alloc(chunk * world);
        });
        if (rc) return rc;
        m->m.tp = tp;
        m->m.tp_part[0] = static_cast<bf16_t*>(buf[0]);
        m->m.tp_part[1] = static_cast<bf16_t*>(buf[1]);
        // all-reduce form: two-shot from 8 ranks on (each rank reduces T / world rows), one-shot
        // below (Qwen3-8B decode at batch 128 on B200: TP8 3.80 ms two-shot vs 4.07 one-shot,
        // TP4 4.53 ms one-shot vs 4.81 two-shot); MSGL_TP_ALLREDUCE=1 or 2 forces one
        const char* env = std::getenv("MSGL_TP_ALLREDUCE");
        const bool two = env && (env[0] == '1' || env[0] == '2') ? env[0] == '2' : world >= 8;
        if (two) {
            void* xs = nullptr;
            msgl_tp_p2p_buffer(tp, 2, &xs, &have);
            m->m.tp_x = static_cast<bf16_t*>(xs);
        }
        m->m.graphs_reset();
    }
    return MSGL_OK;
}

int msgl_model_set_num_layers_run(msgl_model* m, int n) {
    if (!m) return msgl::set_error(MSGL_ERR_INVALID_ARG, "null model");
    m->m.layers_run = n;
    return MSGL_OK;
}

}  // extern "C"
