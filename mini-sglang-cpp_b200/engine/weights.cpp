// weights.cpp -- safetensors checkpoint ingest for the executor.
//
// WeightLoader (src/model/weight.cpp:32-105) indexes every *.safetensors file of a model
// directory by its JSON header (8-byte little-endian header size, then a JSON object
// name -> {dtype, shape, data_offsets}; data follows the header) and reads a tensor's bytes on
// demand. Qwen3ForCausalLM::load_weights (src/model/qwen3.cpp:94-166) and
// Qwen3MoEForCausalLM::load_weights (src/model/qwen3_moe.cpp:123-199) map the Hugging Face names
// onto the layers, concatenating q | k | v and gate | up rows when the checkpoint stores them
// separately. This file does the same through the executor's public ABI
// (msgl_model_set_weight: full tensors, host bf16; the executor keeps its tensor-parallel shard)
// with three differences, all deliberate: F32 / F16 tensors are rounded to bf16 (nearest even)
// instead of copied as raw bytes into an fp32 tensor; the Qwen3 per-head norms
// (self_attn.q_norm / k_norm, which the reference never loads) are loaded; a missing
// lm_head.weight falls back to the embedding (tied embeddings). A tensor the executor needs and
// the checkpoint lacks is an error, not a silently uninitialised weight.
#include <dirent.h>

#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "msgl_engine.h"

namespace msgl {
int set_error(int code, const char* msg);

namespace {

// ------------------------------------------------------------------ minimal JSON reader
// Enough of RFC 8259 for safetensors headers: objects, arrays, strings (escapes, \u to UTF-8),
// integers / numbers, true / false / null.
struct JVal {
    enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
    bool b = false;
    double num = 0;
    int64_t inum = 0;
    bool is_int = false;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal* get(const std::string& k) const {
        for (auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

class JReader {
  public:
    JReader(const char* p, const char* e) : p_(p), e_(e) {}
    JVal parse() {
        JVal v = value();
        ws();
        if (p_ != e_) fail("trailing characters");
        return v;
    }

  private:
    const char *p_, *e_;
    int depth_ = 0;
    [[noreturn]] void fail(const char* what) {
        throw std::runtime_error(std::string("safetensors header: ") + what);
    }
    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    char peek() {
        ws();
        if (p_ >= e_) fail("unexpected end");
        return *p_;
    }
    void expect(char c) {
        if (peek() != c) fail("unexpected character");
        ++p_;
    }
    JVal value() {
        if (++depth_ > 64) fail("nesting too deep");
        JVal v;
        const char c = peek();
        if (c == '{') {
            v.kind = JVal::kObj;
            ++p_;
            if (peek() == '}') {
                ++p_;
            } else {
                for (;;) {
                    if (peek() != '"') fail("object key");
                    std::string k = string();
                    expect(':');
                    v.obj.emplace_back(std::move(k), value());
                    const char d = peek();
                    ++p_;
                    if (d == '}') break;
                    if (d != ',') fail("object separator");
                }
            }
        } else if (c == '[') {
            v.kind = JVal::kArr;
            ++p_;
            if (peek() == ']') {
                ++p_;
            } else {
                for (;;) {
                    v.arr.push_back(value());
                    const char d = peek();
                    ++p_;
                    if (d == ']') break;
                    if (d != ',') fail("array separator");
                }
            }
        } else if (c == '"') {
            v.kind = JVal::kStr;
            v.str = string();
        } else if (c == 't' || c == 'f' || c == 'n') {
            static const char* words[3] = {"true", "false", "null"};
            const int w = c == 't' ? 0 : c == 'f' ? 1 : 2;
            const size_t n = std::strlen(words[w]);
            if (static_cast<size_t>(e_ - p_) < n || std::strncmp(p_, words[w], n)) fail("literal");
            p_ += n;
            v.kind = w == 2 ? JVal::kNull : JVal::kBool;
            v.b = w == 0;
        } else {
            number(v);
        }
        --depth_;
        return v;
    }
    void number(JVal& v) {
        const char* s = p_;
        bool integral = true;
        while (p_ < e_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                           *p_ == '-' || *p_ == '+')) {
            if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') integral = false;
            ++p_;
        }
        if (p_ == s) fail("value");
        const std::string tok(s, p_);
        v.kind = JVal::kNum;
        v.is_int = integral;
        try {
            v.num = std::stod(tok);
            if (integral) v.inum = std::stoll(tok);
        } catch (...) {
            fail("number");
        }
    }
    static void utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) {
            out += static_cast<char>(cp);
        } else if (cp < 0x800) {
            out += static_cast<char>(0xC0 | (cp >> 6));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += static_cast<char>(0xE0 | (cp >> 12));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else {
            out += static_cast<char>(0xF0 | (cp >> 18));
            out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        }
    }
    uint32_t hex4() {
        if (e_ - p_ < 4) fail("\\u escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i, ++p_) {
            const char h = *p_;
            v <<= 4;
            if (h >= '0' && h <= '9') v |= h - '0';
            else if (h >= 'a' && h <= 'f') v |= h - 'a' + 10;
            else if (h >= 'A' && h <= 'F') v |= h - 'A' + 10;
            else fail("\\u escape");
        }
        return v;
    }
    std::string string() {
        expect('"');
        std::string out;
        for (;;) {
            if (p_ >= e_) fail("unterminated string");
            const char c = *p_++;
            if (c == '"') break;
            if (c != '\\') {
                out += c;
                continue;
            }
            if (p_ >= e_) fail("escape");
            const char x = *p_++;
            switch (x) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00 && e_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                        p_ += 2;
                        const uint32_t lo = hex4();
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(out, cp);
                    break;
                }
                default: fail("escape");
            }
        }
        return out;
    }
};

// ------------------------------------------------------------------ checkpoint index
struct TensorInfo {
    std::string file, dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // absolute byte offsets in the file
    int64_t numel() const {
        int64_t n = 1;
        for (int64_t d : shape) n *= d;
        return n;
    }
};

int dtype_bytes(const std::string& d) {
    if (d == "BF16" || d == "F16") return 2;
    if (d == "F32") return 4;
    return 0;  // not a weight dtype this loader converts
}

void index_file(const std::string& path, std::map<std::string, TensorInfo>& out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open " + path);
    f.seekg(0, std::ios::end);
    const uint64_t fsize = static_cast<uint64_t>(f.tellg());
    f.seekg(0);
    if (fsize < 8) throw std::runtime_error(path + ": no header size");
    unsigned char b8[8];
    if (!f.read(reinterpret_cast<char*>(b8), 8)) throw std::runtime_error(path + ": no header size");
    uint64_t hsize = 0;
    for (int i = 7; i >= 0; --i) hsize = (hsize << 8) | b8[i];  // little-endian
    if (hsize == 0 || hsize > fsize - 8 || hsize > (256ull << 20))
        throw std::runtime_error(path + ": bad header size");
    std::string hdr(hsize, '\0');
    if (!f.read(&hdr[0], static_cast<std::streamsize>(hsize)))
        throw std::runtime_error(path + ": short header");
    const JVal root = JReader(hdr.data(), hdr.data() + hdr.size()).parse();
    if (root.kind != JVal::kObj) throw std::runtime_error(path + ": header is not an object");
    const uint64_t base = 8 + hsize;
    for (auto& kv : root.obj) {
        if (kv.first == "__metadata__") continue;
        const JVal& t = kv.second;
        const JVal* dt = t.get("dtype");
        const JVal* sh = t.get("shape");
        const JVal* off = t.get("data_offsets");
        if (t.kind != JVal::kObj || !dt || dt->kind != JVal::kStr || !sh || sh->kind != JVal::kArr ||
            !off || off->kind != JVal::kArr || off->arr.size() != 2)
            throw std::runtime_error(path + ": malformed entry " + kv.first);
        TensorInfo info;
        info.file = path;
        info.dtype = dt->str;
        for (auto& d : sh->arr) {
            if (d.kind != JVal::kNum || !d.is_int || d.inum < 0)
                throw std::runtime_error(path + ": bad shape of " + kv.first);
            info.shape.push_back(d.inum);
        }
        const JVal &o0 = off->arr[0], &o1 = off->arr[1];
        if (o0.kind != JVal::kNum || o1.kind != JVal::kNum || !o0.is_int || !o1.is_int ||
            o0.inum < 0 || o1.inum < o0.inum)
            throw std::runtime_error(path + ": bad data_offsets of " + kv.first);
        info.begin = base + static_cast<uint64_t>(o0.inum);
        info.end = base + static_cast<uint64_t>(o1.inum);
        if (info.end > fsize) throw std::runtime_error(path + ": data of " + kv.first + " past the end");
        const int eb = dtype_bytes(info.dtype);
        if (eb && static_cast<uint64_t>(info.numel()) * eb != info.end - info.begin)
            throw std::runtime_error(path + ": size of " + kv.first + " does not match its shape");
        out[kv.first] = std::move(info);
    }
}

std::map<std::string, TensorInfo> index_dir(const std::string& dir) {
    std::map<std::string, TensorInfo> idx;
    DIR* d = opendir(dir.c_str());
    if (!d) throw std::runtime_error("cannot open model directory " + dir);
    std::vector<std::string> files;
    while (dirent* e = readdir(d)) {
        const std::string n = e->d_name;
        if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0)
            files.push_back(dir + "/" + n);
    }
    closedir(d);
    if (files.empty()) throw std::runtime_error("no .safetensors file in " + dir);
    for (auto& f : files) index_file(f, idx);
    return idx;
}

uint16_t f32_to_bf16(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu))
        return static_cast<uint16_t>((u >> 16) | 0x40);  // NaN stays NaN
    u += 0x7FFFu + ((u >> 16) & 1u);                   // round to nearest even
    return static_cast<uint16_t>(u >> 16);
}

float f16_to_f32(uint16_t h) {
    const uint32_t s = static_cast<uint32_t>(h & 0x8000u) << 16, e = (h >> 10) & 0x1F, m = h & 0x3FF;
    uint32_t u;
    if (e == 0) {
        if (m == 0) {
            u = s;
        } else {  // subnormal: normalise
            int sh = 0;
            uint32_t mm = m;
            while (!(mm & 0x400)) {
                mm <<= 1;
                ++sh;
            }
            u = s | static_cast<uint32_t>(127 - 15 - sh + 1) << 23 | (mm & 0x3FF) << 13;
        }
    } else if (e == 31) {
        u = s | 0x7F800000u | m << 13;
    } else {
        u = s | (e + 127 - 15) << 23 | m << 13;
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// Appends the tensor's values, as bf16 bit patterns, to `out`.
void read_bf16(const TensorInfo& t, const std::string& name, std::vector<uint16_t>& out) {
    const int eb = dtype_bytes(t.dtype);
    if (!eb) throw std::runtime_error(name + ": dtype " + t.dtype + " is not BF16 / F16 / F32");
    std::ifstream f(t.file, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open " + t.file);
    f.seekg(static_cast<std::streamoff>(t.begin));
    const size_t n = static_cast<size_t>(t.numel());
    const size_t at = out.size();
    out.resize(at + n);
    if (t.dtype == "BF16") {
        if (!f.read(reinterpret_cast<char*>(out.data() + at), static_cast<std::streamsize>(n * 2)))
            throw std::runtime_error(name + ": short read");
        return;
    }
    std::vector<char> raw(n * eb);
    if (!f.read(raw.data(), static_cast<std::streamsize>(raw.size())))
        throw std::runtime_error(name + ": short read");
    for (size_t i = 0; i < n; ++i) {
        if (t.dtype == "F32") {
            float x;
            std::memcpy(&x, raw.data() + 4 * i, 4);
            out[at + i] = f32_to_bf16(x);
        } else {
            uint16_t h;
            std::memcpy(&h, raw.data() + 2 * i, 2);
            out[at + i] = f32_to_bf16(f16_to_f32(h));
        }
    }
}

struct Loader {
    msgl_model* m;
    msgl_stream_t s;
    const std::map<std::string, TensorInfo>& idx;
    const TensorInfo* find(const std::string& n) const {
        auto it = idx.find(n);
        return it == idx.end() ? nullptr : &it->second;
    }
    // rows of the listed tensors, concatenated (q | k | v, gate | up), into executor tensor `dst`
    void put(const std::string& dst, const std::vector<std::string>& parts) {
        std::vector<uint16_t> buf;
        for (auto& p : parts) {
            const TensorInfo* t = find(p);
            if (!t) throw std::runtime_error("checkpoint lacks " + p);
            read_bf16(*t, p, buf);
        }
        const int rc = msgl_model_set_weight(m, dst.c_str(), buf.data(),
                                             static_cast<int64_t>(buf.size()), s);
        if (rc != MSGL_OK)
            throw std::runtime_error(std::string("set_weight ") + dst + ": " + msgl_last_error());
    }
    // a fused tensor if the checkpoint has one, else its separate parts
    void fused(const std::string& dst, const std::string& whole, const std::vector<std::string>& parts) {
        if (find(whole)) put(dst, {whole});
        else put(dst, parts);
    }
};

template <typename F>
int guarded(F&& f) {
    try {
        return f();
    } catch (const std::exception& e) {
        return set_error(MSGL_ERR_INVALID_ARG, e.what());
    }
}

}  // namespace
}  // namespace msgl

using namespace msgl;

extern "C" {

int msgl_safetensors_index(const char* model_dir, int64_t* num_tensors, int64_t* total_bytes) {
    if (!model_dir) return set_error(MSGL_ERR_INVALID_ARG, "safetensors_index: null directory");
    return guarded([&] {
        const auto idx = index_dir(model_dir);
        int64_t bytes = 0;
        for (auto& kv : idx) bytes += static_cast<int64_t>(kv.second.end - kv.second.begin);
        if (num_tensors) *num_tensors = static_cast<int64_t>(idx.size());
        if (total_bytes) *total_bytes = bytes;
        return static_cast<int>(MSGL_OK);
    });
}

int msgl_model_load_safetensors(msgl_model* m, const char* model_dir, msgl_stream_t stream) {
    if (!m || !model_dir) return set_error(MSGL_ERR_INVALID_ARG, "load_safetensors: null");
    msgl_model_config c;
    const int rc = msgl_model_get_config(m, &c);
    if (rc) return rc;
    return guarded([&] {
        const auto idx = index_dir(model_dir);
        Loader L{m, stream, idx};
        L.put("embed", {"model.embed_tokens.weight"});
        L.put("norm", {"model.norm.weight"});
        L.put("lm_head", {L.find("lm_head.weight") ? "lm_head.weight" : "model.embed_tokens.weight"});
        for (int l = 0; l < c.num_layers; ++l) {
            const std::string p = "model.layers." + std::to_string(l) + ".";
            const std::string q = "layers." + std::to_string(l) + ".";
            L.put(q + "input_ln", {p + "input_layernorm.weight"});
            L.put(q + "post_ln", {p + "post_attention_layernorm.weight"});
            L.fused(q + "qkv", p + "self_attn.qkv_proj.weight",
                    {p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                     p + "self_attn.v_proj.weight"});
            L.put(q + "q_norm", {p + "self_attn.q_norm.weight"});
            L.put(q + "k_norm", {p + "self_attn.k_norm.weight"});
            L.put(q + "o", {p + "self_attn.o_proj.weight"});
            if (c.num_experts > 0) {
                L.put(q + "router", {p + "mlp.gate.weight"});
                for (int e = 0; e < c.num_experts; ++e) {
                    const std::string ep = p + "mlp.experts." + std::to_string(e) + ".";
                    const std::string eq = q + "experts." + std::to_string(e) + ".";
                    L.fused(eq + "gate_up", ep + "gate_up_proj.weight",
                            {ep + "gate_proj.weight", ep + "up_proj.weight"});
                    L.put(eq + "down", {ep + "down_proj.weight"});
                }
            } else {
                L.fused(q + "gate_up", p + "mlp.gate_up_proj.weight",
                        {p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"});
                L.put(q + "down", {p + "mlp.down_proj.weight"});
            }
        }
        return static_cast<int>(MSGL_OK);
    });
}

}  // extern "C"
