// rope.cu -- RoPE, KV page store, and the fused QK-norm + RoPE + KV-page-store kernel.
//
//  * msgl_launch_rope            launch_rope          (kernels/cuda/rotary.cu:43-51), math of
//                                RotaryEmbedding::forward (src/layer/layer.cpp:191-198)
//  * msgl_launch_store_kv_page   launch_store_kv_page (kernels/cuda/radix.cu:28-36)
//  * msgl_qknorm_rope_store_kv   split (src/model/qwen3.cpp:28-45) + per-head RMSNorm over D
//                                (layer.cpp:57-69 with size D) + RoPE + pool store, one pass.
#include "common.cuh"

namespace msgl {
namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p);
template <>
__device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
    return __bfloat162float(*p);
}
__device__ __forceinline__ void st(float* p, float v) { *p = v; }
__device__ __forceinline__ void st(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// One thread per (token, head, d < D/2) over q then k, as rotary.cu:17-34 but with each tensor's
// own head count.
template <typename T>
__global__ void rope_kernel(T* __restrict__ q, T* __restrict__ k, const int* __restrict__ pos,
                            const float* __restrict__ cs_table, int num_tokens, int hq, int hkv,
                            int head_dim) {
    int half = head_dim / 2;
    int64_t nq = static_cast<int64_t>(num_tokens) * hq * half;
    int64_t nk = k ? static_cast<int64_t>(num_tokens) * hkv * half : 0;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < nq + nk;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        bool is_q = idx < nq;
        int64_t i = is_q ? idx : idx - nq;
        int heads = is_q ? hq : hkv;
        int d = static_cast<int>(i % half);
        int64_t th = i / half;  // token * heads + head
        int t = static_cast<int>(th / heads);
        T* x = (is_q ? q : k) + th * head_dim;
        const float* cs = cs_table + static_cast<int64_t>(pos[t]) * head_dim;
        float c = cs[d], s = cs[half + d];
        float x0 = ld(x + d), x1 = ld(x + half + d);
        st(x + d, x0 * c - x1 * s);
        st(x + half + d, x0 * s + x1 * c);
    }
}

template <typename T>
__global__ void store_kv_page_kernel(const T* __restrict__ k, const T* __restrict__ v,
                                     T* __restrict__ kc, T* __restrict__ vc,
                                     const int* __restrict__ page_table, int page_size,
                                     int64_t row, int num_tokens) {
    int64_t total = static_cast<int64_t>(num_tokens) * row;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int t = static_cast<int>(idx / row);
        int64_t hd = idx % row;
        int64_t dst = (static_cast<int64_t>(page_table[t / page_size]) * page_size +
                       t % page_size) * row + hd;
        kc[dst] = k[idx];
        vc[dst] = v[idx];
    }
}

// One warp per (token, head) of the fused QKV row; head_dim 128: lane l owns elements
// {2l, 2l+1} of the first half and {64+2l, 64+2l+1} of the second (the rotate-half partners).
// PARTS: the row is the sum, in split order, of `nparts` fp32 split-K partials of the QKV
// projection ([nparts][T][(Hq + 2 Hkv) D]) instead of one bf16 row.
constexpr int kQkvWarps = 8;

template <bool PARTS>
__global__ void __launch_bounds__(kQkvWarps * 32)
qknorm_rope_store_kernel(const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ parts,
                         int nparts, __nv_bfloat16* __restrict__ q_out,
                         __nv_bfloat16* __restrict__ k_pool, __nv_bfloat16* __restrict__ v_pool,
                         int64_t num_slots, const int* __restrict__ positions,
                         const int* __restrict__ slots, const float* __restrict__ cs_table,
                         const __nv_bfloat16* __restrict__ qn, const __nv_bfloat16* __restrict__ kn,
                         int num_tokens, int hq, int hkv, float eps, int* err) {
    pdl_wait();
    pdl_trigger();
    const int nh = hq + 2 * hkv;
    const int lane = threadIdx.x & 31;
    const int64_t wid = static_cast<int64_t>(blockIdx.x) * kQkvWarps + (threadIdx.x >> 5);
    if (wid >= static_cast<int64_t>(num_tokens) * nh) return;
    const int t = static_cast<int>(wid / nh);
    const int h = static_cast<int>(wid % nh);
    float a0, a1, b0, b1;
    if (PARTS) {
        const int64_t stride = static_cast<int64_t>(num_tokens) * nh * 128;
        const float* src = parts + wid * 128;
        float2 pa = make_float2(0.f, 0.f), pb = make_float2(0.f, 0.f);
        int p = 0;
        for (; p + 4 <= nparts; p += 4) {  // four partials' loads in flight, added in order
            float2 ta[4], tb[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                ta[u] = *reinterpret_cast<const float2*>(src + (p + u) * stride + 2 * lane);
                tb[u] = *reinterpret_cast<const float2*>(src + (p + u) * stride + 64 + 2 * lane);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                pa.x += ta[u].x; pa.y += ta[u].y; pb.x += tb[u].x; pb.y += tb[u].y;
            }
        }
        for (; p < nparts; ++p) {
            const float2 ta = *reinterpret_cast<const float2*>(src + p * stride + 2 * lane);
            const float2 tb = *reinterpret_cast<const float2*>(src + p * stride + 64 + 2 * lane);
            pa.x += ta.x; pa.y += ta.y; pb.x += tb.x; pb.y += tb.y;
        }
        a0 = pa.x; a1 = pa.y; b0 = pb.x; b1 = pb.y;
    } else {
        const __nv_bfloat16* src = qkv + wid * 128;
        uint32_t ua = *reinterpret_cast<const uint32_t*>(src + 2 * lane);
        uint32_t ub = *reinterpret_cast<const uint32_t*>(src + 64 + 2 * lane);
        a0 = bf16lo(ua); a1 = bf16hi(ua); b0 = bf16lo(ub); b1 = bf16hi(ub);
    }

    __nv_bfloat16* dst;
    if (h < hq + hkv) {
        // RMSNorm over the head (RMSNorm(D, eps), layer.cpp:57-69)
        float ss = warp_sum(a0 * a0 + a1 * a1 + b0 * b0 + b1 * b1);
        float inv = 1.0f / sqrtf(ss / 128.0f + eps);
        const __nv_bfloat16* w = h < hq ? qn : kn;
        uint32_t wa = *reinterpret_cast<const uint32_t*>(w + 2 * lane);
        uint32_t wb = *reinterpret_cast<const uint32_t*>(w + 64 + 2 * lane);
        a0 = a0 * inv * bf16lo(wa);
        a1 = a1 * inv * bf16hi(wa);
        b0 = b0 * inv * bf16lo(wb);
        b1 = b1 * inv * bf16hi(wb);
        // rotate-half RoPE (layer.cpp:191-198)
        const float* cs = cs_table + static_cast<int64_t>(positions[t]) * 128;
        float2 c = *reinterpret_cast<const float2*>(cs + 2 * lane);
        float2 s = *reinterpret_cast<const float2*>(cs + 64 + 2 * lane);
        float r0 = a0 * c.x - b0 * s.x, r1 = a1 * c.y - b1 * s.y;
        float r2 = a0 * s.x + b0 * c.x, r3 = a1 * s.y + b1 * c.y;
        a0 = r0; a1 = r1; b0 = r2; b1 = r3;
        if (h < hq) {
            dst = q_out + (static_cast<int64_t>(t) * hq + h) * 128;
        } else {
            int64_t slot = slots[t];
            if (slot < 0) return;
            if (slot >= num_slots) {
                if (lane == 0) record_error(err, MSGL_ERR_BOUNDS, 100);
                return;
            }
            dst = k_pool + (slot * hkv + (h - hq)) * 128;
        }
    } else {
        int64_t slot = slots[t];
        if (slot < 0) return;
        if (slot >= num_slots) {
            if (lane == 0) record_error(err, MSGL_ERR_BOUNDS, 101);
            return;
        }
        dst = v_pool + (slot * hkv + (h - hq - hkv)) * 128;
    }
    *reinterpret_cast<uint32_t*>(dst + 2 * lane) = pack_bf16x2(a0, a1);
    *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = pack_bf16x2(b0, b1);
}

int grid_for(int64_t n, int threads) {
    int64_t b = (n + threads - 1) / threads;
    return static_cast<int>(b > 148 * 32 ? 148 * 32 : (b < 1 ? 1 : b));
}

}  // namespace
}  // namespace msgl

using namespace msgl;

extern "C" {

int msgl_launch_rope(void* query, void* key, const int* positions, const float* cos_sin_cache,
                     int num_tokens, int num_q_heads, int num_kv_heads, int head_dim, int dtype,
                     msgl_stream_t stream) {
    if (num_tokens < 0 || head_dim <= 0 || head_dim % 2 || num_q_heads <= 0 ||
        (key && num_kv_heads <= 0))
        return set_error(MSGL_ERR_INVALID_ARG, "rope: bad sizes");
    if (num_tokens == 0) return MSGL_OK;
    int64_t n = static_cast<int64_t>(num_tokens) * (num_q_heads + (key ? num_kv_heads : 0)) *
                (head_dim / 2);
    if (dtype == MSGL_BF16)
        rope_kernel<__nv_bfloat16><<<grid_for(n, 256), 256, 0, stream>>>(
            static_cast<__nv_bfloat16*>(query), static_cast<__nv_bfloat16*>(key), positions,
            cos_sin_cache, num_tokens, num_q_heads, num_kv_heads, head_dim);
    else if (dtype == MSGL_F32)
        rope_kernel<float><<<grid_for(n, 256), 256, 0, stream>>>(
            static_cast<float*>(query), static_cast<float*>(key), positions, cos_sin_cache,
            num_tokens, num_q_heads, num_kv_heads, head_dim);
    else
        return set_error(MSGL_ERR_INVALID_ARG, "rope: unknown dtype");
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

int msgl_launch_store_kv_page(const void* k, const void* v, void* k_cache, void* v_cache,
                              const int* page_table, int page_size, int num_heads, int head_dim,
                              int num_tokens, int dtype, msgl_stream_t stream) {
    if (num_tokens < 0 || page_size <= 0 || num_heads <= 0 || head_dim <= 0)
        return set_error(MSGL_ERR_INVALID_ARG, "store_kv_page: bad sizes");
    if (num_tokens == 0) return MSGL_OK;
    int64_t row = static_cast<int64_t>(num_heads) * head_dim;
    int64_t n = row * num_tokens;
    if (dtype == MSGL_BF16)
        store_kv_page_kernel<__nv_bfloat16><<<grid_for(n, 256), 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v),
            static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), page_table,
            page_size, row, num_tokens);
    else if (dtype == MSGL_F32)
        store_kv_page_kernel<float><<<grid_for(n, 256), 256, 0, stream>>>(
            static_cast<const float*>(k), static_cast<const float*>(v),
            static_cast<float*>(k_cache), static_cast<float*>(v_cache), page_table, page_size, row,
            num_tokens);
    else
        return set_error(MSGL_ERR_INVALID_ARG, "store_kv_page: unknown dtype");
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

static int launch_qknorm_rope(const void* qkv, const float* parts, int nparts, void* q_out,
                              void* k_pool, void* v_pool, int64_t num_slots, const int* positions,
                              const int* slot_mapping, const float* cos_sin_cache,
                              const void* q_norm_w, const void* k_norm_w, int num_tokens,
                              int num_q_heads, int num_kv_heads, int head_dim, float eps,
                              msgl_stream_t stream) {
    if (head_dim != 128) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "qknorm_rope: head_dim != 128");
    if (num_tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0)
        return set_error(MSGL_ERR_INVALID_ARG, "qknorm_rope: bad sizes");
    if (num_tokens == 0) return MSGL_OK;
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    int64_t warps = static_cast<int64_t>(num_tokens) * (num_q_heads + 2 * num_kv_heads);
    int blocks = static_cast<int>((warps + kQkvWarps - 1) / kQkvWarps);
    auto kern = parts ? qknorm_rope_store_kernel<true> : qknorm_rope_store_kernel<false>;
    launch_pdl(kern, dim3(blocks), dim3(kQkvWarps * 32), 0, stream,
        static_cast<const __nv_bfloat16*>(qkv), parts, nparts, static_cast<__nv_bfloat16*>(q_out),
        static_cast<__nv_bfloat16*>(k_pool), static_cast<__nv_bfloat16*>(v_pool), num_slots,
        positions, slot_mapping, cos_sin_cache, static_cast<const __nv_bfloat16*>(q_norm_w),
        static_cast<const __nv_bfloat16*>(k_norm_w), num_tokens, num_q_heads, num_kv_heads, eps,
        err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

int msgl_qknorm_rope_store_kv(const void* qkv, void* q_out, void* k_pool, void* v_pool,
                              int64_t num_slots, const int* positions, const int* slot_mapping,
                              const float* cos_sin_cache, const void* q_norm_w,
                              const void* k_norm_w, int num_tokens, int num_q_heads,
                              int num_kv_heads, int head_dim, float eps, msgl_stream_t stream) {
    return launch_qknorm_rope(qkv, nullptr, 0, q_out, k_pool, v_pool, num_slots, positions,
                              slot_mapping, cos_sin_cache, q_norm_w, k_norm_w, num_tokens,
                              num_q_heads, num_kv_heads, head_dim, eps, stream);
}

int msgl_qknorm_rope_store_kv_partials(const float* parts, int nparts, void* q_out, void* k_pool,
                                       void* v_pool, int64_t num_slots, const int* positions,
                                       const int* slot_mapping, const float* cos_sin_cache,
                                       const void* q_norm_w, const void* k_norm_w, int num_tokens,
                                       int num_q_heads, int num_kv_heads, int head_dim, float eps,
                                       msgl_stream_t stream) {
    if (head_dim != 128) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "qknorm_rope: head_dim != 128");
    if (!parts || nparts < 1 || nparts > 64)
        return set_error(MSGL_ERR_INVALID_ARG, "qknorm_rope_partials: parts / nparts in [1, 64]");
    if (reinterpret_cast<uintptr_t>(parts) & 7)
        return set_error(MSGL_ERR_INVALID_ARG, "qknorm_rope_partials: parts must be 8-byte aligned");
    return launch_qknorm_rope(nullptr, parts, nparts, q_out, k_pool, v_pool, num_slots, positions,
                              slot_mapping, cos_sin_cache, q_norm_w, k_norm_w, num_tokens,
                              num_q_heads, num_kv_heads, head_dim, eps, stream);
}

}  // extern "C"
