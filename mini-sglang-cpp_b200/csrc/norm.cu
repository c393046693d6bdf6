// norm.cu -- RMSNorm family and the embedding gather.
//
//  * msgl_launch_rmsnorm      RMSNorm::forward            (src/layer/layer.cpp:48-77)
//  * msgl_add_rmsnorm         RMSNorm::forward_fused_add  (src/layer/layer.cpp:79-112)
//  * msgl_embed_rmsnorm       Embedding::forward + the first layer's fused norm
//  * msgl_launch_index_gather launch_index_gather         (kernels/cuda/index.cu:21-28)
//
// One 128-thread CTA per token row; each thread owns up to 8 row vectors of 8 elements
// (16-byte bf16 loads, fp32 math), the row's sum of squares is a warp-shuffle + shared-memory
// reduction. Bound: HBM (a few bytes per element, no reuse).
#include "common.cuh"

namespace msgl {
namespace {

constexpr int kNormThreads = 128;

__device__ __forceinline__ float block_sum_128(float v, float* red) {
    v = warp_sum(v);
    int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float s = red[0] + red[1] + red[2] + red[3];
    __syncthreads();
    return s;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    v[0] = bf16lo(u.x); v[1] = bf16hi(u.x); v[2] = bf16lo(u.y); v[3] = bf16hi(u.y);
    v[4] = bf16lo(u.z); v[5] = bf16hi(u.z); v[6] = bf16lo(u.w); v[7] = bf16hi(u.w);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]); u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]); u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
    float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// MODE 0: y = rmsnorm(x)                        (x, w, y of type T)
// MODE 1: r += x; x = rmsnorm(r)                (x bf16 in/out, r fp32 in/out)
// MODE 2: r = x;  x = rmsnorm(x)                (first fused call)
// MODE 3: r = E[id]; x = rmsnorm(r)             (embedding + first norm; x = E (bf16) rows)
template <typename T, int MODE, int VPT>
__global__ void __launch_bounds__(kNormThreads)
rmsnorm_kernel(const T* x_in, T* x_out, float* __restrict__ resid,
               const T* __restrict__ w, const int* __restrict__ ids, int vocab, int hidden,
               float eps) {
    __shared__ float red[4];
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x;
    const int nvec = hidden >> 3;
    const T* src = x_in + static_cast<int64_t>(row) * hidden;
    bool zero_row = false;
    if (MODE == 3) {
        int id = ids[row];
        zero_row = (id < 0 || id >= vocab);
        src = x_in + static_cast<int64_t>(zero_row ? 0 : id) * hidden;
    }
    float v[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        int vi = threadIdx.x + i * kNormThreads;
        if (vi < nvec) {
            load8(src + vi * 8, v[i]);
            if (MODE == 3 && zero_row) {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
            }
            if (MODE == 1) {
                float r[8];
                load8(resid + static_cast<int64_t>(row) * hidden + vi * 8, r);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] += r[j];
            }
            if (MODE >= 1) store8(resid + static_cast<int64_t>(row) * hidden + vi * 8, v[i]);
#pragma unroll
            for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
        }
    }
    ss = block_sum_128(ss, red);
    const float inv_rms = 1.0f / sqrtf(ss / static_cast<float>(hidden) + eps);
    T* dst = x_out + static_cast<int64_t>(row) * hidden;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        int vi = threadIdx.x + i * kNormThreads;
        if (vi < nvec) {
            float wv[8], o[8];
            load8(w + vi * 8, wv);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv_rms * wv[j];
            store8(dst + vi * 8, o);
        }
    }
}

template <typename T, int MODE>
int launch_norm(const T* x_in, T* x_out, float* resid, const T* w, const int* ids, int vocab,
                int num_tokens, int hidden, float eps, cudaStream_t stream) {
    if (num_tokens < 0 || hidden <= 0 || hidden % 8 != 0 || hidden > 8 * 8 * kNormThreads)
        return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "rmsnorm: hidden must be a multiple of 8, <= 8192");
    if (num_tokens == 0) return MSGL_OK;
    if ((reinterpret_cast<uintptr_t>(x_in) | reinterpret_cast<uintptr_t>(x_out) |
         reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(resid)) & 15)
        return set_error(MSGL_ERR_INVALID_ARG, "rmsnorm: pointers must be 16-byte aligned");
    int vpt = (hidden / 8 + kNormThreads - 1) / kNormThreads;
    dim3 grid(num_tokens), block(kNormThreads);
#define MSGL_NORM_CASE(N)                                                                   \
    case N:                                                                                 \
        launch_pdl(rmsnorm_kernel<T, MODE, N>, grid, block, 0, stream, x_in, x_out, resid, w, \
                   ids, vocab, hidden, eps);                                                \
        break;
    switch (vpt) {
        MSGL_NORM_CASE(1) MSGL_NORM_CASE(2) MSGL_NORM_CASE(3) MSGL_NORM_CASE(4)
        MSGL_NORM_CASE(5) MSGL_NORM_CASE(6) MSGL_NORM_CASE(7) MSGL_NORM_CASE(8)
        default: return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "rmsnorm: hidden too large");
    }
#undef MSGL_NORM_CASE
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

// The same for rows of up to 4096 elements with at most 16 partials: one thread per 4 elements
// (float4), up to 10 partial loads of a thread issued before the first add, so a row of up to
// 10 partials costs one L2 round trip.
constexpr int kPartNormWide = 1024;
constexpr int kPartNormWideMaxParts = 16;
constexpr int kPartNormWideBatch = 10;  // loads in flight per thread (64 registers at 1024 threads)

__global__ void __launch_bounds__(kPartNormWide, 1)
add_partials_rmsnorm_wide_kernel(const float* __restrict__ parts, int nparts,
                                 __nv_bfloat16* __restrict__ x_out, float* __restrict__ resid,
                                 const __nv_bfloat16* __restrict__ w, int hidden, float eps) {
    __shared__ float red[32];
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x;
    const int e0 = threadIdx.x * 4;
    const bool active = e0 < hidden;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * hidden;
    const int64_t off = static_cast<int64_t>(row) * hidden + e0;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    float ss = 0.f;
    uint2 wb = make_uint2(0u, 0u);
    if (active) {
        const float4 r = *reinterpret_cast<const float4*>(resid + off);
        wb = *reinterpret_cast<const uint2*>(w + e0);
        for (int p0 = 0; p0 < nparts; p0 += kPartNormWideBatch) {
            float4 t[kPartNormWideBatch];
#pragma unroll
            for (int u = 0; u < kPartNormWideBatch; ++u)
                if (p0 + u < nparts) t[u] = *reinterpret_cast<const float4*>(parts + (p0 + u) * stride + off);
#pragma unroll
            for (int u = 0; u < kPartNormWideBatch; ++u)
                if (p0 + u < nparts) {
                    v.x += t[u].x; v.y += t[u].y; v.z += t[u].z; v.w += t[u].w;
                }
        }
        v.x += r.x; v.y += r.y; v.z += r.z; v.w += r.w;
        ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        *reinterpret_cast<float4*>(resid + off) = v;
    }
    ss = warp_sum(ss);
    const int nw = (blockDim.x + 31) >> 5;
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < nw; ++i) tot += red[i];
    const float inv_rms = 1.0f / sqrtf(tot / static_cast<float>(hidden) + eps);
    if (active) {
        uint2 o;
        o.x = pack_bf16x2(v.x * inv_rms * bf16lo(wb.x), v.y * inv_rms * bf16hi(wb.x));
        o.y = pack_bf16x2(v.z * inv_rms * bf16lo(wb.y), v.w * inv_rms * bf16hi(wb.y));
        *reinterpret_cast<uint2*>(x_out + off) = o;
    }
}

// residual += sum_p P[p]; x = rmsnorm(residual) * w, with P the fp32 split-K partials
// [nparts][rows][hidden] of the projection before the norm, added in p order, then the residual
// (as forward_fused_add adds x to the residual). One CTA of up to 512 threads per row, VPT
// vectors of 8 elements per thread. The residual and weight loads go out first, then the
// partials eight at a time, so that a row costs about two L2 round trips per vector.
constexpr int kPartNormThreads = 512;

template <int VPT>
__global__ void __launch_bounds__(kPartNormThreads, 1)
add_partials_rmsnorm_kernel(const float* __restrict__ parts, int nparts, __nv_bfloat16* __restrict__ x_out,
                            float* __restrict__ resid, const __nv_bfloat16* __restrict__ w,
                            int hidden, float eps) {
    __shared__ float red[32];
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * hidden;
    float v[VPT][8], r[VPT][8], wv[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int vi = threadIdx.x + i * blockDim.x;
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
        if (vi * 8 >= hidden) continue;
        const int64_t off = static_cast<int64_t>(row) * hidden + vi * 8;
        load8(resid + off, r[i]);
        load8(w + vi * 8, wv[i]);
        const float* pp = parts + off;
        int p = 0;
        for (; p + 8 <= nparts; p += 8) {
            float t[8][8];
#pragma unroll
            for (int u = 0; u < 8; ++u) load8(pp + (p + u) * stride, t[u]);
#pragma unroll
            for (int u = 0; u < 8; ++u)
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] += t[u][j];
        }
        if (p + 4 <= nparts) {
            float t[4][8];
#pragma unroll
            for (int u = 0; u < 4; ++u) load8(pp + (p + u) * stride, t[u]);
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] += t[u][j];
            p += 4;
        }
        for (; p < nparts; ++p) {
            float t[8];
            load8(pp + p * stride, t);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] += t[j];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            v[i][j] += r[i][j];
            ss += v[i][j] * v[i][j];
        }
        store8(resid + off, v[i]);
    }
    ss = warp_sum(ss);
    const int nw = (blockDim.x + 31) >> 5;
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < nw; ++i) tot += red[i];
    const float inv_rms = 1.0f / sqrtf(tot / static_cast<float>(hidden) + eps);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int vi = threadIdx.x + i * blockDim.x;
        if (vi * 8 >= hidden) continue;
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv_rms * wv[i][j];
        store8(x_out + static_cast<int64_t>(row) * hidden + vi * 8, o);
    }
}

template <typename T>
__global__ void index_gather_kernel(const T* __restrict__ in, const int* __restrict__ idx,
                                    T* __restrict__ out, int hidden, int num_rows) {
    pdl_wait();
    pdl_trigger();
    int i = blockIdx.x;
    int id = idx[i];
    bool valid = id >= 0 && id < num_rows;
    const T* src = in + static_cast<int64_t>(valid ? id : 0) * hidden;
    T* dst = out + static_cast<int64_t>(i) * hidden;
    if ((hidden * sizeof(T)) % 16 == 0 && (reinterpret_cast<uintptr_t>(in) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(out) & 15) == 0) {  // 16-byte rows: one uint4 per thread
        const int n16 = static_cast<int>(hidden * sizeof(T) / 16);
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        uint4* d4 = reinterpret_cast<uint4*>(dst);
        for (int h = threadIdx.x; h < n16; h += blockDim.x)
            d4[h] = valid ? s4[h] : make_uint4(0u, 0u, 0u, 0u);
        return;
    }
    for (int h = threadIdx.x; h < hidden; h += blockDim.x) dst[h] = valid ? src[h] : T(0.0f);
}

}  // namespace
}  // namespace msgl

using namespace msgl;

extern "C" {

int msgl_launch_rmsnorm(const void* input, const void* weight, void* output, int num_tokens,
                        int hidden_size, float eps, int dtype, msgl_stream_t stream) {
    if (dtype == MSGL_BF16)
        return launch_norm<__nv_bfloat16, 0>(static_cast<const __nv_bfloat16*>(input),
                                             static_cast<__nv_bfloat16*>(output), nullptr,
                                             static_cast<const __nv_bfloat16*>(weight), nullptr, 0,
                                             num_tokens, hidden_size, eps, stream);
    if (dtype == MSGL_F32)
        return launch_norm<float, 0>(static_cast<const float*>(input),
                                     static_cast<float*>(output), nullptr,
                                     static_cast<const float*>(weight), nullptr, 0, num_tokens,
                                     hidden_size, eps, stream);
    return set_error(MSGL_ERR_INVALID_ARG, "rmsnorm: unknown dtype");
}

int msgl_add_rmsnorm(void* x, float* residual, const void* weight, int num_tokens, int hidden,
                     float eps, int first, msgl_stream_t stream) {
    if (!x || !residual || !weight) return set_error(MSGL_ERR_INVALID_ARG, "add_rmsnorm: null");
    auto* xb = static_cast<__nv_bfloat16*>(x);
    auto* wb = static_cast<const __nv_bfloat16*>(weight);
    if (first)
        return launch_norm<__nv_bfloat16, 2>(xb, xb, residual, wb, nullptr, 0, num_tokens, hidden,
                                             eps, stream);
    return launch_norm<__nv_bfloat16, 1>(xb, xb, residual, wb, nullptr, 0, num_tokens, hidden, eps,
                                         stream);
}

int msgl_add_partials_rmsnorm(const float* parts, int nparts, void* x_out, float* residual,
                              const void* weight, int num_tokens, int hidden, float eps,
                              msgl_stream_t stream) {
    if (!parts || !x_out || !residual || !weight)
        return set_error(MSGL_ERR_INVALID_ARG, "add_partials_rmsnorm: null");
    if (nparts < 1 || nparts > 64)
        return set_error(MSGL_ERR_INVALID_ARG, "add_partials_rmsnorm: nparts must be in [1, 64]");
    if (num_tokens < 0 || hidden <= 0 || hidden % 8 != 0 || hidden > 8 * 1024)
        return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "add_partials_rmsnorm: hidden must be a multiple of 8, <= 8192");
    if ((reinterpret_cast<uintptr_t>(parts) | reinterpret_cast<uintptr_t>(x_out) |
         reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(residual)) & 15)
        return set_error(MSGL_ERR_INVALID_ARG, "add_partials_rmsnorm: pointers must be 16-byte aligned");
    if (num_tokens == 0) return MSGL_OK;
    if (hidden <= 4 * kPartNormWide && nparts <= kPartNormWideMaxParts) {
        const int threads = ((hidden / 4 + 31) / 32) * 32;
        launch_pdl(add_partials_rmsnorm_wide_kernel, dim3(num_tokens), dim3(threads), 0, stream,
                   parts, nparts, static_cast<__nv_bfloat16*>(x_out), residual,
                   static_cast<const __nv_bfloat16*>(weight), hidden, eps);
        MSGL_LAUNCH_CHECK();
        return MSGL_OK;
    }
    const int vecs = hidden / 8;
    const int vpt = vecs > kPartNormThreads ? 2 : 1;
    const int threads = ((vecs / vpt + (vecs % vpt ? 1 : 0) + 31) / 32) * 32;
    auto kern = vpt == 1 ? add_partials_rmsnorm_kernel<1> : add_partials_rmsnorm_kernel<2>;
    launch_pdl(kern, dim3(num_tokens), dim3(threads), 0, stream, parts, nparts,
               static_cast<__nv_bfloat16*>(x_out), residual,
               static_cast<const __nv_bfloat16*>(weight), hidden, eps);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

int msgl_embed_rmsnorm(const void* embed, const int* ids, int num_tokens, int vocab, int hidden,
                       const void* weight, float eps, void* x_out, float* residual_out,
                       msgl_stream_t stream) {
    if (!embed || !ids || !weight || !x_out || !residual_out)
        return set_error(MSGL_ERR_INVALID_ARG, "embed_rmsnorm: null");
    return launch_norm<__nv_bfloat16, 3>(
        static_cast<const __nv_bfloat16*>(embed), static_cast<__nv_bfloat16*>(x_out), residual_out,
        static_cast<const __nv_bfloat16*>(weight), ids, vocab, num_tokens, hidden, eps, stream);
}

int msgl_launch_index_gather(const void* input, const int* indices, void* output,
                             int hidden_size, int num_indices, int num_rows, int dtype,
                             msgl_stream_t stream) {
    if (num_indices < 0 || hidden_size <= 0) return set_error(MSGL_ERR_INVALID_ARG, "index_gather: sizes");
    if (num_indices == 0) return MSGL_OK;
    if (dtype == MSGL_BF16)
        launch_pdl(index_gather_kernel<__nv_bfloat16>, dim3(num_indices), dim3(128), 0, stream,
                   static_cast<const __nv_bfloat16*>(input), indices,
                   static_cast<__nv_bfloat16*>(output), hidden_size, num_rows);
    else if (dtype == MSGL_F32)
        launch_pdl(index_gather_kernel<float>, dim3(num_indices), dim3(128), 0, stream,
                   static_cast<const float*>(input), indices, static_cast<float*>(output),
                   hidden_size, num_rows);
    else
        return set_error(MSGL_ERR_INVALID_ARG, "index_gather: unknown dtype");
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

}  // extern "C"
