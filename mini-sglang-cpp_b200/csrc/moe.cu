// moe.cu -- MoE routing around the grouped tcgen05 GEMMs of gemm.cu.
//
//  * msgl_moe_route_topk   MoERouter::route top-k and weights (src/layer/layer.cpp:283-305)
//                          on fp32 router logits (the logits GEMM is msgl_gemm_bf16 with an
//                          fp32 output, or its split-K partials, summed here in part order):
//                          descending logit, equal logits -> larger expert id first
//                          (std::greater on pair<float,int>), w = exp(l), divided by the top-k
//                          sum when norm_topk.
//  * msgl_moe_permute      counting sort of the (token, k) pairs by expert, stable in pair
//                          order: expert row offsets, the token of each sorted row, and the
//                          sorted position of each pair (deterministic, no atomics on output).
//  * msgl_moe_combine      out[t] = sum_k w[t,k] * y_sorted[pos(t,k)], k in order, fp32
//                          accumulation (the expert loop of src/model/qwen3_moe.cpp:74-108).
//  * msgl_moe_combine_add_rmsnorm  the combine, then the decoder layer's residual add and the
//                          next RMSNorm of the same row in the same CTA (qwen3.cpp:19 on the
//                          MoE output, layer.cpp:79-112): equal bit for bit to msgl_moe_combine
//                          followed by msgl_add_rmsnorm.
#include "common.cuh"

namespace msgl {
namespace {

// key: larger logit wins; equal logits -> larger index wins (std::greater<pair<float,int>>).
// NaN never wins.
__device__ __forceinline__ bool key_greater(float va, int ia, float vb, int ib) {
    return va > vb || (!(vb > va) && !(va != va) && ia > ib);
}

// One warp per token; E <= 32 * kMaxPerLane experts, top_k <= 32.
constexpr int kMaxPerLane = 8;

// The logits are the sum of `nparts` fp32 split-K partials [nparts][T][E], added in part order
// (nparts = 1: plain logits).
__global__ void route_topk_kernel(const float* __restrict__ logits, int nparts, int T, int E,
                                  int top_k, int norm_topk, int* __restrict__ ids,
                                  float* __restrict__ w) {
    pdl_wait();
    pdl_trigger();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float* row = logits + static_cast<int64_t>(warp) * E;
    const int64_t pstride = static_cast<int64_t>(T) * E;
    float v[kMaxPerLane];
    bool taken[kMaxPerLane];
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
        int e = lane + 32 * i;
        v[i] = e < E ? row[e] : -__builtin_huge_valf();
        taken[i] = e >= E;
    }
    // further partials, added in part order; four parts' loads in flight at a time
    for (int pp = 1; pp < nparts; pp += 4) {
        float t[4][kMaxPerLane];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int i = 0; i < kMaxPerLane; ++i) {
                const int e = lane + 32 * i;
                t[u][i] = (pp + u < nparts && e < E) ? row[(pp + u) * pstride + e] : 0.f;
            }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int i = 0; i < kMaxPerLane; ++i)
                if (pp + u < nparts && lane + 32 * i < E) v[i] += t[u][i];
    }
    float sel_v = 0.f, first_v = 0.f;
    int sel_i = 0;
    float sum = 0.f;
    for (int k = 0; k < top_k; ++k) {
        // this lane's best untaken candidate
        float bv = -__builtin_huge_valf();
        int bi = -1;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            int e = lane + 32 * i;
            if (!taken[i] && (bi < 0 || key_greater(v[i], e, bv, bi))) {
                bv = v[i];
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && (bi < 0 || key_greater(ov, oi, bv, bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if (bi >= 0 && (bi & 31) == lane) taken[bi >> 5] = true;
        if (k == 0) first_v = bv;
        if (lane == k) {
            sel_v = bv;
            sel_i = bi;
        }
    }
    // weights: exp(l) (layer.cpp:297); normalised form evaluated as exp(l - l_max) / sum
    float e_l = 0.f;
    if (lane < top_k) e_l = norm_topk ? expf(sel_v - first_v) : expf(sel_v);
    sum = warp_sum(e_l);
    if (lane < top_k) {
        ids[static_cast<int64_t>(warp) * top_k + lane] = sel_i;
        w[static_cast<int64_t>(warp) * top_k + lane] = norm_topk ? e_l / sum : e_l;
    }
}

// Single CTA, 1024 threads: histogram, block scan, then stable placement chunk by chunk
// (per-warp expert counts in shared memory, prefix over warps, rank inside the warp by
// __match_any_sync).
constexpr int kPermThreads = 1024;
constexpr int kPermWarps = kPermThreads / 32;

__global__ void __launch_bounds__(kPermThreads)
permute_kernel(const int* __restrict__ ids, int num_pairs, int top_k, int E,
               int* __restrict__ offsets, int* __restrict__ sorted_token,
               int* __restrict__ pair_pos, int* err) {
    extern __shared__ int sm[];
    __shared__ int scan_sh[32];
    pdl_wait();
    pdl_trigger();
    int* base = sm;                       // [E] running start of each expert
    int* wcnt = sm + E;                   // [kPermWarps][E]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < E; e += kPermThreads) base[e] = 0;
    __syncthreads();
    for (int p = tid; p < num_pairs; p += kPermThreads) {
        int e = ids[p];
        if (static_cast<unsigned>(e) >= static_cast<unsigned>(E)) {
            record_error(err, MSGL_ERR_BOUNDS, 400);
            continue;
        }
        atomicAdd(&base[e], 1);
    }
    __syncthreads();
    {  // exclusive scan of the expert counts -> offsets (E <= 256 < kPermThreads)
        const int c = tid < E ? base[tid] : 0;
        int total;
        const int before = block_excl_scan(c, scan_sh, total);
        if (tid < E) {
            offsets[tid] = before;
            base[tid] = before;
        }
        if (tid == 0) offsets[E] = total;
    }
    __syncthreads();
    for (int c0 = 0; c0 < num_pairs; c0 += kPermThreads) {
        for (int i = tid; i < kPermWarps * E; i += kPermThreads) wcnt[i] = 0;
        __syncthreads();
        const int p = c0 + tid;
        const bool valid = p < num_pairs;
        int e = valid ? ids[p] : -1;
        if (static_cast<unsigned>(e) >= static_cast<unsigned>(E)) e = -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1));
        if (e >= 0 && rank == 0) wcnt[warp * E + e] = __popc(peers);
        __syncthreads();
        for (int x = tid; x < E; x += kPermThreads) {  // prefix over warps, per expert
            int run = base[x];
            for (int w = 0; w < kPermWarps; ++w) {
                int c = wcnt[w * E + x];
                wcnt[w * E + x] = run;
                run += c;
            }
            base[x] = run;
        }
        __syncthreads();
        if (e >= 0) {
            const int pos = wcnt[warp * E + e] + rank;
            sorted_token[pos] = p / top_k;
            pair_pos[p] = pos;
        } else if (valid) {
            pair_pos[p] = -1;
        }
        __syncthreads();
    }
}

// One CTA per token: out[t, h] = sum_k w[t, k] * y[pair_pos[t k + k], h] (k in order). The
// token's k (row, weight) pairs are staged in shared memory first, so each thread's k row loads
// are independent and go out together.
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ pair_pos,
                               const float* __restrict__ w, int top_k, int hidden,
                               __nv_bfloat16* __restrict__ out) {
    __shared__ int s_pos[32];
    __shared__ float s_w[32];
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    if (threadIdx.x < top_k) {
        s_pos[threadIdx.x] = pair_pos[static_cast<int64_t>(t) * top_k + threadIdx.x];
        s_w[threadIdx.x] = w[static_cast<int64_t>(t) * top_k + threadIdx.x];
    }
    __syncthreads();
    for (int h8 = threadIdx.x; h8 * 8 < hidden; h8 += blockDim.x) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll 8
        for (int k = 0; k < top_k; ++k) {
            const int pos = s_pos[k];
            if (pos < 0) continue;
            const float wk = s_w[k];
            uint4 u = *reinterpret_cast<const uint4*>(y + static_cast<int64_t>(pos) * hidden + h8 * 8);
            acc[0] += wk * bf16lo(u.x); acc[1] += wk * bf16hi(u.x);
            acc[2] += wk * bf16lo(u.y); acc[3] += wk * bf16hi(u.y);
            acc[4] += wk * bf16lo(u.z); acc[5] += wk * bf16hi(u.z);
            acc[6] += wk * bf16lo(u.w); acc[7] += wk * bf16hi(u.w);
        }
        uint4 o;
        o.x = pack_bf16x2(acc[0], acc[1]); o.y = pack_bf16x2(acc[2], acc[3]);
        o.z = pack_bf16x2(acc[4], acc[5]); o.w = pack_bf16x2(acc[6], acc[7]);
        *reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * hidden + h8 * 8) = o;
    }
}

// combine_kernel fused with the residual add and the RMSNorm that follow it: one 128-thread CTA
// per token row, thread t owning the row vectors t + 128 i (i < VPT), as the add + RMSNorm kernel
// does. Per vector: m = bf16(sum_k w_k y[pos_k]) (rounded as combine_kernel stores it),
// r += m, and r's squares go into the row sum in the same order; the block reduction and the
// scaling x = bf16(r * inv_rms * g) are that kernel's too, so the output equals the two kernels
// run back to back.
constexpr int kCombNormThreads = 128;

template <int VPT>
__global__ void __launch_bounds__(kCombNormThreads)
combine_add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ pair_pos,
                           const float* __restrict__ w, int top_k, int hidden,
                           float* __restrict__ resid, const __nv_bfloat16* __restrict__ g,
                           float eps, __nv_bfloat16* __restrict__ x_out) {
    __shared__ int s_pos[32];
    __shared__ float s_w[32];
    __shared__ float red[kCombNormThreads / 32];
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    if (threadIdx.x < top_k) {
        s_pos[threadIdx.x] = pair_pos[static_cast<int64_t>(t) * top_k + threadIdx.x];
        s_w[threadIdx.x] = w[static_cast<int64_t>(t) * top_k + threadIdx.x];
    }
    __syncthreads();
    const int nvec = hidden >> 3;
    float* rrow = resid + static_cast<int64_t>(t) * hidden;
    float v[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int vi = threadIdx.x + i * kCombNormThreads;
        if (vi < nvec) {
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll 8
            for (int k = 0; k < top_k; ++k) {
                const int pos = s_pos[k];
                if (pos < 0) continue;
                const float wk = s_w[k];
                uint4 u = *reinterpret_cast<const uint4*>(y + static_cast<int64_t>(pos) * hidden + vi * 8);
                acc[0] += wk * bf16lo(u.x); acc[1] += wk * bf16hi(u.x);
                acc[2] += wk * bf16lo(u.y); acc[3] += wk * bf16hi(u.y);
                acc[4] += wk * bf16lo(u.z); acc[5] += wk * bf16hi(u.z);
                acc[6] += wk * bf16lo(u.w); acc[7] += wk * bf16hi(u.w);
            }
            const float4 r0 = reinterpret_cast<const float4*>(rrow + vi * 8)[0];
            const float4 r1 = reinterpret_cast<const float4*>(rrow + vi * 8)[1];
            const float r[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                const uint32_t m = pack_bf16x2(acc[j], acc[j + 1]);
                v[i][j] = bf16lo(m) + r[j];
                v[i][j + 1] = bf16hi(m) + r[j + 1];
            }
            reinterpret_cast<float4*>(rrow + vi * 8)[0] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
            reinterpret_cast<float4*>(rrow + vi * 8)[1] = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
#pragma unroll
            for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
        }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = red[0] + red[1] + red[2] + red[3];
    const float inv_rms = 1.0f / sqrtf(ss / static_cast<float>(hidden) + eps);
    __nv_bfloat16* dst = x_out + static_cast<int64_t>(t) * hidden;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int vi = threadIdx.x + i * kCombNormThreads;
        if (vi < nvec) {
            const uint4 gu = *reinterpret_cast<const uint4*>(g + vi * 8);
            const float gv[8] = {bf16lo(gu.x), bf16hi(gu.x), bf16lo(gu.y), bf16hi(gu.y),
                                 bf16lo(gu.z), bf16hi(gu.z), bf16lo(gu.w), bf16hi(gu.w)};
            float o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv_rms * gv[j];
            uint4 u;
            u.x = pack_bf16x2(o[0], o[1]); u.y = pack_bf16x2(o[2], o[3]);
            u.z = pack_bf16x2(o[4], o[5]); u.w = pack_bf16x2(o[6], o[7]);
            *reinterpret_cast<uint4*>(dst + vi * 8) = u;
        }
    }
}

}  // namespace
}  // namespace msgl

using namespace msgl;

extern "C" {

int msgl_moe_route_topk_partials(const float* router_parts, int nparts, int num_tokens,
                                 int num_experts, int top_k, int norm_topk, int* topk_ids,
                                 float* topk_weights, msgl_stream_t stream) {
    if (num_tokens < 0 || num_experts <= 0 || num_experts > 32 * kMaxPerLane || top_k <= 0 ||
        top_k > 32 || top_k > num_experts)
        return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "moe_route_topk: E <= 256, top_k <= min(32, E)");
    if (nparts < 1 || nparts > 64) return set_error(MSGL_ERR_INVALID_ARG, "moe_route_topk: nparts in [1, 64]");
    if (num_tokens == 0) return MSGL_OK;
    const int threads = 256;
    const int blocks = (num_tokens * 32 + threads - 1) / threads;
    launch_pdl(route_topk_kernel, dim3(blocks), dim3(threads), 0, stream, router_parts, nparts,
               num_tokens, num_experts, top_k, norm_topk, topk_ids, topk_weights);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

int msgl_moe_route_topk(const float* router_logits, int num_tokens, int num_experts, int top_k,
                        int norm_topk, int* topk_ids, float* topk_weights, msgl_stream_t stream) {
    return msgl_moe_route_topk_partials(router_logits, 1, num_tokens, num_experts, top_k,
                                        norm_topk, topk_ids, topk_weights, stream);
}

int msgl_moe_permute(const int* topk_ids, int num_tokens, int top_k, int num_experts,
                     int* expert_offsets, int* sorted_token, int* pair_pos, msgl_stream_t stream) {
    if (num_tokens < 0 || top_k <= 0 || num_experts <= 0 || num_experts > 256)
        return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "moe_permute: num_experts <= 256");
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    const size_t smem = static_cast<size_t>(num_experts) * (kPermWarps + 1) * sizeof(int);
    cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    launch_pdl(permute_kernel, dim3(1), dim3(kPermThreads), smem, stream, topk_ids,
               num_tokens * top_k, top_k, num_experts, expert_offsets, sorted_token, pair_pos, err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

int msgl_moe_combine(const void* y_sorted, const int* pair_pos, const float* topk_weights,
                     int num_tokens, int top_k, int hidden, void* out, msgl_stream_t stream) {
    if (num_tokens < 0 || top_k <= 0 || top_k > 32 || hidden <= 0 || hidden % 8)
        return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "moe_combine: hidden % 8, top_k <= 32");
    if (num_tokens == 0) return MSGL_OK;
    launch_pdl(combine_kernel, dim3(num_tokens), dim3(128), 0, stream,
               static_cast<const __nv_bfloat16*>(y_sorted), pair_pos, topk_weights, top_k, hidden,
               static_cast<__nv_bfloat16*>(out));
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

int msgl_moe_combine_add_rmsnorm(const void* y_sorted, const int* pair_pos,
                                 const float* topk_weights, int num_tokens, int top_k, int hidden,
                                 float* residual, const void* norm_weight, float eps, void* x_out,
                                 msgl_stream_t stream) {
    if (!y_sorted || !pair_pos || !topk_weights || !residual || !norm_weight || !x_out)
        return set_error(MSGL_ERR_INVALID_ARG, "moe_combine_add_rmsnorm: null");
    if (num_tokens < 0 || top_k <= 0 || top_k > 32 || hidden <= 0 || hidden % 8 ||
        hidden > 8 * 8 * kCombNormThreads)
        return set_error(MSGL_ERR_UNSUPPORTED_SHAPE,
                         "moe_combine_add_rmsnorm: hidden % 8, hidden <= 8192, top_k <= 32");
    if ((reinterpret_cast<uintptr_t>(y_sorted) | reinterpret_cast<uintptr_t>(residual) |
         reinterpret_cast<uintptr_t>(norm_weight) | reinterpret_cast<uintptr_t>(x_out)) & 15)
        return set_error(MSGL_ERR_INVALID_ARG, "moe_combine_add_rmsnorm: pointers must be 16-byte aligned");
    if (num_tokens == 0) return MSGL_OK;
    const int vpt = (hidden / 8 + kCombNormThreads - 1) / kCombNormThreads;
    const auto* y = static_cast<const __nv_bfloat16*>(y_sorted);
    const auto* g = static_cast<const __nv_bfloat16*>(norm_weight);
    auto* xo = static_cast<__nv_bfloat16*>(x_out);
    const dim3 grid(num_tokens), block(kCombNormThreads);
#define MSGL_COMB_CASE(N)                                                                      \
    case N:                                                                                    \
        launch_pdl(combine_add_rmsnorm_kernel<N>, grid, block, 0, stream, y, pair_pos,          \
                   topk_weights, top_k, hidden, residual, g, eps, xo);                          \
        break;
    switch (vpt) {
        MSGL_COMB_CASE(1) MSGL_COMB_CASE(2) MSGL_COMB_CASE(3) MSGL_COMB_CASE(4)
        MSGL_COMB_CASE(5) MSGL_COMB_CASE(6) MSGL_COMB_CASE(7) MSGL_COMB_CASE(8)
        default: return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "moe_combine_add_rmsnorm: hidden");
    }
#undef MSGL_COMB_CASE
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

}  // extern "C"
