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

// Single CTA, 1024 threads: histogram, scan, then stable placement chunk by chunk
// (per-warp expert counts in shared memory, prefix over warps, rank inside the warp by
// __match_any_sync).
constexpr int kPermThreads = 1024;
constexpr int kPermWarps = kPermThreads / 32;

__global__ void __launch_bounds__(kPermThreads)
permute_kernel(const int* __restrict__ ids, int num_pairs, int top_k, int E,
               int* __restrict__ offsets, int* __restrict__ sorted_token,
               int* __restrict__ pair_pos, int* err) {
    extern __shared__ int sm[];
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
    if (tid == 0) {  // exclusive scan -> offsets
        int run = 0;
        for (int e = 0; e < E; ++e) {
            int c = base[e];
            offsets[e] = run;
            base[e] = run;
            run += c;
        }
        offsets[E] = run;
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

}  // extern "C"
