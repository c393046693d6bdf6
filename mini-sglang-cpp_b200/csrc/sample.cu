// sample.cu -- token sampling from fp32 logits with temperature / top-k / top-p.
//
// SamplingParams (include/minisgl/core/types.h:12-20) carries temperature, top_k and top_p; the
// reference samples greedily only (Scheduler::step, src/scheduler/scheduler.cpp:110-124: first
// index of the maximum). msgl_sample keeps that for greedy rows (temperature <= 0 or top_k == 1)
// and otherwise draws from the temperature softmax restricted to a candidate set:
//   1. candidates: the K largest logits, K = top_k if 1 < top_k <= 1024 else min(V, 1024) (ties
//      at the K-th value: the lower ids), in order of (logit descending, id ascending);
//   2. weights w_i = exp((l_i - l_max) / temperature), cumulative sums c_i in that order;
//   3. top-p: the first n candidates with c_{n-1} >= top_p * c_{K-1} (n >= 1; all when top_p >= 1);
//   4. u = uniform from SplitMix64 (Steele, Lea, Flood, OOPSLA 2014) of (seed, step, row), 24 bits;
//      the token is the first candidate i < n with c_i > u * c_{n-1}.
// One CTA of 1024 threads per row: a four-pass 8-bit radix select finds the K-th largest logit
// key, a block scan places the candidates, a bitonic sort orders them in shared memory, and one
// thread accumulates the weights in order (the same order as the host restatement).
#include "common.cuh"

namespace msgl {
namespace {

constexpr int kSampThreads = 1024;
constexpr int kMaxCand = 1024;

__device__ __forceinline__ uint32_t ord_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // larger float -> larger key
}

__device__ __forceinline__ float uniform24(uint64_t seed, uint64_t step, uint64_t row) {
    uint64_t z = seed ^ (step * 0x9E3779B97F4A7C15ull) ^ (row * 0xC2B2AE3D27D4EB4Full);
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return static_cast<float>(z >> 40) * (1.0f / 16777216.0f);
}

__global__ void __launch_bounds__(kSampThreads)
sample_kernel(const float* __restrict__ logits, int V, const float* __restrict__ temperature,
              const int* __restrict__ top_k, const float* __restrict__ top_p, uint64_t seed,
              uint64_t step, int* __restrict__ out) {
    __shared__ int hist[256];
    __shared__ int sh[32];
    __shared__ unsigned long long cand[kMaxCand];  // (key << 32) | (0xFFFFFFFF - id)
    __shared__ float csum[kMaxCand];
    __shared__ uint32_t sel_prefix;
    __shared__ int sel_remaining;
    __shared__ unsigned long long best;
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x, tid = threadIdx.x;
    const float* l = logits + static_cast<int64_t>(row) * V;
    const float T = temperature[row];
    const int k = top_k[row];
    const float p = top_p[row];
    const int chunk = (V + kSampThreads - 1) / kSampThreads;
    const int beg = min(V, tid * chunk), end = min(V, beg + chunk);

    if (T <= 0.f || k == 1) {  // greedy: the first index of the maximum
        if (tid == 0) best = 0ull;
        __syncthreads();
        unsigned long long b = 0ull;
        for (int i = beg; i < end; ++i) {
            const unsigned long long key =
                (static_cast<unsigned long long>(ord_key(l[i])) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
            b = key > b ? key : b;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long y = __shfl_xor_sync(0xffffffffu, b, o);
            b = y > b ? y : b;
        }
        if ((tid & 31) == 0) atomicMax(&best, b);
        __syncthreads();
        if (tid == 0) out[row] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
        return;
    }

    const int K = (k > 1 && k <= kMaxCand) ? min(k, V) : min(V, kMaxCand);
    // 1. the K-th largest key: radix select, 8 bits per pass from the top
    if (tid == 0) {
        sel_prefix = 0;
        sel_remaining = K;
    }
    uint32_t mask = 0;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int b = tid; b < 256; b += kSampThreads) hist[b] = 0;
        __syncthreads();
        const uint32_t prefix = sel_prefix;
        for (int i = beg; i < end; ++i) {
            const uint32_t key = ord_key(l[i]);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1);
        }
        __syncthreads();
        if (tid == 0) {
            int cum = 0, rem = sel_remaining;
            for (int b = 255; b >= 0; --b) {
                if (cum + hist[b] >= rem) {
                    sel_prefix = prefix | (static_cast<uint32_t>(b) << shift);
                    sel_remaining = rem - cum;
                    break;
                }
                cum += hist[b];
            }
        }
        mask |= 255u << shift;
        __syncthreads();
    }
    const uint32_t t = sel_prefix;
    const int ties = sel_remaining;  // how many keys equal to t join (the lowest ids)
    // 2. place the candidates: all keys > t, then the first `ties` keys == t in id order
    int gt = 0, eq = 0;
    for (int i = beg; i < end; ++i) {
        const uint32_t key = ord_key(l[i]);
        gt += key > t;
        eq += key == t;
    }
    int gt_total, eq_total;
    int gt_off = block_excl_scan(gt, sh, gt_total);
    int eq_off = block_excl_scan(eq, sh, eq_total);
    for (int i = beg; i < end; ++i) {
        const uint32_t key = ord_key(l[i]);
        const unsigned long long e =
            (static_cast<unsigned long long>(key) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
        if (key > t) {
            cand[gt_off++] = e;
        } else if (key == t) {
            if (eq_off < ties) cand[gt_total + eq_off] = e;
            ++eq_off;
        }
    }
    for (int i = K + tid; i < kMaxCand; i += kSampThreads) cand[i] = 0ull;  // padding sorts last
    __syncthreads();
    // 3. bitonic sort, descending
    for (int size = 2; size <= kMaxCand; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const int i = tid, j = i ^ stride;
            if (j > i) {
                const bool desc = (i & size) == 0;
                const unsigned long long a = cand[i], b = cand[j];
                if (desc ? a < b : a > b) {
                    cand[i] = b;
                    cand[j] = a;
                }
            }
            __syncthreads();
        }
    }
    // 4. weights and their running sums, in candidate order, by one thread
    if (tid == 0) {
        auto val = [&](int i) {
            const uint32_t key = static_cast<uint32_t>(cand[i] >> 32);
            return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
        };
        const float mx = val(0);
        const float inv_t = 1.0f / T;
        float c = 0.f;
        for (int i = 0; i < K; ++i) {
            c += expf((val(i) - mx) * inv_t);
            csum[i] = c;
        }
        int n = K;
        if (p < 1.f) {
            const float cut = p * csum[K - 1];
            n = 1;
            while (n < K && csum[n - 1] < cut) ++n;
        }
        const float target = uniform24(seed, step, static_cast<uint64_t>(row)) * csum[n - 1];
        int pick = n - 1;
        for (int i = 0; i < n; ++i)
            if (csum[i] > target) {
                pick = i;
                break;
            }
        out[row] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(cand[pick] & 0xFFFFFFFFull));
    }
}

}  // namespace
}  // namespace msgl

using namespace msgl;

extern "C" {

int msgl_sample(const float* logits, int num_rows, int vocab, const float* temperature,
                const int* top_k, const float* top_p, uint64_t seed, uint64_t step, int* out,
                msgl_stream_t stream) {
    if (num_rows < 0 || vocab <= 0) return set_error(MSGL_ERR_INVALID_ARG, "sample: bad sizes");
    if (num_rows == 0) return MSGL_OK;
    if (!logits || !temperature || !top_k || !top_p || !out)
        return set_error(MSGL_ERR_INVALID_ARG, "sample: null pointer");
    launch_pdl(sample_kernel, dim3(num_rows), dim3(kSampThreads), 0, stream, logits, vocab,
               temperature, top_k, top_p, seed, step, out);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

}  // extern "C"
