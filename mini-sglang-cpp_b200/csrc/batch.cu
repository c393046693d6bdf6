// batch.cu -- device-side decode batch metadata.
//
//  * msgl_decode_advance   the decode branch of Scheduler::step's host flatten
//                          (src/scheduler/scheduler.cpp:83-106: input ids, positions) plus the
//                          slot formula of launch_store_kv_page (kernels/cuda/radix.cu:19-22)
//                          and KVCachePool::allocate (src/cache/kvcache.cpp:21-28, LIFO pops)
//                          for the page a request enters, all on the device, so consecutive
//                          decode steps need no host page tables and no host-to-device copies.
//
// One CTA of up to 1024 threads walks the requests in blocks of blockDim; a block-wide scan
// gives each request that starts a new page its rank among this step's allocations, so pages
// leave the free stack in request order, as the host pool hands them out. The step is
// all-or-nothing: if the free stack cannot serve every new page, or a new page would land past
// the page-table width, nothing is written and the error word records why.
#include "common.cuh"

namespace msgl {
namespace {

constexpr int kAdvThreads = 1024;

__device__ __forceinline__ int block_excl_scan(int v, int* sh, int& total) {
    // inclusive warp scan, then the warp totals
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[w] = x;
    __syncthreads();
    if (w == 0) {
        const int nw = (blockDim.x + 31) >> 5;
        int t = lane < nw ? sh[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        if (lane < nw) sh[lane] = t;  // inclusive prefix of the warp totals
    }
    __syncthreads();
    const int before = (w > 0 ? sh[w - 1] : 0) + x - v;
    total = sh[((blockDim.x + 31) >> 5) - 1];
    __syncthreads();  // sh is reused by the next block of requests
    return before;
}

__global__ void __launch_bounds__(kAdvThreads)
decode_advance_kernel(const int* __restrict__ next_tokens, int* __restrict__ input_ids,
                      int* __restrict__ positions, int* __restrict__ slot_mapping,
                      int* __restrict__ page_table, int max_pages, int* __restrict__ seq_lens,
                      const int* __restrict__ free_pages, int* __restrict__ free_top, int B,
                      int page_size, int* err) {
    __shared__ int sh[32];
    __shared__ int bad;
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    const int top = *free_top;
    // pass 1: count the new pages and check every request (no writes)
    int base = 0;
    for (int r0 = 0; r0 < B; r0 += blockDim.x) {
        const int r = r0 + threadIdx.x;
        int need = 0;
        if (r < B) {
            const int L = seq_lens[r];  // tokens in the cache after this step's token is added
            need = (L % page_size) == 0;
            if (L < 0 || L / page_size >= max_pages) atomicOr(&bad, 2);
        }
        int total;
        const int k = base + block_excl_scan(need, sh, total);
        if (need && top - 1 - k < 0) atomicOr(&bad, 1);
        base += total;
    }
    __syncthreads();
    if (bad) {
        if (threadIdx.x == 0) {
            if (bad & 2) record_error(err, MSGL_ERR_BOUNDS, 701);
            else record_error(err, MSGL_ERR_WORKSPACE, 700);
        }
        return;
    }
    // pass 2: pop pages in request order, write the next step's metadata
    base = 0;
    for (int r0 = 0; r0 < B; r0 += blockDim.x) {
        const int r = r0 + threadIdx.x;
        int need = 0, L = 0;
        if (r < B) {
            L = seq_lens[r];
            need = (L % page_size) == 0;
        }
        int total;
        const int k = base + block_excl_scan(need, sh, total);
        if (r < B) {
            int* row = page_table + static_cast<int64_t>(r) * max_pages;
            const int pi = L / page_size;
            if (need) row[pi] = free_pages[top - 1 - k];
            input_ids[r] = next_tokens[r];
            positions[r] = L;
            slot_mapping[r] = row[pi] * page_size + L % page_size;
            seq_lens[r] = L + 1;
        }
        base += total;
    }
    if (threadIdx.x == 0) *free_top = top - base;
}

}  // namespace
}  // namespace msgl

using namespace msgl;

extern "C" {

int msgl_decode_advance(const int* next_tokens, int* input_ids, int* positions, int* slot_mapping,
                        int* page_table, int max_pages, int* seq_lens, const int* free_pages,
                        int* free_top, int num_reqs, int page_size, msgl_stream_t stream) {
    if (num_reqs < 0 || max_pages <= 0 || page_size <= 0)
        return set_error(MSGL_ERR_INVALID_ARG, "decode_advance: bad sizes");
    if (num_reqs == 0) return MSGL_OK;
    if (!next_tokens || !input_ids || !positions || !slot_mapping || !page_table || !seq_lens ||
        !free_pages || !free_top)
        return set_error(MSGL_ERR_INVALID_ARG, "decode_advance: null pointer");
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    const int threads = num_reqs >= kAdvThreads ? kAdvThreads : ((num_reqs + 31) / 32) * 32;
    launch_pdl(decode_advance_kernel, dim3(1), dim3(threads), 0, stream, next_tokens, input_ids,
               positions, slot_mapping, page_table, max_pages, seq_lens, free_pages, free_top,
               num_reqs, page_size, err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

}  // extern "C"
