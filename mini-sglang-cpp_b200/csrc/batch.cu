// batch.cu -- device-side decode batch metadata.
//
//  * msgl_decode_advance   the decode branch of Scheduler::step's host flatten
//                          (src/scheduler/scheduler.cpp:83-106: input ids, positions) plus the
//                          slot formula of launch_store_kv_page (kernels/cuda/radix.cu:19-22)
//                          and KVCachePool::allocate (src/cache/kvcache.cpp:21-28, LIFO pops)
//                          for the page a request enters, all on the device, so consecutive
//                          decode steps need no host page tables and no host-to-device copies.
//
//  * msgl_decode_advance_masked / msgl_decode_finish
//                          the same with finished requests held in place, and the stop rules
//                          (max_tokens, stop ids, ignore_eos) applied on the device.
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

// finished (optional, [B]): requests with a nonzero entry are held where they are -- no page,
// no new position, same input id -- so the next step recomputes their last step (writing the
// same K/V to the same slot) and their output is ignored.
__global__ void __launch_bounds__(kAdvThreads)
decode_advance_kernel(const int* __restrict__ next_tokens, int* __restrict__ input_ids,
                      int* __restrict__ positions, int* __restrict__ slot_mapping,
                      int* __restrict__ page_table, int max_pages, int* __restrict__ seq_lens,
                      const int* __restrict__ free_pages, int* __restrict__ free_top, int B,
                      int page_size, const int* __restrict__ finished, int* err) {
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
        if (r < B && !(finished && finished[r])) {
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
        const bool held = r < B && finished && finished[r];
        if (r < B && !held) {
            L = seq_lens[r];
            need = (L % page_size) == 0;
        }
        int total;
        const int k = base + block_excl_scan(need, sh, total);
        if (r < B && !held) {
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

// Stop rules of one step (Scheduler::step, scheduler.cpp:126-131, with SamplingParams,
// types.h:12-20): a request that had not finished takes next_tokens[r] as its new token
// (token_out[r]), counts it, and finishes once it has generated max_new_tokens[r] tokens or,
// unless ignore_eos[r], when the token is one of the stop ids (the reference checks length
// only, D17). A request that had finished gets token_out[r] = -1.
__global__ void decode_finish_kernel(const int* __restrict__ next_tokens, int* __restrict__ token_out,
                                     const int* __restrict__ max_new_tokens,
                                     const int* __restrict__ ignore_eos,
                                     const int* __restrict__ stop_ids, int num_stop,
                                     int* __restrict__ finished, int* __restrict__ generated, int B) {
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= B) return;
    if (finished[r]) {
        token_out[r] = -1;
        return;
    }
    const int t = next_tokens[r];
    token_out[r] = t;
    const int g = generated[r] + 1;
    generated[r] = g;
    bool stop = g >= max_new_tokens[r];
    if (!(ignore_eos && ignore_eos[r]))
        for (int i = 0; i < num_stop; ++i) stop |= t == stop_ids[i];
    if (stop) finished[r] = 1;
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
               num_reqs, page_size, static_cast<const int*>(nullptr), err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

int msgl_decode_advance_masked(const int* next_tokens, int* input_ids, int* positions,
                               int* slot_mapping, int* page_table, int max_pages, int* seq_lens,
                               const int* free_pages, int* free_top, const int* finished,
                               int num_reqs, int page_size, msgl_stream_t stream) {
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
               num_reqs, page_size, finished, err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

int msgl_decode_finish(const int* next_tokens, int* token_out, const int* max_new_tokens,
                       const int* ignore_eos, const int* stop_ids, int num_stop_ids, int* finished,
                       int* generated, int num_reqs, msgl_stream_t stream) {
    if (num_reqs < 0 || num_stop_ids < 0 || (num_stop_ids > 0 && !stop_ids))
        return set_error(MSGL_ERR_INVALID_ARG, "decode_finish: bad sizes");
    if (num_reqs == 0) return MSGL_OK;
    if (!next_tokens || !token_out || !max_new_tokens || !finished || !generated)
        return set_error(MSGL_ERR_INVALID_ARG, "decode_finish: null pointer");
    launch_pdl(decode_finish_kernel, dim3((num_reqs + 127) / 128), dim3(128), 0, stream,
               next_tokens, token_out, max_new_tokens, ignore_eos, stop_ids, num_stop_ids,
               finished, generated, num_reqs);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

}  // extern "C"
