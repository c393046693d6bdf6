/*
 * msgl_kernels.h -- C ABI of libmsgl, the sm_100a (B200) kernels of the mini-sglang-cpp
 * per-layer Qwen3 / Qwen3-MoE forward path.
 *
 * Conventions (all entry points):
 *  - plain pointers and sizes; every device pointer is a CUDA device address on the current
 *    device; the caller owns every buffer (inputs, outputs, workspaces) -- no entry point
 *    allocates device memory;
 *  - each call is asynchronous on the given stream and returns an msgl_status; on failure
 *    msgl_last_error() returns a message (thread-local);
 *  - kernel-side failures (a bounded wait that ran out, an index outside a pool) never trap:
 *    they are recorded in a per-device error word read by msgl_device_error();
 *  - activations and weights are bf16 unless a dtype argument says otherwise; accumulation is
 *    fp32; the residual stream is fp32.
 *
 * The four reference launchers (include/minisgl/kernel/kernels.h:13-21 of mini-sglang-cpp) keep
 * their names (prefixed msgl_), argument order and meaning, plus a dtype tag and a status.
 */
#ifndef MSGL_KERNELS_H
#define MSGL_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#if defined(__CUDACC__) || defined(CUDART_VERSION)
#include <cuda_runtime.h>
typedef cudaStream_t msgl_stream_t;
#else
typedef void* msgl_stream_t; /* a cudaStream_t */
#endif

#if defined(__GNUC__)
#define MSGL_API __attribute__((visibility("default")))
#else
#define MSGL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    MSGL_OK = 0,
    MSGL_ERR_INVALID_ARG = 1,
    MSGL_ERR_UNSUPPORTED_SHAPE = 2,
    MSGL_ERR_CUDA = 3,
    MSGL_ERR_NCCL = 4,
    MSGL_ERR_TIMEOUT = 5,
    MSGL_ERR_BOUNDS = 6,
    MSGL_ERR_WORKSPACE = 7
} msgl_status;

typedef enum { MSGL_F32 = 0, MSGL_BF16 = 1 } msgl_dtype;

/* ---------------------------------------------------------------- library */
MSGL_API const char* msgl_version(void);
/* Message of the last failing call on this host thread ("" if none). */
MSGL_API const char* msgl_last_error(void);
/* Synchronises `stream`, then reads the device error word of the current device (code and an
 * info word naming the failing site); reset != 0 clears it. */
MSGL_API int msgl_device_error(int* code, int* info, int reset, msgl_stream_t stream);
/* Number of kernels this library has launched from the host so far, over all threads and
 * devices (replays of a captured CUDA graph launch nothing from the host and are not counted;
 * NCCL's own kernels are not counted). */
MSGL_API unsigned long long msgl_kernel_launches(void);

/* ---------------------------------------------------------------- reference launchers */
/* launch_rmsnorm (kernels.h:13-14; kernels/cuda/rmsnorm.cu:37-43; semantics of
 * RMSNorm::forward, src/layer/layer.cpp:48-77). input/weight/output share `dtype`. */
MSGL_API int msgl_launch_rmsnorm(const void* input, const void* weight, void* output, int num_tokens,
                        int hidden_size, float eps, int dtype, msgl_stream_t stream);

/* launch_rope (kernels.h:15-16; kernels/cuda/rotary.cu:43-51). Rotate-half RoPE in place on
 * query [T, num_q_heads, D] and key [T, num_kv_heads, D] (key may be NULL) with the fp32 table
 * cos_sin_cache [max_pos, D] (RotaryEmbedding ctor, layer.cpp:163-176) and per-token positions.
 * The reference passes one head count for both tensors; K has its own here. */
MSGL_API int msgl_launch_rope(void* query, void* key, const int* positions, const float* cos_sin_cache,
                     int num_tokens, int num_q_heads, int num_kv_heads, int head_dim, int dtype,
                     msgl_stream_t stream);

/* launch_index_gather (kernels.h:17-18; kernels/cuda/index.cu:21-28): out[i,:] = in[idx[i],:].
 * Ids outside [0, num_rows) give a zero row, as Embedding::forward does (layer.cpp:26-31). */
MSGL_API int msgl_launch_index_gather(const void* input, const int* indices, void* output,
                             int hidden_size, int num_indices, int num_rows, int dtype,
                             msgl_stream_t stream);

/* launch_store_kv_page (kernels.h:19-21; kernels/cuda/radix.cu:28-36): token t of k/v
 * [T, heads*D] goes to pool row page_table[t / page_size] * page_size + t % page_size. */
MSGL_API int msgl_launch_store_kv_page(const void* k, const void* v, void* k_cache, void* v_cache,
                              const int* page_table, int page_size, int num_heads, int head_dim,
                              int num_tokens, int dtype, msgl_stream_t stream);

/* ---------------------------------------------------------------- fused norm / RoPE / KV */
/* RMSNorm::forward_fused_add (layer.cpp:79-112): residual += x; x = rmsnorm(residual) * w.
 * x bf16 [T,H] in/out, residual fp32 [T,H] in/out, weight bf16 [H].
 * first != 0 is the aliasing first call (layer.cpp:80-84): residual = x; x = rmsnorm(x). */
MSGL_API int msgl_add_rmsnorm(void* x, float* residual, const void* weight, int num_tokens, int hidden,
                     float eps, int first, msgl_stream_t stream);

/* forward_fused_add (layer.cpp:79-112) whose input is the sum of fp32 split-K partials
 * parts [nparts][num_tokens][hidden] (msgl_gemm_bf16_partials): residual += sum_p parts[p]
 * (added in p order); x_out = rmsnorm(residual) * weight (bf16). 1 <= nparts <= 64; parts
 * 16-byte aligned. */
MSGL_API int msgl_add_partials_rmsnorm(const float* parts, int nparts, void* x_out, float* residual,
                                       const void* weight, int num_tokens, int hidden, float eps,
                                       msgl_stream_t stream);

/* Embedding::forward (layer.cpp:15-42) fused with the first layer's input norm:
 * residual = embed[ids]; x = rmsnorm(residual) * w. Out-of-range ids give zero rows. */
MSGL_API int msgl_embed_rmsnorm(const void* embed, const int* ids, int num_tokens, int vocab, int hidden,
                       const void* weight, float eps, void* x_out, float* residual_out,
                       msgl_stream_t stream);

/* QK-norm + RoPE + KV page store, one pass over the QKV projection output (split of
 * src/model/qwen3.cpp:28-45, RoPE of :48, store of kernels/cuda/radix.cu:19-22):
 *   qkv [T, (Hq + 2 Hkv) D] bf16, rows q | k | v per token;
 *   q_out [T, Hq, D] = rope(rmsnorm_D(q) * q_norm);
 *   k_pool[slot_mapping[t], :] = rope(rmsnorm_D(k) * k_norm);  v_pool[slot_mapping[t], :] = v.
 * Pools are [num_slots, Hkv * D] bf16; a negative slot skips the store (padding token), a slot
 * >= num_slots is skipped and recorded as MSGL_ERR_BOUNDS in the device error word.
 * head_dim must be 128. */
MSGL_API int msgl_qknorm_rope_store_kv(const void* qkv, void* q_out, void* k_pool, void* v_pool,
                              int64_t num_slots, const int* positions, const int* slot_mapping,
                              const float* cos_sin_cache, const void* q_norm_w,
                              const void* k_norm_w, int num_tokens, int num_q_heads,
                              int num_kv_heads, int head_dim, float eps, msgl_stream_t stream);
/* The same, with the QKV row the sum (in p order) of fp32 split-K partials
 * parts [nparts][T][(Hq + 2 Hkv) D] of the QKV projection (msgl_gemm_bf16_partials). */
MSGL_API int msgl_qknorm_rope_store_kv_partials(const float* parts, int nparts, void* q_out,
                                                void* k_pool, void* v_pool, int64_t num_slots,
                                                const int* positions, const int* slot_mapping,
                                                const float* cos_sin_cache, const void* q_norm_w,
                                                const void* k_norm_w, int num_tokens,
                                                int num_q_heads, int num_kv_heads, int head_dim,
                                                float eps, msgl_stream_t stream);

/* ---------------------------------------------------------------- sampling */
/* Next-token sampling per row of fp32 logits [num_rows, vocab] with per-row SamplingParams
 * (include/minisgl/core/types.h:12-20; device arrays temperature, top_k, top_p). Rows with
 * temperature <= 0 or top_k == 1 take the first index of the maximum (the reference's greedy
 * scan, scheduler.cpp:110-124). Other rows: candidates = the K largest logits (K = top_k if
 * 1 < top_k <= 1024, else min(vocab, 1024); ties at the K-th value to the lower ids) ordered by
 * (logit desc, id asc); weights exp((l - l_max) / temperature) summed in that order into c_i;
 * top-p keeps the first n candidates with c_{n-1} >= top_p * c_{K-1}; with u the 24-bit
 * SplitMix64 uniform of (seed, step, row), the token is the first i < n with c_i > u * c_{n-1}.
 * Deterministic for a given (seed, step). */
MSGL_API int msgl_sample(const float* logits, int num_rows, int vocab, const float* temperature,
                         const int* top_k, const float* top_p, uint64_t seed, uint64_t step,
                         int* out, msgl_stream_t stream);

/* ---------------------------------------------------------------- batch metadata */
/* Advances a decode batch on the device (the decode branch of Scheduler::step's host flatten,
 * src/scheduler/scheduler.cpp:83-106, with KVCachePool::allocate, src/cache/kvcache.cpp:21-28,
 * and the slot formula of kernels/cuda/radix.cu:19-22): for request r with L = seq_lens[r]
 * (its length in the step just run), input_ids[r] = next_tokens[r], positions[r] = L,
 * seq_lens[r] = L + 1, and when L % page_size == 0 a page is popped from the free stack
 * free_pages[0 .. *free_top) (top first, requests in order: the host pool's LIFO order) into
 * page_table[r][L / page_size]; slot_mapping[r] = page_table[r][L / page_size] * page_size +
 * L % page_size. All-or-nothing: if the stack runs out (MSGL_ERR_WORKSPACE, site 700) or a page
 * would land past max_pages (MSGL_ERR_BOUNDS, site 701), nothing is written and the device
 * error word records it. All arrays are device int32; page_table is [num_reqs, max_pages]. */
MSGL_API int msgl_decode_advance(const int* next_tokens, int* input_ids, int* positions,
                                 int* slot_mapping, int* page_table, int max_pages, int* seq_lens,
                                 const int* free_pages, int* free_top, int num_reqs, int page_size,
                                 msgl_stream_t stream);
/* msgl_decode_advance with finished [num_reqs] (device, may be NULL): requests whose entry is
 * nonzero are held -- no page is popped for them and their input id, position, slot and length
 * stay -- so a fixed-shape (graph-replayed) batch keeps running them, recomputing their last step
 * (the same K/V into the same slot) until the host retires them. */
MSGL_API int msgl_decode_advance_masked(const int* next_tokens, int* input_ids, int* positions,
                                        int* slot_mapping, int* page_table, int max_pages,
                                        int* seq_lens, const int* free_pages, int* free_top,
                                        const int* finished, int num_reqs, int page_size,
                                        msgl_stream_t stream);
/* The finish rule of Scheduler::step (scheduler.cpp:126-131) with the SamplingParams of
 * include/minisgl/core/types.h:12-20, on the device, for one decode step: for every request not
 * yet finished, token_out[r] = next_tokens[r], generated[r] += 1, and finished[r] = 1 once
 * generated[r] >= max_new_tokens[r] (the reference's max_tokens) or, unless ignore_eos[r] (NULL:
 * all zero), next_tokens[r] is one of stop_ids[0 .. num_stop_ids) (the model's end-of-sequence
 * ids; the reference never checks them, D17). Finished requests get token_out[r] = -1. All
 * arrays device int32 [num_reqs]; finished / generated are read and written. */
MSGL_API int msgl_decode_finish(const int* next_tokens, int* token_out, const int* max_new_tokens,
                                const int* ignore_eos, const int* stop_ids, int num_stop_ids,
                                int* finished, int* generated, int num_reqs, msgl_stream_t stream);

/* ---------------------------------------------------------------- paged attention */
/* Replaces Attention::forward (src/layer/layer.cpp:214-262) with attention over the paged KV
 * pool. Pools: [num_slots, Hkv * D] bf16, slot = page * page_size + offset (radix.cu:19-22).
 * page_table [num_reqs, max_pages] int32; seq_lens [num_reqs] = context length including this
 * step's tokens (already stored). head_dim 128, page_size 16, num_q_heads / num_kv_heads <= 8.
 *
 * Decode: one query token per request, q/out [num_reqs, Hq, D] bf16. max_seq_len bounds
 * seq_lens (it sizes the grid and the workspace). The workspace must be zero-filled once before
 * its first use; every call leaves it zero-filled again. */
MSGL_API size_t msgl_paged_attention_workspace_size(int num_reqs, int max_seq_len, int num_q_heads,
                                           int num_kv_heads, int head_dim);
MSGL_API int msgl_paged_attention_decode(const void* q, const void* k_pool, const void* v_pool,
                                int64_t num_slots, const int* page_table, int max_pages,
                                const int* seq_lens, int num_reqs, int max_seq_len,
                                int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                                float scale, void* out, void* workspace,
                                size_t workspace_bytes, msgl_stream_t stream);

/* Cascade decode for a batch whose first `shared_pages` page-table columns hold the same pages
 * in every row (a prefix shared through the radix cache, RadixCache::match_prefix) and whose
 * contexts all cover them. Same result as msgl_paged_attention_decode: the shared pages are
 * attended once per kv head for all requests' query heads together (full MMA rows), each
 * request's remaining pages as in plain decode, and the partial softmax states merged in a fixed
 * order. The kernel checks the sharing (a row that differs, or a context shorter than the prefix,
 * is recorded as MSGL_ERR_BOUNDS in the error word, sites 204 / 205). No counterpart in the
 * reference; workspace: msgl_paged_attention_cascade_workspace_size, zero-filled once, left
 * zero-filled. */
MSGL_API size_t msgl_paged_attention_cascade_workspace_size(int num_reqs, int max_seq_len,
                                                           int shared_pages, int num_q_heads,
                                                           int num_kv_heads, int head_dim);
MSGL_API int msgl_paged_attention_decode_cascade(const void* q, const void* k_pool,
                                                 const void* v_pool, int64_t num_slots,
                                                 const int* page_table, int max_pages,
                                                 const int* seq_lens, int num_reqs,
                                                 int max_seq_len, int shared_pages,
                                                 int num_q_heads, int num_kv_heads, int head_dim,
                                                 int page_size, float scale, void* out,
                                                 void* workspace, size_t workspace_bytes,
                                                 msgl_stream_t stream);

/* Decode without a caller workspace. No counterpart in the reference (its launchers take no
 * workspace); this is an addition for callers that cannot hand in device memory. Same arguments
 * and results as msgl_paged_attention_decode minus the workspace: the scratch is a file-scope
 * 8 MiB device array of the library. Batches whose msgl_paged_attention_workspace_size exceeds
 * 8 MiB are rejected with MSGL_ERR_WORKSPACE. No cudaMalloc / cudaFree or other allocating call;
 * each call clears (cudaMemsetAsync on `stream`) the split-KV arrival counters it uses. The first
 * call on a device looks up the array's address (cudaGetSymbolAddress) with that device current;
 * make that first call before any stream capture. Every call on a device shares the one array,
 * which keeps the last call's partial results; calls that overlap on the GPU (other streams, other
 * host threads) race on it and must be serialised by the caller. */
MSGL_API int msgl_paged_attention_decode_noalloc(const void* q, const void* k_pool,
                                                 const void* v_pool, int64_t num_slots,
                                                 const int* page_table, int max_pages,
                                                 const int* seq_lens, int num_reqs,
                                                 int max_seq_len, int num_q_heads,
                                                 int num_kv_heads, int head_dim, int page_size,
                                                 float scale, void* out, msgl_stream_t stream);

/* Extend / prefill: request r owns query rows [q_indptr[r], q_indptr[r+1]) of q/out
 * [total_q, Hq, D]; row i of an n-row request sits at position seq_lens[r] - n + i and attends
 * causally to context tokens 0..that position. max_q_len bounds the per-request row count. */
MSGL_API int msgl_paged_attention_extend(const void* q, const void* k_pool, const void* v_pool,
                                int64_t num_slots, const int* page_table, int max_pages,
                                const int* seq_lens, const int* q_indptr, int num_reqs,
                                int max_q_len, int num_q_heads, int num_kv_heads, int head_dim,
                                int page_size, float scale, void* out, msgl_stream_t stream);

/* ---------------------------------------------------------------- tcgen05 GEMMs */
/* Linear::forward (layer.cpp:122-143): y[M,N] = x[M,K] * W[N,K]^T, W in the reference's
 * [out, in] row-major layout. x, W bf16; y bf16 (out_dtype MSGL_BF16) or fp32 (MSGL_F32).
 * K % 64 == 0, N % 128 == 0, x/W/y 16-byte aligned. Split-K partial sums go through `workspace`
 * (msgl_gemm_workspace_size bytes; zero-filled once before first use, left zero-filled). */
MSGL_API size_t msgl_gemm_workspace_size(int M, int N, int K);
MSGL_API int msgl_gemm_bf16(const void* x, const void* w, void* y, int M, int N, int K, int out_dtype,
                   void* workspace, size_t workspace_bytes, msgl_stream_t stream);

/* gate_up projection + split + SwiGLU (qwen3.cpp:60-79, layer.cpp:145-161) in one GEMM:
 * y[M, I] = silu(x W_gate^T) * (x W_up^T), with w_packed the gate_up weight re-laid out by
 * msgl_pack_gate_up. I % 16 == 0 and 2I % 128 == 0. */
MSGL_API int msgl_pack_gate_up(const void* w_gate_up, void* w_packed, int inter, int hidden,
                      msgl_stream_t stream);
MSGL_API int msgl_gemm_gate_up_silu(const void* x, const void* w_packed, void* y, int M, int inter, int K,
                           void* workspace, size_t workspace_bytes, msgl_stream_t stream);

/* Linear::forward (layer.cpp:122-143) as split-K partials for decode-sized batches whose next
 * kernel adds them (msgl_add_partials_rmsnorm, msgl_qknorm_rope_store_kv_partials):
 * parts[s][M][N] (fp32) = x[:, Ks] W[:, Ks]^T over the s-th of `splits` equal k-block ranges, so
 * that sum_s parts[s] = x W^T. No cross-CTA reduction, no workspace. 1 <= M <= 256 (tokens
 * in tiles of 128),
 * 1 <= splits <= min(64, ceil(K / 64)); msgl_gemm_partials_splits gives the split count that
 * fills the GPU in one wave (0 for unsupported sizes). */
MSGL_API int msgl_gemm_partials_splits(int M, int N, int K);
MSGL_API int msgl_gemm_bf16_partials(const void* x, const void* w, float* parts, int M, int N, int K,
                                     int splits, msgl_stream_t stream);

/* lm_head (qwen3.cpp:178) fused with greedy sampling (scheduler.cpp:117-124): ids[m] = argmax_n
 * of the fp32 logits x[m] . W[n]; ties to the lowest id. `packed` is [M] uint64 scratch. */
MSGL_API int msgl_lm_head_argmax(const void* x, const void* w, int M, int vocab, int K,
                        unsigned long long* packed, int* ids, void* workspace,
                        size_t workspace_bytes, msgl_stream_t stream);

/* ---------------------------------------------------------------- MoE */
/* MoERouter::route (layer.cpp:270-309) after the router logits GEMM (msgl_gemm_bf16 with
 * out_dtype MSGL_F32): per token the top_k experts by logit, equal logits resolved to the larger
 * expert id (std::greater on pair<float,int>, layer.cpp:291-292); weight exp(logit), divided by
 * the top-k sum when norm_topk (layer.cpp:294-305). num_experts <= 256, top_k <= 32. */
MSGL_API int msgl_moe_route_topk(const float* router_logits, int num_tokens, int num_experts,
                                 int top_k, int norm_topk, int* topk_ids, float* topk_weights,
                                 msgl_stream_t stream);
/* The same on the router GEMM's split-K partials (msgl_gemm_bf16_partials, [nparts][T][E] fp32),
 * summed in part order before the selection; 1 <= nparts <= 64. */
MSGL_API int msgl_moe_route_topk_partials(const float* router_parts, int nparts, int num_tokens,
                                          int num_experts, int top_k, int norm_topk,
                                          int* topk_ids, float* topk_weights, msgl_stream_t stream);

/* Counting sort of the num_tokens * top_k (token, k) pairs by expert, stable in pair order:
 * expert_offsets [E+1] (rows of each expert in the sorted matrix), sorted_token [T*k] (token of
 * each sorted row; gather x with msgl_launch_index_gather), pair_pos [T*k] (sorted row of pair
 * t*k+j). Replaces the per-token expert loop of src/model/qwen3_moe.cpp:74-108. */
MSGL_API int msgl_moe_permute(const int* topk_ids, int num_tokens, int top_k, int num_experts,
                              int* expert_offsets, int* sorted_token, int* pair_pos,
                              msgl_stream_t stream);

/* Grouped tcgen05 GEMM over the expert-sorted rows: for expert e, rows
 * [offsets[e], offsets[e+1]) of x_sorted [max_rows, K] times W_e^T, W = [E, N, K] (each expert
 * in Linear's [out, in] layout), into y [max_rows, N]. The gate_up form takes per-expert weights
 * packed by msgl_pack_gate_up and writes silu(gate) * up [max_rows, inter]. The workspace
 * (msgl_grouped_gemm_workspace_size) holds the device-built tile list. */
MSGL_API size_t msgl_grouped_gemm_workspace_size(int max_rows, int num_experts);
MSGL_API int msgl_grouped_gemm_bf16(const void* x_sorted, const void* w, void* y,
                                    const int* expert_offsets, int num_experts, int N, int K,
                                    int max_rows, void* workspace, size_t workspace_bytes,
                                    msgl_stream_t stream);
MSGL_API int msgl_grouped_gemm_gate_up_silu(const void* x_sorted, const void* w_packed, void* y,
                                            const int* expert_offsets, int num_experts, int inter,
                                            int K, int max_rows, void* workspace,
                                            size_t workspace_bytes, msgl_stream_t stream);
/* msgl_grouped_gemm_bf16 over the tile list that the previous grouped call on this stream left in
 * the same workspace for the same expert_offsets, num_experts and max_rows (the expert down
 * projection after msgl_grouped_gemm_gate_up_silu): the per-call tile-list kernel is not launched
 * again where the schedule needs nothing else from it. A workspace filled for other offsets or
 * sizes gives wrong rows. */
MSGL_API int msgl_grouped_gemm_bf16_reuse_tiles(const void* x_sorted, const void* w, void* y,
                                                const int* expert_offsets, int num_experts, int N,
                                                int K, int max_rows, void* workspace,
                                                size_t workspace_bytes, msgl_stream_t stream);

/* out[t] = sum_j topk_weights[t,j] * y_sorted[pair_pos[t*k+j]], j in order, fp32 accumulation
 * (qwen3_moe.cpp:102-106). out [T, hidden] bf16; hidden % 8 == 0, top_k <= 32. */
MSGL_API int msgl_moe_combine(const void* y_sorted, const int* pair_pos, const float* topk_weights,
                              int num_tokens, int top_k, int hidden, void* out,
                              msgl_stream_t stream);

/* msgl_moe_combine fused with the residual add and the RMSNorm that follow it (the next decoder
 * layer's input_layernorm, src/layer/layer.cpp:79-112): m = combine row rounded to bf16,
 * residual += m (fp32 [T, hidden]), x_out = rmsnorm(residual) * norm_weight (bf16). Equal bit for
 * bit to msgl_moe_combine into x followed by msgl_add_rmsnorm(x, residual, ..., first = 0).
 * hidden % 8 == 0, hidden <= 8192, top_k <= 32; 16-byte aligned rows. */
MSGL_API int msgl_moe_combine_add_rmsnorm(const void* y_sorted, const int* pair_pos,
                                          const float* topk_weights, int num_tokens, int top_k,
                                          int hidden, float* residual, const void* norm_weight,
                                          float eps, void* x_out, msgl_stream_t stream);

/* Vocab-parallel lm_head: this rank's rows W [vocab_local, K] cover token ids
 * [vocab_offset, vocab_offset + vocab_local). packed[m] receives the rank's best
 * (logit, id) key, ties to the lowest id; combine the ranks with msgl_tp_argmax_combine. */
MSGL_API int msgl_lm_head_argmax_partial(const void* x, const void* w, int M, int vocab_local,
                                         int K, int vocab_offset, unsigned long long* packed,
                                         void* workspace, size_t workspace_bytes,
                                         msgl_stream_t stream);

/* ---------------------------------------------------------------- tensor parallelism */
/* TPCommunicator (include/minisgl/distributed/tp.h:9-25; a stub in the reference,
 * src/distributed/tp.cpp:13-47) over NCCL, one process per GPU. Rank 0 creates the id
 * (msgl_tp_unique_id_size() bytes) and the launcher broadcasts it to every rank. */
typedef struct msgl_tp msgl_tp;
MSGL_API size_t msgl_tp_unique_id_size(void);
MSGL_API int msgl_tp_get_unique_id(void* out);
MSGL_API int msgl_tp_init(int rank, int world, const void* unique_id, msgl_tp** out);
MSGL_API int msgl_tp_destroy(msgl_tp* tp);
MSGL_API int msgl_tp_rank(const msgl_tp* tp);
MSGL_API int msgl_tp_world(const msgl_tp* tp);
/* TPCommunicator::all_reduce_sum (tp.cpp:18-31): in-place sum of bf16 x [n] over the ranks. */
MSGL_API int msgl_tp_all_reduce_sum(msgl_tp* tp, void* x, int64_t n, msgl_stream_t stream);
/* TPCommunicator::all_gather (tp.cpp:33-47; a stub in the reference): every rank contributes
 * `bytes` bytes of `send`; `recv` receives world * bytes, rank q's contribution at q * bytes. */
MSGL_API int msgl_tp_all_gather(msgl_tp* tp, const void* send, void* recv, size_t bytes,
                                msgl_stream_t stream);
/* Row-parallel projection output x [T, H] (this rank's partial sum) all-reduced, then
 * msgl_add_rmsnorm (residual += x; x = rmsnorm(residual) * w; first as in msgl_add_rmsnorm). */
MSGL_API int msgl_tp_allreduce_add_rmsnorm(msgl_tp* tp, void* x, float* residual,
                                           const void* weight, int num_tokens, int hidden,
                                           float eps, int first, msgl_stream_t stream);
/* packed [num_rows] uint64 keys (msgl_lm_head_argmax_partial) max-reduced over the ranks and
 * unpacked to ids [num_rows]: greedy sampling over the full vocabulary. */
/* One-kernel all-reduce + add + RMSNorm over NVLink peer memory (no counterpart in the
 * reference, whose TPCommunicator is a stub; it replaces NCCL all-reduce + msgl_add_rmsnorm).
 * msgl_tp_enable_p2p (collective, every rank the same `bytes`) allocates this rank's
 * peer-mapped region -- three slots of `bytes` (two for partial rows, one for the two-shot
 * form's output rows) plus flags -- exchanges cudaIpc
 * handles with an NCCL all-gather on `stream` and maps every other rank's region (plain peer
 * loads; no multicast). msgl_tp_p2p_buffer returns slot 0 or 1: the row-parallel GEMM writes its
 * partial [T, H] bf16 rows there, and CONSECUTIVE fused calls must use alternate slots (checked).
 * msgl_tp_fused_allreduce_add_rmsnorm (every rank, same calls in the same order) computes, on
 * every rank, residual (+)= sum over ranks (rank order, fp32) of the partial rows and
 * x_out = RMSNorm(residual) * weight (bf16; `first` as msgl_add_rmsnorm); all ranks get the same
 * bits. The ranks meet through per-CTA epoch flags in the regions (bounded waits: a rank that does
 * not arrive within ~2 s gives MSGL_ERR_TIMEOUT in the error word, site 500). */
/* After MSGL_ERR_TIMEOUT from any of the fused calls (site 500 / 503) the ranks' call pairing is
 * undefined: destroy the communicator and create a new one (msgl_tp_destroy, msgl_tp_init,
 * msgl_tp_enable_p2p) before the next collective call. A CTA whose wait ran out does not advance
 * its epoch, so a late peer never reads rows that a later call is rewriting.
 *
 * msgl_tp_fused_allreduce_add_rmsnorm_2shot: the same result, computed two-shot. With
 * per = ceil(num_tokens / world), rank r reduces only rows [r per, min(T, (r + 1) per)): it
 * reads those rows of every rank's partial, adds its residual rows, normalises, and stores the
 * bf16 rows into slot 2 of EVERY rank; x_out must be this rank's slot 2 (msgl_tp_p2p_buffer),
 * which afterwards holds all T rows on every rank. The residual is row-partitioned: this call
 * reads and writes only the rows rank r owns, so a caller that uses only the two-shot form keeps
 * each residual row on its owning rank. NVLink bytes per rank: (W-1)/W of the rows read and
 * written once (the one-shot form reads W-1 full copies). */
MSGL_API int msgl_tp_enable_p2p(msgl_tp* tp, size_t bytes, msgl_stream_t stream);
MSGL_API int msgl_tp_p2p_buffer(msgl_tp* tp, int slot, void** ptr, size_t* bytes);
MSGL_API int msgl_tp_fused_allreduce_add_rmsnorm(msgl_tp* tp, const void* partial, void* x_out,
                                                 float* residual, const void* weight,
                                                 int num_tokens, int hidden, float eps, int first,
                                                 msgl_stream_t stream);
MSGL_API int msgl_tp_fused_allreduce_add_rmsnorm_2shot(msgl_tp* tp, const void* partial,
                                                       void* x_out, float* residual,
                                                       const void* weight, int num_tokens,
                                                       int hidden, float eps, int first,
                                                       msgl_stream_t stream);
MSGL_API int msgl_tp_argmax_combine(msgl_tp* tp, unsigned long long* packed, int* ids,
                                    int num_rows, msgl_stream_t stream);
/* Host only: the shard of `rank` as 8 ints {q_head0, q_heads, kv_head0, kv_heads, inter0,
 * inter_cols, vocab0, vocab_rows} (column-parallel qkv / gate_up, row-parallel o / down,
 * vocab-parallel lm_head; kv heads replicated when world > num_kv_heads). */
MSGL_API int msgl_tp_shard_plan(int num_q_heads, int num_kv_heads, int inter, int vocab,
                                int rank, int world, int* out8);

/* ---------------------------------------------------------------- sampling / utilities */
/* Greedy argmax over logits [num_rows, vocab] (scheduler.cpp:117-124): first maximum wins. */
MSGL_API int msgl_argmax(const void* logits, int num_rows, int vocab, int dtype, int* out,
                msgl_stream_t stream);

/* Fill a bf16 buffer with N(mean, std) values from a counter-based generator
 * (Philox4x32-10 keyed by (seed, stream_id), Box-Muller). Used for random-init weights and
 * synthetic KV contents. */
MSGL_API int msgl_fill_normal_bf16(void* out, int64_t n, uint64_t seed, uint64_t stream_id, float mean,
                          float std, msgl_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* MSGL_KERNELS_H */
