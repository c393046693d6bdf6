/*
 * msgl_engine.h -- C ABI of the device-side Qwen3 executor in libmsgl.
 *
 * The executor is the B200 counterpart of Qwen3ForCausalLM / Qwen3MoEForCausalLM
 * (include/minisgl/model/qwen3.h:34-50, qwen3_moe.h:35-51 of mini-sglang-cpp): it owns bf16
 * weights, one paged K/V pool per layer (layout of src/cache/kvcache.cpp:8-19, bf16, token-major
 * [num_pages * page_size, Hkv * D]) and a preallocated workspace, and runs the per-layer forward
 * (src/model/qwen3.cpp:16-83, 168-180) entirely through the kernels of msgl_kernels.h.
 *
 * A step is described by msgl_batch: the flattened token ids / positions of the scheduled
 * requests (Scheduler::step, src/scheduler/scheduler.cpp:83-106) plus the paged-KV metadata
 * the reference never passes down (page table, context lengths, query offsets, pool slots).
 * The executor allocates all of its device memory at create / alloc_kv time; forward() itself
 * allocates nothing and is capturable into a CUDA graph.
 */
#ifndef MSGL_ENGINE_H
#define MSGL_ENGINE_H

#include "msgl_kernels.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct msgl_model msgl_model;

/* Model shape (fields of ModelConfig, include/minisgl/model/config.h:18-36) plus capacity. */
typedef struct {
    int num_layers, hidden, num_q_heads, num_kv_heads, head_dim, inter, vocab;
    int num_experts, top_k, moe_inter, norm_topk; /* num_experts == 0: dense */
    float eps, rope_base;
    int max_position;      /* RoPE table rows; bounds every position */
    int max_tokens;        /* capacity: tokens per step */
    int max_reqs;          /* capacity: requests per step */
    int tp_rank, tp_size;  /* tensor parallel shard of this process (1 GPU each) */
} msgl_model_config;

/* One scheduler step. All pointers are device int32 arrays. */
typedef struct {
    int num_tokens;          /* T */
    int num_reqs;            /* B */
    int is_decode;           /* 1: every request contributes exactly one token */
    int max_pages;           /* page_table row width */
    int max_seq_len;         /* bound on seq_lens */
    int max_q_len;           /* bound on per-request query rows */
    const int* input_ids;    /* [T] */
    const int* positions;    /* [T] */
    const int* slot_mapping; /* [T] pool slot of each token (page * page_size + offset), <0 skip */
    const int* page_table;   /* [B, max_pages] */
    const int* seq_lens;     /* [B] context length including this step's tokens */
    const int* q_indptr;     /* [B+1] */
    const int* last_idx;     /* [B] row of each request's last token (q_indptr[r+1]-1) */
    int shared_prefix_pages; /* > 0: the first n page-table columns are the same pages in every
                                row (a prefix shared through the radix cache) and every context
                                covers them; decode then runs the cascade kernel. 0: none.
                                MSGL_SHARED_PREFIX_DETECT (msgl_model_step_host only): computed
                                from the host page table */
    int decode_tail;         /* mixed (chunked-prefill) batches, is_decode == 0: the last n
                                requests each contribute exactly one query row, the last n rows
                                of the step; attention then runs the split-KV decode kernel on
                                them and the extend kernel on the requests before. 0: no such
                                claim (every request through the extend kernel).
                                MSGL_DECODE_TAIL_DETECT (msgl_model_step_host only): computed
                                from the host q_indptr */
} msgl_batch;
#define MSGL_DECODE_TAIL_DETECT (-1)
#define MSGL_SHARED_PREFIX_DETECT (-1)

/* ------------------------------------------------------------------ prefix cache (host)
 * RadixCache (src/cache/kvcache.cpp:40-115) at page granularity, with its insert / split /
 * eviction defects fixed: match walks the longest cached prefix of whole pages (splitting a
 * node where it ends inside one), insert adds the uncached pages and reports the caller's
 * pages for the cached part that differ from the tree's (to return to the free list), lock
 * (+1 / -1) pins the path of a node for a running request, evict frees up to num_pages pages of
 * unlocked leaves, least recently used first (ties: the lower page id), one page at a time from
 * the leaf's end. Node handles: 0 is the root; a handle stays valid until its node is evicted. */
typedef struct msgl_radix msgl_radix;
MSGL_API int msgl_radix_create(int page_size, msgl_radix** out);
MSGL_API int msgl_radix_destroy(msgl_radix* r);
MSGL_API int msgl_radix_match(msgl_radix* r, const int32_t* tokens, int num_tokens, int32_t* pages_out,
                              int max_pages, int* matched_tokens, int64_t* node);
MSGL_API int msgl_radix_insert(msgl_radix* r, const int32_t* tokens, int num_tokens, const int32_t* pages,
                               int* present_tokens, int32_t* dup_pages_out, int* num_dup, int64_t* node);
MSGL_API int msgl_radix_lock(msgl_radix* r, int64_t node, int delta);
MSGL_API int msgl_radix_evict(msgl_radix* r, int num_pages, int32_t* freed_out, int* num_freed);
MSGL_API int msgl_radix_size(const msgl_radix* r, int* cached_pages, int* evictable_pages);

MSGL_API int msgl_model_create(const msgl_model_config* cfg, msgl_model** out);
MSGL_API int msgl_model_destroy(msgl_model* m);

/* Weights. random_init: every matrix N(0, std) from the counter-based generator keyed by
 * (seed, tensor index), every norm gain 1.0. set_weight: host bf16 bit patterns of the FULL
 * (unsharded) tensor named as in the reference's loader (qwen3.cpp:94-166) shortened:
 *   embed, norm, lm_head, layers.<l>.{input_ln, qkv, q_norm, k_norm, o, post_ln, gate_up, down,
 *   router}, layers.<l>.experts.<e>.{gate_up, down}
 * (gate_up rows gate | up; qkv rows q | k | v). The executor keeps its tensor-parallel shard. */
MSGL_API int msgl_model_random_init(msgl_model* m, uint64_t seed, float std, msgl_stream_t stream);
MSGL_API int msgl_model_set_weight(msgl_model* m, const char* name, const uint16_t* host_bf16,
                                   int64_t numel, msgl_stream_t stream);
/* Checkpoint ingest (WeightLoader, src/model/weight.cpp:32-105, with the name maps of
 * qwen3.cpp:94-166 / qwen3_moe.cpp:123-199): every *.safetensors file of model_dir is indexed
 * by its JSON header; model.embed_tokens / model.norm / lm_head (the embedding when absent:
 * tied) and per layer input_layernorm, post_attention_layernorm, self_attn.{qkv_proj | q_proj +
 * k_proj + v_proj, q_norm, k_norm, o_proj}, mlp.{gate_up_proj | gate_proj + up_proj, down_proj}
 * (MoE: mlp.gate and mlp.experts.<e>.{gate_up_proj | gate_proj + up_proj, down_proj}) go
 * through msgl_model_set_weight. BF16 is copied, F16 / F32 rounded to bf16 (nearest even). A
 * missing tensor or a malformed header is MSGL_ERR_INVALID_ARG with the name in
 * msgl_last_error(). msgl_safetensors_index only reads the headers (host only, no device). */
MSGL_API int msgl_model_load_safetensors(msgl_model* m, const char* model_dir, msgl_stream_t stream);
MSGL_API int msgl_safetensors_index(const char* model_dir, int64_t* num_tensors, int64_t* total_bytes);
/* The configuration the executor was created with. */
MSGL_API int msgl_model_get_config(const msgl_model* m, msgl_model_config* out);
/* Device bytes held by weights / KV pools / workspace. */
MSGL_API int64_t msgl_model_weight_bytes(const msgl_model* m);

/* KV pools: num_pages pages of page_size (16) tokens per layer, zero-filled. */
MSGL_API int msgl_model_alloc_kv(msgl_model* m, int num_pages, int page_size, msgl_stream_t stream);
MSGL_API int msgl_model_kv_pool(msgl_model* m, int layer, void** k_pool, void** v_pool,
                                int64_t* num_slots);

/* One forward step: next_tokens [B] (device) = greedy tokens of each request's last row
 * (scheduler.cpp:117-124 on the last token, fixing D10); logits (optional, device fp32
 * [B, vocab]) receives the final logits of those rows (under tensor parallelism every rank
 * computes its vocab rows and the shards are all-gathered, so every rank gets all of them).
 * flags & MSGL_FWD_GRAPH: run the step as a CUDA graph, captured on first use and replayed
 * while the batch's pointers and shape fields are unchanged (stream must not be the legacy
 * default stream). */
#define MSGL_FWD_GRAPH 1
MSGL_API int msgl_model_forward(msgl_model* m, const msgl_batch* batch, int* next_tokens,
                                float* logits, int flags, msgl_stream_t stream);

/* The scheduler-facing step (Scheduler::step -> model_->forward, scheduler.cpp:108-124):
 * `host_batch` holds HOST pointers (pinned for asynchronous copies); the executor copies them
 * into its own device buffers, runs the step (as a CUDA graph when flags & MSGL_FWD_GRAPH and
 * the step is a decode), copies the greedy tokens back into host_next_tokens [B] and
 * synchronises the stream. */
MSGL_API int msgl_model_step_host(msgl_model* m, const msgl_batch* host_batch,
                                  int* host_next_tokens, int flags, msgl_stream_t stream);
/* Overlap scheduling (SchedulerConfig::overlap_scheduling, include/minisgl/scheduler/
 * scheduler.h:23, which the reference never acts on): msgl_model_step_host without the wait.
 * The copies, the step and the D2H of the greedy tokens are queued on `stream` and the call
 * returns with a ticket; msgl_model_step_wait(ticket) waits for that step (one of the last two
 * submitted). Consecutive submissions use the executor's two staging sets in turn, so the host
 * can build and submit step N+1 while step N runs; the host arrays of a step (pinned for
 * asynchronous copies) and its host_next_tokens must stay untouched until its wait returns.
 * flags & MSGL_STEP_TOKENS_FROM_PREV (a decode step after a submitted step): input_ids is not
 * read from the host -- row r takes the greedy token of row r of the previous submitted step,
 * on the device -- so a decode step can be submitted before the previous step's tokens reach
 * the host. */
#define MSGL_STEP_TOKENS_FROM_PREV 2
MSGL_API int msgl_model_step_host_async(msgl_model* m, const msgl_batch* host_batch,
                                        int* host_next_tokens, int flags, msgl_stream_t stream,
                                        uint64_t* ticket);
MSGL_API int msgl_model_step_wait(msgl_model* m, uint64_t ticket);
/* Decode steps without the host in between (Scheduler::step's decode loop with the flatten of
 * scheduler.cpp:83-106 on the device): from one decode step's device arrays (*batch, e.g. built
 * on the host once), run num_steps greedy steps back to back; step s writes its ids to
 * token_log[s * num_reqs ...] and, before step s + 1, msgl_decode_advance moves the arrays of
 * *batch on in place (new pages come off the device free stack free_pages[0 .. *free_top)).
 * Every step runs with max_seq_len = max_pages * page_size (capped at max_position), so with
 * MSGL_FWD_GRAPH one captured graph serves every step. Nothing waits on the host: the caller
 * synchronises the stream before reading token_log. */
MSGL_API int msgl_model_decode_steps(msgl_model* m, const msgl_batch* batch, int num_steps,
                                     int* token_log, const int* free_pages, int* free_top,
                                     int flags, msgl_stream_t stream);
/* The same with the finish rules of Scheduler::step (scheduler.cpp:126-131) and SamplingParams
 * (include/minisgl/core/types.h:12-20) applied on the device after every step
 * (msgl_decode_finish): a request finishes after max_new_tokens[r] tokens or, unless
 * ignore_eos[r], on a stop id. From then on its token_log entries are -1 and the advance holds it
 * in place (msgl_decode_advance_masked: no new page, its last step recomputed), so the batch keeps
 * its shape (and its captured graph) until the host retires the request. finished [B] and
 * generated [B] are read and written (zero-fill them for fresh requests); all device int32. */
typedef struct {
    const int* max_new_tokens; /* [B] tokens each request may generate (the reference's max_tokens) */
    const int* ignore_eos;     /* [B] nonzero: stop ids do not finish the request; NULL: none set */
    const int* stop_ids;       /* [num_stop_ids] end-of-sequence token ids */
    int num_stop_ids;
    int* finished;             /* [B] in / out */
    int* generated;            /* [B] in / out */
} msgl_stop_rules;
MSGL_API int msgl_model_decode_steps_stop(msgl_model* m, const msgl_batch* batch, int num_steps,
                                          int* token_log, const int* free_pages, int* free_top,
                                          const msgl_stop_rules* stop, int flags,
                                          msgl_stream_t stream);

/* Debug: device pointer to the hidden state [max_tokens, hidden] bf16 after the most recent
 * forward (the last layer's output before the final norm) -- used by per-layer parity tests
 * together with num_layers_override. */
MSGL_API int msgl_model_debug_hidden(msgl_model* m, void** x, float** residual);

/* Attach the tensor-parallel communicator of this rank (required when cfg.tp_size > 1; its rank
 * and world must match the config). The executor then all-reduces the row-parallel o_proj /
 * down_proj outputs (fused with the following add + RMSNorm) and combines the vocab-parallel
 * lm_head argmax over the ranks. */
MSGL_API int msgl_model_set_tp(msgl_model* m, msgl_tp* tp);
MSGL_API int msgl_model_set_num_layers_run(msgl_model* m, int n);

#ifdef __cplusplus
}
#endif
#endif /* MSGL_ENGINE_H */
