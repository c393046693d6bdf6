// tp.cu -- tensor-parallel communicator (TPCommunicator, src/distributed/tp.cpp:13-47, which is a
// stub in the reference) over NCCL on NVLink / NVSwitch, one process per GPU.
//
//  * msgl_tp_all_reduce_sum   TPCommunicator::all_reduce_sum (tp.cpp:18-31): in-place sum of a
//                             bf16 [n] buffer over all ranks
//  * msgl_tp_allreduce_add_rmsnorm   the row-parallel o_proj / down_proj output all-reduced and
//                             fused with the following residual add + RMSNorm (layer.cpp:79-112)
//  * msgl_tp_argmax_combine   vocab-parallel greedy sampling: each rank's packed (logit, id) keys
//                             reduced with a 64-bit max, then unpacked to token ids
//  * msgl_tp_shard_plan       which rows / columns of every weight a rank owns (host only)
#include <nccl.h>

#include <cstring>
#include <string>

#include "common.cuh"

struct msgl_tp {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
};

namespace msgl {
namespace {

int nccl_err(ncclResult_t r, const char* what) {
    std::string m = std::string(what) + ": " + ncclGetErrorString(r);
    return set_error(MSGL_ERR_NCCL, m.c_str());
}

__global__ void unpack_keys_kernel(const unsigned long long* __restrict__ packed,
                                   int* __restrict__ ids, int M) {
    pdl_wait();
    pdl_trigger();
    int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m < M) ids[m] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(packed[m] & 0xFFFFFFFFull));
}

}  // namespace
}  // namespace msgl

using namespace msgl;

extern "C" {

size_t msgl_tp_unique_id_size(void) { return sizeof(ncclUniqueId); }

int msgl_tp_get_unique_id(void* out) {
    if (!out) return set_error(MSGL_ERR_INVALID_ARG, "tp_get_unique_id: null");
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return nccl_err(r, "ncclGetUniqueId");
    std::memcpy(out, &id, sizeof(id));
    return MSGL_OK;
}

int msgl_tp_init(int rank, int world, const void* unique_id, msgl_tp** out) {
    if (!out || !unique_id || world < 1 || rank < 0 || rank >= world)
        return set_error(MSGL_ERR_INVALID_ARG, "tp_init: bad rank / world");
    *out = nullptr;
    auto* tp = new msgl_tp();
    tp->rank = rank;
    tp->world = world;
    if (world > 1) {
        ncclUniqueId id;
        std::memcpy(&id, unique_id, sizeof(id));
        ncclResult_t r = ncclCommInitRank(&tp->comm, world, id, rank);
        if (r != ncclSuccess) {
            delete tp;
            return nccl_err(r, "ncclCommInitRank");
        }
    }
    *out = tp;
    return MSGL_OK;
}

int msgl_tp_destroy(msgl_tp* tp) {
    if (!tp) return MSGL_OK;
    if (tp->comm) ncclCommDestroy(tp->comm);
    delete tp;
    return MSGL_OK;
}

int msgl_tp_rank(const msgl_tp* tp) { return tp ? tp->rank : 0; }
int msgl_tp_world(const msgl_tp* tp) { return tp ? tp->world : 1; }

int msgl_tp_all_reduce_sum(msgl_tp* tp, void* x, int64_t n, msgl_stream_t stream) {
    if (!tp || n < 0) return set_error(MSGL_ERR_INVALID_ARG, "tp_all_reduce_sum: bad args");
    if (tp->world == 1 || n == 0) return MSGL_OK;
    ncclResult_t r = ncclAllReduce(x, x, static_cast<size_t>(n), ncclBfloat16, ncclSum, tp->comm,
                                   stream);
    return r == ncclSuccess ? MSGL_OK : nccl_err(r, "ncclAllReduce");
}

int msgl_tp_allreduce_add_rmsnorm(msgl_tp* tp, void* x, float* residual, const void* weight,
                                  int num_tokens, int hidden, float eps, int first,
                                  msgl_stream_t stream) {
    int rc = msgl_tp_all_reduce_sum(tp, x, static_cast<int64_t>(num_tokens) * hidden, stream);
    if (rc) return rc;
    return msgl_add_rmsnorm(x, residual, weight, num_tokens, hidden, eps, first, stream);
}

int msgl_tp_argmax_combine(msgl_tp* tp, unsigned long long* packed, int* ids, int num_rows,
                           msgl_stream_t stream) {
    if (!tp || num_rows < 0) return set_error(MSGL_ERR_INVALID_ARG, "tp_argmax_combine: bad args");
    if (num_rows == 0) return MSGL_OK;
    if (tp->world > 1) {
        ncclResult_t r = ncclAllReduce(packed, packed, static_cast<size_t>(num_rows), ncclUint64,
                                       ncclMax, tp->comm, stream);
        if (r != ncclSuccess) return nccl_err(r, "ncclAllReduce(max)");
    }
    launch_pdl(unpack_keys_kernel, dim3((num_rows + 255) / 256), dim3(256), 0, stream, packed, ids,
               num_rows);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

// Megatron-style shard of one rank (host only, no device work):
//  q heads [q0, q0 + hq_l), kv heads [kv0, kv0 + hkv_l) (replicated when tp > Hkv: each rank
//  keeps the kv head of its query group), intermediate columns [i0, i0 + inter_l) of gate, up
//  and down, vocab rows [v0, v0 + vocab_l) of lm_head.
int msgl_tp_shard_plan(int num_q_heads, int num_kv_heads, int inter, int vocab, int rank,
                       int world, int* out8) {
    if (!out8 || world < 1 || rank < 0 || rank >= world || num_kv_heads <= 0 ||
        num_q_heads % num_kv_heads || num_q_heads % world || inter % world)
        return set_error(MSGL_ERR_INVALID_ARG, "tp_shard_plan: shape not divisible by world");
    const int hq_l = num_q_heads / world;
    const int group = num_q_heads / num_kv_heads;
    int hkv_l, kv0;
    if (num_kv_heads >= world) {
        if (num_kv_heads % world) return set_error(MSGL_ERR_INVALID_ARG, "tp_shard_plan: Hkv % world");
        hkv_l = num_kv_heads / world;
        kv0 = rank * hkv_l;
    } else {
        if (hq_l > group || group % hq_l)
            return set_error(MSGL_ERR_INVALID_ARG, "tp_shard_plan: a rank's q heads span kv heads");
        hkv_l = 1;
        kv0 = (rank * hq_l) / group;
    }
    const int inter_l = inter / world;
    const int vocab_l = (vocab + world - 1) / world;
    const int v0 = rank * vocab_l;
    out8[0] = rank * hq_l;
    out8[1] = hq_l;
    out8[2] = kv0;
    out8[3] = hkv_l;
    out8[4] = rank * inter_l;
    out8[5] = inter_l;
    out8[6] = v0;
    out8[7] = v0 >= vocab ? 0 : (v0 + vocab_l > vocab ? vocab - v0 : vocab_l);
    return MSGL_OK;
}

}  // extern "C"
