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
//  * msgl_tp_enable_p2p / msgl_tp_p2p_buffer / msgl_tp_fused_allreduce_add_rmsnorm
//                             the same all-reduce + add + RMSNorm as ONE kernel over NVLink peer
//                             memory: every rank reads the other ranks' partial rows directly
//                             (cudaIpc mappings, plain loads, no multicast) -- see below.
//  * msgl_tp_fused_allreduce_add_rmsnorm_2shot
//                             the two-shot form: each rank reduces and normalises only its block
//                             of rows and stores the normed rows into every rank's x buffer.
#include <nccl.h>

#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"

constexpr int kTpMaxWorld = 8;

struct msgl_tp {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    // peer-mapped region (msgl_tp_enable_p2p):
    //   [slot 0: data_bytes][slot 1: data_bytes][slot 2 (x rows of the two-shot): data_bytes][flags]
    void* sym = nullptr;
    size_t data_bytes = 0;
    void* peer[kTpMaxWorld] = {};  // every rank's region in this process (peer[rank] = sym)
    int last_slot = -1;            // slot of the previous fused call (calls must alternate)
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

// ------------------------------------------------------------------ P2P all-reduce + norm
// Region of each rank: two slots of partial rows (consecutive calls alternate slots), then
// flags (4-byte words, zero at setup), one per CTA index b < kTpMaxCtas so that CTA b of every
// rank pairs with CTA b of the others and no two CTAs write the same word:
//   ready[q][b]  = e + 1 once CTA b of rank q starts call e (its partial rows are complete)
//   epoch[b]     calls CTA b has taken part in on this rank (the same on every rank: all ranks
//                run the same calls with the same row count, hence the same grid)
// Why two slots and no end-of-call handshake: a slot is rewritten two calls later, after this
// rank's call in between waited for every peer's ready flag of that call -- raised only once the
// peer's previous call, the one that read the slot, had completed.
//   done[q][b]   = e + 1 once CTA b of rank q has stored its normed rows of call e into every
//                rank's slot 2 (two-shot only)
constexpr int kTpMaxCtas = 148;
constexpr int kSlots = 3;
constexpr size_t kReadyOff = 0;                                          // [kTpMaxWorld][kTpMaxCtas]
constexpr size_t kEpochOff = static_cast<size_t>(kTpMaxWorld) * kTpMaxCtas;  // [kTpMaxCtas]
constexpr size_t kDoneOff = kEpochOff + kTpMaxCtas;                      // [kTpMaxWorld][kTpMaxCtas]
constexpr size_t kFlagBytes = (kDoneOff + static_cast<size_t>(kTpMaxWorld) * kTpMaxCtas) * 4;
struct TpPeers {
    const __nv_bfloat16* part[kTpMaxWorld];  // every rank's partial rows (this call's slot)
    unsigned* flags[kTpMaxWorld];            // every rank's flag area
    __nv_bfloat16* xrows[kTpMaxWorld];       // every rank's slot 2 (two-shot output rows)
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread t < world (t != rank) of CTA b: raise word [rank][b] of the flag array at `off` on rank
// t, then wait (bounded) until rank t raised this rank's word [t][b]; the CTA then synchronises.
// Returns false on every thread when any wait of the CTA ran out (MSGL_ERR_TIMEOUT, `site`).
__device__ __forceinline__ bool flag_exchange(const TpPeers& peers, const unsigned* local,
                                              size_t off, int world, int rank, unsigned value,
                                              int* err, int site) {
    const int t = threadIdx.x;
    bool ok = true;
    if (t < world && t != rank) {
        st_release_sys(peers.flags[t] + off + rank * kTpMaxCtas + blockIdx.x, value);
        const unsigned* mine = local + off + t * kTpMaxCtas + blockIdx.x;
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_sys(mine) < value) {
            if (globaltimer_ns() - t0 > 2000000000ull) {
                record_error(err, MSGL_ERR_TIMEOUT, site);
                ok = false;
                break;
            }
        }
    }
    return __syncthreads_and(ok) != 0;
}

// One CTA (128 threads, VPT 8-element vectors per thread) per row, rows strided over the grid.
// x[row] = RMSNorm(residual[row] (+)= sum over ranks, in rank order, of partial_q[row]) * w.
// Every rank sums the same values in the same order, so every rank gets the same bits. The row
// of every rank (its own included) comes into shared memory with one bulk copy each
// (cp.async.bulk from the peer-mapped region, no multicast): a few large NVLink transfers per
// row instead of one 16-byte request per thread and vector.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

template <int VPT>
__global__ void __launch_bounds__(128)
tp_fused_ar_norm_kernel(TpPeers peers, int world, int rank, __nv_bfloat16* __restrict__ x_out,
                        float* __restrict__ resid, const __nv_bfloat16* __restrict__ w, int T,
                        int H, float eps, int first, unsigned* __restrict__ local, int* err) {
    extern __shared__ __align__(16) uint8_t ar_smem[];
    const __nv_bfloat16* rows = reinterpret_cast<const __nv_bfloat16*>(ar_smem);  // [world][H]
    uint64_t* bar = reinterpret_cast<uint64_t*>(ar_smem + static_cast<size_t>(world) * H * 2);
    __shared__ float red[4];
    pdl_wait();  // this rank's partial (the previous kernel's output) is complete
    pdl_trigger();
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }
    unsigned* epoch_p = local + kEpochOff + blockIdx.x;
    const unsigned e = *reinterpret_cast<volatile unsigned*>(epoch_p);
    // every rank's partial is complete
    const bool ok = flag_exchange(peers, local, kReadyOff, world, rank, e + 1, err, 500);
    const int nvec = H >> 3;
    const uint32_t row_bytes = static_cast<uint32_t>(H) * 2;
    uint32_t phase = 0;
    for (int row = blockIdx.x; row < T; row += gridDim.x) {
        const int64_t rbase = static_cast<int64_t>(row) * H;
        if (threadIdx.x == 0) {
            fence_proxy_async_global();  // the acquired peer rows, read through the async proxy
            fence_proxy_async();         // this CTA's reads of the previous row's copies are done
            mbar_arrive_expect_tx(bar, row_bytes * world);
            for (int q = 0; q < world; ++q)
                bulk_load(ar_smem + static_cast<size_t>(q) * row_bytes, peers.part[q] + rbase, row_bytes, bar);
        }
        float v[VPT][8];
        float rr[VPT][8];
#pragma unroll
        for (int i = 0; i < VPT; ++i) {  // residual loads overlap the copies
            const int vi = threadIdx.x + i * 128;
            if (vi >= nvec || first) continue;
            const float4* r4 = reinterpret_cast<const float4*>(resid + rbase + vi * 8);
            const float4 a = r4[0], b = r4[1];
            rr[i][0] = a.x; rr[i][1] = a.y; rr[i][2] = a.z; rr[i][3] = a.w;
            rr[i][4] = b.x; rr[i][5] = b.y; rr[i][6] = b.z; rr[i][7] = b.w;
        }
        mbar_wait(bar, phase, err, 502);
        phase ^= 1;
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int vi = threadIdx.x + i * 128;
            if (vi >= nvec) continue;
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
            for (int q = 0; q < world; ++q) {
                const uint4 u = *reinterpret_cast<const uint4*>(rows + static_cast<int64_t>(q) * H + vi * 8);
                v[i][0] += bf16lo(u.x); v[i][1] += bf16hi(u.x);
                v[i][2] += bf16lo(u.y); v[i][3] += bf16hi(u.y);
                v[i][4] += bf16lo(u.z); v[i][5] += bf16hi(u.z);
                v[i][6] += bf16lo(u.w); v[i][7] += bf16hi(u.w);
            }
            if (!first) {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] += rr[i][j];
            }
            float4* r4 = reinterpret_cast<float4*>(resid + rbase + vi * 8);
            r4[0] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
            r4[1] = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
#pragma unroll
            for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
        }
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();  // also: every thread is done reading this row's copies
        const float tot = red[0] + red[1] + red[2] + red[3];
        __syncthreads();
        const float inv = 1.0f / sqrtf(tot / static_cast<float>(H) + eps);
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int vi = threadIdx.x + i * 128;
            if (vi >= nvec) continue;
            const uint4 wu = *reinterpret_cast<const uint4*>(w + vi * 8);
            uint4 o;
            o.x = pack_bf16x2(v[i][0] * inv * bf16lo(wu.x), v[i][1] * inv * bf16hi(wu.x));
            o.y = pack_bf16x2(v[i][2] * inv * bf16lo(wu.y), v[i][3] * inv * bf16hi(wu.y));
            o.z = pack_bf16x2(v[i][4] * inv * bf16lo(wu.z), v[i][5] * inv * bf16hi(wu.z));
            o.w = pack_bf16x2(v[i][6] * inv * bf16lo(wu.w), v[i][7] * inv * bf16hi(wu.w));
            *reinterpret_cast<uint4*>(x_out + rbase + vi * 8) = o;
        }
    }
    // a CTA whose wait ran out keeps its epoch: the communicator is then out of step and must be
    // rebuilt (documented with MSGL_ERR_TIMEOUT)
    if (threadIdx.x == 0 && ok) *reinterpret_cast<volatile unsigned*>(epoch_p) = e + 1;
}

// Two-shot: with per = ceil(T / world), rank r owns rows [r per, min(T, (r + 1) per)). CTA b of
// every rank pairs with CTA b of the others (same grid on every rank). After the ready exchange a
// CTA brings each of its owned rows from every rank (bulk copies into shared memory), sums them in
// rank order in fp32, adds the residual (this rank's rows only), normalises, and stores the bf16
// row into slot 2 of every rank (16-byte stores over NVLink, its own included). The done
// exchange then tells each peer that this CTA's rows have landed; once CTA b has seen every
// peer's done flag, the rows of CTA b of every rank are in this rank's slot 2, so when the grid
// completes the whole [T, H] block is there. NVLink traffic per rank and call: (W - 1) / W of the
// rows read once and written once, instead of (W - 1) full copies read by the one-shot kernel.
template <int VPT>
__global__ void __launch_bounds__(128)
tp_ar2_norm_kernel(TpPeers peers, int world, int rank, float* __restrict__ resid,
                   const __nv_bfloat16* __restrict__ w, int T, int H, float eps, int first,
                   unsigned* __restrict__ local, int* err) {
    extern __shared__ __align__(16) uint8_t ar_smem[];
    const __nv_bfloat16* rows = reinterpret_cast<const __nv_bfloat16*>(ar_smem);  // [world][H]
    uint64_t* bar = reinterpret_cast<uint64_t*>(ar_smem + static_cast<size_t>(world) * H * 2);
    __shared__ float red[4];
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }
    pdl_wait();  // this rank's partial (the previous kernel's output) is complete
    pdl_trigger();
    unsigned* epoch_p = local + kEpochOff + blockIdx.x;
    const unsigned e = *reinterpret_cast<volatile unsigned*>(epoch_p);
    bool ok = flag_exchange(peers, local, kReadyOff, world, rank, e + 1, err, 500);
    const int per = (T + world - 1) / world;
    const int r_end = min(T, (rank + 1) * per);
    const int nvec = H >> 3;
    const uint32_t row_bytes = static_cast<uint32_t>(H) * 2;
    uint32_t phase = 0;
    for (int row = rank * per + blockIdx.x; ok && row < r_end; row += gridDim.x) {
        const int64_t rbase = static_cast<int64_t>(row) * H;
        if (threadIdx.x == 0) {
            fence_proxy_async_global();  // the acquired peer rows, read through the async proxy
            fence_proxy_async();         // this CTA's reads of the previous row's copies are done
            mbar_arrive_expect_tx(bar, row_bytes * world);
            for (int q = 0; q < world; ++q)
                bulk_load(ar_smem + static_cast<size_t>(q) * row_bytes, peers.part[q] + rbase, row_bytes, bar);
        }
        float v[VPT][8];
        float rr[VPT][8];
#pragma unroll
        for (int i = 0; i < VPT; ++i) {  // residual loads overlap the copies
            const int vi = threadIdx.x + i * 128;
            if (vi >= nvec || first) continue;
            const float4* r4 = reinterpret_cast<const float4*>(resid + rbase + vi * 8);
            const float4 a = r4[0], b = r4[1];
            rr[i][0] = a.x; rr[i][1] = a.y; rr[i][2] = a.z; rr[i][3] = a.w;
            rr[i][4] = b.x; rr[i][5] = b.y; rr[i][6] = b.z; rr[i][7] = b.w;
        }
        mbar_wait(bar, phase, err, 502);
        phase ^= 1;
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int vi = threadIdx.x + i * 128;
            if (vi >= nvec) continue;
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
            for (int q = 0; q < world; ++q) {
                const uint4 u = *reinterpret_cast<const uint4*>(rows + static_cast<int64_t>(q) * H + vi * 8);
                v[i][0] += bf16lo(u.x); v[i][1] += bf16hi(u.x);
                v[i][2] += bf16lo(u.y); v[i][3] += bf16hi(u.y);
                v[i][4] += bf16lo(u.z); v[i][5] += bf16hi(u.z);
                v[i][6] += bf16lo(u.w); v[i][7] += bf16hi(u.w);
            }
            if (!first) {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] += rr[i][j];
            }
            float4* r4 = reinterpret_cast<float4*>(resid + rbase + vi * 8);
            r4[0] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
            r4[1] = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
#pragma unroll
            for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
        }
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();  // also: every thread is done reading this row's copies
        const float tot = red[0] + red[1] + red[2] + red[3];
        __syncthreads();
        const float inv = 1.0f / sqrtf(tot / static_cast<float>(H) + eps);
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int vi = threadIdx.x + i * 128;
            if (vi >= nvec) continue;
            const uint4 wu = *reinterpret_cast<const uint4*>(w + vi * 8);
            uint4 o;
            o.x = pack_bf16x2(v[i][0] * inv * bf16lo(wu.x), v[i][1] * inv * bf16hi(wu.x));
            o.y = pack_bf16x2(v[i][2] * inv * bf16lo(wu.y), v[i][3] * inv * bf16hi(wu.y));
            o.z = pack_bf16x2(v[i][4] * inv * bf16lo(wu.z), v[i][5] * inv * bf16hi(wu.z));
            o.w = pack_bf16x2(v[i][6] * inv * bf16lo(wu.w), v[i][7] * inv * bf16hi(wu.w));
            for (int q = 0; q < world; ++q)  // start with the next rank: spread the link load
                *reinterpret_cast<uint4*>(peers.xrows[(rank + 1 + q) % world] + rbase + vi * 8) = o;
        }
    }
    // the stores above precede (barrier, then each flag's release) the done flags
    ok = flag_exchange(peers, local, kDoneOff, world, rank, e + 1, err, 503) && ok;
    if (threadIdx.x == 0) {
        fence_proxy_async_global();  // peers' rows in slot 2, read by the next kernel's TMA
        if (ok) *reinterpret_cast<volatile unsigned*>(epoch_p) = e + 1;
    }
}

template <int VPT>
cudaError_t launch_ar(int grid, cudaStream_t stream, const TpPeers& pr, const msgl_tp* tp,
                      void* x_out, float* residual, const void* weight, int T, int H, float eps,
                      int first, unsigned* local, int* err) {
    const size_t smem = static_cast<size_t>(tp->world) * H * 2 + 16;
    static std::atomic<int> optin[kMaxDevices];
    const cudaError_t e = smem_optin(tp_fused_ar_norm_kernel<VPT>, smem, optin);
    if (e != cudaSuccess) return e;
    return launch_pdl(tp_fused_ar_norm_kernel<VPT>, dim3(grid), dim3(128), smem, stream, pr,
                      tp->world, tp->rank, static_cast<__nv_bfloat16*>(x_out), residual,
                      static_cast<const __nv_bfloat16*>(weight), T, H, eps, first, local, err);
}

template <int VPT>
cudaError_t launch_ar2(int grid, cudaStream_t stream, const TpPeers& pr, const msgl_tp* tp,
                       float* residual, const void* weight, int T, int H, float eps, int first,
                       unsigned* local, int* err) {
    const size_t smem = static_cast<size_t>(tp->world) * H * 2 + 16;
    static std::atomic<int> optin[kMaxDevices];
    const cudaError_t e = smem_optin(tp_ar2_norm_kernel<VPT>, smem, optin);
    if (e != cudaSuccess) return e;
    return launch_pdl(tp_ar2_norm_kernel<VPT>, dim3(grid), dim3(128), smem, stream, pr, tp->world,
                      tp->rank, residual, static_cast<const __nv_bfloat16*>(weight), T, H, eps,
                      first, local, err);
}

TpPeers peers_of(const msgl_tp* tp, int slot) {
    TpPeers pr{};
    for (int q = 0; q < tp->world; ++q) {
        uint8_t* base = static_cast<uint8_t*>(tp->peer[q]);
        pr.part[q] = reinterpret_cast<const __nv_bfloat16*>(base + slot * tp->data_bytes);
        pr.flags[q] = reinterpret_cast<unsigned*>(base + kSlots * tp->data_bytes);
        pr.xrows[q] = reinterpret_cast<__nv_bfloat16*>(base + 2 * tp->data_bytes);
    }
    return pr;
}

// Checks shared by the one- and two-shot calls: MSGL_OK with *slot the partial's slot (0 / 1),
// or the error status.
int check_fused(msgl_tp* tp, const void* partial, float* residual, const void* weight,
                int num_tokens, int hidden, int* slot) {
    if (!tp || !residual || !weight || num_tokens < 0 || hidden <= 0 || hidden % 8 ||
        hidden > 8 * 8 * 128)
        return set_error(MSGL_ERR_INVALID_ARG, "tp_fused_allreduce: bad args");
    if (!tp->sym) return set_error(MSGL_ERR_INVALID_ARG, "tp_fused_allreduce: msgl_tp_enable_p2p not called");
    *slot = -1;
    for (int k = 0; k < 2; ++k)
        if (partial == static_cast<uint8_t*>(tp->sym) + k * tp->data_bytes) *slot = k;
    if (*slot < 0)
        return set_error(MSGL_ERR_INVALID_ARG,
                         "tp_fused_allreduce: partial must be a msgl_tp_p2p_buffer slot (0 or 1)");
    if (*slot == tp->last_slot)
        return set_error(MSGL_ERR_INVALID_ARG, "tp_fused_allreduce: consecutive calls must alternate slots");
    if (static_cast<size_t>(num_tokens) * hidden * 2 > tp->data_bytes)
        return set_error(MSGL_ERR_WORKSPACE, "tp_fused_allreduce: rows exceed the peer-mapped region");
    return MSGL_OK;
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
    for (int q = 0; q < tp->world && q < kTpMaxWorld; ++q)
        if (q != tp->rank && tp->peer[q]) cudaIpcCloseMemHandle(tp->peer[q]);
    if (tp->sym) cudaFree(tp->sym);
    if (tp->comm) ncclCommDestroy(tp->comm);
    delete tp;
    return MSGL_OK;
}

// Collective (every rank, same bytes): allocate this rank's peer-mapped region, exchange the
// cudaIpc handles with an NCCL all-gather, and map every other rank's region.
int msgl_tp_enable_p2p(msgl_tp* tp, size_t bytes, msgl_stream_t stream) {
    if (!tp || bytes == 0 || bytes % 16) return set_error(MSGL_ERR_INVALID_ARG, "tp_enable_p2p: bad args");
    if (tp->world > kTpMaxWorld) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "tp_enable_p2p: world > 8");
    if (tp->sym) return set_error(MSGL_ERR_INVALID_ARG, "tp_enable_p2p: already enabled");
    const size_t total = kSlots * bytes + kFlagBytes;
    if (cudaMalloc(&tp->sym, total) != cudaSuccess || cudaMemset(tp->sym, 0, total) != cudaSuccess) {
        tp->sym = nullptr;
        return set_error(MSGL_ERR_CUDA, "tp_enable_p2p: region allocation failed");
    }
    tp->data_bytes = bytes;
    tp->peer[tp->rank] = tp->sym;
    if (tp->world == 1) return MSGL_OK;
    cudaIpcMemHandle_t mine;
    if (cudaIpcGetMemHandle(&mine, tp->sym) != cudaSuccess)
        return set_error(MSGL_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    void* dev = nullptr;
    if (cudaMalloc(&dev, hb * (tp->world + 1)) != cudaSuccess)
        return set_error(MSGL_ERR_CUDA, "tp_enable_p2p: handle buffer");
    uint8_t* d8 = static_cast<uint8_t*>(dev);
    std::vector<uint8_t> all(hb * tp->world);
    int rc = MSGL_OK;
    if (cudaMemcpy(d8 + hb * tp->world, &mine, hb, cudaMemcpyHostToDevice) != cudaSuccess) {
        rc = set_error(MSGL_ERR_CUDA, "tp_enable_p2p: handle copy");
    } else {
        ncclResult_t r = ncclAllGather(d8 + hb * tp->world, d8, hb, ncclUint8, tp->comm, stream);
        if (r != ncclSuccess) rc = nccl_err(r, "ncclAllGather(ipc handles)");
        else if (cudaStreamSynchronize(stream) != cudaSuccess ||
                 cudaMemcpy(all.data(), d8, hb * tp->world, cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = set_error(MSGL_ERR_CUDA, "tp_enable_p2p: handle gather");
    }
    cudaFree(dev);
    if (rc) return rc;
    for (int q = 0; q < tp->world; ++q) {
        if (q == tp->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, all.data() + hb * q, hb);
        if (cudaIpcOpenMemHandle(&tp->peer[q], h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            tp->peer[q] = nullptr;
            return set_error(MSGL_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
        }
    }
    return MSGL_OK;
}

int msgl_tp_p2p_buffer(msgl_tp* tp, int slot, void** ptr, size_t* bytes) {
    if (!tp || !ptr || slot < 0 || slot >= kSlots) return set_error(MSGL_ERR_INVALID_ARG, "tp_p2p_buffer: bad args");
    *ptr = tp->sym ? static_cast<uint8_t*>(tp->sym) + slot * tp->data_bytes : nullptr;
    if (bytes) *bytes = tp->data_bytes;
    return tp->sym ? MSGL_OK : set_error(MSGL_ERR_INVALID_ARG, "tp_p2p_buffer: msgl_tp_enable_p2p not called");
}

int msgl_tp_fused_allreduce_add_rmsnorm(msgl_tp* tp, const void* partial, void* x_out,
                                        float* residual, const void* weight, int num_tokens,
                                        int hidden, float eps, int first, msgl_stream_t stream) {
    if (!x_out) return set_error(MSGL_ERR_INVALID_ARG, "tp_fused_allreduce: bad args");
    int slot = -1;
    const int rc = check_fused(tp, partial, residual, weight, num_tokens, hidden, &slot);
    if (rc) return rc;
    if (num_tokens == 0) return MSGL_OK;
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    const TpPeers pr = peers_of(tp, slot);
    unsigned* local = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(tp->sym) + kSlots * tp->data_bytes);
    const int grid = num_tokens < kTpMaxCtas ? num_tokens : kTpMaxCtas;
    const int vpt = (hidden / 8 + 127) / 128;
    cudaError_t e;
#define MSGL_TP_CASE(N)                                                                          \
    case N:                                                                                      \
        e = launch_ar<N>(grid, stream, pr, tp, x_out, residual, weight, num_tokens, hidden, eps, \
                         first, local, err);                                                     \
        break;
    switch (vpt) {
        MSGL_TP_CASE(1) MSGL_TP_CASE(2) MSGL_TP_CASE(3) MSGL_TP_CASE(4)
        MSGL_TP_CASE(5) MSGL_TP_CASE(6) MSGL_TP_CASE(7) MSGL_TP_CASE(8)
        default: return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "tp_fused_allreduce: hidden too large");
    }
#undef MSGL_TP_CASE
    if (e != cudaSuccess) return set_error(MSGL_ERR_CUDA, cudaGetErrorString(e));
    tp->last_slot = slot;
    return MSGL_OK;
}

int msgl_tp_fused_allreduce_add_rmsnorm_2shot(msgl_tp* tp, const void* partial, void* x_out,
                                              float* residual, const void* weight, int num_tokens,
                                              int hidden, float eps, int first,
                                              msgl_stream_t stream) {
    int slot = -1;
    const int rc = check_fused(tp, partial, residual, weight, num_tokens, hidden, &slot);
    if (rc) return rc;
    if (x_out != static_cast<uint8_t*>(tp->sym) + 2 * tp->data_bytes)
        return set_error(MSGL_ERR_INVALID_ARG, "tp_fused_allreduce_2shot: x_out must be msgl_tp_p2p_buffer slot 2");
    if (num_tokens == 0) return MSGL_OK;
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    const TpPeers pr = peers_of(tp, slot);
    unsigned* local = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(tp->sym) + kSlots * tp->data_bytes);
    const int per = (num_tokens + tp->world - 1) / tp->world;
    const int grid = per < kTpMaxCtas ? per : kTpMaxCtas;
    const int vpt = (hidden / 8 + 127) / 128;
    cudaError_t e;
#define MSGL_TP_CASE(N)                                                                       \
    case N:                                                                                   \
        e = launch_ar2<N>(grid, stream, pr, tp, residual, weight, num_tokens, hidden, eps,    \
                          first, local, err);                                                 \
        break;
    switch (vpt) {
        MSGL_TP_CASE(1) MSGL_TP_CASE(2) MSGL_TP_CASE(3) MSGL_TP_CASE(4)
        MSGL_TP_CASE(5) MSGL_TP_CASE(6) MSGL_TP_CASE(7) MSGL_TP_CASE(8)
        default: return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "tp_fused_allreduce_2shot: hidden too large");
    }
#undef MSGL_TP_CASE
    if (e != cudaSuccess) return set_error(MSGL_ERR_CUDA, cudaGetErrorString(e));
    tp->last_slot = slot;
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

int msgl_tp_all_gather(msgl_tp* tp, const void* send, void* recv, size_t bytes,
                       msgl_stream_t stream) {
    if (!tp || (bytes && (!send || !recv))) return set_error(MSGL_ERR_INVALID_ARG, "tp_all_gather: bad args");
    if (bytes == 0) return MSGL_OK;
    if (tp->world == 1) {
        if (send != recv &&
            cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
            return set_error(MSGL_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
        return MSGL_OK;
    }
    ncclResult_t r = ncclAllGather(send, recv, bytes, ncclUint8, tp->comm, stream);
    return r == ncclSuccess ? MSGL_OK : nccl_err(r, "ncclAllGather");
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
