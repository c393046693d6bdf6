// gemm.cu -- tcgen05 / TMEM bf16 GEMMs for the dense projections.
//
// Linear::forward (src/layer/layer.cpp:122-143): y[M,N] = x[M,K] W[N,K]^T with W in the
// reference's [out, in] layout; every weight byte crosses HBM once per call. All kernels share
// one structure: a TMA producer warp (weight and token tiles, SW128, k-blocks of 64), a warp that
// allocates TMEM and issues tcgen05.mma from one thread (fp32 accumulator in TMEM), and
// epilogue warps that read the accumulator with tcgen05.ld. Schedules, chosen per call
// (run_gemm):
//   gemm_rows_kernel   M <= 128, many weight rows (or a short K): whole tiles of 16 hs weight
//                      rows per CTA over the full K; tokens are the UMMA M dimension, the tile's
//                      rows N; at 129..256 tokens (argmax) one token tile per grid row
//   gemm_part_kernel   M <= 256: split-K fp32 partials (tokens as M in tiles of 128, 256 weight
//                      rows as N), summed by the next kernel or by partials_reduce_kernel
//   gemm_cl_kernel     M <= 128 otherwise: cluster split-K, partials exchanged over DSMEM
//   (129..256 tokens: the partials + reduce; argmax on the row kernel; else two passes of the
//   schedules above, 128 tokens and the rest)
//   gemm_sk_kernel     stream-K (prefill-sized M; 128 weight rows as M, up to 256 tokens as N)
//   gemm_kernel        one CTA per tile (very large grids) and the grouped MoE GEMM
// Epilogues: bf16 store, fp32 store, SwiGLU (gate/up rows interleaved in 16-row groups by
// msgl_pack_gate_up; split of qwen3.cpp:62-77 + SwiGLU of layer.cpp:155-158), argmax
// (scheduler.cpp:117-124).
#include <algorithm>
#include <cstdlib>

#include <string>

#include "common.cuh"
#include "tmap.h"

namespace msgl {
namespace {

constexpr int kBM = 128;       // weight rows per tile (UMMA M)
constexpr int kBK = 64;        // K per stage: one 128-byte swizzle row
constexpr int kGemmThreads = 192;
// Stream-K kernel: producer warp, MMA warp, then kSkEpiWarps epilogue warps -- two per TMEM lane
// quarter, splitting the tile's columns, so each SM sub-partition runs two epilogue warps and
// hides the latency of the TMEM-load / convert / store chains.
constexpr int kSkEpiWarps = 8;
constexpr int kSkThreads = (2 + kSkEpiWarps) * 32;
constexpr int kTileA = kBM * kBK * 2;  // 16 KB
// K-blocks per ring stage of the persistent kernels (one mbarrier phase carries kKps weight and
// kKps activation tiles). Measured on B200 with the decode shapes: 2 per stage with half the
// stages was no faster than 1 per stage with a deeper ring, so the ring keeps single k-blocks.
constexpr int kKps = 1;
constexpr int kRingBudget = 192 * 1024;  // shared memory for the ring (and cluster part buffer)
constexpr size_t kCounterBytes = 16384;  // split-K arrival counters: up to 4096 tiles

enum Epi { EPI_BF16 = 0, EPI_F32 = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

template <int BN>
struct GemmCfg {
    static constexpr int kTileB = BN * kBK * 2;
    static constexpr int kStageBytes = kTileA + kTileB;
    static constexpr int kStages = BN >= 256 ? 4 : (BN == 16 ? 3 : (96 * 1024) / kStageBytes);
    static constexpr int kTmemCols = BN < 32 ? 32 : BN;
    static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStageBytes + 1024 + 256;
};

__device__ __forceinline__ void named_bar(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Named barrier that also ORs a predicate over its `count` threads: every participant gets the
// same answer, so a decision taken on it is uniform across the warps.
__device__ __forceinline__ bool named_bar_or(int id, int count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(n));
}

// Epilogue on one 16-column chunk of the accumulator held by this thread (row `row` of the
// tile = weight row n). vals[j] is column col0 + j (token m0 + col0 + j).
template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const float (&vals)[16], int n, int N, int m_base,
                                               int M, void* y, unsigned long long* amax,
                                               int lane, int warp_q, int n_tile, int id_off) {
    if (EPI == EPI_BF16 || EPI == EPI_F32) {
        if (n >= N) return;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            int m = m_base + j;
            if (m < M) {
                if (EPI == EPI_BF16)
                    static_cast<__nv_bfloat16*>(y)[static_cast<int64_t>(m) * N + n] =
                        __float2bfloat16_rn(vals[j]);
                else
                    static_cast<float*>(y)[static_cast<int64_t>(m) * N + n] = vals[j];
            }
        }
    } else if (EPI == EPI_SWIGLU) {
        // rows of each 16-row group: 8 gate rows then the 8 matching up rows; lane l pairs with
        // lane l ^ 8, the even token going to the gate lane and the odd one to the up lane
        const int inter = N >> 1;
        const int f = n_tile * (kBM / 2) + warp_q * 16 + (lane >> 4) * 8 + (lane & 7);
        const bool lo = (lane & 8) == 0;
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            float send = lo ? vals[j + 1] : vals[j];
            float recv = __shfl_xor_sync(0xffffffffu, send, 8);
            float g = lo ? vals[j] : recv;
            float u = lo ? recv : vals[j + 1];
            int m = m_base + j + (lo ? 0 : 1);
            if (m < M && f < inter)
                static_cast<__nv_bfloat16*>(y)[static_cast<int64_t>(m) * inter + f] =
                    __float2bfloat16_rn(g / (1.0f + expf(-g)) * u);
        }
    } else {  // EPI_ARGMAX
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            unsigned long long key = n < N ? argmax_key(vals[j], n + id_off) : 0ull;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                key = other > key ? other : key;
            }
            int m = m_base + j;
            if (lane == 0 && m < M) atomicMax(amax + m, key);
        }
    }
}

// Grouped (MoE) mode: CTA x of the grid takes tile `tiles[x]` = (expert, first row) of the
// expert-sorted token matrix; rows past the expert's end are masked, weight rows are offset by
// expert * N. CTAs beyond *num_tiles exit at once.
struct GroupArgs {
    const int2* tiles = nullptr;
    const int* num_tiles = nullptr;
    const int* offsets = nullptr;  // [E + 1] row offsets of each expert
};

// One CTA per 128 x BN tile of y^T = W x^T (192 threads: warp 0 TMA, warp 1 TMEM + MMA, warps
// 2-5 epilogue, one TMEM lane = one weight row). Split K: partial tiles go to the workspace and
// the last CTA to arrive (self-resetting counter) sums them in split order and runs the epilogue.
template <int BN, int EPI, bool GROUPED>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
            void* __restrict__ y, unsigned long long* __restrict__ amax, int M, int N, int K,
            int kb_per_split, int splits, float* __restrict__ ws, int* __restrict__ ws_cnt,
            GroupArgs grp, int id_off, int* err) {
    using Cfg = GemmCfg<BN>;
    constexpr int ST = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + ST * kTileA;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * Cfg::kStageBytes);
    uint64_t* empty = full + ST;
    uint64_t* accum_full = empty + ST;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_full + 1);
    int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);

    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tile = blockIdx.x, n_tile = blockIdx.y, split = blockIdx.z;
    int m0 = m_tile * BN;
    const int n0 = n_tile * kBM;
    int w_row0 = 0;
    if (GROUPED) {
        if (m_tile >= *grp.num_tiles) return;  // uniform: before any barrier or TMEM use
        const int2 t = grp.tiles[m_tile];
        m0 = t.y;
        M = grp.offsets[t.x + 1];
        w_row0 = t.x * N;
    }
    const int kbs = (K + kBK - 1) / kBK;
    const int kb0 = split * kb_per_split;
    const int kb1 = min(kbs, kb0 + kb_per_split);
    const int nkb = kb1 - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum_full, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmap_w);
            tma_prefetch_desc(&tmap_x);
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            for (int i = 0; i < nkb; ++i) {
                const int s = i % ST;
                if (i >= ST && !mbar_wait(&empty[s], ((i / ST) - 1) & 1, err, 300)) break;
                mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
                const int kx = (kb0 + i) * kBK;
                tma_load_2d_hint(sA + s * kTileA, &tmap_w, &full[s], kx, w_row0 + n0, pol_w);
                tma_load_2d_hint(sB + s * Cfg::kTileB, &tmap_x, &full[s], kx, m0, pol_x);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
            for (int i = 0; i < nkb; ++i) {
                const int s = i % ST;
                if (!mbar_wait(&full[s], (i / ST) & 1, err, 310)) break;
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sA + s * kTileA);
                const uint32_t b_addr = smem_u32(sB + s * Cfg::kTileB);
#pragma unroll
                for (int k = 0; k < kBK / 16; ++k) {
                    umma_bf16(tmem, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                              idesc, (i > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(accum_full);
        }
    } else {
        // ---------------- epilogue warps 2..5
        const int warp_q = warp & 3;  // TMEM lane quarter this warp may access
        const int row = warp_q * 32 + lane;
        const int n = n0 + row;
        const int et = threadIdx.x - 64;  // 0..127
        const bool have = nkb > 0 && mbar_wait(accum_full, 0, err, 320);
        tc_fence_after();
        const uint32_t taddr = tmem + (static_cast<uint32_t>(warp_q * 32) << 16);
        if (splits == 1) {
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t r[16];
                float v[16];
                tmem_ld16(taddr + c0, r);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = have ? __uint_as_float(r[j]) : 0.f;
                epilogue_chunk<EPI>(v, n, N, m0 + c0, M, y, amax, lane, warp_q, n_tile, id_off);
            }
        } else {
            const int64_t tile_id = static_cast<int64_t>(n_tile) * gridDim.x + m_tile;
            float* part = ws + (tile_id * splits + split) * (static_cast<int64_t>(BN) * kBM);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t r[16];
                tmem_ld16(taddr + c0, r);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    __stcg(part + (c0 + j) * kBM + row, have ? __uint_as_float(r[j]) : 0.f);
            }
            __threadfence();
            named_bar(1, 128);
            if (et == 0) {
                int old = atomicAdd(ws_cnt + tile_id, 1);
                *last_flag = (old == splits - 1);
            }
            named_bar(1, 128);
            if (*last_flag) {
                __threadfence();
                const float* base = ws + tile_id * splits * (static_cast<int64_t>(BN) * kBM);
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = 0.f;
                    for (int sp = 0; sp < splits; ++sp) {
                        const float* p = base + static_cast<int64_t>(sp) * BN * kBM;
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] += __ldcg(p + (c0 + j) * kBM + row);
                    }
                    epilogue_chunk<EPI>(v, n, N, m0 + c0, M, y, amax, lane, warp_q, n_tile, id_off);
                }
                if (et == 0) ws_cnt[tile_id] = 0;
            }
        }
        tc_fence_before();
    }
    // Lane 0 of warps 0 and 1 ran the producer / MMA loops alone: reconverge every warp before
    // the block barrier (bar.sync counts whole warps), so TMEM is freed only after the epilogue.
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

// Grouped (MoE) GEMM, persistent with dynamic work: G CTAs (as many as fit) take work items
// (tile, 128-row weight slab), item = slab * num_tiles + tile, from a counter in the workspace
// (zeroed by group_tiles_kernel), so CTAs that finish early take more and the last wave is not a
// fixed split. Adjacent items are the tiles of one expert on one slab, so CTAs that run together
// read the same weights (the second read comes from L2). The TMA ring runs on across items and
// the accumulator is double-buffered in TMEM (an item's epilogue overlaps the next mainloop).
// The producer lane passes each item's index to the MMA and epilogue warps through a small ring
// in shared memory (id < 0: no more work). 192 threads: warp 0 TMA, warp 1 TMEM + MMA, warps
// 2-5 epilogue.
constexpr int kItemQ = 4;
template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_grouped_dyn_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                        void* __restrict__ y, int N, int K, GroupArgs grp, int* __restrict__ counter,
                        int* err) {
    using Cfg = GemmCfg<BN>;
    constexpr int ST = Cfg::kStages;
    constexpr int kCols = BN < 32 ? 32 : BN;  // TMEM columns of one accumulator
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + ST * kTileA;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * Cfg::kStageBytes);
    uint64_t* empty = full + ST;
    uint64_t* tfull = empty + ST;        // [2] accumulator ready
    uint64_t* tempty = tfull + 2;        // [2] accumulator drained
    uint64_t* ifull = tempty + 2;        // [kItemQ] item index published
    uint64_t* iempty = ifull + kItemQ;   // [kItemQ] item index slot free again
    int* items = reinterpret_cast<int*>(iempty + kItemQ);      // [kItemQ]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(items + kItemQ);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);  // the four epilogue warps
        }
        for (int q = 0; q < kItemQ; ++q) {
            mbar_init(&ifull[q], 1);
            mbar_init(&iempty[q], 4);  // the four epilogue warps release an index slot
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // the tile list and the zeroed counter come from the kernel before
    pdl_trigger();
    const int nt = *grp.num_tiles;
    const int total = nt * ((N + kBM - 1) / kBM);
    const int KB = (K + kBK - 1) / kBK;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmap_w);
            tma_prefetch_desc(&tmap_x);
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            int it = 0;
            bool ok = true;
            int item = atomicAdd(counter, 1);
            for (int j = 0; ok; ++j) {
                const int q = j % kItemQ;
                if (j >= kItemQ && !mbar_wait(&iempty[q], ((j / kItemQ) - 1) & 1, err, 340)) break;
                const int cur = item < total ? item : -1;
                items[q] = cur;
                mbar_arrive(&ifull[q]);  // release: the index store precedes the arrive
                if (cur < 0) break;
                item = atomicAdd(counter, 1);  // the next index, in flight during this item
                const int2 t = grp.tiles[cur % nt];
                const int wrow = t.x * N + (cur / nt) * kBM;
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const int s = it % ST;
                    if (it >= ST && !mbar_wait(&empty[s], ((it / ST) - 1) & 1, err, 341)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
                    tma_load_2d_hint(sA + s * kTileA, &tmap_w, &full[s], kb * kBK, wrow, pol_w);
                    tma_load_2d_hint(sB + s * Cfg::kTileB, &tmap_x, &full[s], kb * kBK, t.y, pol_x);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
            int it = 0;
            for (int j = 0;; ++j) {
                const int q = j % kItemQ;
                if (!mbar_wait(&ifull[q], (j / kItemQ) & 1, err, 342)) break;
                if (items[q] < 0) break;
                const int a = j & 1;
                if (j >= 2 && !mbar_wait(&tempty[a], ((j >> 1) - 1) & 1, err, 343)) break;
                tc_fence_after();
                const uint32_t acc = tmem + a * kCols;
                bool ok = true;
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const int s = it % ST;
                    if (!mbar_wait(&full[s], (it / ST) & 1, err, 344)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * kTileA);
                    const uint32_t b_addr = smem_u32(sB + s * Cfg::kTileB);
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)
                        umma_bf16(acc, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                                  idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                umma_commit(&tfull[a]);
            }
        }
    } else {
        // ---------------- epilogue warps 2..5
        const int warp_q = warp & 3;
        const int row = warp_q * 32 + lane;
        for (int j = 0;; ++j) {
            const int q = j % kItemQ;
            if (!mbar_wait(&ifull[q], (j / kItemQ) & 1, err, 345)) break;
            const int cur = items[q];
            if (cur < 0) break;
            const int a = j & 1;
            if (!mbar_wait(&tfull[a], (j >> 1) & 1, err, 346)) break;
            tc_fence_after();
            const int2 t = grp.tiles[cur % nt];
            const int slab = cur / nt;
            const int M = grp.offsets[t.x + 1];  // rows past the expert's end are masked
            const uint32_t taddr = tmem + a * kCols + (static_cast<uint32_t>(warp_q * 32) << 16);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t r[16];
                float v[16];
                tmem_ld16(taddr + c0, r);
                tmem_ld_wait();
#pragma unroll
                for (int u = 0; u < 16; ++u) v[u] = __uint_as_float(r[u]);
                epilogue_chunk<EPI>(v, slab * kBM + row, N, t.y + c0, M, y, nullptr, lane, warp_q,
                                    slab, 0);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tempty[a]);
                mbar_arrive(&iempty[q]);
            }
        }
        tc_fence_before();
    }
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * kCols);
    }
}

// ============================================================================ stream-K kernel
// Persistent: one CTA per SM. Hybrid schedule: the T output tiles split into full waves of G
// whole tiles (data-parallel: CTA c takes tiles c, c + G, ...) and a remainder of T_rem tiles
// whose (tile, k-block) units are cut into G_sk equal contiguous ranges (stream-K), so every SM
// streams about the same number of weight bytes whatever the tile count. A CTA's stream-K range
// is [tail of a tile] [whole tiles] [head of a tile]:
//  * the tail part (k-blocks [x, KB)) of a tile that an earlier CTA starts: its fp32 part goes to
//    this CTA's workspace slot and a flag is raised -- done FIRST, at the start of the kernel;
//  * the head part (k-blocks [0, y)) of a tile: this CTA owns the tile. It runs it LAST, then
//    waits (bounded) for the flags of the tile's other contributors -- the following CTAs, which
//    published their parts at their start -- and adds their parts, in CTA order
//    (deterministic), to its own accumulator before the epilogue.
// Segment order of a CTA: its stream-K segments but the last, its whole data-parallel tiles, its
// last stream-K segment. Each segment accumulates into one of two TMEM buffers (the epilogue of
// segment j overlaps the mainloop of segment j + 1).
template <int BN>
struct SkCfg {
    static constexpr int kTileB = BN * kBK * 2;
    static constexpr int kStageBytes = kKps * (kTileA + kTileB);
    static constexpr int kStages = kRingBudget / kStageBytes > 8 ? 8 : kRingBudget / kStageBytes;
    static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStageBytes + 1024 + 256;
};

constexpr size_t kSkFlagBytes = 4096;  // one flag per CTA (<= 1024 CTAs), then the parts
constexpr int kSkMaxCtas = static_cast<int>(kSkFlagBytes / sizeof(int));

__device__ __forceinline__ int sk_cta_of(int64_t u, int64_t U, int G) {
    return static_cast<int>(((u + 1) * G + U - 1) / U - 1);
}

struct SkWork {
    int T, KB, G, c;
    int T_dp, T_rem, G_sk;
    int64_t U_sk, u0, u1;  // this CTA's stream-K units (relative to tile T_dp)
    int n_sk, n_dp, lead;  // stream-K segments, whole data-parallel tiles, SK segments run first
    __device__ __forceinline__ void init(int T_, int KB_, int G_, int c_) {
        T = T_; KB = KB_; G = G_; c = c_;
        T_dp = T >= G ? (T / G) * G : 0;
        T_rem = T - T_dp;
        U_sk = static_cast<int64_t>(T_rem) * KB;
        const int64_t min_units = max(1, KB / 8);
        G_sk = T_rem > 0 ? static_cast<int>(min(static_cast<int64_t>(G), max(static_cast<int64_t>(1), U_sk / min_units))) : 0;
        if (c < G_sk) {
            u0 = static_cast<int64_t>(c) * U_sk / G_sk;
            u1 = static_cast<int64_t>(c + 1) * U_sk / G_sk;
            n_sk = static_cast<int>((u1 - 1) / KB - u0 / KB + 1);
        } else {
            u0 = u1 = 0;
            n_sk = 0;
        }
        n_dp = c < T_dp ? (T_dp - c + G - 1) / G : 0;
        // the last stream-K segment waits for the data-parallel tiles only when it is the head
        // of a tile this CTA owns (starts at a tile boundary, ends inside the tile)
        const bool last_is_head = n_sk > 0 && (u1 % KB) != 0 && ((u1 - 1) / KB) * KB >= u0;
        lead = n_sk - (last_is_head ? 1 : 0);
    }
    __device__ __forceinline__ int num_segs() const { return n_sk + n_dp; }
    // segment j: tile t, k-blocks [kb_s, kb_e); tr = stream-K tile index (relative to T_dp), or
    // -1 for a data-parallel tile
    __device__ __forceinline__ void seg(int j, int& t, int& kb_s, int& kb_e, int& tr) const {
        if (j >= lead && j < lead + n_dp) {
            t = c + (j - lead) * G;
            kb_s = 0;
            kb_e = KB;
            tr = -1;
            return;
        }
        const int js = j < lead ? j : j - n_dp;
        tr = static_cast<int>(u0 / KB) + js;
        const int64_t tb = static_cast<int64_t>(tr) * KB;
        kb_s = static_cast<int>(max(u0, tb) - tb);
        kb_e = static_cast<int>(min(u1, tb + KB) - tb);
        t = T_dp + tr;
    }
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kSkThreads, 1)
gemm_sk_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
               void* __restrict__ y, unsigned long long* __restrict__ amax, int M, int N, int K,
               int m_tiles, int* __restrict__ ws_flag, float* __restrict__ ws_part, int id_off,
               int* err) {
    using Cfg = SkCfg<BN>;
    constexpr int ST = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;                      // [ST][kKps] weight tiles
    uint8_t* sB = smem + ST * kKps * kTileA;  // [ST][kKps] activation tiles
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * Cfg::kStageBytes);
    uint64_t* empty = full + ST;
    uint64_t* tfull = empty + ST;   // [2] accumulator ready
    uint64_t* tempty = tfull + 2;   // [2] accumulator drained
    uint64_t* pfull = tempty + 2;   // contributors' parts landed in the (drained) ring
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pfull + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    SkWork wk;
    wk.init(m_tiles * ((N + kBM - 1) / kBM), (K + kBK - 1) / kBK, gridDim.x, blockIdx.x);
    const int nseg = wk.num_segs();

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], kSkEpiWarps);
        }
        mbar_init(pfull, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmap_w);
            tma_prefetch_desc(&tmap_x);
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            // Weight tiles of the first ST stages go out before the dependency wait: weights
            // are never written by a preceding kernel, so their fetch overlaps its tail. A stage
            // holds up to kKps consecutive k-blocks of one segment.
            constexpr uint32_t kKbBytes = kTileA + Cfg::kTileB;
            int npre = 0;
            for (int j = 0; j < nseg && npre < ST; ++j) {
                int t, kb_s, kb_e, tr;
                wk.seg(j, t, kb_s, kb_e, tr);
                const int wrow = (t / m_tiles) * kBM;
                for (int kb = kb_s; kb < kb_e && npre < ST; kb += kKps, ++npre) {
                    const int nk = min(kKps, kb_e - kb);
                    mbar_arrive_expect_tx(&full[npre], nk * kKbBytes);
                    for (int u = 0; u < nk; ++u)
                        tma_load_2d_hint(sA + (npre * kKps + u) * kTileA, &tmap_w, &full[npre],
                                         (kb + u) * kBK, wrow, pol_w);
                }
            }
            pdl_wait();
            pdl_trigger();
            int i = 0;
            bool ok = true;
            for (int j = 0; j < nseg && ok; ++j) {
                int t, kb_s, kb_e, tr;
                wk.seg(j, t, kb_s, kb_e, tr);
                const int wrow = (t / m_tiles) * kBM, xrow = (t % m_tiles) * BN;
                for (int kb = kb_s; kb < kb_e; kb += kKps, ++i) {
                    const int s = i % ST;
                    const int nk = min(kKps, kb_e - kb);
                    if (i >= npre) {
                        if (i >= ST && !mbar_wait(&empty[s], ((i / ST) - 1) & 1, err, 330)) { ok = false; break; }
                        mbar_arrive_expect_tx(&full[s], nk * kKbBytes);
                        for (int u = 0; u < nk; ++u)
                            tma_load_2d_hint(sA + (s * kKps + u) * kTileA, &tmap_w, &full[s],
                                             (kb + u) * kBK, wrow, pol_w);
                    }
                    for (int u = 0; u < nk; ++u)  // (stages armed above get their activations here)
                        tma_load_2d_hint(sB + (s * kKps + u) * Cfg::kTileB, &tmap_x, &full[s],
                                         (kb + u) * kBK, xrow, pol_x);
                }
            }
        } else {
            pdl_wait();
            pdl_trigger();
        }
    } else if (warp == 1) {
        pdl_wait();
        pdl_trigger();
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
            int i = 0;
            bool ok = true;
            for (int j = 0; j < nseg && ok; ++j) {
                int t, kb_s, kb_e, tr;
                wk.seg(j, t, kb_s, kb_e, tr);
                const int a = j & 1;
                if (j >= 2 && !mbar_wait(&tempty[a], ((j >> 1) - 1) & 1, err, 340)) break;
                tc_fence_after();
                const uint32_t acc = tmem + a * BN;
                for (int kb = kb_s; kb < kb_e; kb += kKps, ++i) {
                    const int s = i % ST;
                    const int nk = min(kKps, kb_e - kb);
                    if (!mbar_wait(&full[s], (i / ST) & 1, err, 341)) { ok = false; break; }
                    tc_fence_after();
                    for (int u = 0; u < nk; ++u) {
                        const uint32_t a_addr = smem_u32(sA + (s * kKps + u) * kTileA);
                        const uint32_t b_addr = smem_u32(sB + (s * kKps + u) * Cfg::kTileB);
#pragma unroll
                        for (int k = 0; k < kBK / 16; ++k)
                            umma_bf16(acc, umma_desc_sw128(a_addr + k * 32),
                                      umma_desc_sw128(b_addr + k * 32), idesc,
                                      (kb > kb_s || u > 0 || k > 0) ? 1u : 0u);
                    }
                    umma_commit(&empty[s]);
                }
                umma_commit(&tfull[a]);
            }
        }
    } else {
        // ---------------- epilogue warps 2..9 (named barrier 1 among them): warp w reads TMEM
        // lane quarter w % 4 (rows) and every other 16-column chunk, starting at chunk eg
        pdl_wait();
        pdl_trigger();
        const int warp_q = warp & 3;
        const int eg = (warp - 2) >> 2;
        const int row = warp_q * 32 + lane;
        const int et = threadIdx.x - 64;
        constexpr int kEpiThreads = kSkEpiWarps * 32;
        constexpr int64_t kPart = static_cast<int64_t>(kBM) * BN;  // floats of one part
        for (int j = 0; j < nseg; ++j) {
            int t, kb_s, kb_e, tr;
            wk.seg(j, t, kb_s, kb_e, tr);
            const int a = j & 1;
            const bool have = mbar_wait(&tfull[a], (j >> 1) & 1, err, 350);
            tc_fence_after();
            const int n_tile = t / m_tiles, m_tile = t % m_tiles;
            const int n = n_tile * kBM + row, m0 = m_tile * BN;
            const uint32_t taddr = tmem + a * BN + (static_cast<uint32_t>(warp_q * 32) << 16);
            if (kb_s > 0) {
                // ---- tail part of a tile owned by an earlier CTA: publish it (column-major
                // [BN][128], so one warp store covers 32 consecutive rows) and raise the flag
                float* part = ws_part + wk.c * kPart + row;
#pragma unroll 1
                for (int c0 = eg * 16; c0 < BN; c0 += 32) {
                    uint32_t r[16];
                    tmem_ld16(taddr + c0, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int q = 0; q < 16; ++q)
                        __stcg(part + (c0 + q) * kBM, have ? __uint_as_float(r[q]) : 0.f);
                }
                tc_fence_before();
                __threadfence();
                named_bar(1, kEpiThreads);
                if (et == 0) st_release_gpu(ws_flag + wk.c, 1);
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[a]);  // TMEM buffer free for segment j + 2
                continue;
            }
            // ---- whole tile, or the head of a tile this CTA owns (always its last segment, so
            // the smem ring has drained): pull the contributors' parts -- later CTAs, which
            // published them at their start -- into the ring with bulk copies, as many per round
            // trip as fit, and add them in CTA order to the accumulator (kept in TMEM between
            // rounds), then run the epilogue.
            const int ncontrib = kb_e < wk.KB
                ? sk_cta_of(static_cast<int64_t>(tr) * wk.KB + wk.KB - 1, wk.U_sk, wk.G_sk) - wk.c : 0;
            constexpr uint32_t kPartBytes = static_cast<uint32_t>(kPart * sizeof(float));
            constexpr int kPerRound = (ST * Cfg::kStageBytes) / kPartBytes;
            static_assert(kPerRound >= 1, "ring smaller than one part");
            int done = 0, round = 0;
            do {
                const int nb = min(kPerRound, ncontrib - done);
                if (nb > 0) {
                    if (et == 0) {
                        if (round > 0) fence_proxy_async();  // earlier reads before the overwrite
                        mbar_arrive_expect_tx(pfull, nb * kPartBytes);
                        for (int k = 0; k < nb; ++k) {
                            const int cc = wk.c + 1 + done + k;
                            const uint64_t t0 = globaltimer_ns();
                            while (ld_acquire_gpu(ws_flag + cc) == 0) {
                                if (globaltimer_ns() - t0 > 2000000000ull) {
                                    record_error(err, MSGL_ERR_TIMEOUT, 360);
                                    break;
                                }
                            }
                            ws_flag[cc] = 0;  // consumed: the workspace is left zero-filled
                            bulk_load(smem + k * kPartBytes, ws_part + cc * kPart, kPartBytes, pfull);
                        }
                    }
                    // every thread acquires the copies; a timeout anywhere stops all of them
                    const bool timed_out = !mbar_wait(pfull, round & 1, err, 361);
                    if (named_bar_or(1, kEpiThreads, timed_out)) break;
                }
                const bool final_round = done + nb >= ncontrib;
                const float* sp = reinterpret_cast<const float*>(smem) + row;
#pragma unroll 1
                for (int c0 = eg * 16; c0 < BN; c0 += 32) {
                    uint32_t r[16];
                    float v[16];
                    tmem_ld16(taddr + c0, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int q = 0; q < 16; ++q) v[q] = have ? __uint_as_float(r[q]) : 0.f;
                    for (int k = 0; k < nb; ++k)
#pragma unroll
                        for (int q = 0; q < 16; ++q) v[q] += sp[k * kPart + (c0 + q) * kBM];
                    if (final_round) {
                        epilogue_chunk<EPI>(v, n, N, m0 + c0, M, y, amax, lane, warp_q, n_tile, id_off);
                    } else {
#pragma unroll
                        for (int q = 0; q < 16; ++q) r[q] = __float_as_uint(v[q]);
                        tmem_st16(taddr + c0, r);
                    }
                }
                if (final_round) break;
                tmem_st_wait();
                named_bar(1, kEpiThreads);  // every thread has read this round's parts
                done += nb;
                ++round;
            } while (true);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[a]);
        }
        tc_fence_before();
    }
    // Lane 0 of warps 0 and 1 ran the producer / MMA loops alone: reconverge every warp before
    // the block barrier (bar.sync counts whole warps), so TMEM is freed only after the epilogue.
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

// ============================================================================ cluster split-K
// Decode-sized GEMMs (M <= 128 tokens, so one token tile): every output tile is computed by a
// cluster of C CTAs, CTA rank r accumulating k-blocks [r KB / C, (r + 1) KB / C) in TMEM. The
// tile's 16-column chunks are owned round-robin by the ranks (chunk ci by rank ci % C). After
// its mainloop a CTA publishes the chunks it does not own (fp32, column-major [BN][128]) in its
// own shared memory and arrives on the owners' `pready` mbarriers (remote arrive, release at
// cluster scope); each owner then adds the peers' chunks -- read over distributed shared memory,
// in rank order (deterministic) -- to its own TMEM accumulator and runs 1/C of the epilogue, and
// arrives on the peers' `pfree` mbarriers once it no longer needs their buffers. No fp32
// partials go to global memory and no second kernel runs. The cluster is persistent over tiles
// q, q + n_clusters, ...; TMEM is double-buffered, so a tile's reduction and epilogue overlap
// the next tile's mainloop. Producer warp, MMA warp and 8 epilogue warps as in the stream-K
// kernel. A CTA exits once its peers are done with its last published chunks.
template <int BN>
struct ClCfg {
    static constexpr int kTileB = BN * kBK * 2;
    static constexpr int kStageBytes = kKps * (kTileA + kTileB);
    static constexpr int kPartBytes = kBM * BN * 4;
    static constexpr int kStages = (kRingBudget - kPartBytes) / kStageBytes > 8
                                       ? 8 : (kRingBudget - kPartBytes) / kStageBytes;
    static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr size_t kSmem =
        static_cast<size_t>(kStages) * kStageBytes + kPartBytes + 1024 + 256;
};
constexpr int kClMaxC = 8;

template <int BN, int EPI>
__global__ void __launch_bounds__(kSkThreads, 1)
gemm_cl_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
               void* __restrict__ y, unsigned long long* __restrict__ amax, int M, int N, int K,
               int id_off, int* err) {
    using Cfg = ClCfg<BN>;
    constexpr int ST = Cfg::kStages;
    constexpr int NCH = BN / 16;  // 16-column chunks per tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;                      // [ST][kKps] weight tiles
    uint8_t* sB = smem + ST * kKps * kTileA;  // [ST][kKps] activation tiles
    float* part = reinterpret_cast<float*>(smem + ST * Cfg::kStageBytes);  // [BN][128]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * Cfg::kStageBytes + Cfg::kPartBytes);
    uint64_t* empty = full + ST;
    uint64_t* tfull = empty + ST;   // [2] accumulator ready
    uint64_t* tempty = tfull + 2;   // [2] accumulator drained
    uint64_t* pready = tempty + 2;  // peers' chunks for me are published
    uint64_t* pfree = pready + 1;   // peers are done with my published chunks
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pfree + 1);
    volatile int* verdict = reinterpret_cast<volatile int*>(tmem_slot + 1);  // epilogue broadcast

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int C = static_cast<int>(cluster_nctarank());
    const int rank = static_cast<int>(cluster_ctarank());
    const int n_clusters = static_cast<int>(nclusters_x());
    const int q = static_cast<int>(cluster_id_x());
    const int n_tiles = (N + kBM - 1) / kBM;
    const int KB = (K + kBK - 1) / kBK;
    const int kb0 = rank * KB / C, kb1 = (rank + 1) * KB / C;
    const int my_tiles = q < n_tiles ? (n_tiles - q + n_clusters - 1) / n_clusters : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], kSkEpiWarps);
        }
        mbar_init(pready, C > 1 ? C - 1 : 1);
        mbar_init(pfree, C > 1 ? C - 1 : 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    cluster_sync_all();  // barriers of every CTA initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmap_w);
            tma_prefetch_desc(&tmap_x);
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            // weight tiles of the first ST stages before the dependency wait (see gemm_sk_kernel)
            constexpr uint32_t kKbBytes = kTileA + Cfg::kTileB;
            int npre = 0;
            for (int i = 0; i < my_tiles && npre < ST; ++i) {
                const int wrow = (q + i * n_clusters) * kBM;
                for (int kb = kb0; kb < kb1 && npre < ST; kb += kKps, ++npre) {
                    const int nk = min(kKps, kb1 - kb);
                    mbar_arrive_expect_tx(&full[npre], nk * kKbBytes);
                    for (int u = 0; u < nk; ++u)
                        tma_load_2d_hint(sA + (npre * kKps + u) * kTileA, &tmap_w, &full[npre],
                                         (kb + u) * kBK, wrow, pol_w);
                }
            }
            pdl_wait();
            pdl_trigger();
            int it = 0;
            bool ok = true;
            for (int i = 0; i < my_tiles && ok; ++i) {
                const int wrow = (q + i * n_clusters) * kBM;
                for (int kb = kb0; kb < kb1; kb += kKps, ++it) {
                    const int s = it % ST;
                    const int nk = min(kKps, kb1 - kb);
                    if (it >= npre) {
                        if (it >= ST && !mbar_wait(&empty[s], ((it / ST) - 1) & 1, err, 430)) { ok = false; break; }
                        mbar_arrive_expect_tx(&full[s], nk * kKbBytes);
                        for (int u = 0; u < nk; ++u)
                            tma_load_2d_hint(sA + (s * kKps + u) * kTileA, &tmap_w, &full[s],
                                             (kb + u) * kBK, wrow, pol_w);
                    }
                    for (int u = 0; u < nk; ++u)
                        tma_load_2d_hint(sB + (s * kKps + u) * Cfg::kTileB, &tmap_x, &full[s],
                                         (kb + u) * kBK, 0, pol_x);
                }
            }
        } else {
            pdl_wait();
            pdl_trigger();
        }
    } else if (warp == 1) {
        pdl_wait();
        pdl_trigger();
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
            int it = 0;
            bool ok = true;
            for (int i = 0; i < my_tiles && ok; ++i) {
                const int a = i & 1;
                if (i >= 2 && !mbar_wait(&tempty[a], ((i >> 1) - 1) & 1, err, 440)) break;
                tc_fence_after();
                const uint32_t acc = tmem + a * BN;
                for (int kb = kb0; kb < kb1; kb += kKps, ++it) {
                    const int s = it % ST;
                    const int nk = min(kKps, kb1 - kb);
                    if (!mbar_wait(&full[s], (it / ST) & 1, err, 441)) { ok = false; break; }
                    tc_fence_after();
                    for (int u = 0; u < nk; ++u) {
                        const uint32_t a_addr = smem_u32(sA + (s * kKps + u) * kTileA);
                        const uint32_t b_addr = smem_u32(sB + (s * kKps + u) * Cfg::kTileB);
#pragma unroll
                        for (int k = 0; k < kBK / 16; ++k)
                            umma_bf16(acc, umma_desc_sw128(a_addr + k * 32),
                                      umma_desc_sw128(b_addr + k * 32), idesc,
                                      (kb > kb0 || u > 0 || k > 0) ? 1u : 0u);
                    }
                    umma_commit(&empty[s]);
                }
                umma_commit(&tfull[a]);
            }
        }
    } else {
        // ---------------- epilogue warps 2..9: warp w reads TMEM lane quarter w % 4; the two warp
        // groups eg = 0, 1 take alternate chunks of the lists below
        pdl_wait();
        pdl_trigger();
        const int warp_q = warp & 3;
        const int eg = (warp - 2) >> 2;
        const int row = warp_q * 32 + lane;
        const int et = threadIdx.x - 64;
        constexpr int kEpiThreads = kSkEpiWarps * 32;
        const uint32_t part_u32 = smem_u32(part);
        for (int i = 0; i < my_tiles; ++i) {
            const int a = i & 1;
            const int n_tile = q + i * n_clusters;
            const int n = n_tile * kBM + row;
            // One thread waits (bounded) for the accumulator and, from tile 1 on, for the peers to
            // be done with this CTA's buffer; the verdict is broadcast so that every epilogue warp
            // takes the same path through the named barriers below.
            if (et == 0)
                *verdict = mbar_wait(&tfull[a], (i >> 1) & 1, err, 450) &&
                           (C == 1 || i == 0 || mbar_wait_cluster(pfree, (i - 1) & 1, err, 451));
            named_bar(1, kEpiThreads);
            const bool ok_acc = *verdict != 0;
            named_bar(1, kEpiThreads);  // verdict read by all before it is rewritten
            if (!ok_acc) break;
            tc_fence_after();
            const uint32_t taddr = tmem + a * BN + (static_cast<uint32_t>(warp_q * 32) << 16);
            if (C > 1) {
                // publish the chunks the peers own: chunk ci is [4 quarters][128 rows][4 floats],
                // so one warp's 16-byte store (or a peer's load) covers 512 contiguous bytes
                int j = 0;
                for (int ci = 0; ci < NCH; ++ci) {
                    if (ci % C == rank) continue;
                    if ((j++ & 1) != eg) continue;
                    uint32_t r[16];
                    tmem_ld16(taddr + ci * 16, r);
                    tmem_ld_wait();
                    float4* dst = reinterpret_cast<float4*>(part) + ci * 4 * kBM + row;
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4)
                        dst[q4 * kBM] =
                            make_float4(__uint_as_float(r[4 * q4]), __uint_as_float(r[4 * q4 + 1]),
                                        __uint_as_float(r[4 * q4 + 2]), __uint_as_float(r[4 * q4 + 3]));
                }
                fence_acq_rel_cluster();
                named_bar(1, kEpiThreads);
                if (et < C && et != rank)  // one thread per peer
                    mbar_remote_arrive(mapa_shared(smem_u32(pready), et));
                if (et == 0) *verdict = mbar_wait_cluster(pready, i & 1, err, 452);
                named_bar(1, kEpiThreads);
                const bool ok_peers = *verdict != 0;
                named_bar(1, kEpiThreads);
                if (!ok_peers) break;
            }
            // my chunks: own accumulator + the peers' published parts, in rank order
            int j = 0;
            for (int ci = rank; ci < NCH; ci += C) {
                if ((j++ & 1) != eg) continue;
                uint32_t r[16];
                float v[16];
                tmem_ld16(taddr + ci * 16, r);
                tmem_ld_wait();
#pragma unroll
                for (int qq = 0; qq < 16; ++qq) v[qq] = 0.f;
                for (int pr = 0; pr < C; ++pr) {
                    if (pr == rank) {
#pragma unroll
                        for (int qq = 0; qq < 16; ++qq) v[qq] += __uint_as_float(r[qq]);
                    } else {
                        const uint32_t src = mapa_shared(part_u32 + (ci * 4 * kBM + row) * 16, pr);
                        float4 pv[4];
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) pv[q4] = ld_dsmem_v4(src + q4 * kBM * 16);
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {
                            v[4 * q4] += pv[q4].x;
                            v[4 * q4 + 1] += pv[q4].y;
                            v[4 * q4 + 2] += pv[q4].z;
                            v[4 * q4 + 3] += pv[q4].w;
                        }
                    }
                }
                epilogue_chunk<EPI>(v, n, N, ci * 16, M, y, amax, lane, warp_q, n_tile, id_off);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[a]);
            if (C > 1) {
                fence_acq_rel_cluster();
                named_bar(1, kEpiThreads);
                if (et < C && et != rank)  // done reading peer et's buffer
                    mbar_remote_arrive(mapa_shared(smem_u32(pfree), et));
            }
        }
        // no CTA leaves while a peer may still read its buffer: wait until every peer is done
        // with the last tile's (every remote access to this CTA's shared memory precedes it)
        if (C > 1 && my_tiles > 0 && et == 0) mbar_wait_cluster(pfree, (my_tiles - 1) & 1, err, 453);
        tc_fence_before();
    }
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

// ============================================================================ split-K partials
// Decode-sized GEMMs (M <= 256 tokens) whose consumer can take the K-split reduction over. The
// operands are swapped relative to the other kernels: the tokens are the UMMA M dimension (128,
// rows past M zero-filled by TMA) and 256 weight rows the N dimension, so a ring stage holds a
// 16 KB token tile and a 32 KB weight tile -- 1.5 bytes staged per weight byte instead of 2,
// which is what bounds a decode GEMM when every SM streams weights (per-SM TMA ingest).
// CTA (blockIdx.x = tile * S + s, blockIdx.y = token tile) accumulates k-blocks
// [s KB / S, (s + 1) KB / S) of weight rows [256 tile, 256 tile + 256) for tokens
// [128 y, 128 y + 128) in TMEM (lane = token, column = weight row) and stores the fp32 partial
// into parts[s][M][N]; the two token tiles of a 256-token step read each weight tile at about the
// same time, the second mostly from L2. No CTA waits for another; the next kernel on the stream
// (fused add + RMSNorm, QK-norm + RoPE) adds the S partials in split order (deterministic).
// Producer warp, MMA warp, 8 epilogue warps as in the stream-K kernel.
constexpr int kPartBN = 256;                        // weight rows per tile (UMMA N)
constexpr int kPartTileX = kBM * kBK * 2;           // 16 KB token tile (UMMA A, M = 128)
constexpr int kPartTileW = kPartBN * kBK * 2;       // 32 KB weight tile (UMMA B)
constexpr int kPartStage = kPartTileX + kPartTileW;
constexpr int kPartStages = kRingBudget / kPartStage;  // 4
constexpr size_t kPartSmem = static_cast<size_t>(kPartStages) * kPartStage + 1024 + 256;
constexpr int kPartPitch = kPartBN + 4;  // floats per token row of the epilogue staging tile
static_assert(kBM * kPartPitch * 4 <= kPartStages * kPartStage, "staging tile exceeds the ring");

__global__ void __launch_bounds__(kSkThreads, 1)
gemm_part_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                 const __grid_constant__ CUtensorMap tmap_x2, float* __restrict__ parts, int M,
                 int N, int K, int S, int xbox, int xbox2, int* err) {
    constexpr int ST = kPartStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sW = smem;                     // [ST] weight tiles (B)
    uint8_t* sX = smem + ST * kPartTileW;   // [ST] token tiles (A)
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * kPartStage);
    uint64_t* empty = full + ST;
    uint64_t* tfull = empty + ST;  // accumulator ready
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x / S, sp = blockIdx.x % S;
    const int KB = (K + kBK - 1) / kBK;
    const int kb0 = sp * KB / S, kb1 = (sp + 1) * KB / S;  // S <= KB: never empty
    const int wrow = tile * kPartBN;
    const int m0 = blockIdx.y * kBM;          // this CTA's 128-token tile
    const int Mt = min(kBM, M - m0);
    // the token box holds xbox rows (M rounded up to 8 when M < 128; the second token tile has
    // its own map, xbox2 rows): the tile's other rows are stale shared memory, whose MMA rows
    // are never stored
    const CUtensorMap* tmx = blockIdx.y ? &tmap_x2 : &tmap_x;
    const uint32_t stage_tx =
        kPartTileW + static_cast<uint32_t>(blockIdx.y ? xbox2 : xbox) * kBK * 2;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tfull, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kPartBN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmap_w);
            tma_prefetch_desc(tmx);
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            // weight tiles of the first ST stages before the dependency wait (see gemm_sk_kernel)
            const int npre = min(ST, kb1 - kb0);
            for (int i = 0; i < npre; ++i) {
                mbar_arrive_expect_tx(&full[i], stage_tx);
                tma_load_2d_hint(sW + i * kPartTileW, &tmap_w, &full[i], (kb0 + i) * kBK, wrow, pol_w);
            }
            pdl_wait();
            pdl_trigger();
            for (int kb = kb0, i = 0; kb < kb1; ++kb, ++i) {
                const int s = i % ST;
                if (i >= npre) {
                    if (!mbar_wait(&empty[s], ((i / ST) - 1) & 1, err, 470)) break;
                    mbar_arrive_expect_tx(&full[s], stage_tx);
                    tma_load_2d_hint(sW + s * kPartTileW, &tmap_w, &full[s], kb * kBK, wrow, pol_w);
                }
                tma_load_2d_hint(sX + s * kPartTileX, tmx, &full[s], kb * kBK, m0, pol_x);
            }
        } else {
            pdl_wait();
            pdl_trigger();
        }
    } else if (warp == 1) {
        pdl_wait();
        pdl_trigger();
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(kBM, kPartBN);
            bool ok = true;
            for (int kb = kb0, i = 0; kb < kb1; ++kb, ++i) {
                const int s = i % ST;
                if (!mbar_wait(&full[s], (i / ST) & 1, err, 471)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sX + s * kPartTileX);
                const uint32_t b_addr = smem_u32(sW + s * kPartTileW);
#pragma unroll
                for (int k = 0; k < kBK / 16; ++k)
                    umma_bf16(tmem, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                              idesc, (kb > kb0 || k > 0) ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            if (ok) umma_commit(tfull);
        }
    } else {
        // ---------------- epilogue warps 2..9: warp w reads TMEM lane quarter w % 4 (32 tokens)
        // and every other 16-column chunk (16 weight rows) into the drained ring, laid out
        // [token][kPartPitch] (rows padded by 16 B: a warp's 16-byte stores hit distinct banks);
        // then each warp writes whole token rows to global memory, 512 contiguous bytes per store
        pdl_wait();
        pdl_trigger();
        const int warp_q = warp & 3;
        const int eg = (warp - 2) >> 2;
        const int ew = warp - 2;
        constexpr int kEpiThreads = kSkEpiWarps * 32;
        const bool have = mbar_wait(tfull, 0, err, 472);
        tc_fence_after();
        float* stage = reinterpret_cast<float*>(smem);  // the ring is drained once tfull fired
        if (warp_q * 32 < Mt) {  // warp-uniform: quarters past the last token load nothing
            const uint32_t taddr = tmem + (static_cast<uint32_t>(warp_q * 32) << 16);
            float4* srow = reinterpret_cast<float4*>(stage + (warp_q * 32 + lane) * kPartPitch);
#pragma unroll 1
            for (int ci = eg; ci < kPartBN / 16; ci += 4) {  // two chunks per TMEM round trip
                uint32_t r[2][16];
                tmem_ld16(taddr + ci * 16, r[0]);
                tmem_ld16(taddr + (ci + 2) * 16, r[1]);
                tmem_ld_wait();
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4)
                        srow[(ci + 2 * h) * 4 + q4] =
                            have ? make_float4(__uint_as_float(r[h][4 * q4]), __uint_as_float(r[h][4 * q4 + 1]),
                                               __uint_as_float(r[h][4 * q4 + 2]), __uint_as_float(r[h][4 * q4 + 3]))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        tc_fence_before();
        named_bar(1, kEpiThreads);
        const bool vec = (N & 3) == 0 && wrow + kPartBN <= N;
        for (int m = ew; m < Mt; m += kSkEpiWarps) {
            const float* src = stage + m * kPartPitch;
            float* dst = parts + (static_cast<int64_t>(sp) * M + m0 + m) * N + wrow;
#pragma unroll
            for (int c = lane * 4; c < kPartBN; c += 128) {
                const float4 v = *reinterpret_cast<const float4*>(src + c);
                if (vec) {
                    *reinterpret_cast<float4*>(dst + c) = v;
                } else {
                    if (wrow + c < N) dst[c] = v.x;
                    if (wrow + c + 1 < N) dst[c + 1] = v.y;
                    if (wrow + c + 2 < N) dst[c + 2] = v.z;
                    if (wrow + c + 3 < N) dst[c + 3] = v.w;
                }
            }
        }
    }
    // lane 0 of warps 0 and 1 ran their loops alone: reconverge before the block barrier
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kPartBN);
    }
}

// ============================================================================ row ranges
// Decode-sized GEMMs with many weight rows (gate_up, lm_head): every CTA owns whole tiles of BR
// consecutive weight rows (BR = 16 hs, hs <= 16, chosen on the host so that the tiles fill the
// GPU's CTAs in near-equal rounds) over the full K, so there is no K split and no cross-CTA
// reduction. Operands as in the partials kernel: tokens are the UMMA M dimension (128) and the
// tile's weight rows the N dimension (BR), a ring stage holding a 16 KB token tile and a
// BR x 64 weight tile. The CTA walks its tiles t = blockIdx.x, + gridDim.x, ... with the
// accumulator double-buffered in TMEM (2 x 256 columns), so a tile's epilogue overlaps the next
// tile's mainloop. Epilogue thread = token (TMEM lane), 16 consecutive weight rows per chunk:
//   BF16 / F32  y[m][n .. n + 15]
//   SWIGLU      packed rows (16-row groups: 8 gate, then the 8 matching up rows) ->
//               y[m][f .. f + 7] = silu(gate) * up for the group's 8 features
//   ARGMAX      running best (logit, lowest id) over the thread's rows, one atomicMax per token
constexpr int kRowsTileX = kBM * kBK * 2;         // 16 KB token tile (UMMA A)
constexpr int kRowsTileW = 256 * kBK * 2;         // room for a 256-row weight tile (UMMA B)
constexpr int kRowsStage = kRowsTileX + kRowsTileW;
constexpr int kRowsStages = kRingBudget / kRowsStage;  // 4
constexpr size_t kRowsSmem = static_cast<size_t>(kRowsStages) * kRowsStage + 1024 + 256;

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

template <int EPI>
__global__ void __launch_bounds__(kSkThreads, 1)
gemm_rows_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                 void* __restrict__ y, unsigned long long* __restrict__ amax, int M, int N, int K,
                 int BR, int xbox, int id_off, int* err) {
    constexpr int ST = kRowsStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sW = smem;                     // [ST] weight tiles (B)
    uint8_t* sX = smem + ST * kRowsTileW;   // [ST] token tiles (A)
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * kRowsStage);
    uint64_t* empty = full + ST;
    uint64_t* tfull = empty + ST;   // [2] accumulator ready
    uint64_t* tempty = tfull + 2;   // [2] accumulator drained
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int T = (N + BR - 1) / BR;
    const int KB = (K + kBK - 1) / kBK;
    const int G = gridDim.x;
    const int my_tiles = static_cast<int>(blockIdx.x) < T ? (T - blockIdx.x + G - 1) / G : 0;
    const int m0 = blockIdx.y * kBM;  // token tile (129..256 tokens: two, each with its own CTAs)
    // token box of xbox rows (M rounded up to 8): the tile's other rows are never stored
    const uint32_t stage_tx = static_cast<uint32_t>(xbox + BR) * kBK * 2;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], kSkEpiWarps);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmap_w);
            tma_prefetch_desc(&tmap_x);
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            // weight tiles of the first ST stages before the dependency wait (see gemm_sk_kernel)
            const int npre = my_tiles > 0 ? min(ST, my_tiles * KB) : 0;
            for (int i = 0; i < npre; ++i) {
                const int t = blockIdx.x + (i / KB) * G;
                mbar_arrive_expect_tx(&full[i], stage_tx);
                tma_load_2d_hint(sW + i * kRowsTileW, &tmap_w, &full[i], (i % KB) * kBK, t * BR, pol_w);
            }
            pdl_wait();
            pdl_trigger();
            int i = 0;
            bool ok = true;
            for (int it = 0; it < my_tiles && ok; ++it) {
                const int wrow = (blockIdx.x + it * G) * BR;
                for (int kb = 0; kb < KB; ++kb, ++i) {
                    const int s = i % ST;
                    if (i >= npre) {
                        if (!mbar_wait(&empty[s], ((i / ST) - 1) & 1, err, 480)) { ok = false; break; }
                        mbar_arrive_expect_tx(&full[s], stage_tx);
                        tma_load_2d_hint(sW + s * kRowsTileW, &tmap_w, &full[s], kb * kBK, wrow, pol_w);
                    }
                    tma_load_2d_hint(sX + s * kRowsTileX, &tmap_x, &full[s], kb * kBK, m0, pol_x);
                }
            }
        } else {
            pdl_wait();
            pdl_trigger();
        }
    } else if (warp == 1) {
        pdl_wait();
        pdl_trigger();
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(kBM, BR);
            int i = 0;
            bool ok = true;
            for (int it = 0; it < my_tiles && ok; ++it) {
                const int a = it & 1;
                if (it >= 2 && !mbar_wait(&tempty[a], ((it >> 1) - 1) & 1, err, 481)) break;
                tc_fence_after();
                const uint32_t acc = tmem + a * 256;
                for (int kb = 0; kb < KB; ++kb, ++i) {
                    const int s = i % ST;
                    if (!mbar_wait(&full[s], (i / ST) & 1, err, 482)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sX + s * kRowsTileX);
                    const uint32_t b_addr = smem_u32(sW + s * kRowsTileW);
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)
                        umma_bf16(acc, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                                  idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&tfull[a]);
            }
        }
    } else {
        // ---------------- epilogue warps 2..9: warp w reads TMEM lane quarter w % 4 (32 tokens);
        // the two warps of a quarter take alternate 16-row chunks
        pdl_wait();
        pdl_trigger();
        const int warp_q = warp & 3;
        const int eg = (warp - 2) >> 2;
        const int m = m0 + warp_q * 32 + lane;
        const bool live = m0 + warp_q * 32 < M;  // warp-uniform
        const int nch = BR / 16;
        unsigned long long best = 0ull;
        for (int it = 0; it < my_tiles; ++it) {
            const int a = it & 1;
            const int wrow = (blockIdx.x + it * G) * BR;
            const bool have = mbar_wait(&tfull[a], (it >> 1) & 1, err, 483);
            tc_fence_after();
            if (live) {
                const uint32_t taddr = tmem + a * 256 + (static_cast<uint32_t>(warp_q * 32) << 16);
#pragma unroll 1
                for (int ci = eg; ci < nch; ci += 2) {
                    uint32_t r[16];
                    __syncwarp();  // converged for the warp-collective TMEM load
                    tmem_ld16(taddr + ci * 16, r);
                    tmem_ld_wait();
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = have ? __uint_as_float(r[j]) : 0.f;
                    const int n0 = wrow + ci * 16;
                    if (m >= M || n0 >= N) {
                    } else if (EPI == EPI_ARGMAX) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const unsigned long long key =
                                n0 + j < N ? argmax_key(v[j], n0 + j + id_off) : 0ull;
                            best = key > best ? key : best;
                        }
                    } else if (EPI == EPI_SWIGLU) {
                        const int inter = N >> 1;
                        const int f0 = n0 >> 1;  // the group's first feature
                        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(y) + static_cast<int64_t>(m) * inter + f0;
                        if ((inter & 7) == 0) {
                            uint4 o;
                            o.x = pack_bf16x2(silu_mul(v[0], v[8]), silu_mul(v[1], v[9]));
                            o.y = pack_bf16x2(silu_mul(v[2], v[10]), silu_mul(v[3], v[11]));
                            o.z = pack_bf16x2(silu_mul(v[4], v[12]), silu_mul(v[5], v[13]));
                            o.w = pack_bf16x2(silu_mul(v[6], v[14]), silu_mul(v[7], v[15]));
                            *reinterpret_cast<uint4*>(dst) = o;
                        } else {
#pragma unroll
                            for (int k = 0; k < 8; ++k)
                                if (f0 + k < inter) dst[k] = __float2bfloat16_rn(silu_mul(v[k], v[k + 8]));
                        }
                    } else if (EPI == EPI_BF16) {
                        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(y) + static_cast<int64_t>(m) * N + n0;
                        if ((N & 7) == 0 && n0 + 16 <= N) {
                            uint4 o[2];
                            uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
                            for (int j = 0; j < 8; ++j) ow[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
                            reinterpret_cast<uint4*>(dst)[0] = o[0];
                            reinterpret_cast<uint4*>(dst)[1] = o[1];
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                if (n0 + j < N) dst[j] = __float2bfloat16_rn(v[j]);
                        }
                    } else {  // EPI_F32
                        float* dst = static_cast<float*>(y) + static_cast<int64_t>(m) * N + n0;
                        if ((N & 3) == 0 && n0 + 16 <= N) {
#pragma unroll
                            for (int q4 = 0; q4 < 4; ++q4)
                                reinterpret_cast<float4*>(dst)[q4] =
                                    make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                if (n0 + j < N) dst[j] = v[j];
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[a]);
        }
        if (EPI == EPI_ARGMAX && live && m < M && best) atomicMax(amax + m, best);
        tc_fence_before();
    }
    // lane 0 of warps 0 and 1 ran their loops alone: reconverge before the block barrier
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// MSGL_GEMM_ROWS=0 turns the row-range schedule off (the cluster / stream-K schedules run).
// MSGL_GEMM_DECODE (tuning override, default automatic): the schedule of decode-sized GEMMs
// (M <= 128): "rows", "parts" (split-K partials + reduce), "cl" (cluster split-K) or "sk"
// (stream-K); a schedule that does not apply to the shape falls through to the automatic choice.
int decode_schedule() {
    static const int v = [] {
        const char* e = std::getenv("MSGL_GEMM_DECODE");
        if (!e) return 0;
        const std::string x(e);
        return x == "rows" ? 1 : x == "parts" ? 2 : x == "cl" ? 3 : x == "sk" ? 4 : 0;
    }();
    return v;
}

// K up to which decode GEMMs take narrow row tiles (no K split); MSGL_GEMM_SHORTK_ROWS=0 turns
// that off (read on every call). Measured on B200 at 128 tokens against split-K partials +
// reduce: 4096 x 512 4.9 vs 8.8 us, 4096 x 1024 7.2 vs 9.4, 4096 x 1536 9.6 vs 10.2; at
// 4096 x 2048 the partials win (10.9 vs 11.8).
constexpr int kRowsShortK = 1536;
bool small_k_rows() {
    const char* e = std::getenv("MSGL_GEMM_SHORTK_ROWS");
    return !(e && e[0] == '0');
}


bool rows_disabled() {
    static const bool off = [] {
        const char* e = std::getenv("MSGL_GEMM_ROWS");
        return e && e[0] == '0';
    }();
    return off;
}

int num_sms() {
    static int n[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!n[dev]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
            cudaGetLastError();  // no device (host-only query): a 148-SM B200
            v = 148;
        }
        n[dev] = v;
    }
    return n[dev];
}

// Stream-K workspace: one flag per CTA (zero when idle), then one fp32 part slot per CTA.
size_t sk_workspace_bytes(int bn, int sms) {
    return kSkFlagBytes + static_cast<size_t>(sms) * kBM * bn * sizeof(float);
}

struct GemmPlan {
    int bn, m_tiles, n_tiles, splits, kb_per_split;
    size_t ws_part_bytes, ws_cnt_off, ws_bytes;
};

int pick_bn(int M) {
    if (M <= 16) return 16;
    if (M <= 32) return 32;
    if (M <= 64) return 64;
    if (M <= 128) return 128;
    return 256;
}

GemmPlan plan_gemm(int M, int N, int K) {
    GemmPlan p{};
    p.bn = pick_bn(M);
    p.m_tiles = (M + p.bn - 1) / p.bn;
    p.n_tiles = (N + kBM - 1) / kBM;
    const int kbs = (K + kBK - 1) / kBK;
    const int tiles = p.m_tiles * p.n_tiles;
    const int slots = p.bn >= 256 ? 148 : 2 * 148;  // resident CTAs (smem-bound)
    int splits = 1;
    if (tiles < slots) splits = std::max(1, std::min(slots / tiles, std::max(1, kbs / 4)));
    splits = std::min(splits, 32);
    p.kb_per_split = (kbs + splits - 1) / splits;
    p.splits = (kbs + p.kb_per_split - 1) / p.kb_per_split;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    // Workspace layout: arrival counters at a FIXED offset (0) for every GEMM shape, partial
    // tiles after them. One workspace serves GEMMs of different shapes in stream order; a
    // shape-dependent counter offset would let one GEMM's partials overwrite another's
    // (self-resetting, hence persistent) counters.
    if (p.splits > 1) {
        p.ws_cnt_off = 0;
        p.ws_part_bytes = up(static_cast<size_t>(tiles) * p.splits * p.bn * kBM * sizeof(float));
        p.ws_bytes = kCounterBytes + p.ws_part_bytes;
    }
    return p;
}

template <int BN, int EPI, bool GROUPED = false>
int launch_bn(const GemmPlan& p, const CUtensorMap& tw, const CUtensorMap& tx, void* y,
              unsigned long long* amax, int M, int N, int K, void* ws, cudaStream_t stream,
              GroupArgs grp = GroupArgs{}, int id_off = 0) {
    using Cfg = GemmCfg<BN>;
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    cudaFuncSetAttribute(gemm_kernel<BN, EPI, GROUPED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(Cfg::kSmem));
    dim3 grid(p.m_tiles, p.n_tiles, p.splits);
    uint8_t* w8 = static_cast<uint8_t*>(ws);
    launch_pdl(gemm_kernel<BN, EPI, GROUPED>, grid, dim3(kGemmThreads), Cfg::kSmem, stream,
        tw, tx, y, amax, M, N, K, p.kb_per_split, p.splits,
        p.splits > 1 ? reinterpret_cast<float*>(w8 + kCounterBytes) : nullptr,
        p.splits > 1 ? reinterpret_cast<int*>(w8 + p.ws_cnt_off) : nullptr, grp, id_off, err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

// Grouped GEMM schedule: the persistent kernel with dynamic work for prefill-sized tiles, one
// CTA per tile for decode-sized ones. Measured on B200, Qwen3-30B-A3B experts (128 x 1536 x 2048
// gate_up + SwiGLU, 128 x 2048 x 768 down), persistent vs per-tile, in us:
//   tokens x top-8  rows/tile  gate_up       down
//   4096            256        408 vs 480    200 vs 309
//   2048            128        249 vs 233    130 vs 138
//   1024 / 512      64 / 32    176 vs 156    99 vs 100  (and 166 vs 138, 92 vs 86)
//   256             16         151 vs 130    83 vs 76
// so: 256-row tiles, and the plain (non-SwiGLU) epilogue from 128-row tiles.
// MSGL_GROUPED_PERSISTENT=0 / 1 forces either (read on every call).
bool grouped_persistent(int bn, bool swiglu) {
    const char* e = std::getenv("MSGL_GROUPED_PERSISTENT");
    if (e && (e[0] == '0' || e[0] == '1')) return e[0] == '1';
    return bn >= 256 || (bn >= 128 && !swiglu);
}

template <int BN, int EPI>
int launch_grouped_dyn(const CUtensorMap& tw, const CUtensorMap& tx, void* y, int N, int K,
                       const GroupArgs& g, int* counter, int64_t max_items, cudaStream_t stream) {
    using Cfg = GemmCfg<BN>;
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    cudaFuncSetAttribute(gemm_grouped_dyn_kernel<BN, EPI>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(Cfg::kSmem));
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemm_grouped_dyn_kernel<BN, EPI>,
                                                      kGemmThreads, Cfg::kSmem) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        per_sm = 1;
    }
    const int G = static_cast<int>(std::min<int64_t>(static_cast<int64_t>(num_sms()) * per_sm,
                                                     std::max<int64_t>(1, max_items)));
    launch_pdl(gemm_grouped_dyn_kernel<BN, EPI>, dim3(G), dim3(kGemmThreads), Cfg::kSmem, stream,
               tw, tx, y, N, K, g, counter, err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

template <int BN, int EPI>
int launch_sk(const CUtensorMap& tw, const CUtensorMap& tx, void* y, unsigned long long* amax,
              int M, int N, int K, void* ws, int sms, cudaStream_t stream, int id_off = 0) {
    using Cfg = SkCfg<BN>;
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    cudaFuncSetAttribute(gemm_sk_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(Cfg::kSmem));
    const int m_tiles = (M + BN - 1) / BN;
    const int64_t units = static_cast<int64_t>(m_tiles) * ((N + kBM - 1) / kBM) * ((K + kBK - 1) / kBK);
    const int G = static_cast<int>(std::min<int64_t>(std::min(sms, kSkMaxCtas), units));
    uint8_t* w8 = static_cast<uint8_t*>(ws);
    launch_pdl(gemm_sk_kernel<BN, EPI>, dim3(G), dim3(kSkThreads), Cfg::kSmem, stream,
        tw, tx, y, amax, M, N, K, m_tiles, reinterpret_cast<int*>(w8),
        reinterpret_cast<float*>(w8 + kSkFlagBytes), id_off, err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

// Cluster split-K launch: grid = n_clusters clusters of C CTAs (cluster dims C x 1 x 1),
// programmatic stream serialisation as every kernel of the forward path.
template <int BN, int EPI>
cudaError_t launch_cl_raw(const CUtensorMap& tw, const CUtensorMap& tx, void* y,
                          unsigned long long* amax, int M, int N, int K, int C, int n_clusters,
                          int id_off, int* err, cudaStream_t stream) {
    using Cfg = ClCfg<BN>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_clusters * C);
    cfg.blockDim = dim3(kSkThreads);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    launch_counter().fetch_add(1, std::memory_order_relaxed);
    return cudaLaunchKernelEx(&cfg, gemm_cl_kernel<BN, EPI>, tw, tx, y, amax, M, N, K, id_off, err);
}

// Co-resident clusters of C CTAs of gemm_cl_kernel<BN, EPI> on this device (cached).
template <int BN, int EPI>
int cl_max_clusters(int C) {
    static int cache[64][kClMaxC + 1] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cache[dev][C]) return cache[dev][C] > 0 ? cache[dev][C] : 0;
    using Cfg = ClCfg<BN>;
    cudaFuncSetAttribute(gemm_cl_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(Cfg::kSmem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C * 64);
    cfg.blockDim = dim3(kSkThreads);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_cl_kernel<BN, EPI>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    cache[dev][C] = n > 0 ? n : -1;
    return n;
}

// Cluster size for a decode GEMM of T tiles x KB k-blocks: the C in 1..8 (C <= KB) with the
// fewest k-blocks per CTA over all waves, ceil(T / clusters) * ceil(KB / C); ties go to the
// smaller C (less reduction traffic). Returns that cost (k-blocks on the busiest CTA).
template <int BN, int EPI>
int64_t plan_cl(int T, int KB, int& C_best, int& n_clusters) {
    int64_t best = -1;
    C_best = 1;
    n_clusters = 0;
    for (int C = 1; C <= kClMaxC && C <= KB; ++C) {
        const int nc = cl_max_clusters<BN, EPI>(C);
        if (nc <= 0) continue;
        const int64_t cost = static_cast<int64_t>((T + nc - 1) / nc) * ((KB + C - 1) / C);
        if (best < 0 || cost < best) {
            best = cost;
            C_best = C;
            n_clusters = std::min(nc, T);
        }
    }
    return best;
}

// Launches the cluster kernel when its wave-quantised cost is within 20% of a perfect balance
// of the T * KB k-blocks over the SMs; returns -1 (nothing launched) otherwise, so that the
// caller runs the stream-K kernel, whose balance is exact but whose cross-CTA reduction goes
// through global memory.
template <int BN, int EPI>
int launch_cl(const CUtensorMap& tw, const CUtensorMap& tx, void* y, unsigned long long* amax,
              int M, int N, int K, cudaStream_t stream, int id_off) {
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    const int T = (N + kBM - 1) / kBM, KB = (K + kBK - 1) / kBK;
    int C = 1, nc = 0;
    const int64_t cost = plan_cl<BN, EPI>(T, KB, C, nc);
    const int64_t sms = num_sms();
    const int64_t balanced = (static_cast<int64_t>(T) * KB + sms - 1) / sms;
    if (nc <= 0 || (decode_schedule() != 3 && cost * 5 > balanced * 6)) return -1;
    cudaError_t e = launch_cl_raw<BN, EPI>(tw, tx, y, amax, M, N, K, C, nc, id_off, err, stream);
    if (e != cudaSuccess) return set_error(MSGL_ERR_CUDA, cudaGetErrorString(e));
    return MSGL_OK;
}

// Sum of the S fp32 split-K partials parts[S][M][N] of a decode GEMM, in split order, in the
// form the GEMM's caller asked for: BF16 / F32 y[m][n] (4 columns per thread), SWIGLU the packed
// gate/up rows in 16-column groups (8 gate, then the 8 matching up columns) -> y[m][f] =
// silu(gate) * up for the group's 8 features (one group per thread). Partial loads go out four
// splits at a time.
template <int EPI>
__global__ void __launch_bounds__(256)
partials_reduce_kernel(const float* __restrict__ parts, int S, void* __restrict__ y, int M, int N) {
    pdl_wait();
    pdl_trigger();
    const int64_t stride = static_cast<int64_t>(M) * N;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (EPI == EPI_SWIGLU) {
        const int groups = N >> 4;
        if (idx >= static_cast<int64_t>(M) * groups) return;
        const int m = static_cast<int>(idx / groups), g = static_cast<int>(idx % groups);
        const float4* src = reinterpret_cast<const float4*>(parts + static_cast<int64_t>(m) * N + g * 16);
        float4 acc[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        int sp = 0;
        for (; sp + 2 <= S; sp += 2) {
            float4 t[2][4];
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int q = 0; q < 4; ++q) t[u][q] = src[(sp + u) * (stride >> 2) + q];
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    acc[q].x += t[u][q].x; acc[q].y += t[u][q].y;
                    acc[q].z += t[u][q].z; acc[q].w += t[u][q].w;
                }
        }
        for (; sp < S; ++sp)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 t = src[sp * (stride >> 2) + q];
                acc[q].x += t.x; acc[q].y += t.y; acc[q].z += t.z; acc[q].w += t.w;
            }
        const float* v = reinterpret_cast<const float*>(acc);  // 8 gate, then 8 up
        const int inter = N >> 1;
        uint4 o;
        o.x = pack_bf16x2(silu_mul(v[0], v[8]), silu_mul(v[1], v[9]));
        o.y = pack_bf16x2(silu_mul(v[2], v[10]), silu_mul(v[3], v[11]));
        o.z = pack_bf16x2(silu_mul(v[4], v[12]), silu_mul(v[5], v[13]));
        o.w = pack_bf16x2(silu_mul(v[6], v[14]), silu_mul(v[7], v[15]));
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(y) + static_cast<int64_t>(m) * inter + g * 8) = o;
    } else {
        // 4 columns per thread when rows are float4-aligned, else one
        const bool vec = (N & 3) == 0;
        const int per = vec ? 4 : 1;
        const int64_t cols = N / per;
        if (idx >= static_cast<int64_t>(M) * cols) return;
        const int64_t e0 = (idx / cols) * N + (idx % cols) * per;  // first element
        float a[4] = {0.f, 0.f, 0.f, 0.f};
        if (vec) {
            const float4* src = reinterpret_cast<const float4*>(parts + e0);
            int sp = 0;
            for (; sp + 4 <= S; sp += 4) {
                float4 t[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) t[u] = src[(sp + u) * (stride >> 2)];
#pragma unroll
                for (int u = 0; u < 4; ++u) { a[0] += t[u].x; a[1] += t[u].y; a[2] += t[u].z; a[3] += t[u].w; }
            }
            for (; sp < S; ++sp) {
                const float4 t = src[sp * (stride >> 2)];
                a[0] += t.x; a[1] += t.y; a[2] += t.z; a[3] += t.w;
            }
        } else {
            for (int sp = 0; sp < S; ++sp) a[0] += parts[sp * stride + e0];
        }
        for (int j = 0; j < per; ++j) {
            if (EPI == EPI_BF16) static_cast<__nv_bfloat16*>(y)[e0 + j] = __float2bfloat16_rn(a[j]);
            else static_cast<float*>(y)[e0 + j] = a[j];
        }
    }
}

// Decode-sized GEMM as split-K partials in the caller's workspace (after the counter region,
// which must stay zero-filled) plus the reduce kernel above. Returns -1 (nothing launched) when
// the shape gives fewer than 2 splits or the workspace is too small.
template <int EPI>
int launch_part_reduce(const void* x, const void* w, void* y, int M, int N, int K, void* ws,
                       size_t ws_bytes, cudaStream_t stream);

// Split count of the partials kernel: as many splits as keep one tile-split per SM in a single
// wave, at least 4 k-blocks per split, at most 16 partials for the consumer to add.
// Rows of the token box of the kernels that take tokens as the UMMA M dimension: M rounded up to
// 8 below 128 tokens. The TMA then brings only those rows (out-of-range rows of a 128-row box
// cost as much as real ones: lm_head + argmax over 151936 x 1024 took 80 us at 4 tokens against
// 58 us at 64).
int token_box(int M) { return M >= kBM ? kBM : std::max(8, (M + 7) & ~7); }

int part_splits(int M, int N, int K) {
    const int MT = std::max(1, (M + kBM - 1) / kBM);
    const int T = (N + kPartBN - 1) / kPartBN * MT, KB = (K + kBK - 1) / kBK, sms = num_sms();
    if (T >= sms) return 1;
    return std::max(1, std::min({sms / T, std::max(1, KB / 4), 16}));
}

// Token maps: tokens [0, 128) with a box of token_box(M) rows, and (M > 128) tokens [128, M)
// with a box of token_box(M - 128) rows -- the byte counts the kernel expects.
int launch_part(const void* x, const CUtensorMap& tw, float* parts, int M, int N, int K, int S,
                cudaStream_t stream) {
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    CUtensorMap tx, tx2;
    const int xbox = token_box(std::min(M, kBM));
    const int xbox2 = M > kBM ? token_box(M - kBM) : xbox;
    int rc = make_tmap_2d_bf16(&tx, x, K, M, static_cast<uint64_t>(K) * 2, kBK, xbox, true);
    if (rc) return rc;
    rc = make_tmap_2d_bf16(&tx2, x, K, M, static_cast<uint64_t>(K) * 2, kBK, xbox2, true);
    if (rc) return rc;
    cudaFuncSetAttribute(gemm_part_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(kPartSmem));
    const int T = (N + kPartBN - 1) / kPartBN;
    launch_pdl(gemm_part_kernel, dim3(T * S, (M + kBM - 1) / kBM), dim3(kSkThreads), kPartSmem,
               stream, tw, tx, tx2, parts, M, N, K, S, xbox, xbox2, err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

// Tile height (in 16-row groups) of the row-range kernel for N weight rows on `sms` CTAs: the
// hs in [6, 16] whose tiles spread over the CTAs with the least staged bytes on the busiest
// CTA (rounds x (16 KB token tile + 2 KB x hs weight tile) per k-block), among those that keep
// the CTAs at least 85% evenly loaded; 0 when none does (the caller uses another schedule).
// Below 6 groups the token tile would be most of what a stage brings in.
int plan_rows(int N, int sms, int& tiles, int min_hs = 6) {
    const int n = (N + 15) / 16;
    int best_hs = 0;
    int64_t best = -1;
    tiles = 0;
    for (int hs = min_hs; hs <= 16; ++hs) {
        const int T = (n + hs - 1) / hs;
        const int rounds = (T + sms - 1) / sms;
        if (static_cast<int64_t>(T) * 100 < static_cast<int64_t>(rounds) * sms * 85) continue;
        const int64_t cost = static_cast<int64_t>(rounds) * (16 + 2 * hs);
        if (best < 0 || cost < best) {
            best = cost;
            best_hs = hs;
            tiles = T;
        }
    }
    return best_hs;
}

template <int EPI>
int launch_rows(const void* x, const void* w, void* y, unsigned long long* amax, int M, int N,
                int K, int hs, int tiles, int sms, cudaStream_t stream, int id_off) {
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    const int BR = hs * 16;
    CUtensorMap tw, tx;
    int rc = make_tmap_2d_bf16(&tw, w, K, N, static_cast<uint64_t>(K) * 2, kBK, BR, true);
    if (rc) return rc;
    rc = make_tmap_2d_bf16(&tx, x, K, M, static_cast<uint64_t>(K) * 2, kBK, token_box(M), true);
    if (rc) return rc;
    cudaFuncSetAttribute(gemm_rows_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(kRowsSmem));
    // grid.y = token tiles of 128 (two at 129..256 tokens; `sms` is then the CTAs per tile)
    launch_pdl(gemm_rows_kernel<EPI>, dim3(std::min(tiles, sms), (M + kBM - 1) / kBM),
               dim3(kSkThreads), kRowsSmem, stream, tw, tx, y, amax, M, N, K, BR, token_box(M),
               id_off, err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

size_t part_reduce_bytes(int M, int N, int K) {
    if (M > 256) return 0;
    // 129..256 tokens: one pass over both token tiles, or (fewer than 2 splits) two passes of 128
    const int S = part_splits(M, N, K), S1 = part_splits(std::min(M, 128), N, K);
    size_t b = 0;
    if (S >= 2) b = static_cast<size_t>(S) * M * N * sizeof(float);
    if (S1 >= 2) b = std::max(b, static_cast<size_t>(S1) * std::min(M, 128) * N * sizeof(float));
    return b ? kCounterBytes + b : 0;
}

template <int EPI>
int launch_part_reduce(const void* x, const void* w, void* y, int M, int N, int K, void* ws,
                       size_t ws_bytes, cudaStream_t stream) {
    const int S = part_splits(M, N, K);
    if (S < 2 || (EPI == EPI_SWIGLU && N % 16) || !ws || (reinterpret_cast<uintptr_t>(ws) & 15) ||
        ws_bytes < kCounterBytes + static_cast<size_t>(S) * M * N * sizeof(float))
        return -1;
    float* parts = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kCounterBytes);
    CUtensorMap tw;
    int rc = make_tmap_2d_bf16(&tw, w, K, N, static_cast<uint64_t>(K) * 2, kBK, kPartBN, true);
    if (rc) return rc;
    rc = launch_part(x, tw, parts, M, N, K, S, stream);
    if (rc) return rc;
    const int64_t work = EPI == EPI_SWIGLU ? static_cast<int64_t>(M) * (N / 16)
                                           : static_cast<int64_t>(M) * ((N & 3) == 0 ? N / 4 : N);
    launch_pdl(partials_reduce_kernel<EPI>, dim3(static_cast<unsigned>((work + 255) / 256)), dim3(256), 0,
               stream, static_cast<const float*>(parts), S, y, M, N);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

template <int EPI>
int run_gemm(const void* x, const void* w, void* y, unsigned long long* amax, int M, int N, int K,
             void* ws, size_t ws_bytes, cudaStream_t stream, int id_off = 0) {
    if (M < 0 || N <= 0 || K <= 0) return set_error(MSGL_ERR_INVALID_ARG, "gemm: bad sizes");
    if (K % 8) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "gemm: K must be a multiple of 8");
    if (M == 0) return MSGL_OK;
    if (M > 65535 * 256) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "gemm: M too large");
    if (M > 128 && M <= 256 && decode_schedule() == 0 && !rows_disabled()) {
        // 129..256 tokens (a large decode batch): split-K partials over both 128-token tiles in
        // one grid, summed by the reduce kernel (the partials kernel alone, measured on B200 at
        // 256 tokens, against stream-K: 5120 x 2048 10.0 vs 25.1 us, 6144 x 4096 15.3 vs 27.7,
        // 4096 x 12288 26.3 vs 41.3)
        if (EPI != EPI_ARGMAX) {
            const int r = launch_part_reduce<EPI>(x, w, y, M, N, K, ws, ws_bytes, stream);
            if (r != -1) return r;
        } else {
            // argmax needs whole rows: row tiles for both token tiles in one launch, half of
            // the SMs on each, so the two CTAs of a weight tile read it at about the same time
            const int half = std::max(1, num_sms() / 2);
            int tiles = 0;
            const int hs = plan_rows(N, half, tiles);
            if (hs > 0)
                return launch_rows<EPI>(x, w, y, amax, M, N, K, hs, tiles, half, stream, id_off);
        }
    }
    if (M > 128 && M <= 256 && decode_schedule() == 0 && !rows_disabled() &&
        (EPI == EPI_ARGMAX || static_cast<int64_t>(N) * K * 2 < (int64_t(40) << 20))) {
        // otherwise (argmax, which needs whole rows, or fewer than 2 splits): two passes of the
        // decode-sized schedules over tokens [0, 128) and [128, M), the second reading weights
        // under 40 MB from L2 (lm_head + argmax 151936 x 2048 at 256 tokens: 199 us vs 338 on
        // stream-K; from 50 MB up stream-K is faster for the other epilogues)
        int rc = run_gemm<EPI>(x, w, y, amax, 128, N, K, ws, ws_bytes, stream, id_off);
        if (rc) return rc;
        const auto* x2 = static_cast<const __nv_bfloat16*>(x) + static_cast<int64_t>(128) * K;
        void* y2 = y;
        if (EPI == EPI_F32) y2 = static_cast<float*>(y) + static_cast<int64_t>(128) * N;
        else if (EPI == EPI_SWIGLU)
            y2 = static_cast<__nv_bfloat16*>(y) + static_cast<int64_t>(128) * (N / 2);
        else if (EPI == EPI_BF16)
            y2 = static_cast<__nv_bfloat16*>(y) + static_cast<int64_t>(128) * N;
        return run_gemm<EPI>(x2, w, y2, amax ? amax + 128 : nullptr, M - 128, N, K, ws, ws_bytes,
                             stream, id_off);
    }
    const int force = M <= 128 ? decode_schedule() : 0;
    // Small gate_up + SwiGLU (a wide tensor-parallel rank's shard, e.g. 3072 x 4096): the
    // cluster schedule reduces in shared memory and needs no second kernel; measured at M 128,
    // 3072 x 4096: 14.0 us cluster vs 19.8 us partials + reduce (at 6144 x 4096 partials win,
    // 20.8 vs 23.5 us). With a short K and at least 32 tokens narrow row tiles beat both
    // (Qwen3-0.6B's 6144 x 1024: 8.2 vs 9.4 us at 64 tokens, 8.3 vs 11.3 at 128; at 4 tokens
    // the cluster / partials path stays faster, 7.0 vs 8.2).
    const bool small_swiglu = EPI == EPI_SWIGLU && M <= 128 && force == 0 &&
                              static_cast<int64_t>(N) * K <= (int64_t(16) << 20) &&
                              !(K <= kRowsShortK && M >= 32 && small_k_rows());
    if (M <= 128 && !rows_disabled() && force <= 2 && !small_swiglu) {
        // decode-sized: many weight rows -> whole row tiles per CTA (no K split); otherwise
        // split-K partials summed by a second small kernel (not for argmax, which needs whole
        // rows); row tiles of 6-9 groups only when the partials do not apply
        const int sms = num_sms();
        int tiles = 0;
        // short K (a wide tensor-parallel rank's row-parallel projection): narrow row tiles over
        // the whole K in one launch beat split-K partials + reduce (two launches)
        const bool short_k = K <= kRowsShortK && small_k_rows();
        const int hs = plan_rows(N, sms, tiles, short_k ? 2 : 6);
        if ((hs >= 10 || (short_k && hs > 0)) && force != 2)
            return launch_rows<EPI>(x, w, y, amax, M, N, K, hs, tiles, sms, stream, id_off);
        if (EPI != EPI_ARGMAX && force != 1) {
            const int r = launch_part_reduce<EPI>(x, w, y, M, N, K, ws, ws_bytes, stream);
            if (r != -1) return r;
        }
        if (hs) return launch_rows<EPI>(x, w, y, amax, M, N, K, hs, tiles, sms, stream, id_off);
    }
    const int bn = pick_bn(M);
    const int64_t tiles = static_cast<int64_t>((M + bn - 1) / bn) * ((N + kBM - 1) / kBM);
    CUtensorMap tw, tx;
    int rc = make_tmap_2d_bf16(&tw, w, K, N, static_cast<uint64_t>(K) * 2, kBK, kBM, true);
    if (rc) return rc;
    rc = make_tmap_2d_bf16(&tx, x, K, M, static_cast<uint64_t>(K) * 2, kBK, bn, true);
    if (rc) return rc;
    if (bn <= 128 && force != 4) {  // one token tile: cluster split-K when it balances well (no workspace)
        int r;
        switch (bn) {
            case 16: r = launch_cl<16, EPI>(tw, tx, y, amax, M, N, K, stream, id_off); break;
            case 32: r = launch_cl<32, EPI>(tw, tx, y, amax, M, N, K, stream, id_off); break;
            case 64: r = launch_cl<64, EPI>(tw, tx, y, amax, M, N, K, stream, id_off); break;
            default: r = launch_cl<128, EPI>(tw, tx, y, amax, M, N, K, stream, id_off); break;
        }
        if (r != -1) return r;
        if (small_swiglu) {  // the cluster plan did not balance: partials + reduce after all
            r = launch_part_reduce<EPI>(x, w, y, M, N, K, ws, ws_bytes, stream);
            if (r != -1) return r;
        }
    }
    if (tiles <= static_cast<int64_t>(kCounterBytes / sizeof(int))) {
        const int sms = num_sms();
        if (!ws || ws_bytes < sk_workspace_bytes(bn, sms))
            return set_error(MSGL_ERR_WORKSPACE, "gemm: workspace too small");
        if (reinterpret_cast<uintptr_t>(ws) & 15)
            return set_error(MSGL_ERR_INVALID_ARG, "gemm: workspace must be 16-byte aligned");
        switch (bn) {
            case 16: return launch_sk<16, EPI>(tw, tx, y, amax, M, N, K, ws, sms, stream, id_off);
            case 32: return launch_sk<32, EPI>(tw, tx, y, amax, M, N, K, ws, sms, stream, id_off);
            case 64: return launch_sk<64, EPI>(tw, tx, y, amax, M, N, K, ws, sms, stream, id_off);
            case 128: return launch_sk<128, EPI>(tw, tx, y, amax, M, N, K, ws, sms, stream, id_off);
            default: return launch_sk<256, EPI>(tw, tx, y, amax, M, N, K, ws, sms, stream, id_off);
        }
    }
    // very large grids: one CTA per tile, no K split, no workspace
    GemmPlan p = plan_gemm(M, N, K);
    p.splits = 1;
    p.kb_per_split = (K + kBK - 1) / kBK;
    switch (p.bn) {
        case 16: return launch_bn<16, EPI>(p, tw, tx, y, amax, M, N, K, ws, stream, GroupArgs{}, id_off);
        case 32: return launch_bn<32, EPI>(p, tw, tx, y, amax, M, N, K, ws, stream, GroupArgs{}, id_off);
        case 64: return launch_bn<64, EPI>(p, tw, tx, y, amax, M, N, K, ws, stream, GroupArgs{}, id_off);
        case 128: return launch_bn<128, EPI>(p, tw, tx, y, amax, M, N, K, ws, stream, GroupArgs{}, id_off);
        default: return launch_bn<256, EPI>(p, tw, tx, y, amax, M, N, K, ws, stream, GroupArgs{}, id_off);
    }
}

// One thread per expert: the expert's row tiles of height bn, as (expert, first row) pairs.
__global__ void group_tiles_kernel(const int* __restrict__ offsets, int E, int bn,
                                   int2* __restrict__ tiles, int* __restrict__ num_tiles) {
    // one thread per expert (the block is E rounded up to whole warps): its tile count, the
    // block's exclusive scan of the counts, then its tiles at that position
    __shared__ int sh[32];
    pdl_wait();
    pdl_trigger();
    const int e = threadIdx.x;
    int cnt = 0, beg = 0;
    if (e < E) {
        beg = offsets[e];
        cnt = (offsets[e + 1] - beg + bn - 1) / bn;
    }
    int total;
    const int first = block_excl_scan(cnt, sh, total);
    if (e == 0) {
        num_tiles[0] = total;
        num_tiles[1] = 0;  // the persistent grouped kernel's work counter
    }
    for (int i = 0; i < cnt; ++i) tiles[first + i] = make_int2(e, beg + i * bn);
}

// reuse_tiles: the workspace already holds the tile list of an earlier grouped call with the same
// offsets, max_rows and E (so the same bn); the tile kernel is skipped unless the persistent
// schedule runs, which needs the work counter that kernel zeroes.
template <int EPI>
int run_grouped(const void* x, const void* w, void* y, const int* offsets, int E, int N, int K,
                int max_rows, void* ws, size_t ws_bytes, cudaStream_t stream,
                bool reuse_tiles = false) {
    if (E <= 0 || E > 1024 || N <= 0 || K <= 0 || max_rows < 0)
        return set_error(MSGL_ERR_INVALID_ARG, "grouped gemm: bad sizes");
    if (K % 8) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "grouped gemm: K % 8");
    if (max_rows == 0) return MSGL_OK;
    const int avg = (max_rows + E - 1) / E;
    const int bn = pick_bn(avg);
    const int max_tiles = (max_rows + bn - 1) / bn + E;
    const size_t need = static_cast<size_t>(max_tiles) * sizeof(int2) + 256;
    if (!ws || ws_bytes < need) return set_error(MSGL_ERR_WORKSPACE, "grouped gemm: workspace too small");
    if (max_tiles > 65535 * 8) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "grouped gemm: too many tiles");
    int* num_tiles = static_cast<int*>(ws);
    int2* tiles = reinterpret_cast<int2*>(static_cast<uint8_t*>(ws) + 256);
    const bool persistent = grouped_persistent(bn, EPI == EPI_SWIGLU);
    if (!reuse_tiles || persistent) {
        launch_pdl(group_tiles_kernel, dim3(1), dim3((E + 31) & ~31), 0, stream, offsets, E, bn, tiles,
                   num_tiles);
        MSGL_LAUNCH_CHECK();
    }
    CUtensorMap tw, tx;
    int rc = make_tmap_2d_bf16(&tw, w, K, static_cast<uint64_t>(E) * N, static_cast<uint64_t>(K) * 2,
                               kBK, kBM, true);
    if (rc) return rc;
    rc = make_tmap_2d_bf16(&tx, x, K, max_rows, static_cast<uint64_t>(K) * 2, kBK, bn, true);
    if (rc) return rc;
    GemmPlan p{};
    p.bn = bn;
    p.m_tiles = max_tiles;
    p.n_tiles = (N + kBM - 1) / kBM;
    p.splits = 1;
    p.kb_per_split = (K + kBK - 1) / kBK;
    GroupArgs g{tiles, num_tiles, offsets};
    if (persistent) {
        const int64_t max_items = static_cast<int64_t>(max_tiles) * p.n_tiles;
        switch (bn) {
            case 16: return launch_grouped_dyn<16, EPI>(tw, tx, y, N, K, g, num_tiles + 1, max_items, stream);
            case 32: return launch_grouped_dyn<32, EPI>(tw, tx, y, N, K, g, num_tiles + 1, max_items, stream);
            case 64: return launch_grouped_dyn<64, EPI>(tw, tx, y, N, K, g, num_tiles + 1, max_items, stream);
            case 128: return launch_grouped_dyn<128, EPI>(tw, tx, y, N, K, g, num_tiles + 1, max_items, stream);
            default: return launch_grouped_dyn<256, EPI>(tw, tx, y, N, K, g, num_tiles + 1, max_items, stream);
        }
    }
    switch (bn) {
        case 16: return launch_bn<16, EPI, true>(p, tw, tx, y, nullptr, max_rows, N, K, nullptr, stream, g);
        case 32: return launch_bn<32, EPI, true>(p, tw, tx, y, nullptr, max_rows, N, K, nullptr, stream, g);
        case 64: return launch_bn<64, EPI, true>(p, tw, tx, y, nullptr, max_rows, N, K, nullptr, stream, g);
        case 128: return launch_bn<128, EPI, true>(p, tw, tx, y, nullptr, max_rows, N, K, nullptr, stream, g);
        default: return launch_bn<256, EPI, true>(p, tw, tx, y, nullptr, max_rows, N, K, nullptr, stream, g);
    }
}

__global__ void pack_gate_up_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                    int inter, int row_vecs) {
    const int r = blockIdx.x;  // packed row: groups of 16 = 8 gate rows, then the 8 up rows
    const int grp = r >> 4, within = r & 15;
    const int srow = within < 8 ? grp * 8 + within : inter + grp * 8 + within - 8;
    for (int v = threadIdx.x; v < row_vecs; v += blockDim.x)
        dst[static_cast<int64_t>(r) * row_vecs + v] = src[static_cast<int64_t>(srow) * row_vecs + v];
}

__global__ void unpack_argmax_kernel(unsigned long long* __restrict__ packed, int* __restrict__ ids,
                                     int M) {
    pdl_wait();
    pdl_trigger();
    int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m < M) ids[m] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(packed[m] & 0xFFFFFFFFull));
}

template <typename T>
__global__ void argmax_rows_kernel(const T* __restrict__ logits, int vocab, int* __restrict__ out) {
    __shared__ unsigned long long red[8];
    pdl_wait();
    pdl_trigger();
    const T* r = logits + static_cast<int64_t>(blockIdx.x) * vocab;
    unsigned long long best = 0ull;
    for (int v = threadIdx.x; v < vocab; v += blockDim.x) {
        float x;
        if constexpr (sizeof(T) == 4) x = r[v];
        else x = __bfloat162float(r[v]);
        unsigned long long k = argmax_key(x, v);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
        best = red[0] > best ? red[0] : best;
        out[blockIdx.x] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
    }
}

}  // namespace
}  // namespace msgl

using namespace msgl;

extern "C" {

size_t msgl_gemm_workspace_size(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    const int bn = pick_bn(M);
    const int64_t tiles = static_cast<int64_t>((M + bn - 1) / bn) * ((N + kBM - 1) / kBM);
    if (tiles > static_cast<int64_t>(kCounterBytes / sizeof(int))) return 0;
    int sms = 148;
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
        sms = v;
    else
        cudaGetLastError();  // no device (host-only query): size for a 148-SM B200
    return std::max(sk_workspace_bytes(bn, sms), part_reduce_bytes(M, N, K));
}

int msgl_gemm_bf16(const void* x, const void* w, void* y, int M, int N, int K, int out_dtype,
                   void* workspace, size_t workspace_bytes, msgl_stream_t stream) {
    if (out_dtype == MSGL_BF16)
        return run_gemm<EPI_BF16>(x, w, y, nullptr, M, N, K, workspace, workspace_bytes, stream);
    if (out_dtype == MSGL_F32)
        return run_gemm<EPI_F32>(x, w, y, nullptr, M, N, K, workspace, workspace_bytes, stream);
    return set_error(MSGL_ERR_INVALID_ARG, "gemm: unknown out_dtype");
}

int msgl_pack_gate_up(const void* w_gate_up, void* w_packed, int inter, int hidden,
                      msgl_stream_t stream) {
    if (inter <= 0 || inter % 16 || hidden <= 0 || hidden % 8)
        return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "pack_gate_up: inter % 16, hidden % 8");
    if (w_gate_up == w_packed) return set_error(MSGL_ERR_INVALID_ARG, "pack_gate_up: in place");
    pack_gate_up_kernel<<<2 * inter, 128, 0, stream>>>(static_cast<const uint4*>(w_gate_up),
                                                       static_cast<uint4*>(w_packed), inter,
                                                       hidden / 8);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

int msgl_gemm_gate_up_silu(const void* x, const void* w_packed, void* y, int M, int inter, int K,
                           void* workspace, size_t workspace_bytes, msgl_stream_t stream) {
    if (inter <= 0 || inter % 16) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "gate_up: inter % 16");
    return run_gemm<EPI_SWIGLU>(x, w_packed, y, nullptr, M, 2 * inter, K, workspace,
                                workspace_bytes, stream);
}

int msgl_gemm_partials_splits(int M, int N, int K) {
    if (M <= 0 || M > 256 || N <= 0 || K <= 0) return 0;
    return part_splits(M, N, K);
}

int msgl_gemm_bf16_partials(const void* x, const void* w, float* parts, int M, int N, int K,
                            int splits, msgl_stream_t stream) {
    if (M < 0 || N <= 0 || K <= 0 || !x || !w || !parts)
        return set_error(MSGL_ERR_INVALID_ARG, "gemm_partials: bad arguments");
    if (M > 256) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "gemm_partials: M must be <= 256");
    if (K % 8) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "gemm_partials: K must be a multiple of 8");
    const int KB = (K + kBK - 1) / kBK;
    if (splits < 1 || splits > KB || splits > 64)
        return set_error(MSGL_ERR_INVALID_ARG, "gemm_partials: splits must be in [1, min(64, K / 64)]");
    if (M == 0) return MSGL_OK;
    CUtensorMap tw;
    int rc = make_tmap_2d_bf16(&tw, w, K, N, static_cast<uint64_t>(K) * 2, kBK, kPartBN, true);
    if (rc) return rc;
    return launch_part(x, tw, parts, M, N, K, splits, stream);
}

size_t msgl_grouped_gemm_workspace_size(int max_rows, int num_experts) {
    if (max_rows < 0 || num_experts <= 0) return 0;
    const int bn = pick_bn((max_rows + num_experts - 1) / num_experts);
    return static_cast<size_t>((max_rows + bn - 1) / bn + num_experts) * sizeof(int2) + 256;
}

int msgl_grouped_gemm_bf16(const void* x_sorted, const void* w, void* y,
                           const int* expert_offsets, int num_experts, int N, int K, int max_rows,
                           void* workspace, size_t workspace_bytes, msgl_stream_t stream) {
    return run_grouped<EPI_BF16>(x_sorted, w, y, expert_offsets, num_experts, N, K, max_rows,
                                 workspace, workspace_bytes, stream);
}

int msgl_grouped_gemm_bf16_reuse_tiles(const void* x_sorted, const void* w, void* y,
                                       const int* expert_offsets, int num_experts, int N, int K,
                                       int max_rows, void* workspace, size_t workspace_bytes,
                                       msgl_stream_t stream) {
    return run_grouped<EPI_BF16>(x_sorted, w, y, expert_offsets, num_experts, N, K, max_rows,
                                 workspace, workspace_bytes, stream, true);
}

int msgl_grouped_gemm_gate_up_silu(const void* x_sorted, const void* w_packed, void* y,
                                   const int* expert_offsets, int num_experts, int inter, int K,
                                   int max_rows, void* workspace, size_t workspace_bytes,
                                   msgl_stream_t stream) {
    if (inter <= 0 || inter % 16) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "grouped gate_up: inter % 16");
    return run_grouped<EPI_SWIGLU>(x_sorted, w_packed, y, expert_offsets, num_experts, 2 * inter,
                                   K, max_rows, workspace, workspace_bytes, stream);
}

int msgl_lm_head_argmax(const void* x, const void* w, int M, int vocab, int K,
                        unsigned long long* packed, int* ids, void* workspace,
                        size_t workspace_bytes, msgl_stream_t stream) {
    if (M <= 0) return M == 0 ? MSGL_OK : set_error(MSGL_ERR_INVALID_ARG, "lm_head: M < 0");
    if (cudaMemsetAsync(packed, 0, static_cast<size_t>(M) * sizeof(unsigned long long), stream) !=
        cudaSuccess)
        return set_error(MSGL_ERR_CUDA, "lm_head: memset failed");
    int rc = run_gemm<EPI_ARGMAX>(x, w, nullptr, packed, M, vocab, K, workspace, workspace_bytes,
                                  stream);
    if (rc) return rc;
    launch_pdl(unpack_argmax_kernel, dim3((M + 255) / 256), dim3(256), 0, stream, packed, ids, M);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

int msgl_lm_head_argmax_partial(const void* x, const void* w, int M, int vocab_local, int K,
                                int vocab_offset, unsigned long long* packed, void* workspace,
                                size_t workspace_bytes, msgl_stream_t stream) {
    if (M <= 0) return M == 0 ? MSGL_OK : set_error(MSGL_ERR_INVALID_ARG, "lm_head: M < 0");
    if (vocab_offset < 0) return set_error(MSGL_ERR_INVALID_ARG, "lm_head: vocab_offset < 0");
    if (cudaMemsetAsync(packed, 0, static_cast<size_t>(M) * sizeof(unsigned long long), stream) !=
        cudaSuccess)
        return set_error(MSGL_ERR_CUDA, "lm_head: memset failed");
    return run_gemm<EPI_ARGMAX>(x, w, nullptr, packed, M, vocab_local, K, workspace,
                                workspace_bytes, stream, vocab_offset);
}

int msgl_argmax(const void* logits, int num_rows, int vocab, int dtype, int* out,
                msgl_stream_t stream) {
    if (num_rows < 0 || vocab <= 0) return set_error(MSGL_ERR_INVALID_ARG, "argmax: bad sizes");
    if (num_rows == 0) return MSGL_OK;
    if (dtype == MSGL_F32)
        launch_pdl(argmax_rows_kernel<float>, dim3(num_rows), dim3(256), 0, stream,
                   static_cast<const float*>(logits), vocab, out);
    else if (dtype == MSGL_BF16)
        launch_pdl(argmax_rows_kernel<__nv_bfloat16>, dim3(num_rows), dim3(256), 0, stream,
                   static_cast<const __nv_bfloat16*>(logits), vocab, out);
    else
        return set_error(MSGL_ERR_INVALID_ARG, "argmax: unknown dtype");
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

}  // extern "C"
