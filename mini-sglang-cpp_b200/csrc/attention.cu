// attention.cu -- paged-KV decode and extend attention over the page pool.
//
// Replaces Attention::forward (src/layer/layer.cpp:214-262). Same math -- scale 1/sqrt(D),
// softmax with max subtraction, fp32 accumulation -- evaluated online (flash style) per request
// over the paged pool [num_slots, Hkv * 128] (slot = page * 16 + offset, the layout of
// kernels/cuda/radix.cu:19-22), with GQA (query head h reads kv head h / (Hq / Hkv)).
//
// Data movement: a producer warp walks the request's page-table row and stages pages of K and
// V into shared memory with TMA loads (SWIZZLE_128B, no multicast) on an mbarrier ring; four
// consumer warps compute S = Q K^T and O += P V with warp-level bf16 MMA (m16n8k16, fp32
// accumulate; fragments read with ldmatrix from the swizzled tiles, conflict-free) and a
// warp-shuffle online softmax. The query group of one kv head (Hq / Hkv <= 8 heads) fills the MMA
// rows. Decode: one 3-D TMA per pool brings a whole page of up to four kv heads (16 KB) -- TMA
// throughput per CTA is set by the number of boxes in flight, not their size -- and the pages of
// a request are split over `chunks` CTAs (split-KV) whose partial (m, l, O) the last CTA to
// finish merges (a self-resetting arrival counter). Extend: one CTA per (query tile, kv head),
// one page (2-D TMA, 4 x 2 KB) per stage.
//
// Bound: HBM. Per (request, kv head, token) the kernel reads 512 B of K/V; the tensor work per
// byte is ~4 FLOP, far below the MMA rate.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "tmap.h"

namespace msgl {
namespace {

constexpr int kPage = 16;
constexpr int kHd = 128;
constexpr int kPageSlotBytes = 4 * 2048;  // K lo, K hi, V lo, V hi halves of one page
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kExtendStages = 8;          // x 1 page per stage
constexpr int kMaxChunkPages = 512;       // decode split-KV chunk bound (page ids in smem)
constexpr int kExtendPageBatch = 1024;    // extend: page ids staged per batch
constexpr float kNegInf = -__builtin_huge_valf();

__device__ __forceinline__ void named_bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// One page (16 tokens) for one warp: S = Q K^T (2 x 8 MMAs), masked online softmax, O += P V
// (16 MMAs). Rows g (lane >> 2) and g + 8 of the MMA tile are query rows; TWO selects whether
// rows g + 8 carry data. lim0 / lim1: last kv token index visible to row g / g + 8.
template <bool TWO>
__device__ __forceinline__ void attend_page(uint32_t k_base, uint32_t v_base,
                                            const uint32_t (&qa)[8][4], float (&o)[16][4],
                                            float (&m)[2], float (&l)[2], int tok0, int lim0,
                                            int lim1, float sl2e, int lane) {
    float s[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[n][e] = 0.f;

    const int mi = lane >> 3;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
        const int row = ((mi >> 1) << 3) + (lane & 7);
        const int chunk = ((kk & 3) << 1) + (mi & 1);
        uint32_t addr = k_base + ((kk >> 2) << 11) + row * 128 + ((chunk ^ (row & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(addr, b0, b1, b2, b3);
        mma_bf16_16816(s[0], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
        mma_bf16_16816(s[1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
    }

    const int c = lane & 3;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            int tk = tok0 + n * 8 + 2 * c + e;
            s[n][e] = tk <= lim0 ? s[n][e] * sl2e : kNegInf;
            if (TWO) s[n][2 + e] = tk <= lim1 ? s[n][2 + e] * sl2e : kNegInf;
        }

    float p[2][4];
#pragma unroll
    for (int r = 0; r < (TWO ? 2 : 1); ++r) {
        float mx = fmaxf(fmaxf(s[0][2 * r], s[0][2 * r + 1]), fmaxf(s[1][2 * r], s[1][2 * r + 1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        float m_new = fmaxf(m[r], mx);
        float alpha = 1.f, base = 0.f;
        if (m_new != kNegInf) {
            alpha = exp2f(m[r] - m_new);
            base = m_new;
        }
        float ps = 0.f;
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float v = exp2f(s[n][2 * r + e] - base);
                p[n][2 * r + e] = v;
                ps += v;
            }
        l[r] = l[r] * alpha + ps;
        m[r] = m_new;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            o[j][2 * r] *= alpha;
            o[j][2 * r + 1] *= alpha;
        }
    }
    const uint32_t pa0 = pack_bf16x2(p[0][0], p[0][1]);
    const uint32_t pa2 = pack_bf16x2(p[1][0], p[1][1]);
    const uint32_t pa1 = TWO ? pack_bf16x2(p[0][2], p[0][3]) : 0u;
    const uint32_t pa3 = TWO ? pack_bf16x2(p[1][2], p[1][3]) : 0u;

#pragma unroll
    for (int j2 = 0; j2 < 8; ++j2) {
        const int row = ((mi & 1) << 3) + (lane & 7);
        const int chunk = ((j2 & 3) << 1) + (mi >> 1);
        uint32_t addr = v_base + ((j2 >> 2) << 11) + row * 128 + ((chunk ^ (row & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(addr, b0, b1, b2, b3);
        mma_bf16_16816(o[2 * j2], pa0, pa1, pa2, pa3, b0, b1);
        mma_bf16_16816(o[2 * j2 + 1], pa0, pa1, pa2, pa3, b2, b3);
    }
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void issue_page(uint8_t* dst, const CUtensorMap* tk,
                                           const CUtensorMap* tv, uint64_t* bar, int kvh, int page) {
    const int x = kvh * kHd, y = page * kPage;
    tma_load_2d(dst, tk, bar, x, y);
    tma_load_2d(dst + 2048, tk, bar, x + 64, y);
    tma_load_2d(dst + 4096, tv, bar, x, y);
    tma_load_2d(dst + 6144, tv, bar, x + 64, y);
}

__device__ __forceinline__ void store_bf16x8(__nv_bfloat16* dst, const float (&v)[8]) {
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(dst) = u;
}

// ------------------------------------------------------------------------------ decode
// grid (max_chunks, Hkv / hc, B); block 160 = 4 consumer warps + 1 TMA producer warp. One CTA
// covers a chunk of one request's pages for a group of hc = min(Hkv, 4) kv heads. A page of the
// group is ONE 3-D TMA box per pool -- {64 dims, 16 token rows, 2 hc head halves}, token rows
// 2 * Hkv * 128 B apart, head halves 128 B apart -- landing head-major ([hh][token][64], the
// same 2 KB swizzled tiles the MMA fragments read), so the ring moves 16 KB per TMA instead of
// 2 KB. A stage holds pps = 4 / hc pages; warp w attends local kv head w % hc on page w / hc.
constexpr int kDecWarps = 4;
constexpr int kDecThreads = (kDecWarps + 1) * 32;
constexpr int kDecHeads = 4;                                 // kv heads per CTA (max)
constexpr int kDecHalfStage = kDecHeads * 2 * 2048;          // 16 KB of K (or of V) per stage
constexpr int kDecStageBytes = 2 * kDecHalfStage;            // 32 KB: K then V
constexpr int kDecStages = 3;                                // 96 KB ring: 2 CTAs per SM

// Merge of split-KV partials by the 128 consumer threads of the last CTA to arrive: for each
// (query head, 8-wide slice) item, O = sum_k exp2(m_k - M) O_k / sum_k exp2(m_k - M) l_k over the
// `total` chunks k in order (M = max_k m_k; a chunk with m = -inf adds nothing). Partial k of
// query head qh sits at index chunk_of(k) * hq + qh of ws_ml (pairs m, l) / ws_o (rows of 128).
// Each thread takes two items at a time and issues a batch's loads (8 maxima, then 4 chunks of
// l and O) before using any of them, so a merge costs a few L2 round trips, not one per chunk
// and item; the sums keep the chunk order (same bits as a chunk-by-chunk loop).
template <class ChunkBase>
__device__ __forceinline__ void merge_partials(int total, int nq, int qh0, int hq,
                                               ChunkBase chunk_base, const float* ws_o,
                                               const float* ws_ml, __nv_bfloat16* out_row0) {
    constexpr int kT = kDecWarps * 32;
    const int nitems = nq * 16;
    for (int base = threadIdx.x; base < nitems; base += 2 * kT) {
        const int it[2] = {base, base + kT};
        const bool live[2] = {it[0] < nitems, it[1] < nitems};
        int64_t qoff[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) qoff[u] = qh0 + (live[u] ? (it[u] >> 4) : 0);
        float M[2] = {kNegInf, kNegInf};
        for (int k0 = 0; k0 < total; k0 += 8) {
            float mv[2][8];
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    mv[u][j] = (live[u] && k0 + j < total)
                                   ? __ldcg(ws_ml + (chunk_base(k0 + j) * hq + qoff[u]) * 2)
                                   : kNegInf;
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int j = 0; j < 8; ++j) M[u] = fmaxf(M[u], mv[u][j]);
        }
        float O[2][8], Ls[2] = {0.f, 0.f};
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int e = 0; e < 8; ++e) O[u][e] = 0.f;
        for (int k0 = 0; k0 < total; k0 += 4) {
            float mc[2][4], lc[2][4];
            float4 x0[2][4], x1[2][4];
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const bool ok = live[u] && k0 + j < total;
                    const int64_t pi = ok ? chunk_base(k0 + j) * hq + qoff[u] : 0;
                    const int d0 = (it[u] & 15) * 8;
                    mc[u][j] = ok ? __ldcg(ws_ml + pi * 2) : kNegInf;
                    lc[u][j] = ok ? __ldcg(ws_ml + pi * 2 + 1) : 0.f;
                    const float4* src = reinterpret_cast<const float4*>(ws_o + pi * kHd + d0);
                    x0[u][j] = ok ? __ldcg(src) : make_float4(0.f, 0.f, 0.f, 0.f);
                    x1[u][j] = ok ? __ldcg(src + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (!(live[u] && k0 + j < total)) continue;
                    const float sc = (mc[u][j] == kNegInf) ? 0.f : exp2f(mc[u][j] - M[u]);
                    Ls[u] += lc[u][j] * sc;
                    O[u][0] += x0[u][j].x * sc; O[u][1] += x0[u][j].y * sc;
                    O[u][2] += x0[u][j].z * sc; O[u][3] += x0[u][j].w * sc;
                    O[u][4] += x1[u][j].x * sc; O[u][5] += x1[u][j].y * sc;
                    O[u][6] += x1[u][j].z * sc; O[u][7] += x1[u][j].w * sc;
                }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (!live[u]) continue;
            const float inv = Ls[u] > 0.f ? 1.f / Ls[u] : 0.f;
            float r[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) r[e] = O[u][e] * inv;
            store_bf16x8(out_row0 + qoff[u] * kHd + (it[u] & 15) * 8, r);
        }
    }
}


__global__ void __launch_bounds__(kDecThreads, 2)
paged_decode_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                    const __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ out,
                    const int* __restrict__ page_table, int max_pages,
                    const int* __restrict__ seq_lens, int pool_pages, int hq, int hkv, int hc,
                    int chunk_pages, int max_chunks, float sl2e, float* __restrict__ ws_o,
                    float* __restrict__ ws_ml, int* __restrict__ ws_cnt, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDecStages * kDecStageBytes);
    uint64_t* empty = full + kDecStages;
    int* flag = reinterpret_cast<int*>(empty + kDecStages);
    int* pages = flag + 4;  // [chunk_pages <= kMaxChunkPages]

    const int b = blockIdx.z, hg = blockIdx.y, chunk = blockIdx.x;
    const int group = hq / hkv;
    const int pps = kDecWarps / hc;   // pages per stage
    const int nq = hc * group;        // query heads of this CTA
    const int qh0 = hg * nq;          // first of them
    // prologue overlapping the previous kernel: barriers only (the page table and context
    // lengths are step inputs, but they may be written by a preceding kernel of the caller)
    if (threadIdx.x == 0) {
        for (int s = 0; s < kDecStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kDecWarps);
        }
        fence_barrier_init();
    }
    pdl_wait();
    pdl_trigger();
    int L = seq_lens[b];
    if (L < 0 || L > max_pages * kPage) {  // context longer than the page-table row
        if (threadIdx.x == 0 && chunk == 0 && hg == 0) record_error(err, MSGL_ERR_BOUNDS, 202);
        L = L < 0 ? 0 : max_pages * kPage;
    }
    const int npages = (L + kPage - 1) / kPage;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (npages == 0) {  // empty context: output zeros (chunk 0 only)
        if (chunk == 0)
            for (int i = threadIdx.x; i < nq * 16; i += blockDim.x) {
                float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                store_bf16x8(out + (static_cast<int64_t>(b) * hq + qh0 + (i >> 4)) * kHd + (i & 15) * 8, z);
            }
        return;
    }
    const int p0 = chunk * chunk_pages;
    if (p0 >= npages) return;
    const int np = min(npages - p0, chunk_pages);
    const int nchunks = (npages + chunk_pages - 1) / chunk_pages;
    const int nsteps = (np + pps - 1) / pps;
    __syncthreads();

    if (warp == kDecWarps) {
        // ---------------- TMA producer: page ids staged in shared memory first
        const int* pt = page_table + static_cast<int64_t>(b) * max_pages + p0;
        for (int i = lane; i < np; i += 32) {
            int page = pt[i];
            if (static_cast<unsigned>(page) >= static_cast<unsigned>(pool_pages)) {
                record_error(err, MSGL_ERR_BOUNDS, 201);
                page = 0;
            }
            pages[i] = page;
        }
        __syncwarp();
        if (lane == 0) {
            tma_prefetch_desc(&tk);
            tma_prefetch_desc(&tv);
            const int page_half = hc * 4096;  // K (or V) bytes of one page of the head group
            for (int it = 0; it < nsteps; ++it) {
                const int s = it % kDecStages;
                if (it >= kDecStages && !mbar_wait(&empty[s], ((it / kDecStages) - 1) & 1, err, 200))
                    break;
                const int cnt = min(pps, np - it * pps);
                mbar_arrive_expect_tx(&full[s], cnt * 2 * page_half);
                uint8_t* st = smem + s * kDecStageBytes;
                for (int p = 0; p < cnt; ++p) {
                    const int y = pages[it * pps + p] * kPage;
                    tma_load_3d(st + p * page_half, &tk, &full[s], 0, y, 2 * hc * hg);
                    tma_load_3d(st + kDecHalfStage + p * page_half, &tv, &full[s], 0, y, 2 * hc * hg);
                }
            }
        }
        return;
    }

    // ---------------- consumers: local kv head `head`, page `psub` of every stage
    const int head = warp % hc, psub = warp / hc;
    const int g = lane >> 2, c = lane & 3;
    uint32_t qa[8][4];
    {
        const bool real = g < group;
        const __nv_bfloat16* qr =
            q + (static_cast<int64_t>(b) * hq + qh0 + head * group + (real ? g : 0)) * kHd;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            qa[kk][0] = real ? *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 2 * c) : 0u;
            qa[kk][2] = real ? *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 8 + 2 * c) : 0u;
            qa[kk][1] = 0u;
            qa[kk][3] = 0u;
        }
    }
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m[2] = {kNegInf, kNegInf}, l[2] = {0.f, 0.f};

    const uint32_t my_off = (psub * hc + head) * 4096;
    for (int it = 0; it < nsteps; ++it) {
        const int s = it % kDecStages;
        if (!mbar_wait(&full[s], (it / kDecStages) & 1, err, 210)) break;
        const int pidx = it * pps + psub;
        if (pidx < np) {
            const uint32_t base = smem_u32(smem + s * kDecStageBytes) + my_off;
            attend_page<false>(base, base + kDecHalfStage, qa, o, m, l, (p0 + pidx) * kPage, L - 1,
                               -1, sl2e, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---------------- combine the pps warps of each head (shared memory over the drained ring)
    float lsum = l[0];
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
    named_bar_sync(1, kDecWarps * 32);
    float* mo = reinterpret_cast<float*>(smem);      // [4 warps][8 rows][128]
    float* mm = mo + kDecWarps * 8 * kHd;             // [4][8]
    float* ml = mm + kDecWarps * 8;                   // [4][8]
    if (g < group) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            mo[(warp * 8 + g) * kHd + 8 * j + 2 * c] = o[j][0];
            mo[(warp * 8 + g) * kHd + 8 * j + 2 * c + 1] = o[j][1];
        }
        if (c == 0) {
            mm[warp * 8 + g] = m[0];
            ml[warp * 8 + g] = lsum;
        }
    }
    named_bar_sync(1, kDecWarps * 32);

    // items: (local query head, 8-wide d chunk) over the 128 consumer threads
    for (int item = threadIdx.x; item < nq * 16; item += kDecWarps * 32) {
        const int lq = item >> 4, d0 = (item & 15) * 8;
        const int h = lq / group, r = lq % group;
        const int qh = qh0 + lq;
        float M = kNegInf;
        for (int ps = 0; ps < pps; ++ps) M = fmaxf(M, mm[(ps * hc + h) * 8 + r]);
        float O[8] = {0, 0, 0, 0, 0, 0, 0, 0}, Ls = 0.f;
        for (int ps = 0; ps < pps; ++ps) {
            const int w = ps * hc + h;
            const float mw = mm[w * 8 + r];
            const float sc = (mw == kNegInf) ? 0.f : exp2f(mw - M);
            Ls += ml[w * 8 + r] * sc;
#pragma unroll
            for (int e = 0; e < 8; ++e) O[e] += mo[(w * 8 + r) * kHd + d0 + e] * sc;
        }
        if (nchunks == 1) {
            const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) O[e] *= inv;
            store_bf16x8(out + (static_cast<int64_t>(b) * hq + qh) * kHd + d0, O);
        } else {
            const int64_t pi = (static_cast<int64_t>(b) * max_chunks + chunk) * hq + qh;
            float4* dst = reinterpret_cast<float4*>(ws_o + pi * kHd + d0);
            dst[0] = make_float4(O[0], O[1], O[2], O[3]);
            dst[1] = make_float4(O[4], O[5], O[6], O[7]);
            if ((item & 15) == 0) {
                ws_ml[pi * 2] = M;
                ws_ml[pi * 2 + 1] = Ls;
            }
        }
    }
    if (nchunks == 1) return;

    // ---------------- split-KV: the last chunk CTA of (request, head group) merges all chunks
    __threadfence();
    named_bar_sync(1, kDecWarps * 32);
    int* cnt = ws_cnt + static_cast<int64_t>(b) * gridDim.y + hg;
    if (threadIdx.x == 0) {
        const int old = atomicAdd(cnt, 1);
        *flag = (old == nchunks - 1);
    }
    named_bar_sync(1, kDecWarps * 32);
    if (!*flag) return;
    __threadfence();
    const int64_t cbase = static_cast<int64_t>(b) * max_chunks;
    merge_partials(nchunks, nq, qh0, hq, [cbase](int k) { return cbase + k; }, ws_o, ws_ml,
                   out + static_cast<int64_t>(b) * hq * kHd);
    if (threadIdx.x == 0) *cnt = 0;
}

// ------------------------------------------------------------------------------ extend
// grid (q tiles, Hkv, B); each warp owns 16 MMA rows = (16 / group) query tokens x group heads;
// all four warps walk the same pages 0..(last visible page of the tile).
__global__ void __launch_bounds__(kThreads)
paged_extend_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                    const __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ out,
                    const int* __restrict__ page_table, int max_pages,
                    const int* __restrict__ seq_lens, const int* __restrict__ q_indptr,
                    int pool_pages, int hq, int hkv, float sl2e, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kExtendStages * kPageSlotBytes);
    uint64_t* empty = full + kExtendStages;

    const int b = blockIdx.z, kvh = blockIdx.y;
    const int group = hq / hkv;
    const int tpw = 16 / group;  // query tokens per warp
    if (threadIdx.x == 0) {
        for (int s = 0; s < kExtendStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    pdl_wait();
    pdl_trigger();
    const int qbeg = q_indptr[b];
    const int nq = q_indptr[b + 1] - qbeg;
    const int tile0 = blockIdx.x * kConsumerWarps * tpw;
    if (tile0 >= nq) return;
    const int L = seq_lens[b];
    const int last_tok = min(nq, tile0 + kConsumerWarps * tpw) - 1;
    const int last_pos = L - nq + last_tok;  // visible kv tokens 0..last_pos
    if (last_pos < 0) return;
    int npages = last_pos / kPage + 1;
    if (npages > max_pages) {  // context longer than the page-table row
        if (threadIdx.x == 0) record_error(err, MSGL_ERR_BOUNDS, 222);
        npages = max_pages;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();

    if (warp == kConsumerWarps) {
        if (lane == 0) {
            tma_prefetch_desc(&tk);
            tma_prefetch_desc(&tv);
        }
        // Page ids staged in shared memory, kExtendPageBatch at a time (one coalesced warp load
        // per batch); lane 0 issues the TMA loads.
        int* pages = reinterpret_cast<int*>(empty + kExtendStages);
        const int* pt = page_table + static_cast<int64_t>(b) * max_pages;
        bool ok = true;
        for (int it = 0; it < npages && ok; ++it) {
            if (it % kExtendPageBatch == 0) {
                __syncwarp();
                const int n = min(kExtendPageBatch, npages - it);
                for (int i = lane; i < n; i += 32) {
                    int page = pt[it + i];
                    if (static_cast<unsigned>(page) >= static_cast<unsigned>(pool_pages)) {
                        record_error(err, MSGL_ERR_BOUNDS, 221);
                        page = 0;
                    }
                    pages[i] = page;
                }
                __syncwarp();
            }
            if (lane == 0) {
                const int s = it % kExtendStages;
                if (it >= kExtendStages &&
                    !mbar_wait(&empty[s], ((it / kExtendStages) - 1) & 1, err, 220)) {
                    ok = false;
                } else {
                    mbar_arrive_expect_tx(&full[s], kPageSlotBytes);
                    issue_page(smem + s * kPageSlotBytes, &tk, &tv, &full[s], kvh,
                               pages[it % kExtendPageBatch]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
        }
        return;
    }

    const int g = lane >> 2, c = lane & 3;
    // rows g and g + 8 of this warp: local token r / group, head r % group
    const int r0 = g, r1 = g + 8;
    const int i0 = tile0 + warp * tpw + r0 / group, i1 = tile0 + warp * tpw + r1 / group;
    const bool v0 = i0 < nq, v1 = i1 < nq;
    const int h0 = kvh * group + r0 % group, h1 = kvh * group + r1 % group;
    const int lim0 = v0 ? L - nq + i0 : -1, lim1 = v1 ? L - nq + i1 : -1;
    uint32_t qa[8][4];
    {
        const __nv_bfloat16* q0 = q + (static_cast<int64_t>(qbeg + (v0 ? i0 : 0)) * hq + h0) * kHd;
        const __nv_bfloat16* q1 = q + (static_cast<int64_t>(qbeg + (v1 ? i1 : 0)) * hq + h1) * kHd;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            qa[kk][0] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + 16 * kk + 2 * c) : 0u;
            qa[kk][2] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + 16 * kk + 8 + 2 * c) : 0u;
            qa[kk][1] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + 16 * kk + 2 * c) : 0u;
            qa[kk][3] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + 16 * kk + 8 + 2 * c) : 0u;
        }
    }
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m[2] = {kNegInf, kNegInf}, l[2] = {0.f, 0.f};
    // Last visible kv token of any row of this warp. Warp-uniform on purpose: attend_page is
    // made of warp-collective instructions (ldmatrix, mma.sync, full-mask shuffles), so the
    // whole warp must take the same branch even when only some of its rows are valid.
    const int warp_last = __reduce_max_sync(0xffffffffu, max(lim0, lim1));

    for (int it = 0; it < npages; ++it) {
        const int s = it % kExtendStages;
        if (!mbar_wait(&full[s], (it / kExtendStages) & 1, err, 230)) break;
        if (it * kPage <= warp_last) {
            uint32_t base = smem_u32(smem + s * kPageSlotBytes);
            attend_page<true>(base, base + 4096, qa, o, m, l, it * kPage, lim0, lim1, sl2e, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

#pragma unroll
    for (int r = 0; r < 2; ++r) {
        float ls = l[r];
        ls += __shfl_xor_sync(0xffffffffu, ls, 1);
        ls += __shfl_xor_sync(0xffffffffu, ls, 2);
        const bool valid = r == 0 ? v0 : v1;
        if (!valid) continue;
        const float inv = ls > 0.f ? 1.f / ls : 0.f;
        const int i = r == 0 ? i0 : i1;
        const int h = r == 0 ? h0 : h1;
        __nv_bfloat16* dst = out + (static_cast<int64_t>(qbeg + i) * hq + h) * kHd;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            *reinterpret_cast<uint32_t*>(dst + 8 * j + 2 * c) =
                pack_bf16x2(o[j][2 * r] * inv, o[j][2 * r + 1] * inv);
    }
}

// ------------------------------------------------------------------------------ extend, tcgen05
// Prefill / chunked-prefill attention on the 5th-generation tensor cores. One CTA per (128-row
// query tile, kv head, request); the rows are (128 / group) query tokens x the group's heads,
// token-major, so one UMMA of M = 128 covers every query head of the kv head. Keys go in blocks
// of 128 (8 pages):
//   warp 0   TMA producer: per block 8 pages x 2 dim halves of K into a 3-stage K ring and of V
//            into a 3-stage V ring (2-D boxes of 16 rows x 64 dims, SWIZZLE_128B): a block's tiles
//            are [128 keys][64] halves, the canonical K-major layout for S = Q K^T and MN-major
//            for O += P V. A K stage is released when its S MMA completes, a V stage when its
//            P V MMA completes, so the next block's K lands while the softmax still works;
//   warp 1   MMA issuer (one lane): S(j+1) = Q K^T into the other of two TMEM S buffers while
//            the softmax works on S(j), then O += P(j) V(j) into TMEM with P read from tensor
//            memory (bf16 pairs written over S(j)'s first 64 columns) and V as an MN-major B
//            operand; a K stage is released after its S MMA, a V stage and the S buffer after
//            the P V MMA;
//   warps 2-9 softmax / epilogue: a pair of warps per TMEM lane quarter (warp % 4), each thread of
//            the pair one query row and one half of the 128 keys (and of O's 128 columns): the
//            row's Q half into shared memory once; per block its 64 S columns into registers
//            (one TMEM load), the row max (the two halves meet through shared memory and a named
//            barrier per pair), p = exp2(s - m) as bf16 pairs into TMEM over its S buffer, its part
//            of the running sum,
//            and O *= exp2(m_old - m_new) on its 64 columns; at the end O / l to global.
// TMEM: S / P buffers at columns [0, 128) and [128, 256), O at [256, 384) (512 allocated).
// The online softmax is the reference's (layer.cpp:226-257: scale 1/sqrt(D), max subtraction,
// fp32 accumulation) evaluated per block; causal masking by position L - q_len + i.
constexpr int kTcRows = 128;
constexpr int kTcKeys = 128;
constexpr int kTcPages = kTcKeys / kPage;  // 8
constexpr int kTcHalf = kTcRows * 128;     // 16 KB: 128 rows x 64 bf16
constexpr int kTcTile = 2 * kTcHalf;       // 32 KB: 128 x 128 bf16
constexpr int kTcStages = 3;
constexpr int kTcThreads = 10 * 32;  // producer, MMA, 8 softmax warps
constexpr size_t kTcSmem = 1024 + (1 + 2 * kTcStages) * kTcTile + 256 + 1024;  // Q, K x 3, V x 3, barriers, max exchange

__global__ void __launch_bounds__(kTcThreads, 1)
paged_extend_tc_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                       const __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ out,
                       const int* __restrict__ page_table, int max_pages,
                       const int* __restrict__ seq_lens, const int* __restrict__ q_indptr,
                       int pool_pages, int hq, int hkv, float sl2e, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint8_t* sQ = smem;                                // [2 halves][128 rows][64], SW128
    uint8_t* sK = smem + kTcTile;                      // [kTcStages] tiles
    uint8_t* sV = sK + kTcStages * kTcTile;            // [kTcStages] tiles
    uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kTcStages * kTcTile);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;                     // [kTcStages]
    uint64_t* k_empty = k_full + kTcStages;          // [kTcStages]
    uint64_t* v_full = k_empty + kTcStages;          // [kTcStages]
    uint64_t* v_empty = v_full + kTcStages;          // [kTcStages]
    // one barrier per block parity for every hand-off, so that no waiter can find its barrier
    // two phases ahead of the phase it waits for
    uint64_t* s_full = v_empty + kTcStages;          // [2]
    uint64_t* s_free = s_full + 2;                   // [2]
    uint64_t* p_full = s_free + 2;                   // [2]
    uint64_t* o_ready = p_full + 2;                  // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_ready + 2);
    float* red = reinterpret_cast<float*>(o_ready + 3);  // [2 halves][128 rows]

    const int b = blockIdx.z, kvh = blockIdx.y;
    const int group = hq / hkv;
    const int tpt = kTcRows / group;  // query tokens per tile
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(q_full, 8);
        for (int st = 0; st < kTcStages; ++st) {
            mbar_init(&k_full[st], 1);
            mbar_init(&k_empty[st], 1);
            mbar_init(&v_full[st], 1);
            mbar_init(&v_empty[st], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 1);
            mbar_init(&p_full[i], 8);
            mbar_init(&o_ready[i], 1);
        }
        fence_barrier_init();
    }
    pdl_wait();
    pdl_trigger();
    const int qbeg = q_indptr[b];
    const int nq = q_indptr[b + 1] - qbeg;
    const int tile0 = blockIdx.x * tpt;
    if (tile0 >= nq) return;
    const int L = seq_lens[b];
    const int last_pos = L - nq + min(nq, tile0 + tpt) - 1;  // last key any row of the tile sees
    if (last_pos < 0) {
        if (threadIdx.x == 0) record_error(err, MSGL_ERR_INVALID_ARG, 250);
        return;
    }
    int npages = (L + kPage - 1) / kPage;
    if (npages > max_pages) {  // context longer than the page-table row
        if (threadIdx.x == 0) record_error(err, MSGL_ERR_BOUNDS, 252);
        npages = max_pages;
    }
    const int nblk = min(last_pos / kTcKeys + 1, (npages + kTcPages - 1) / kTcPages);
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer
        const int* pt = page_table + static_cast<int64_t>(b) * max_pages;
        if (lane == 0) {
            tma_prefetch_desc(&tk);
            tma_prefetch_desc(&tv);
        }
        bool ok = true;
        int page_reg = 0;
        for (int j = 0; j < nblk; ++j) {
            if ((j & 3) == 0) {  // page ids of blocks j .. j + 3, one per lane
                const int pi = j * kTcPages + lane;
                int page = 0;  // past the request's pages: page 0, every key there is masked
                if (pi < npages) {
                    page = pt[pi];
                    if (static_cast<unsigned>(page) >= static_cast<unsigned>(pool_pages)) {
                        record_error(err, MSGL_ERR_BOUNDS, 251);
                        page = 0;
                    }
                }
                page_reg = page;
            }
            int pg[kTcPages];
#pragma unroll
            for (int p = 0; p < kTcPages; ++p) pg[p] = __shfl_sync(0xffffffffu, page_reg, (j & 3) * kTcPages + p);
            if (lane == 0) {
                const int st = j % kTcStages;
                const uint32_t par = ((j / kTcStages) - 1) & 1;
                if (j >= kTcStages && !mbar_wait(&k_empty[st], par, err, 253)) {
                    ok = false;
                } else {
                    mbar_arrive_expect_tx(&k_full[st], kTcTile);
                    uint8_t* kd = sK + st * kTcTile;
#pragma unroll
                    for (int p = 0; p < kTcPages; ++p)
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                            tma_load_2d(kd + h * kTcHalf + p * 2048, &tk, &k_full[st], kvh * kHd + h * 64, pg[p] * kPage);
                    if (j >= kTcStages && !mbar_wait(&v_empty[st], par, err, 253)) {
                        ok = false;
                    } else {
                        mbar_arrive_expect_tx(&v_full[st], kTcTile);
                        uint8_t* vd = sV + st * kTcTile;
#pragma unroll
                        for (int p = 0; p < kTcPages; ++p)
#pragma unroll
                            for (int h = 0; h < 2; ++h)
                                tma_load_2d(vd + h * kTcHalf + p * 2048, &tv, &v_full[st], kvh * kHd + h * 64, pg[p] * kPage);
                    }
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (one lane)
        if (lane == 0) {
            constexpr uint32_t idS = umma_idesc_bf16(kTcRows, kTcKeys);
            constexpr uint32_t idO = umma_idesc_bf16_bmn(kTcRows, kHd);
            const uint32_t tO = tmem + 256;
            const uint32_t aQ = smem_u32(sQ);
            // S(j) = Q K(j)^T into S buffer j % 2 (the caller checked that the buffer is free)
            auto issue_s = [&](int j) -> bool {
                const int st = j % kTcStages;
                if (!mbar_wait(&k_full[st], (j / kTcStages) & 1, err, 255)) return false;
                tc_fence_after();
                const uint32_t aK = smem_u32(sK + st * kTcTile);
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    umma_bf16(tmem + (j & 1) * 128, umma_desc_sw128(aQ + (k >> 2) * kTcHalf + (k & 3) * 32),
                              umma_desc_sw128(aK + (k >> 2) * kTcHalf + (k & 3) * 32), idS,
                              k > 0 ? 1u : 0u);
                umma_commit(&s_full[j & 1]);
                umma_commit(&k_empty[st]);
                return true;
            };
            bool ok = mbar_wait(q_full, 0, err, 254) && issue_s(0);
            for (int j = 0; ok && j < nblk; ++j) {
                if (j + 1 < nblk) {  // the next block's S, overlapping the softmax of this one
                    if (j + 1 >= 2 && !mbar_wait(&s_free[(j + 1) & 1], (((j + 1) >> 1) - 1) & 1, err, 256)) break;
                    if (!issue_s(j + 1)) break;
                }
                const int st = j % kTcStages;
                if (!mbar_wait(&v_full[st], (j / kTcStages) & 1, err, 255)) break;
                if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, err, 256)) break;
                tc_fence_after();
                const uint32_t aV = smem_u32(sV + st * kTcTile), tP = tmem + (j & 1) * 128;
#pragma unroll
                for (int k = 0; k < 8; ++k)  // 16 keys per UMMA: P from TMEM (8 columns), V MN-major
                    umma_bf16_ta(tO, tP + k * 8, umma_desc_sw128_mn(aV + k * 2048, kTcHalf, 1024), idO,
                                 (j > 0 || k > 0) ? 1u : 0u);
                umma_commit(&o_ready[j & 1]);
                umma_commit(&v_empty[st]);
                umma_commit(&s_free[j & 1]);  // P(j) read: its S buffer may take S(j + 2)
            }
        }
        __syncwarp();
    } else {
        // ---------------- softmax / epilogue: thread = (TMEM lane = query row, half of the keys)
        const int quarter = warp & 3;
        const int ch = (warp - 2) >> 2;  // key / O-column half of this warp
        const int r = quarter * 32 + lane;
        const int t = r / group, hl = r % group;
        const bool valid = tile0 + t < nq;
        const int qpos = L - nq + tile0 + t;  // the row sees keys 0 .. qpos
        const uint32_t row_t = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        const int pair_bar = 1 + quarter;    // named barrier of the two warps of this quarter
        {   // this half of the row's Q into the SW128 tile
            const uint4* src = reinterpret_cast<const uint4*>(
                q + (static_cast<int64_t>(qbeg + tile0 + (valid ? t : 0)) * hq + kvh * group + hl) * kHd + ch * 64);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint4 v = valid ? src[c] : make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(sQ + ch * kTcHalf + r * 128 + ((c ^ (r & 7)) << 4)) = v;
            }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_full);
        float m = kNegInf, l = 0.f;
        bool ok = true;
        // Every iteration runs the same two pair barriers on both warps of a pair: after a wait
        // that ran out (recorded in the error word) a warp skips the work and the waits but
        // keeps the barrier sequence, so the pair never meets at different barriers.
        for (int j = 0; j < nblk; ++j) {
            ok = ok && __all_sync(0xffffffffu, mbar_wait(&s_full[j & 1], (j >> 1) & 1, err, 257));
            uint32_t sv[64];
            float mx = kNegInf;
            const int kb = j * kTcKeys + ch * 64;
            if (ok) {
                tc_fence_after();
                tmem_ld64(row_t + (j & 1) * 128 + ch * 64, sv);
                tmem_ld_wait();
                float mx8[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) mx8[i] = kNegInf;
#pragma unroll
                for (int e = 0; e < 64; ++e) {  // eight independent max chains
                    const float x = kb + e <= qpos ? __uint_as_float(sv[e]) * sl2e : kNegInf;
                    sv[e] = __float_as_uint(x);
                    mx8[e & 7] = fmaxf(mx8[e & 7], x);
                }
                mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                           fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            }
            red[ch * 128 + r] = mx;
            named_bar_sync(pair_bar, 64);
            mx = fmaxf(mx, red[(1 - ch) * 128 + r]);
            named_bar_sync(pair_bar, 64);  // both read before either writes the next value
            if (!ok) continue;
            // The running max moves only when the block's max exceeds it by more than 2^8 in p:
            // p = exp2(s - m) then stays <= 256 (exact enough in bf16, and O / l uses the same m),
            // and O is rescaled in TMEM only on those (rare, after the first blocks) steps.
            const float m_new = (m == kNegInf || mx > m + 8.f) ? fmaxf(m, mx) : m;
            const float base = m_new == kNegInf ? 0.f : m_new;
            const float alpha = m == kNegInf ? 0.f : exp2f(m - m_new);
            // P(j) as bf16 pairs into the first 64 columns of S(j)'s TMEM buffer (both halves of
            // S(j) are in registers: the pair barriers above came after both loads)
            float sum4[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t pk[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                const float p0 = exp2f(__uint_as_float(sv[2 * e]) - base);
                const float p1 = exp2f(__uint_as_float(sv[2 * e + 1]) - base);
                sum4[e & 3] += p0 + p1;
                pk[e] = pack_bf16x2(p0, p1);
            }
            tmem_st32(row_t + (j & 1) * 128 + ch * 32, pk);
            tmem_st_wait();
            l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
            m = m_new;
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                // O *= alpha once P(j - 1) V(j - 1) has landed (and before P(j) V(j) is issued)
                ok = __all_sync(0xffffffffu, mbar_wait(&o_ready[(j - 1) & 1], ((j - 1) >> 1) & 1, err, 258));
                if (!ok) continue;
                tc_fence_after();
                uint32_t o[64];
                tmem_ld64(row_t + 256 + ch * 64, o);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 64; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                tmem_st64(row_t + 256 + ch * 64, o);
                tmem_st_wait();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[j & 1]);
        }
        if (ok)
            ok = __all_sync(0xffffffffu, mbar_wait(&o_ready[(nblk - 1) & 1], ((nblk - 1) >> 1) & 1, err, 259));
        // the row sum: this half's part plus the partner's (both halves use the same m)
        red[ch * 128 + r] = l;
        named_bar_sync(pair_bar, 64);
        l += red[(1 - ch) * 128 + r];
        if (ok) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            __nv_bfloat16* dst = out + (static_cast<int64_t>(qbeg + tile0 + t) * hq + kvh * group + hl) * kHd + ch * 64;
            uint32_t o[64];
            tmem_ld64(row_t + 256 + ch * 64, o);
            tmem_ld_wait();
            if (valid) {
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    uint4 w;
                    w.x = pack_bf16x2(__uint_as_float(o[8 * c]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
                    w.y = pack_bf16x2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
                    w.z = pack_bf16x2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
                    w.w = pack_bf16x2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
                    reinterpret_cast<uint4*>(dst)[c] = w;
                }
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------------------ cascade decode
// Decode when the first S page-table columns are the same pages for every request (a prefix
// shared through the radix cache). One launch, two kinds of CTA:
//  * prefix CTAs (first in the grid): (prefix chunk, kv head g, 64-row tile) -- the rows are the
//    (request, query head of g) pairs of all requests, so one warp's 16 MMA rows are 16 / group
//    requests x group heads and every row is live; the chunk's shared pages are read once per kv
//    head (4 pages of one head per 32 KB stage, a 3-D box {64, 16, 2}); no mask (every request
//    sees the whole prefix);
//  * suffix CTAs: the decode CTAs of the plain kernel over page columns >= S.
// Both write unnormalised partials (O, m, l) to the workspace; the last CTA to arrive for a
// (request, head group) merges its suffix chunks then its prefix chunks, in that fixed order.
struct CascadePlan {
    int shared_pages;  // S
    int pc_pages;      // prefix pages per prefix chunk
    int n_pchunks;     // prefix chunks
    int row_tiles;     // 64-row tiles of (request, q head) rows of one kv head
    int n_pre;         // prefix CTAs = n_pchunks * Hkv * row_tiles
    int chunk_pages;   // suffix pages per suffix chunk
    int chunks_sfx;    // suffix chunks per (request, head group) in the grid
    int n_hg;          // head groups
    int max_chunks;    // workspace chunk stride = chunks_sfx + n_pchunks
};
constexpr int kPrePagesPerStage = 4;
constexpr int kPreRows = kDecWarps * 16;  // 64 rows per prefix CTA

// The 128 consumer threads merge request b's head group hg: suffix chunks 0..nsfx-1, then prefix
// chunks chunks_sfx .. chunks_sfx + n_pchunks - 1.
__device__ __forceinline__ void cascade_merge(int b, int hg, int nsfx, int hq, int nq,
                                              const CascadePlan& cp, const float* ws_o,
                                              const float* ws_ml, __nv_bfloat16* out) {
    const int64_t cbase = static_cast<int64_t>(b) * cp.max_chunks;
    const int csfx = cp.chunks_sfx;
    merge_partials(nsfx + cp.n_pchunks, nq, hg * nq, hq,
                   [cbase, nsfx, csfx](int k) {
                       return cbase + (k < nsfx ? k : csfx + (k - nsfx));
                   },
                   ws_o, ws_ml, out + static_cast<int64_t>(b) * hq * kHd);
}

// suffix chunks of request b that have pages (the suffix CTAs that arrive)
__device__ __forceinline__ int cascade_nsfx(int L, const CascadePlan& cp) {
    const int npages = (L + kPage - 1) / kPage;
    const int sp = npages - cp.shared_pages;
    return sp > 0 ? (sp + cp.chunk_pages - 1) / cp.chunk_pages : 0;
}

__global__ void __launch_bounds__(kDecThreads, 2)
paged_decode_cascade_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                            const __grid_constant__ CUtensorMap tk1, const __grid_constant__ CUtensorMap tv1,
                            const __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ out,
                            const int* __restrict__ page_table, int max_pages,
                            const int* __restrict__ seq_lens, int num_reqs, int pool_pages, int hq,
                            int hkv, int hc, CascadePlan cp, float sl2e, float* __restrict__ ws_o,
                            float* __restrict__ ws_ml, int* __restrict__ ws_cnt, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDecStages * kDecStageBytes);
    uint64_t* empty = full + kDecStages;
    int* flag = reinterpret_cast<int*>(empty + kDecStages);
    int* mlist = flag + 4;              // [kPreRows] requests this CTA merges
    int* pages = mlist + kPreRows;      // [<= kMaxChunkPages] page ids
    if (threadIdx.x == 0) {
        for (int st = 0; st < kDecStages; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], kDecWarps);
        }
        fence_barrier_init();
    }
    pdl_wait();
    pdl_trigger();
    const int group = hq / hkv;
    const int nq = hc * group;  // query heads per head group
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g4 = lane >> 2, c = lane & 3;
    const int S = cp.shared_pages;
    const int maxL = max_pages * kPage;

    if (blockIdx.x < static_cast<unsigned>(cp.n_pre)) {
        // ======================================================== prefix CTA
        const int pc = blockIdx.x % cp.n_pchunks;
        const int kvh = (blockIdx.x / cp.n_pchunks) % hkv;
        const int rt = blockIdx.x / (cp.n_pchunks * hkv);
        const int hg = kvh / hc;
        const int pbeg = pc * cp.pc_pages;
        const int np = min(S - pbeg, cp.pc_pages);
        const int nsteps = (np + kPrePagesPerStage - 1) / kPrePagesPerStage;
        __syncthreads();
        if (warp == kDecWarps) {
            for (int i = lane; i < np; i += 32) {
                int page = page_table[pbeg + i];  // row 0: the shared columns
                if (static_cast<unsigned>(page) >= static_cast<unsigned>(pool_pages)) {
                    record_error(err, MSGL_ERR_BOUNDS, 206);
                    page = 0;
                }
                pages[i] = page;
            }
            __syncwarp();
            if (lane == 0) {
                tma_prefetch_desc(&tk1);
                tma_prefetch_desc(&tv1);
                for (int it = 0; it < nsteps; ++it) {
                    const int st = it % kDecStages;
                    if (it >= kDecStages && !mbar_wait(&empty[st], ((it / kDecStages) - 1) & 1, err, 240))
                        break;
                    const int cnt = min(kPrePagesPerStage, np - it * kPrePagesPerStage);
                    mbar_arrive_expect_tx(&full[st], cnt * 8192);
                    uint8_t* stg = smem + st * kDecStageBytes;
                    for (int pp = 0; pp < cnt; ++pp) {
                        const int y = pages[it * kPrePagesPerStage + pp] * kPage;
                        tma_load_3d(stg + pp * 4096, &tk1, &full[st], 0, y, 2 * kvh);
                        tma_load_3d(stg + kDecHalfStage + pp * 4096, &tv1, &full[st], 0, y, 2 * kvh);
                    }
                }
            }
            return;
        }
        // rows of this warp: r = rt * 64 + warp * 16 + i -> request r / group, head r % group
        const int rbase = rt * kPreRows + warp * 16;
        const int ra = rbase + g4, rb = rbase + g4 + 8;
        const int ba = ra / group, bb = rb / group;
        const bool va = ba < num_reqs, vb = bb < num_reqs;
        const int qa_h = kvh * group + ra % group, qb_h = kvh * group + rb % group;
        uint32_t qa[8][4];
        {
            const __nv_bfloat16* q0 = q + (static_cast<int64_t>(va ? ba : 0) * hq + qa_h) * kHd;
            const __nv_bfloat16* q1 = q + (static_cast<int64_t>(vb ? bb : 0) * hq + qb_h) * kHd;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                qa[kk][0] = va ? *reinterpret_cast<const uint32_t*>(q0 + 16 * kk + 2 * c) : 0u;
                qa[kk][2] = va ? *reinterpret_cast<const uint32_t*>(q0 + 16 * kk + 8 + 2 * c) : 0u;
                qa[kk][1] = vb ? *reinterpret_cast<const uint32_t*>(q1 + 16 * kk + 2 * c) : 0u;
                qa[kk][3] = vb ? *reinterpret_cast<const uint32_t*>(q1 + 16 * kk + 8 + 2 * c) : 0u;
            }
        }
        float o[16][4];
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        float m[2] = {kNegInf, kNegInf}, l[2] = {0.f, 0.f};
        constexpr int kAll = 0x3fffffff;  // no mask: every request sees the whole prefix
        for (int it = 0; it < nsteps; ++it) {
            const int st = it % kDecStages;
            if (!mbar_wait(&full[st], (it / kDecStages) & 1, err, 241)) break;
            const int cnt = min(kPrePagesPerStage, np - it * kPrePagesPerStage);
            const uint32_t base = smem_u32(smem + st * kDecStageBytes);
            for (int pp = 0; pp < cnt; ++pp)
                attend_page<true>(base + pp * 4096, base + kDecHalfStage + pp * 4096, qa, o, m, l,
                                  0, kAll, kAll, sl2e, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
        // partials of rows ra, rb -> chunk chunks_sfx + pc
        const int ch = cp.chunks_sfx + pc;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float ls = l[r];
            ls += __shfl_xor_sync(0xffffffffu, ls, 1);
            ls += __shfl_xor_sync(0xffffffffu, ls, 2);
            const bool valid = r == 0 ? va : vb;
            if (!valid) continue;
            const int bq = r == 0 ? ba : bb, qh = r == 0 ? qa_h : qb_h;
            const int64_t pi = (static_cast<int64_t>(bq) * cp.max_chunks + ch) * hq + qh;
            float* dst = ws_o + pi * kHd;
#pragma unroll
            for (int j = 0; j < 16; ++j)
                *reinterpret_cast<float2*>(dst + 8 * j + 2 * c) = make_float2(o[j][2 * r], o[j][2 * r + 1]);
            if (c == 0) {
                ws_ml[pi * 2] = m[r];
                ws_ml[pi * 2 + 1] = ls;
            }
        }
        // arrive for every request of the tile; merge those this CTA completes
        __threadfence();
        named_bar_sync(1, kDecWarps * 32);
        const int rq0 = rt * kPreRows / group;
        const int nrq = min(kPreRows / group, num_reqs - rq0);
        if (threadIdx.x == 0) *flag = 0;
        named_bar_sync(1, kDecWarps * 32);
        if (threadIdx.x < nrq) {
            const int bq = rq0 + threadIdx.x;
            int L = seq_lens[bq];
            L = L < 0 ? 0 : (L > maxL ? maxL : L);
            const int expected = cascade_nsfx(L, cp) + cp.n_pchunks * hc;
            const int old = atomicAdd(&ws_cnt[static_cast<int64_t>(bq) * cp.n_hg + hg], 1);
            if (old == expected - 1) mlist[atomicAdd(flag, 1)] = bq;
        }
        named_bar_sync(1, kDecWarps * 32);
        const int nm = *flag;
        if (nm == 0) return;
        __threadfence();
        for (int k = 0; k < nm; ++k) {
            const int bq = mlist[k];
            int L = seq_lens[bq];
            L = L < 0 ? 0 : (L > maxL ? maxL : L);
            cascade_merge(bq, hg, cascade_nsfx(L, cp), hq, nq, cp, ws_o, ws_ml, out);
            if (threadIdx.x == 0) ws_cnt[static_cast<int64_t>(bq) * cp.n_hg + hg] = 0;
        }
        return;
    }

    // ============================================================ suffix CTA
    const int sidx = blockIdx.x - cp.n_pre;
    const int chunk = sidx % cp.chunks_sfx;
    const int hg = (sidx / cp.chunks_sfx) % cp.n_hg;
    const int b = sidx / (cp.chunks_sfx * cp.n_hg);
    const int pps = kDecWarps / hc;
    const int qh0 = hg * nq;
    int L = seq_lens[b];
    if (L < 0 || L > maxL) {
        if (threadIdx.x == 0 && chunk == 0 && hg == 0) record_error(err, MSGL_ERR_BOUNDS, 202);
        L = L < 0 ? 0 : maxL;
    }
    const int npages = (L + kPage - 1) / kPage;
    if (chunk == 0 && hg == 0 && warp == kDecWarps) {  // the batch must really share the prefix
        if (L < S * kPage && lane == 0) record_error(err, MSGL_ERR_BOUNDS, 204);
        for (int i = lane; i < S; i += 32)
            if (page_table[static_cast<int64_t>(b) * max_pages + i] != page_table[i])
                record_error(err, MSGL_ERR_BOUNDS, 205);
    }
    const int p0 = S + chunk * cp.chunk_pages;
    if (p0 >= npages) return;  // no suffix pages for this chunk: it does not arrive
    const int np = min(npages - p0, cp.chunk_pages);
    const int nsteps = (np + pps - 1) / pps;
    __syncthreads();

    if (warp == kDecWarps) {
        const int* pt = page_table + static_cast<int64_t>(b) * max_pages + p0;
        for (int i = lane; i < np; i += 32) {
            int page = pt[i];
            if (static_cast<unsigned>(page) >= static_cast<unsigned>(pool_pages)) {
                record_error(err, MSGL_ERR_BOUNDS, 201);
                page = 0;
            }
            pages[i] = page;
        }
        __syncwarp();
        if (lane == 0) {
            tma_prefetch_desc(&tk);
            tma_prefetch_desc(&tv);
            const int page_half = hc * 4096;
            for (int it = 0; it < nsteps; ++it) {
                const int st = it % kDecStages;
                if (it >= kDecStages && !mbar_wait(&empty[st], ((it / kDecStages) - 1) & 1, err, 200))
                    break;
                const int cnt = min(pps, np - it * pps);
                mbar_arrive_expect_tx(&full[st], cnt * 2 * page_half);
                uint8_t* stg = smem + st * kDecStageBytes;
                for (int pp = 0; pp < cnt; ++pp) {
                    const int y = pages[it * pps + pp] * kPage;
                    tma_load_3d(stg + pp * page_half, &tk, &full[st], 0, y, 2 * hc * hg);
                    tma_load_3d(stg + kDecHalfStage + pp * page_half, &tv, &full[st], 0, y, 2 * hc * hg);
                }
            }
        }
        return;
    }
    const int head = warp % hc, psub = warp / hc;
    uint32_t qa[8][4];
    {
        const bool real = g4 < group;
        const __nv_bfloat16* qr =
            q + (static_cast<int64_t>(b) * hq + qh0 + head * group + (real ? g4 : 0)) * kHd;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            qa[kk][0] = real ? *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 2 * c) : 0u;
            qa[kk][2] = real ? *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 8 + 2 * c) : 0u;
            qa[kk][1] = 0u;
            qa[kk][3] = 0u;
        }
    }
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m[2] = {kNegInf, kNegInf}, l[2] = {0.f, 0.f};
    const uint32_t my_off = (psub * hc + head) * 4096;
    for (int it = 0; it < nsteps; ++it) {
        const int st = it % kDecStages;
        if (!mbar_wait(&full[st], (it / kDecStages) & 1, err, 210)) break;
        const int pidx = it * pps + psub;
        if (pidx < np) {
            const uint32_t base = smem_u32(smem + st * kDecStageBytes) + my_off;
            attend_page<false>(base, base + kDecHalfStage, qa, o, m, l, (p0 + pidx) * kPage, L - 1,
                               -1, sl2e, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    // combine the pps warps of each head, write this chunk's partial
    float lsum = l[0];
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
    named_bar_sync(1, kDecWarps * 32);
    float* mo = reinterpret_cast<float*>(smem);
    float* mm = mo + kDecWarps * 8 * kHd;
    float* ml = mm + kDecWarps * 8;
    if (g4 < group) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            mo[(warp * 8 + g4) * kHd + 8 * j + 2 * c] = o[j][0];
            mo[(warp * 8 + g4) * kHd + 8 * j + 2 * c + 1] = o[j][1];
        }
        if (c == 0) {
            mm[warp * 8 + g4] = m[0];
            ml[warp * 8 + g4] = lsum;
        }
    }
    named_bar_sync(1, kDecWarps * 32);
    for (int item = threadIdx.x; item < nq * 16; item += kDecWarps * 32) {
        const int lq = item >> 4, d0 = (item & 15) * 8;
        const int h = lq / group, r = lq % group;
        const int qh = qh0 + lq;
        float M = kNegInf;
        for (int ps = 0; ps < pps; ++ps) M = fmaxf(M, mm[(ps * hc + h) * 8 + r]);
        float O[8] = {0, 0, 0, 0, 0, 0, 0, 0}, Ls = 0.f;
        for (int ps = 0; ps < pps; ++ps) {
            const int w = ps * hc + h;
            const float mw = mm[w * 8 + r];
            const float sc = (mw == kNegInf) ? 0.f : exp2f(mw - M);
            Ls += ml[w * 8 + r] * sc;
#pragma unroll
            for (int e = 0; e < 8; ++e) O[e] += mo[(w * 8 + r) * kHd + d0 + e] * sc;
        }
        const int64_t pi = (static_cast<int64_t>(b) * cp.max_chunks + chunk) * hq + qh;
        float4* dst = reinterpret_cast<float4*>(ws_o + pi * kHd + d0);
        dst[0] = make_float4(O[0], O[1], O[2], O[3]);
        dst[1] = make_float4(O[4], O[5], O[6], O[7]);
        if ((item & 15) == 0) {
            ws_ml[pi * 2] = M;
            ws_ml[pi * 2 + 1] = Ls;
        }
    }
    __threadfence();
    named_bar_sync(1, kDecWarps * 32);
    int* cnt = ws_cnt + static_cast<int64_t>(b) * cp.n_hg + hg;
    if (threadIdx.x == 0) {
        const int expected = cascade_nsfx(L, cp) + cp.n_pchunks * hc;
        *flag = (atomicAdd(cnt, 1) == expected - 1);
    }
    named_bar_sync(1, kDecWarps * 32);
    if (!*flag) return;
    __threadfence();
    cascade_merge(b, hg, cascade_nsfx(L, cp), hq, nq, cp, ws_o, ws_ml, out);
    if (threadIdx.x == 0) *cnt = 0;
}

// ------------------------------------------------------------------------------ host side
constexpr size_t kDecodeCounterBytes = 262144;  // one int per request: up to 65536

struct DecodePlan {
    int chunk_pages, max_chunks;
    size_t off_o, off_ml, off_cnt, bytes;
};

// kv heads per decode CTA: the largest of 4, 2, 1 that divides Hkv.
int decode_heads_per_cta(int hkv) { return hkv % 4 == 0 ? 4 : (hkv % 2 == 0 ? 2 : 1); }

DecodePlan plan_decode(int B, int max_seq_len, int hq, int hkv) {
    DecodePlan p{};
    const int max_pages_seq = std::max(1, (max_seq_len + kPage - 1) / kPage);
    const int n_hg = hkv / decode_heads_per_cta(hkv);
    // Two CTAs per SM (96 KB ring each): split each request's pages into chunks so that
    // (chunk, head group, request) gives about one wave of CTAs (measured at batch 128,
    // context 2048: 1 wave 101.6 us, 2 waves 109, 4 waves 112, 8 waves 115 -- fewer, longer
    // chunks amortise the pipeline fill and the merge), chunks of at least 16 pages and at most
    // kMaxChunkPages.
    const int slots = 2 * 148;
    const long long rows = static_cast<long long>(std::max(1, B)) * n_hg;
    int chunks = static_cast<int>(std::min<long long>((slots + rows - 1) / rows, 1 << 20));
    chunks = std::max(1, std::min(chunks, (max_pages_seq + 15) / 16));
    // One or two kv heads per CTA: CTAs are short and their own rate (not HBM) bounds them, so a
    // last wave filled below half costs a whole CTA's time for little work; one chunk fewer keeps
    // one wave (128 requests x 2048 at a TP8 / TP4 rank of the 8B decode: 3 chunks = 1.3 waves;
    // 25.3 -> 18.0 us at one kv head, 39.0 -> 30.0 us at two).
    if (decode_heads_per_cta(hkv) <= 2 && chunks > 1) {
        const long long tail = (rows * chunks) % slots;
        if (tail != 0 && tail * 2 < slots && rows * (chunks - 1) * 2 >= slots) --chunks;
    }
    chunks = std::max(chunks, (max_pages_seq + kMaxChunkPages - 1) / kMaxChunkPages);
    p.chunk_pages = (max_pages_seq + chunks - 1) / chunks;
    p.max_chunks = (max_pages_seq + p.chunk_pages - 1) / p.chunk_pages;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    // Layout: arrival counters (one per request and head group) at a fixed offset (0) whatever
    // the batch shape -- they persist (self-resetting) between calls, so no other call's
    // partials may land on them -- then the partial O and (m, l) of every chunk.
    size_t o_bytes = up(static_cast<size_t>(B) * p.max_chunks * hq * kHd * sizeof(float));
    size_t ml_bytes = up(static_cast<size_t>(B) * p.max_chunks * hq * 2 * sizeof(float));
    p.off_cnt = 0;
    p.off_o = kDecodeCounterBytes;
    p.off_ml = kDecodeCounterBytes + o_bytes;
    p.bytes = p.max_chunks > 1 ? kDecodeCounterBytes + o_bytes + ml_bytes : 0;
    return p;
}

int check_common(int hq, int hkv, int head_dim, int page_size, int64_t num_slots) {
    if (head_dim != kHd) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "attention: head_dim must be 128");
    if (page_size != kPage) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "attention: page_size must be 16");
    if (hkv <= 0 || hq <= 0 || hq % hkv) return set_error(MSGL_ERR_INVALID_ARG, "attention: Hq % Hkv != 0");
    int group = hq / hkv;
    if (group > 8 || (16 % group)) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "attention: Hq/Hkv must be 1,2,4 or 8");
    if (num_slots <= 0 || num_slots % kPage || num_slots / kPage > INT32_MAX)
        return set_error(MSGL_ERR_INVALID_ARG, "attention: num_slots must be a positive multiple of 16");
    return MSGL_OK;
}

int make_pool_maps(CUtensorMap* tk, CUtensorMap* tv, const void* k_pool, const void* v_pool,
                   int64_t num_slots, int hkv) {
    const uint64_t row = static_cast<uint64_t>(hkv) * kHd;
    int rc = make_tmap_2d_bf16(tk, k_pool, row, num_slots, row * 2, 64, kPage, true);
    if (rc) return rc;
    return make_tmap_2d_bf16(tv, v_pool, row, num_slots, row * 2, 64, kPage, true);
}

// Decode view of a pool: {64 dims, num_slots token rows (Hkv * 256 B apart), 2 Hkv head halves
// (128 B apart)}, box {64, 16, 2 hc}: one page of hc kv heads, head-major in shared memory.
int make_decode_maps(CUtensorMap* tk, CUtensorMap* tv, const void* k_pool, const void* v_pool,
                     int64_t num_slots, int hkv, int hc) {
    const uint64_t row_bytes = static_cast<uint64_t>(hkv) * kHd * 2;
    int rc = make_tmap_3d_bf16(tk, k_pool, 64, num_slots, 2 * hkv, row_bytes, 128, 64, kPage, 2 * hc);
    if (rc) return rc;
    return make_tmap_3d_bf16(tv, v_pool, 64, num_slots, 2 * hkv, row_bytes, 128, 64, kPage, 2 * hc);
}

// Scratch of msgl_paged_attention_decode_noalloc: one file-scope device array per device (module
// load zero-fills it), shared by every call of that entry point on the device.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) uint8_t g_decode_scratch[kNoAllocScratchBytes];

// Cascade plan: suffix chunks from the plain decode plan of the suffix length. A suffix warp
// attends chunk_pages * hc / 4 (page, head) pairs (its CTA's hc heads over the chunk, split over
// 4 warps); a prefix warp attends every page of its prefix chunk for its 16 rows. Prefix chunks
// therefore get chunk_pages * hc / 4 pages, so both kinds of CTA take about as long (with one
// kv head per CTA, chunks as long as the suffix's made the prefix CTAs 4x longer than the rest
// of the grid) -- but no more than 4 prefix chunks per suffix chunk, which bounds the workspace
// at 5x the plain decode's.
constexpr int kMaxPreChunksPerSfx = 4;
CascadePlan plan_cascade(int B, int max_seq_len, int shared_pages, int hq, int hkv) {
    CascadePlan cp{};
    const int max_pages_seq = std::max(1, (max_seq_len + kPage - 1) / kPage);
    const int sfx_pages = std::max(1, max_pages_seq - shared_pages);
    const DecodePlan dp = plan_decode(B, sfx_pages * kPage, hq, hkv);
    const int group = hq / hkv;
    const int hc = decode_heads_per_cta(hkv);
    cp.shared_pages = shared_pages;
    cp.chunk_pages = dp.chunk_pages;
    cp.chunks_sfx = dp.max_chunks;
    const int balanced = std::max(1, (cp.chunk_pages * hc + kDecWarps - 1) / kDecWarps);
    const int cap = kMaxPreChunksPerSfx * cp.chunks_sfx;
    cp.pc_pages = std::min(kMaxChunkPages, std::max(balanced, (shared_pages + cap - 1) / cap));
    cp.n_pchunks = (shared_pages + cp.pc_pages - 1) / cp.pc_pages;
    cp.row_tiles = (B * group + kPreRows - 1) / kPreRows;
    cp.n_pre = cp.n_pchunks * hkv * cp.row_tiles;
    cp.n_hg = hkv / decode_heads_per_cta(hkv);
    cp.max_chunks = cp.chunks_sfx + cp.n_pchunks;
    return cp;
}

size_t cascade_workspace_bytes(int B, const CascadePlan& cp, int hq) {
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    return kDecodeCounterBytes + up(static_cast<size_t>(B) * cp.max_chunks * hq * kHd * sizeof(float)) +
           up(static_cast<size_t>(B) * cp.max_chunks * hq * 2 * sizeof(float));
}

// Extend kernel choice: the tcgen05 kernel when a request can fill at least half a 128-row tile
// (max_q_len x group >= 64); the warp-level MMA kernel for short extends. MSGL_EXTEND_TC=0 forces
// the warp-level kernel (read on every call).
bool use_extend_tc(int max_q_len, int group) {
    const char* e = std::getenv("MSGL_EXTEND_TC");
    if (e && e[0] == '0') return false;
    return static_cast<int64_t>(max_q_len) * group >= 64;
}

// Argument checks of the plain decode entry points (msgl_paged_attention_decode and the
// no-allocation variant), done before anything is queued on the stream; fills the plan.
int check_decode(int64_t num_slots, int max_pages, int num_reqs, int max_seq_len, int hq, int hkv,
                 int head_dim, int page_size, DecodePlan* plan) {
    int rc = check_common(hq, hkv, head_dim, page_size, num_slots);
    if (rc) return rc;
    if (num_reqs < 0 || max_seq_len < 0 || max_pages <= 0)
        return set_error(MSGL_ERR_INVALID_ARG, "decode: bad sizes");
    if (num_reqs == 0) return MSGL_OK;
    if ((max_seq_len + kPage - 1) / kPage > max_pages)
        return set_error(MSGL_ERR_INVALID_ARG, "decode: max_seq_len exceeds page-table width");
    *plan = plan_decode(num_reqs, max_seq_len, hq, hkv);
    const int n_hg = hkv / decode_heads_per_cta(hkv);
    if (num_reqs > 65535 || n_hg > 65535)
        return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "decode: num_reqs or Hkv too large");
    if (plan->bytes > 0 && static_cast<size_t>(num_reqs) * n_hg * sizeof(int) > kDecodeCounterBytes)
        return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "decode: num_reqs * Hkv / 4 > 65536");
    return MSGL_OK;
}

}  // namespace
}  // namespace msgl

using namespace msgl;

extern "C" {

size_t msgl_paged_attention_workspace_size(int num_reqs, int max_seq_len, int num_q_heads,
                                           int num_kv_heads, int head_dim) {
    if (num_reqs <= 0 || num_kv_heads <= 0 || head_dim != kHd) return 0;
    return plan_decode(num_reqs, max_seq_len, num_q_heads, num_kv_heads).bytes;
}

int msgl_paged_attention_decode(const void* q, const void* k_pool, const void* v_pool,
                                int64_t num_slots, const int* page_table, int max_pages,
                                const int* seq_lens, int num_reqs, int max_seq_len,
                                int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                                float scale, void* out, void* workspace,
                                size_t workspace_bytes, msgl_stream_t stream) {
    DecodePlan p{};
    int rc = check_decode(num_slots, max_pages, num_reqs, max_seq_len, num_q_heads, num_kv_heads,
                          head_dim, page_size, &p);
    if (rc) return rc;
    if (num_reqs == 0) return MSGL_OK;
    if (p.bytes > 0 && (!workspace || workspace_bytes < p.bytes))
        return set_error(MSGL_ERR_WORKSPACE, "decode: workspace too small");
    const int hc = decode_heads_per_cta(num_kv_heads);
    const int n_hg = num_kv_heads / hc;
    CUtensorMap tk, tv;
    rc = make_decode_maps(&tk, &tv, k_pool, v_pool, num_slots, num_kv_heads, hc);
    if (rc) return rc;
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    const size_t smem = kDecStages * kDecStageBytes + 2 * kDecStages * 8 + 16 +
                        kMaxChunkPages * sizeof(int) + 1024;
    static std::atomic<int> optin[kMaxDevices];
    cudaError_t e = smem_optin(paged_decode_kernel, smem, optin);
    if (e != cudaSuccess) return set_error(MSGL_ERR_CUDA, cudaGetErrorString(e));
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    dim3 grid(p.max_chunks, n_hg, num_reqs);
    const float sl2e = scale * 1.4426950408889634f;
    launch_pdl(paged_decode_kernel, grid, dim3(kDecThreads), smem, stream,
        tk, tv, static_cast<const __nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(out), page_table,
        max_pages, seq_lens, static_cast<int>(num_slots / kPage), num_q_heads, num_kv_heads, hc,
        p.chunk_pages, p.max_chunks, sl2e, p.bytes ? reinterpret_cast<float*>(ws + p.off_o) : nullptr,
        p.bytes ? reinterpret_cast<float*>(ws + p.off_ml) : nullptr,
        p.bytes ? reinterpret_cast<int*>(ws + p.off_cnt) : nullptr, err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

int msgl_paged_attention_extend(const void* q, const void* k_pool, const void* v_pool,
                                int64_t num_slots, const int* page_table, int max_pages,
                                const int* seq_lens, const int* q_indptr, int num_reqs,
                                int max_q_len, int num_q_heads, int num_kv_heads, int head_dim,
                                int page_size, float scale, void* out, msgl_stream_t stream) {
    int rc = check_common(num_q_heads, num_kv_heads, head_dim, page_size, num_slots);
    if (rc) return rc;
    if (num_reqs < 0 || max_q_len < 0 || max_pages <= 0)
        return set_error(MSGL_ERR_INVALID_ARG, "extend: bad sizes");
    if (num_reqs == 0 || max_q_len == 0) return MSGL_OK;
    if (num_reqs > 65535) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "extend: num_reqs > 65535");
    CUtensorMap tk, tv;
    rc = make_pool_maps(&tk, &tv, k_pool, v_pool, num_slots, num_kv_heads);
    if (rc) return rc;
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    const size_t smem = kExtendStages * kPageSlotBytes + 2 * kExtendStages * 8 +
                        kExtendPageBatch * sizeof(int) + 1024;
    static std::atomic<int> optin[kMaxDevices];
    cudaError_t e = smem_optin(paged_extend_kernel, smem, optin);
    if (e != cudaSuccess) return set_error(MSGL_ERR_CUDA, cudaGetErrorString(e));
    const int group = num_q_heads / num_kv_heads;
    const float sl2e = scale * 1.4426950408889634f;
    if (use_extend_tc(max_q_len, group)) {  // tcgen05 tiles of 128 query rows
        static std::atomic<int> optin_tc[kMaxDevices];
        cudaError_t e2 = smem_optin(paged_extend_tc_kernel, kTcSmem, optin_tc);
        if (e2 != cudaSuccess) return set_error(MSGL_ERR_CUDA, cudaGetErrorString(e2));
        const int tpt = kTcRows / group;
        dim3 grid_tc((max_q_len + tpt - 1) / tpt, num_kv_heads, num_reqs);
        launch_pdl(paged_extend_tc_kernel, grid_tc, dim3(kTcThreads), kTcSmem, stream, tk, tv,
                   static_cast<const __nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(out),
                   page_table, max_pages, seq_lens, q_indptr, static_cast<int>(num_slots / kPage),
                   num_q_heads, num_kv_heads, sl2e, err);
        MSGL_LAUNCH_CHECK();
        return MSGL_OK;
    }
    const int tile_tokens = kConsumerWarps * (16 / group);
    dim3 grid((max_q_len + tile_tokens - 1) / tile_tokens, num_kv_heads, num_reqs);
    launch_pdl(paged_extend_kernel, grid, dim3(kThreads), smem, stream,
        tk, tv, static_cast<const __nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(out), page_table,
        max_pages, seq_lens, q_indptr, static_cast<int>(num_slots / kPage), num_q_heads,
        num_kv_heads, sl2e, err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

size_t msgl_paged_attention_cascade_workspace_size(int num_reqs, int max_seq_len, int shared_pages,
                                                   int num_q_heads, int num_kv_heads, int head_dim) {
    if (num_reqs <= 0 || num_kv_heads <= 0 || head_dim != kHd || shared_pages <= 0) return 0;
    const CascadePlan cp = plan_cascade(num_reqs, max_seq_len, shared_pages, num_q_heads, num_kv_heads);
    return cascade_workspace_bytes(num_reqs, cp, num_q_heads);
}

int msgl_paged_attention_decode_cascade(const void* q, const void* k_pool, const void* v_pool,
                                        int64_t num_slots, const int* page_table, int max_pages,
                                        const int* seq_lens, int num_reqs, int max_seq_len,
                                        int shared_pages, int num_q_heads, int num_kv_heads,
                                        int head_dim, int page_size, float scale, void* out,
                                        void* workspace, size_t workspace_bytes,
                                        msgl_stream_t stream) {
    int rc = check_common(num_q_heads, num_kv_heads, head_dim, page_size, num_slots);
    if (rc) return rc;
    if (num_reqs < 0 || max_seq_len < 0 || max_pages <= 0)
        return set_error(MSGL_ERR_INVALID_ARG, "decode_cascade: bad sizes");
    if (num_reqs == 0) return MSGL_OK;
    if ((max_seq_len + kPage - 1) / kPage > max_pages)
        return set_error(MSGL_ERR_INVALID_ARG, "decode_cascade: max_seq_len exceeds page-table width");
    if (shared_pages <= 0 || shared_pages > max_pages || shared_pages * kPage > max_seq_len)
        return set_error(MSGL_ERR_INVALID_ARG, "decode_cascade: shared_pages outside the contexts");
    if (num_reqs > 65535) return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "decode_cascade: num_reqs > 65535");
    const CascadePlan cp = plan_cascade(num_reqs, max_seq_len, shared_pages, num_q_heads, num_kv_heads);
    const size_t need = cascade_workspace_bytes(num_reqs, cp, num_q_heads);
    if (!workspace || workspace_bytes < need)
        return set_error(MSGL_ERR_WORKSPACE, "decode_cascade: workspace too small");
    if (static_cast<size_t>(num_reqs) * cp.n_hg * sizeof(int) > kDecodeCounterBytes)
        return set_error(MSGL_ERR_UNSUPPORTED_SHAPE, "decode_cascade: num_reqs * Hkv / 4 > 65536");
    const int hc = decode_heads_per_cta(num_kv_heads);
    CUtensorMap tk, tv, tk1, tv1;
    rc = make_decode_maps(&tk, &tv, k_pool, v_pool, num_slots, num_kv_heads, hc);
    if (rc) return rc;
    rc = make_decode_maps(&tk1, &tv1, k_pool, v_pool, num_slots, num_kv_heads, 1);
    if (rc) return rc;
    int* err = device_error_word();
    if (!err) return set_error(MSGL_ERR_CUDA, "device error word unavailable");
    const size_t smem = kDecStages * kDecStageBytes + 2 * kDecStages * 8 + 16 +
                        (kPreRows + kMaxChunkPages) * sizeof(int) + 1024;
    static std::atomic<int> optin[kMaxDevices];
    cudaError_t e = smem_optin(paged_decode_cascade_kernel, smem, optin);
    if (e != cudaSuccess) return set_error(MSGL_ERR_CUDA, cudaGetErrorString(e));
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const size_t o_bytes = (static_cast<size_t>(num_reqs) * cp.max_chunks * num_q_heads * kHd * sizeof(float) + 255) & ~size_t(255);
    const int grid = cp.n_pre + cp.chunks_sfx * cp.n_hg * num_reqs;
    const float sl2e = scale * 1.4426950408889634f;
    launch_pdl(paged_decode_cascade_kernel, dim3(grid), dim3(kDecThreads), smem, stream, tk, tv, tk1,
               tv1, static_cast<const __nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(out),
               page_table, max_pages, seq_lens, num_reqs, static_cast<int>(num_slots / kPage),
               num_q_heads, num_kv_heads, hc, cp, sl2e,
               reinterpret_cast<float*>(ws + kDecodeCounterBytes),
               reinterpret_cast<float*>(ws + kDecodeCounterBytes + o_bytes),
               reinterpret_cast<int*>(ws), err);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

// The device address of the static scratch is looked up once per device (on the first call with
// that device current) and cached; the call then clears the split-KV arrival counters it will
// use and runs msgl_paged_attention_decode on the scratch.
int msgl_paged_attention_decode_noalloc(const void* q, const void* k_pool, const void* v_pool,
                                        int64_t num_slots, const int* page_table, int max_pages,
                                        const int* seq_lens, int num_reqs, int max_seq_len,
                                        int num_q_heads, int num_kv_heads, int head_dim,
                                        int page_size, float scale, void* out,
                                        msgl_stream_t stream) {
    // every argument check of the workspace entry point runs first: a rejected call queues
    // nothing on the stream
    DecodePlan p{};
    int rc = check_decode(num_slots, max_pages, num_reqs, max_seq_len, num_q_heads, num_kv_heads,
                          head_dim, page_size, &p);
    if (rc) return rc;
    if (num_reqs == 0) return MSGL_OK;
    if (p.bytes > kNoAllocScratchBytes) {
        char buf[256];
        snprintf(buf, sizeof(buf),
                 "decode_noalloc: this batch needs %zu bytes of scratch; the static scratch holds "
                 "%zu (8 MiB) -- use msgl_paged_attention_decode with a workspace",
                 p.bytes, kNoAllocScratchBytes);
        return set_error(MSGL_ERR_WORKSPACE, buf);
    }
    static void* ptrs[kMaxDevices] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return set_error(MSGL_ERR_CUDA, "decode_noalloc: no current device");
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!ptrs[dev]) {
            void* ptr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
            if (e != cudaSuccess || !ptr)
                return set_error(MSGL_ERR_CUDA, e != cudaSuccess ? cudaGetErrorString(e)
                                                                 : "decode_noalloc: null scratch");
            ptrs[dev] = ptr;
        }
        scratch = ptrs[dev];
    }
    if (p.bytes > 0) {  // arrival counters at offset 0 must start at zero
        const size_t cnt_bytes = static_cast<size_t>(num_reqs) *
                                 (num_kv_heads / decode_heads_per_cta(num_kv_heads)) * sizeof(int);
        const cudaError_t e = cudaMemsetAsync(scratch, 0, std::min(cnt_bytes, kDecodeCounterBytes), stream);
        if (e != cudaSuccess) return set_error(MSGL_ERR_CUDA, cudaGetErrorString(e));
    }
    return msgl_paged_attention_decode(q, k_pool, v_pool, num_slots, page_table, max_pages,
                                       seq_lens, num_reqs, max_seq_len, num_q_heads, num_kv_heads,
                                       head_dim, page_size, scale, out, scratch,
                                       kNoAllocScratchBytes, stream);
}

}  // extern "C"
