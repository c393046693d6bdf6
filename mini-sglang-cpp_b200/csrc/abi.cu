// abi.cu -- library-wide C-ABI pieces: status messages, the device error word, version, the
// counter-based normal generator used for random-init weights, and the TMA descriptor helper.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "tmap.h"

namespace msgl {

__device__ int g_device_error[2];  // {code, info}; zero-initialised at module load

static thread_local std::string t_last_error;

int set_error(int code, const char* msg) {
    t_last_error = msg ? msg : "";
    return code;
}

int* device_error_word() {
    static int* ptrs[64] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
        ptrs[dev] = static_cast<int*>(p);
    }
    return ptrs[dev];
}

std::atomic<unsigned long long>& launch_counter() {
    static std::atomic<unsigned long long> n{0};
    return n;
}

bool pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("MSGL_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

// ------------------------------------------------------------------ TMA descriptors
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                      bool swizzle128) {
    EncodeTiledFn fn = get_encode_fn();
    if (!fn) return set_error(MSGL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride_bytes & 15))
        return set_error(MSGL_ERR_INVALID_ARG, "TMA base / row stride not 16-byte aligned");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[160];
        snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu box %u x %u",
                 (int)r, (unsigned long long)inner, (unsigned long long)outer, box_inner,
                 box_outer);
        return set_error(MSGL_ERR_CUDA, buf);
    }
    return MSGL_OK;
}

int make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                      uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2) {
    EncodeTiledFn fn = get_encode_fn();
    if (!fn) return set_error(MSGL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (s1 & 15) || (s2 & 15))
        return set_error(MSGL_ERR_INVALID_ARG, "TMA base / strides not 16-byte aligned");
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1, s2};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[200];
        snprintf(buf, sizeof(buf),
                 "cuTensorMapEncodeTiled (3-D) failed (%d): dims %llu x %llu x %llu strides %llu %llu "
                 "box %u x %u x %u",
                 (int)r, (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2,
                 (unsigned long long)s1, (unsigned long long)s2, b0, b1, b2);
        return set_error(MSGL_ERR_CUDA, buf);
    }
    return MSGL_OK;
}

// ------------------------------------------------------------------ Philox4x32-10
// Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3" (SC'11).
struct U4 { uint32_t x, y, z, w; };

__host__ __device__ inline uint32_t mulhilo(uint32_t a, uint32_t b, uint32_t* hi) {
    uint64_t p = static_cast<uint64_t>(a) * b;
    *hi = static_cast<uint32_t>(p >> 32);
    return static_cast<uint32_t>(p);
}

__host__ __device__ inline U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
    const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        uint32_t hi0, hi1;
        uint32_t lo0 = mulhilo(M0, c.x, &hi0);
        uint32_t lo1 = mulhilo(M1, c.z, &hi1);
        c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
        k0 += W0;
        k1 += W1;
    }
    return c;
}

__global__ void fill_normal_bf16_kernel(__nv_bfloat16* out, int64_t n, uint64_t seed,
                                        uint64_t stream_id, float mean, float std) {
    int64_t i4 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x);
    int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (; i4 * 4 < n; i4 += stride) {
        U4 c{static_cast<uint32_t>(i4), static_cast<uint32_t>(static_cast<uint64_t>(i4) >> 32),
             static_cast<uint32_t>(stream_id), static_cast<uint32_t>(stream_id >> 32)};
        U4 r = philox4x32_10(c, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
        // Box-Muller on (x, y) and (z, w); uniforms in (0, 1].
        const float inv = 2.3283064365386963e-10f;
        float u0 = (r.x + 1.0f) * inv, u1 = r.y * inv, u2 = (r.z + 1.0f) * inv, u3 = r.w * inv;
        float rad0 = sqrtf(-2.0f * logf(u0)), rad1 = sqrtf(-2.0f * logf(u2));
        float s0, c0, s1, c1;
        sincospif(2.0f * u1, &s0, &c0);
        sincospif(2.0f * u3, &s1, &c1);
        float v[4] = {rad0 * c0, rad0 * s0, rad1 * c1, rad1 * s1};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int64_t idx = i4 * 4 + j;
            if (idx < n) out[idx] = __float2bfloat16_rn(mean + std * v[j]);
        }
    }
}

}  // namespace msgl

using namespace msgl;

extern "C" {

const char* msgl_version(void) { return "msgl-b200 0.1.0 (sm_100a)"; }

const char* msgl_last_error(void) { return t_last_error.c_str(); }

unsigned long long msgl_kernel_launches(void) { return launch_counter().load(); }

int msgl_device_error(int* code, int* info, int reset, msgl_stream_t stream) {
    if (cudaStreamSynchronize(stream) != cudaSuccess)
        return set_error(MSGL_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
    int w[2] = {0, 0};
    if (cudaMemcpyFromSymbol(w, g_device_error, sizeof(w)) != cudaSuccess)
        return set_error(MSGL_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
    if (code) *code = w[0];
    if (info) *info = w[1];
    if (reset) {
        int z[2] = {0, 0};
        if (cudaMemcpyToSymbol(g_device_error, z, sizeof(z)) != cudaSuccess)
            return set_error(MSGL_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
    }
    return MSGL_OK;
}

int msgl_fill_normal_bf16(void* out, int64_t n, uint64_t seed, uint64_t stream_id, float mean,
                          float std, msgl_stream_t stream) {
    if (n < 0 || (n > 0 && !out)) return set_error(MSGL_ERR_INVALID_ARG, "fill_normal: bad args");
    if (n == 0) return MSGL_OK;
    int64_t quads = (n + 3) / 4;
    int threads = 256;
    int64_t blocks = (quads + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;
    fill_normal_bf16_kernel<<<static_cast<int>(blocks), threads, 0, stream>>>(
        static_cast<__nv_bfloat16*>(out), n, seed, stream_id, mean, std);
    MSGL_LAUNCH_CHECK();
    return MSGL_OK;
}

}  // extern "C"
