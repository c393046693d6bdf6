// tmap.h -- host helper that encodes 2-D bf16 TMA descriptors (CUtensorMap) through the driver
// entry point (no link-time dependency on libcuda).
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace msgl {
// Tensor of `outer` rows x `inner` bf16 elements, rows `row_stride_bytes` apart; box of
// box_outer rows x box_inner elements. Out-of-range elements of a box read as zero.
int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                      bool swizzle128);
}  // namespace msgl
