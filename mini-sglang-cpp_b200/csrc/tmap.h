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

// 3-D view of bf16 elements: dims {d0 (contiguous), d1, d2}, byte strides s1 / s2 of dims 1 / 2
// (any order: s2 may be smaller than s1, which lets one box gather a page's token rows of several
// heads into a head-major [box2][box1][box0] tile), SWIZZLE_128B.
int make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                      uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2);
}  // namespace msgl
