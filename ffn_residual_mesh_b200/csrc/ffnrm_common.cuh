// Shared device-side definitions for the B200 exact base/residual split kernels.
//
// Device layout of one projection (gate or up) of one layer, rows = d_ff rows held
// by this context, D = d_model, G = D/32:
//   pair    : bits 0-1 of every code, row-packed [F, D/4]; byte j of a row holds codes
//             4j..4j+3 at bit pairs 0,2,4,6 (the reference QLO2 layout,
//             scripts/export_cuda_residual_artifact_v2.py:13-24). Present for r in
//             {2,3} and whenever fallback data is kept.
//   plane   : one bit of every code, row-packed [F, D/8], code 8j+i at bit i of byte j
//             (one plane of scripts/compile_q4k_host_base_gpu_residual.py:17-26):
//             bit 0 for r = 1, bit 2 for r = 3.
//   pair_hi : bits 2-3 of every code in the pair layout (fallback tiles only).
//   alpha   : [F, G] fp16 when lossless, else f32; beta likewise (fallback only).
//
// The residual group dot of row f, group g, token t is
//   r = 1: P = dot(plane, z)      r = 2: P = dot(pair, z)     r = 3: P = dot(pair, z) + 4*dot(plane, z)
// and the unsplit fallback dot is  dot(pair, z) + 4*dot(pair_hi, z).
//
// dp4a operand order. A 32-bit word of `pair` holds 16 codes; (w >> 2i) & 0x03030303
// yields codes {16m+i, 16m+4+i, 16m+8+i, 16m+12+i} (m = word index), so activations
// are stored permuted in shared memory to match (zpair). A 32-bit word of `plane`
// holds one group; (w >> i) & 0x01010101 yields codes {i, 8+i, 16+i, 24+i} (zplane).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ffnrm {

constexpr int kGroup = 32;

struct ProjView {
    const uint8_t *pair;
    const uint8_t *plane;
    const uint8_t *pair_hi;
    const void *alpha;
    const void *beta;
};

template <bool HALF>
__device__ __forceinline__ void load_scale2(const void *base, int64_t index, float &a0, float &a1) {
    if constexpr (HALF) {
        const __half2 v = *reinterpret_cast<const __half2 *>(reinterpret_cast<const __half *>(base) + index);
        const float2 f = __half22float2(v);
        a0 = f.x;
        a1 = f.y;
    } else {
        const float2 v = *reinterpret_cast<const float2 *>(reinterpret_cast<const float *>(base) + index);
        a0 = v.x;
        a1 = v.y;
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ bool row_flagged(const uint8_t *tiles, int row, int tile_rows) {
    return tiles != nullptr && tiles[row / tile_rows] != 0;
}

}  // namespace ffnrm
