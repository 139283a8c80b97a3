// Shared device-side definitions for the B200 exact base/residual split kernels.
//
// Device layouts (chosen at load time; the host converts from the reference's
// artifact formats). C = G/2 chunks of two 32-code groups. Records are tiled by 64-row
// tiles: for row tile rt and chunk c, the 128 records of the gate rows rt*64..+63 and
// then the up rows of the same tile are contiguous, so one 32-row block of one
// projection (a warp's lanes) is 32 consecutive records and one tile's K chunk is a
// single contiguous run for a bulk copy. A projection's view starts at record 64*proj;
// rec_index() gives the record of (32-row block rb, chunk c, lane) from there.
//
//   pair  [F64][C][2][64][16 B]  bits 0-1 of every code. Word j of a record holds group
//         2c + (j>>1), codes 16*(j&1) .. +15; code 4i+b of those 16 sits at bit 8b+2i,
//         so (w >> 2i) & 0x03030303 is the dp4a operand for activations 4i..4i+3 in
//         natural order.
//   plane [F64][C][2][64][8 B]   one bit of every code (bit 0 for r = 1, bit 2 for r = 3).
//         Word j holds group 2c + j; code 4i+b at bit 8b+i, so (w >> i) & 0x01010101
//         pairs with activations 4i..4i+3.
//   pair_hi  like pair, bits 2-3 (fallback tiles only).
//   alpha/beta [F64][C][2][64][2]   fp16 when lossless, else f32.
//
// Rows F..64*F64-1 are zero padding. The residual group dot of row f, group g is
//   r = 1: P = dot(plane, z)   r = 2: P = dot(pair, z)   r = 3: P = dot(pair, z) + 4 dot(plane, z)
// and the unsplit fallback dot is dot(pair, z) + 4 dot(pair_hi, z).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ffnrm {

constexpr int kGroup = 32;

// Asynchronous global -> shared copies (cp.async). The 16-byte form zero-fills when
// `valid` is false.
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src, bool valid) {
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    const int bytes = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(gmem_src), "r"(bytes));
}
template <int BYTES>
__device__ __forceinline__ void cp_async_small(void *smem_dst, const void *gmem_src) {
    static_assert(BYTES == 4 || BYTES == 8, "4 or 8 bytes");
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(dst), "l"(gmem_src), "n"(BYTES));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Record of (32-row block rb, chunk c, lane) relative to a projection's view.
__host__ __device__ __forceinline__ int64_t rec_index(int rb, int C, int c, int lane) {
    return (int64_t(rb >> 1) * C + c) * 128 + (rb & 1) * 32 + lane;
}

struct ProjView {
    const uint4 *pair;
    const uint2 *plane;
    const uint4 *pair_hi;
    const void *alpha;
    const void *beta;
};

template <bool HALF>
__device__ __forceinline__ void load_scale2(const void *base, int64_t record, float &a0, float &a1) {
    if constexpr (HALF) {
        const __half2 v = __ldg(reinterpret_cast<const __half2 *>(base) + record);
        const float2 f = __half22float2(v);
        a0 = f.x;
        a1 = f.y;
    } else {
        const float2 v = __ldg(reinterpret_cast<const float2 *>(base) + record);
        a0 = v.x;
        a1 = v.y;
    }
}

// The same pair of scales from a shared-memory copy of the records.
template <bool HALF>
__device__ __forceinline__ void load_scale2_shared(const void *base, int record, float &a0, float &a1) {
    if constexpr (HALF) {
        const float2 f = __half22float2(reinterpret_cast<const __half2 *>(base)[record]);
        a0 = f.x;
        a1 = f.y;
    } else {
        const float2 v = reinterpret_cast<const float2 *>(base)[record];
        a0 = v.x;
        a1 = v.y;
    }
}

__device__ __forceinline__ bool row_flagged(const uint8_t *tiles, int row, int tile_rows) {
    return tiles != nullptr && tiles[row / tile_rows] != 0;
}

// Exact dot of one 32-code group in the pair layout (words lo = codes 0-15,
// hi = codes 16-31) with 8 natural-order activation words.
__device__ __forceinline__ int dot_pair(uint32_t lo, uint32_t hi, const uint4 &z0, const uint4 &z1) {
    constexpr uint32_t M = 0x03030303u;
    int a = __dp4a(int(lo & M), int(z0.x), 0);
    a = __dp4a(int((lo >> 2) & M), int(z0.y), a);
    a = __dp4a(int((lo >> 4) & M), int(z0.z), a);
    a = __dp4a(int((lo >> 6) & M), int(z0.w), a);
    a = __dp4a(int(hi & M), int(z1.x), a);
    a = __dp4a(int((hi >> 2) & M), int(z1.y), a);
    a = __dp4a(int((hi >> 4) & M), int(z1.z), a);
    a = __dp4a(int((hi >> 6) & M), int(z1.w), a);
    return a;
}

// Exact dot of one 32-code group in the plane layout with 8 activation words.
__device__ __forceinline__ int dot_plane(uint32_t w, const uint4 &z0, const uint4 &z1) {
    constexpr uint32_t M = 0x01010101u;
    int a = __dp4a(int(w & M), int(z0.x), 0);
    a = __dp4a(int((w >> 1) & M), int(z0.y), a);
    a = __dp4a(int((w >> 2) & M), int(z0.z), a);
    a = __dp4a(int((w >> 3) & M), int(z0.w), a);
    a = __dp4a(int((w >> 4) & M), int(z1.x), a);
    a = __dp4a(int((w >> 5) & M), int(z1.y), a);
    a = __dp4a(int((w >> 6) & M), int(z1.z), a);
    a = __dp4a(int((w >> 7) & M), int(z1.w), a);
    return a;
}

__global__ void cast_f16_kernel(const float *src, __half *dst, int64_t n) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}

}  // namespace ffnrm
