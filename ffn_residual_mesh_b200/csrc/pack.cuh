// Load-time repacking on the GPU: the reference's artifact formats -> the row-tiled
// device layouts of ffnrm_common.cuh.
//
// Inputs (device memory): per projection either full Q4 codes [F, D] (one byte each),
// QLO2 row-packed residual codes [F, D/4] (scripts/export_cuda_residual_artifact_v2.py:13-24)
// or r residual bit planes (scripts/compile_q4k_host_base_gpu_residual.py:17-26), plus
// optional (4 - r) high planes; alpha / beta [F, G] f32. Every kernel is a grid-stride
// loop over independent outputs, bounded by the buffer sizes it is given.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "ffnrm_common.cuh"

namespace ffnrm {

// Decode n codes of one projection: lo[i] = the r-bit residual code, and when `full` is
// non-null the complete Q4 code (from the full codes, or the low planes plus `high`).
// fmt: 0 full Q4 bytes, 1 QLO2 row-packed (r = 2), 2 bit planes. Q4 bytes above 15 set *bad.
__global__ void decode_codes_kernel(int fmt, const uint8_t *codes, const uint8_t *high, int r, int64_t n,
                                    uint8_t *lo, uint8_t *full, int *bad) {
    const uint8_t mask = uint8_t((1 << r) - 1);
    const int64_t plane = n / 8;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        uint8_t v;
        if (fmt == 0) {
            const uint8_t q = codes[i];
            if (q > 15) atomicOr(bad, 1);
            lo[i] = q & mask;
            if (full) full[i] = q;
            continue;
        }
        if (fmt == 1) {
            v = (codes[i >> 2] >> (2 * (i & 3))) & 3;
        } else {
            v = 0;
            for (int b = 0; b < r; ++b) v |= uint8_t(((codes[b * plane + (i >> 3)] >> (i & 7)) & 1) << b);
        }
        lo[i] = v;
        if (full) {
            uint8_t h = 0;
            for (int b = 0; b < 4 - r; ++b) h |= uint8_t(((high[b * plane + (i >> 3)] >> (i & 7)) & 1) << b);
            full[i] = uint8_t((h << r) | v);
        }
    }
}

// Pair records [F64][C][2][64][16 B] of bits shift..shift+1 of both projections' code
// bytes q0 (gate), q1 (up) [F, D]: word j of the record of (row, chunk c) holds group
// 2c + (j >> 1), codes 16 (j & 1) .. + 15, code 4i + b at bit 8b + 2i. Rows >= F are zero.
__global__ void pack_pair_kernel(const uint8_t *q0, const uint8_t *q1, int shift, int64_t F, int64_t D, uint4 *out) {
    const int64_t C = D / 64, n = (F + 63) / 64 * C * 128;
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < n; idx += int64_t(gridDim.x) * blockDim.x) {
        const int64_t rt = idx / (C * 128), rem = idx - rt * C * 128, c = rem / 128;
        const int k = int(rem - c * 128), proj = k >> 6;
        const int64_t row = rt * 64 + (k & 63);
        uint32_t w[4] = {0, 0, 0, 0};
        if (row < F) {
            const uint8_t *codes = (proj ? q1 : q0) + row * D + 64 * c;
            for (int j = 0; j < 4; ++j)
                for (int i = 0; i < 4; ++i)
                    for (int b = 0; b < 4; ++b) w[j] |= uint32_t((codes[16 * j + 4 * i + b] >> shift) & 3) << (8 * b + 2 * i);
        }
        out[idx] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// Plane records [F64][C][2][64][8 B] of bit `bit`: word j holds group 2c + j, code 4i + b
// at bit 8b + i.
__global__ void pack_plane_kernel(const uint8_t *q0, const uint8_t *q1, int bit, int64_t F, int64_t D, uint2 *out) {
    const int64_t C = D / 64, n = (F + 63) / 64 * C * 128;
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < n; idx += int64_t(gridDim.x) * blockDim.x) {
        const int64_t rt = idx / (C * 128), rem = idx - rt * C * 128, c = rem / 128;
        const int k = int(rem - c * 128), proj = k >> 6;
        const int64_t row = rt * 64 + (k & 63);
        uint32_t w[2] = {0, 0};
        if (row < F) {
            const uint8_t *codes = (proj ? q1 : q0) + row * D + 64 * c;
            for (int j = 0; j < 2; ++j)
                for (int i = 0; i < 8; ++i)
                    for (int b = 0; b < 4; ++b) w[j] |= uint32_t((codes[32 * j + 4 * i + b] >> bit) & 1) << (8 * b + i);
        }
        out[idx] = make_uint2(w[0], w[1]);
    }
}

// Both projections' per-group scales [F, G] -> [F64][C][2][64][2] (fp16 when `half`).
__global__ void pack_scales_kernel(const float *v0, const float *v1, int64_t F, int64_t G, int half, void *out) {
    const int64_t C = G / 2, n = (F + 63) / 64 * C * 128;
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < n; idx += int64_t(gridDim.x) * blockDim.x) {
        const int64_t rt = idx / (C * 128), rem = idx - rt * C * 128, c = rem / 128;
        const int k = int(rem - c * 128), proj = k >> 6;
        const int64_t row = rt * 64 + (k & 63);
        float a = 0.f, b = 0.f;
        if (row < F) {
            const float *v = (proj ? v1 : v0) + row * G + 2 * c;
            a = v[0];
            b = v[1];
        }
        if (half)
            reinterpret_cast<__half2 *>(out)[idx] = __floats2half2_rn(a, b);
        else
            reinterpret_cast<float2 *>(out)[idx] = make_float2(a, b);
    }
}

// *flag = 1 if some value is not exactly representable in fp16 (NaNs compare as equal).
__global__ void half_exact_kernel(const float *v, int64_t n, int *flag) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const float x = v[i], back = __half2float(__float2half_rn(x));
        if (!(back == x) && !(isnan(x) && isnan(back))) atomicOr(flag, 1);
    }
}

// Byte codes [F64 * 128][D] for the byte-code tensor-core kernel: row 128 rt + 64 proj + r
// = code row 64 rt + r of projection proj (zero past F).
__global__ void pack_codes8_kernel(const uint8_t *q0, const uint8_t *q1, int64_t F, int64_t D, uint4 *out) {
    const int64_t v = D / 16, n = (F + 63) / 64 * 128 * v;
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < n; idx += int64_t(gridDim.x) * blockDim.x) {
        const int64_t orow = idx / v, col = idx - orow * v;
        const int64_t rt = orow / 128, k = orow - rt * 128, row = rt * 64 + (k & 63);
        uint4 x = make_uint4(0, 0, 0, 0);
        if (row < F) x = reinterpret_cast<const uint4 *>((k >> 6 ? q1 : q0) + row * D)[col];
        out[idx] = x;
    }
}

}  // namespace ffnrm
