// Decode residual contraction on CUDA cores: exact int32 group dots with __dp4a,
// warp-shuffle reductions, gate and up in one launch.
//
// Replaces residual_kernel (src/exact_residual_cuda_runner.cu:122-159), which
// evaluates q*alpha*z*s per element in fp32 with byte loads and a shared-memory
// tree. Here each warp owns R rows; its lanes stream 16-byte chunks of packed codes
// (two 32-code groups) with 128-bit loads, unpack them with shift/mask into dp4a
// operands, and accumulate each group dot exactly in int32 before applying
// alpha[row,g]*s[t,g] in fp32. The permuted activations live in shared memory and
// are read once per chunk for all R rows. Rows in flagged fallback tiles compute the
// unsplit projection  sum_g s*(alpha*(P01 + 4*P23) + beta*zsum)  instead.
#pragma once

#include "ffnrm_common.cuh"

namespace ffnrm {

struct ResidualParams {
    ProjView proj[2];
    const int8_t *z;      // [T, D]
    const float *s;       // [T, G]
    float *out[2];        // [T, F]
    int32_t *dots;        // [2, T, F, G] or null
    const uint8_t *fallback_tiles;
    int F, D, G, T, tile_rows;
    int row_blocks;       // CTAs per projection
    int need_pair, need_plane;
};

__device__ __forceinline__ uint32_t pack4(int8_t a, int8_t b, int8_t c, int8_t d) {
    return uint32_t(uint8_t(a)) | (uint32_t(uint8_t(b)) << 8) | (uint32_t(uint8_t(c)) << 16) |
           (uint32_t(uint8_t(d)) << 24);
}

// Group dot of one 32-code group in pair layout: words w0 (codes 0-15), w1 (16-31).
__device__ __forceinline__ int dot_pair(uint32_t w0, uint32_t w1, const uint4 &za, const uint4 &zb) {
    constexpr uint32_t M = 0x03030303u;
    int acc = __dp4a(int(w0 & M), int(za.x), 0);
    acc = __dp4a(int((w0 >> 2) & M), int(za.y), acc);
    acc = __dp4a(int((w0 >> 4) & M), int(za.z), acc);
    acc = __dp4a(int((w0 >> 6) & M), int(za.w), acc);
    acc = __dp4a(int(w1 & M), int(zb.x), acc);
    acc = __dp4a(int((w1 >> 2) & M), int(zb.y), acc);
    acc = __dp4a(int((w1 >> 4) & M), int(zb.z), acc);
    acc = __dp4a(int((w1 >> 6) & M), int(zb.w), acc);
    return acc;
}

// Group dot of one 32-code group in plane layout (one bit per code).
__device__ __forceinline__ int dot_plane(uint32_t w, const uint4 &za, const uint4 &zb) {
    constexpr uint32_t M = 0x01010101u;
    int acc = __dp4a(int(w & M), int(za.x), 0);
    acc = __dp4a(int((w >> 1) & M), int(za.y), acc);
    acc = __dp4a(int((w >> 2) & M), int(za.z), acc);
    acc = __dp4a(int((w >> 3) & M), int(za.w), acc);
    acc = __dp4a(int((w >> 4) & M), int(zb.x), acc);
    acc = __dp4a(int((w >> 5) & M), int(zb.y), acc);
    acc = __dp4a(int((w >> 6) & M), int(zb.z), acc);
    acc = __dp4a(int((w >> 7) & M), int(zb.w), acc);
    return acc;
}

// Shared memory: [zpair TT*G*8 u32][zplane TT*G*8 u32][s TT*G f32][zsum TT*G f32]
inline size_t residual_smem_bytes(int TT, int G, bool need_pair, bool need_plane) {
    return size_t(TT) * G * (8 * 4 * (int(need_pair) + int(need_plane)) + 8);
}

template <int RB, int TT, int R, bool AHALF>
__global__ void __launch_bounds__(256) residual_dp4a_kernel(const ResidualParams p) {
    extern __shared__ __align__(16) uint32_t smem[];
    const int G = p.G, D = p.D, F = p.F, T = p.T;
    const int words = G * 8;
    uint32_t *zpair = smem;
    uint32_t *zplane = zpair + (p.need_pair ? TT * words : 0);
    float *s_sm = reinterpret_cast<float *>(zplane + (p.need_plane ? TT * words : 0));
    float *zsum_sm = s_sm + TT * G;

    const int proj = blockIdx.x / p.row_blocks;
    const int rb = blockIdx.x - proj * p.row_blocks;
    const int t0 = blockIdx.y * TT;

    // Stage the activations of TT tokens, permuted to the dp4a operand order.
    for (int idx = threadIdx.x; idx < TT * words; idx += blockDim.x) {
        const int t = idx / words, w = idx - t * words;
        const int g = w >> 3, sub = w & 7;
        uint32_t vp = 0, vq = 0;
        if (t0 + t < T) {
            const int8_t *zr = p.z + int64_t(t0 + t) * D + g * kGroup;
            if (p.need_pair) {
                const int m = sub >> 2, i = sub & 3;
                vp = pack4(zr[16 * m + i], zr[16 * m + 4 + i], zr[16 * m + 8 + i], zr[16 * m + 12 + i]);
            }
            if (p.need_plane) vq = pack4(zr[sub], zr[8 + sub], zr[16 + sub], zr[24 + sub]);
        }
        if (p.need_pair) zpair[idx] = vp;
        if (p.need_plane) zplane[idx] = vq;
    }
    for (int idx = threadIdx.x; idx < TT * G; idx += blockDim.x) {
        const int t = idx / G, g = idx - t * G;
        float sv = 0.f, zs = 0.f;
        if (t0 + t < T) {
            sv = p.s[int64_t(t0 + t) * G + g];
            if (p.fallback_tiles) {
                const int8_t *zr = p.z + int64_t(t0 + t) * D + g * kGroup;
                int acc = 0;
                for (int i = 0; i < kGroup; ++i) acc += zr[i];
                zs = float(acc);
            }
        }
        s_sm[idx] = sv;
        zsum_sm[idx] = zs;
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (rb * (blockDim.x >> 5) + warp) * R;
    if (row0 >= F) return;
    const ProjView pv = p.proj[proj];
    const int pair_bytes = D / 4, plane_bytes = D / 8;

    bool flag[R];
    bool any_flag = false;
#pragma unroll
    for (int j = 0; j < R; ++j) {
        flag[j] = (row0 + j < F) && row_flagged(p.fallback_tiles, row0 + j, p.tile_rows);
        any_flag |= flag[j];
    }

    float acc[R][TT];
#pragma unroll
    for (int j = 0; j < R; ++j)
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[j][t] = 0.f;

    const int chunks = G / 2;
    for (int c = lane; c < chunks; c += 32) {
        uint4 wp[R], wh[R];
        uint2 wq[R];
        float a0[R], a1[R], b0[R], b1[R];
#pragma unroll
        for (int j = 0; j < R; ++j) {
            const int row = row0 + j;
            const bool valid = row < F;
            wp[j] = make_uint4(0, 0, 0, 0);
            wh[j] = make_uint4(0, 0, 0, 0);
            wq[j] = make_uint2(0, 0);
            a0[j] = a1[j] = b0[j] = b1[j] = 0.f;
            if (valid) {
                if (RB != 1 || flag[j])
                    wp[j] = __ldg(reinterpret_cast<const uint4 *>(pv.pair + int64_t(row) * pair_bytes) + c);
                if (RB != 2)
                    wq[j] = __ldg(reinterpret_cast<const uint2 *>(pv.plane + int64_t(row) * plane_bytes) + c);
                load_scale2<AHALF>(pv.alpha, int64_t(row) * G + 2 * c, a0[j], a1[j]);
                if (flag[j]) {
                    wh[j] = __ldg(reinterpret_cast<const uint4 *>(pv.pair_hi + int64_t(row) * pair_bytes) + c);
                    load_scale2<AHALF>(pv.beta, int64_t(row) * G + 2 * c, b0[j], b1[j]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            uint4 zp0 = make_uint4(0, 0, 0, 0), zp1 = zp0, zp2 = zp0, zp3 = zp0;
            uint4 zq0 = zp0, zq1 = zp0, zq2 = zp0, zq3 = zp0;
            if (RB != 1 || any_flag) {
                const uint4 *src = reinterpret_cast<const uint4 *>(zpair + t * words + 2 * c * 8);
                zp0 = src[0];
                zp1 = src[1];
                zp2 = src[2];
                zp3 = src[3];
            }
            if (RB != 2) {
                const uint4 *src = reinterpret_cast<const uint4 *>(zplane + t * words + 2 * c * 8);
                zq0 = src[0];
                zq1 = src[1];
                zq2 = src[2];
                zq3 = src[3];
            }
            const float s0 = s_sm[t * G + 2 * c], s1 = s_sm[t * G + 2 * c + 1];
#pragma unroll
            for (int j = 0; j < R; ++j) {
                int P0 = 0, P1 = 0;
                if (RB != 1) {
                    P0 = dot_pair(wp[j].x, wp[j].y, zp0, zp1);
                    P1 = dot_pair(wp[j].z, wp[j].w, zp2, zp3);
                }
                if (RB == 1) {
                    P0 = dot_plane(wq[j].x, zq0, zq1);
                    P1 = dot_plane(wq[j].y, zq2, zq3);
                }
                if (RB == 3) {
                    P0 += 4 * dot_plane(wq[j].x, zq0, zq1);
                    P1 += 4 * dot_plane(wq[j].y, zq2, zq3);
                }
                const int row = row0 + j;
                if (p.dots != nullptr && row < F && t0 + t < T)
                    *reinterpret_cast<int2 *>(p.dots + ((int64_t(proj) * T + t0 + t) * F + row) * G + 2 * c) =
                        make_int2(P0, P1);
                if (flag[j]) {
                    const int F0 = dot_pair(wp[j].x, wp[j].y, zp0, zp1) + 4 * dot_pair(wh[j].x, wh[j].y, zp0, zp1);
                    const int F1 = dot_pair(wp[j].z, wp[j].w, zp2, zp3) + 4 * dot_pair(wh[j].z, wh[j].w, zp2, zp3);
                    const float zs0 = zsum_sm[t * G + 2 * c], zs1 = zsum_sm[t * G + 2 * c + 1];
                    acc[j][t] += s0 * (a0[j] * float(F0) + b0[j] * zs0) + s1 * (a1[j] * float(F1) + b1[j] * zs1);
                } else {
                    acc[j][t] = fmaf(float(P0), a0[j] * s0, acc[j][t]);
                    acc[j][t] = fmaf(float(P1), a1[j] * s1, acc[j][t]);
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < R; ++j) {
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            const float v = warp_sum(acc[j][t]);
            if (lane == 0 && row0 + j < F && t0 + t < T) p.out[proj][int64_t(t0 + t) * F + row0 + j] = v;
        }
    }
}

}  // namespace ffnrm
