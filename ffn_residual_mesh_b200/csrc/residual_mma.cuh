// Residual contraction on tensor cores for token batches (T >= 5): exact int32
// group dots with mma.sync m16n8k32 (u8 codes x s8 activations -> s32).
//
// Each 32-code group is exactly one K=32 MMA step, so every MMA result is an exact
// integer group dot P[row, token, g]; the per-group scale alpha[row,g]*s[token,g]
// is applied in fp32 on the accumulator fragment before the next group. The A
// fragment (16 rows x 32 codes) comes straight from the interleaved code records:
// for lane (g = lane/4, t = lane%4), (word >> 2t) & 0x03030303 holds the codes
// 4t..4t+3 of a row, which is the m16n8k32 A register layout. r = 1 and r = 3
// build the same bytes from the bit plane; fallback rows add the high pair
// (q = pair + 4*pair_hi) so one MMA still gives the unsplit dot.
//
// A warp owns one 32-row block (two M tiles) for all tokens of the CTA's token
// tile (NT tiles of 8 tokens); the CTA's warps share activations staged in shared
// memory one K chunk at a time (double-buffered cp.async), so activations cross L2
// once per CTA rather than once per row.
#pragma once

#include "ffnrm_common.cuh"
#include "residual_dp4a.cuh"

namespace ffnrm {

constexpr int kMmaKChunk = 256;             // activations staged per K chunk (codes)
constexpr int kMmaZStride = kMmaKChunk + 16;  // padded row stride in bytes (bank spread)

__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src, bool valid) {
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    const int bytes = valid ? 16 : 0;  // zero-fill when the token is past T
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(gmem_src), "r"(bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Codes 4t..4t+3 (lo half) and 16+4t..16+4t+3 (hi half) of one row and group as u8 bytes.
template <int RB>
__device__ __forceinline__ void group_codes(uint32_t lo, uint32_t hi, uint32_t plane, int t, uint32_t &k0,
                                            uint32_t &k1) {
    constexpr uint32_t M2 = 0x03030303u, M1 = 0x01010101u;
    if (RB == 1) {
        k0 = (plane >> t) & M1;
        k1 = (plane >> (4 + t)) & M1;
    } else {
        k0 = (lo >> (2 * t)) & M2;
        k1 = (hi >> (2 * t)) & M2;
        if (RB == 3) {
            k0 |= ((plane >> t) & M1) << 2;
            k1 |= ((plane >> (4 + t)) & M1) << 2;
        }
    }
}

// Shared memory: [z 2 x TN x kMmaZStride int8][s G x TN f32][zsum G x TN f32 (fallback)]
inline size_t residual_mma_smem_bytes(int TN, int G, bool fallback) {
    return size_t(2) * TN * kMmaZStride + size_t(G) * TN * 4 * (fallback ? 2 : 1);
}

template <int RB, int NT, bool AHALF, bool FB>
__global__ void __launch_bounds__(128) residual_mma_kernel(const ResidualParams p) {
    constexpr int TN = NT * 8;
    extern __shared__ __align__(16) uint8_t smem[];
    const int G = p.G, D = p.D, F = p.F, T = p.T;
    int8_t *z_sm = reinterpret_cast<int8_t *>(smem);
    float *s_sm = reinterpret_cast<float *>(smem + size_t(2) * TN * kMmaZStride);  // [G][TN]
    float *zsum_sm = s_sm + G * TN;                                               // [G][TN]

    const int warps = blockDim.x >> 5;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int t0 = blockIdx.y * TN;
    const int blocks_per_proj = (p.row_blocks + warps - 1) / warps;
    const int proj = blockIdx.x / blocks_per_proj;
    const int rb = (blockIdx.x - proj * blocks_per_proj) * warps + warp;
    const bool active = rb < p.row_blocks;
    const ProjView pv = p.proj[proj];

    // Per-token group scales (and group sums for fallback rows), [G][TN].
    for (int i = threadIdx.x; i < G * TN; i += blockDim.x) {
        const int gg = i / TN, tok = i - gg * TN;
        float sv = 0.f, zs = 0.f;
        if (t0 + tok < T) {
            sv = p.s[int64_t(t0 + tok) * G + gg];
            if (FB) {
                const int8_t *zr = p.z + int64_t(t0 + tok) * D + gg * kGroup;
                int a = 0;
                for (int k = 0; k < kGroup; ++k) a += zr[k];
                zs = float(a);
            }
        }
        s_sm[i] = sv;
        if (FB) zsum_sm[i] = zs;
    }

    auto stage = [&](int kc, int buf) {
        // TN tokens x kMmaKChunk activations -> z_sm[buf], 16 bytes per copy
        const int per_row = kMmaKChunk / 16;
        for (int i = threadIdx.x; i < TN * per_row; i += blockDim.x) {
            const int tok = i / per_row, v = i - tok * per_row;
            const bool ok = t0 + tok < T;
            const int8_t *src = p.z + int64_t(ok ? t0 + tok : 0) * D + kc + v * 16;
            cp_async16(z_sm + (size_t(buf) * TN + tok) * kMmaZStride + v * 16, src, ok);
        }
        cp_async_commit();
    };

    // Rows of this lane: r[0] = g, r[1] = g+8 (M tile 0), r[2] = g+16, r[3] = g+24 (M tile 1)
    int row[4];
    bool flag[4];
    bool any_flag = false;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        row[i] = rb * 32 + g + 8 * i;
        flag[i] = FB && active && row[i] < F && row_flagged(p.fallback_tiles, row[i], p.tile_rows);
        any_flag |= flag[i];
    }
    if (FB) any_flag = __any_sync(0xffffffffu, any_flag);

    float acc[2][NT][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[m][n][e] = 0.f;

    const int C = G / 2;
    const int nchunks = D / kMmaKChunk;
    stage(0, 0);
    for (int kc = 0; kc < nchunks; ++kc) {
        if (kc + 1 < nchunks) {
            stage((kc + 1) * kMmaKChunk, (kc + 1) & 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const int8_t *zb = z_sm + size_t(kc & 1) * TN * kMmaZStride;
        if (active) {
#pragma unroll 1
            for (int cl = 0; cl < kMmaKChunk / 64; ++cl) {
                const int c = kc * (kMmaKChunk / 64) + cl;  // chunk of two groups
                const int64_t rec = (int64_t(rb) * C + c) * 32;
                uint4 L[4], H[4];
                uint2 Q[4];
                float a[4][2], b[4][2];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int ri = g + 8 * i;
                    L[i] = RB != 1 || (FB && any_flag) ? __ldg(pv.pair + rec + ri) : make_uint4(0, 0, 0, 0);
                    Q[i] = RB != 2 ? __ldg(pv.plane + rec + ri) : make_uint2(0, 0);
                    load_scale2<AHALF>(pv.alpha, rec + ri, a[i][0], a[i][1]);
                    if (FB && any_flag) {
                        H[i] = __ldg(pv.pair_hi + rec + ri);
                        load_scale2<AHALF>(pv.beta, rec + ri, b[i][0], b[i][1]);
                    } else {
                        H[i] = make_uint4(0, 0, 0, 0);
                        b[i][0] = b[i][1] = 0.f;
                    }
                }
#pragma unroll
                for (int j = 0; j < 2; ++j) {  // group 2c + j
                    const int grp = 2 * c + j;
                    uint32_t A[2][4], AF[2][4];
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
#pragma unroll
                        for (int h = 0; h < 2; ++h) {  // h = 0: row g(+16m), h = 1: row g+8(+16m)
                            const int i = 2 * m + h;
                            const uint32_t lo = j ? L[i].z : L[i].x, hi = j ? L[i].w : L[i].y;
                            const uint32_t pl = j ? Q[i].y : Q[i].x;
                            uint32_t k0, k1;
                            group_codes<RB>(lo, hi, pl, t, k0, k1);
                            A[m][h] = k0;      // a0 / a1: codes 4t..4t+3
                            A[m][2 + h] = k1;  // a2 / a3: codes 16+4t..
                            if (FB && any_flag) {
                                const uint32_t hlo = j ? H[i].z : H[i].x, hhi = j ? H[i].w : H[i].y;
                                constexpr uint32_t M2 = 0x03030303u;
                                uint32_t f0, f1;
                                group_codes<2>(lo, hi, 0, t, f0, f1);
                                AF[m][h] = f0 | (((hlo >> (2 * t)) & M2) << 2);
                                AF[m][2 + h] = f1 | (((hhi >> (2 * t)) & M2) << 2);
                            }
                        }
                    }
                    const int kk = cl * 64 + 32 * j;  // offset inside the staged chunk
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        const int8_t *zr = zb + (n * 8 + g) * kMmaZStride + kk + 4 * t;
                        const uint32_t b0 = *reinterpret_cast<const uint32_t *>(zr);
                        const uint32_t b1 = *reinterpret_cast<const uint32_t *>(zr + 16);
                        const float2 sv = *reinterpret_cast<const float2 *>(s_sm + grp * TN + n * 8 + 2 * t);
#pragma unroll
                        for (int m = 0; m < 2; ++m) {
                            int d[4];
                            mma_u8s8(d, A[m], b0, b1);
                            const float ar0 = a[2 * m][j], ar1 = a[2 * m + 1][j];
                            if (p.dots != nullptr) {
                                const int tk = t0 + n * 8 + 2 * t;
                                const int r0 = row[2 * m], r1 = row[2 * m + 1];
                                int32_t *dp = p.dots + int64_t(proj) * T * F * G;
                                if (r0 < F && tk < T) dp[(int64_t(tk) * F + r0) * G + grp] = d[0];
                                if (r0 < F && tk + 1 < T) dp[(int64_t(tk + 1) * F + r0) * G + grp] = d[1];
                                if (r1 < F && tk < T) dp[(int64_t(tk) * F + r1) * G + grp] = d[2];
                                if (r1 < F && tk + 1 < T) dp[(int64_t(tk + 1) * F + r1) * G + grp] = d[3];
                            }
                            if (FB && any_flag && (flag[2 * m] || flag[2 * m + 1])) {
                                int e[4];
                                mma_u8s8(e, AF[m], b0, b1);
                                const float2 zs = *reinterpret_cast<const float2 *>(zsum_sm + grp * TN + n * 8 + 2 * t);
                                const float br0 = b[2 * m][j], br1 = b[2 * m + 1][j];
                                if (flag[2 * m]) {
                                    acc[m][n][0] += sv.x * (ar0 * float(e[0]) + br0 * zs.x);
                                    acc[m][n][1] += sv.y * (ar0 * float(e[1]) + br0 * zs.y);
                                } else {
                                    acc[m][n][0] = fmaf(float(d[0]), ar0 * sv.x, acc[m][n][0]);
                                    acc[m][n][1] = fmaf(float(d[1]), ar0 * sv.y, acc[m][n][1]);
                                }
                                if (flag[2 * m + 1]) {
                                    acc[m][n][2] += sv.x * (ar1 * float(e[2]) + br1 * zs.x);
                                    acc[m][n][3] += sv.y * (ar1 * float(e[3]) + br1 * zs.y);
                                } else {
                                    acc[m][n][2] = fmaf(float(d[2]), ar1 * sv.x, acc[m][n][2]);
                                    acc[m][n][3] = fmaf(float(d[3]), ar1 * sv.y, acc[m][n][3]);
                                }
                            } else {
                                acc[m][n][0] = fmaf(float(d[0]), ar0 * sv.x, acc[m][n][0]);
                                acc[m][n][1] = fmaf(float(d[1]), ar0 * sv.y, acc[m][n][1]);
                                acc[m][n][2] = fmaf(float(d[2]), ar1 * sv.x, acc[m][n][2]);
                                acc[m][n][3] = fmaf(float(d[3]), ar1 * sv.y, acc[m][n][3]);
                            }
                        }
                    }
                }
            }
        }
        __syncthreads();  // the buffer just read is refilled by the next iteration's stage
    }
    if (!active) return;
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        const int r0 = row[2 * m], r1 = row[2 * m + 1];
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int tk = t0 + n * 8 + 2 * t;
            float *out = p.out[proj];
            if (r0 < F && tk < T) out[int64_t(tk) * F + r0] = acc[m][n][0];
            if (r0 < F && tk + 1 < T) out[int64_t(tk + 1) * F + r0] = acc[m][n][1];
            if (r1 < F && tk < T) out[int64_t(tk) * F + r1] = acc[m][n][2];
            if (r1 < F && tk + 1 < T) out[int64_t(tk + 1) * F + r1] = acc[m][n][3];
        }
    }
}

}  // namespace ffnrm
