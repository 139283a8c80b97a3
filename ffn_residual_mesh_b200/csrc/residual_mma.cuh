// Residual contraction on tensor cores for token batches (T >= 5): exact int32
// group dots with mma.sync m16n8k32 (u8 codes x s8 activations -> s32).
//
// Each 32-code group is exactly one K=32 MMA step, so every MMA result is an exact
// integer group dot P[row, token, g]; the per-group scale alpha[row,g]*s[token,g]
// is applied in fp32 on the accumulator fragment before the next group. The A
// fragment (16 rows x 32 codes) comes straight from the interleaved code records:
// for lane (g = lane/4, t = lane%4), (word >> 2t) & 0x03030303 holds codes 4t..4t+3
// of a row, which is the m16n8k32 A register layout. r = 1 and r = 3 build the same
// bytes from the bit plane; fallback rows add the high pair (q = pair + 4*pair_hi)
// so one MMA still gives the unsplit dot.
//
// CTA = 4 warps: warps 0/1 take the gate rows of two 32-row blocks, warps 2/3 the up
// rows of the same blocks, all for one tile of TN = 8*NT tokens. Codes, scales and
// activations of each K chunk (kMmaKChunk codes) are staged into shared memory by
// cp.async, kMmaStages deep, so HBM latency overlaps the MMAs. In forward mode the up
// warps hand their accumulators to the gate warps through shared memory and the gate
// warps merge with the base sums and write h = SiLU(g)*u.
#pragma once

#include "ffnrm_common.cuh"
#include "residual_dp4a.cuh"

namespace ffnrm {

constexpr int kMmaKChunk = 256;               // codes per staged K chunk (8 groups)
constexpr int kMmaZStride = kMmaKChunk + 16;  // padded activation row stride in bytes
constexpr int kMmaStages = 3;
constexpr int kMmaChunks = kMmaKChunk / 64;   // 2-group records per row per K chunk

__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Codes 4t..4t+3 (k0) and 16+4t..16+4t+3 (k1) of one row and group as u8 bytes.
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

// Per-stage bytes for one 32-row block: pair records, plane records, scales.
template <int RB, bool AHALF>
struct StageLayout {
    static constexpr int pair = RB != 1 ? kMmaChunks * 32 * 16 : 0;
    static constexpr int plane = RB != 2 ? kMmaChunks * 32 * 8 : 0;
    static constexpr int alpha = kMmaChunks * 32 * (AHALF ? 4 : 8);
    static constexpr int block = pair + plane + alpha;
};

template <int RB, bool AHALF>
inline size_t residual_mma_smem_bytes(int TN, int G, bool fallback) {
    const size_t stage = size_t(TN) * kMmaZStride + 4 * StageLayout<RB, AHALF>::block;
    const size_t xch = size_t(TN) * 256;  // 2 blocks x 2 M tiles x NT x 4 values x 32 lanes x 4 B
    return kMmaStages * stage + size_t(G) * TN * 4 * (fallback ? 2 : 1) + xch;
}

template <int RB, int NT, bool AHALF, bool FB>
__global__ void __launch_bounds__(128) residual_mma_kernel(const ResidualParams p) {
    constexpr int TN = NT * 8;
    using SL = StageLayout<RB, AHALF>;
    extern __shared__ __align__(16) uint8_t smem[];
    const int G = p.G, D = p.D, F = p.F, T = p.T;
    const size_t stage_bytes = size_t(TN) * kMmaZStride + 4 * SL::block;
    float *s_sm = reinterpret_cast<float *>(smem + kMmaStages * stage_bytes);  // [G][TN]
    float *zsum_sm = s_sm + G * TN;                                           // [G][TN] (fallback)
    float *xch = zsum_sm + (FB ? G * TN : 0);                                 // [2 blocks][2*NT*4][32]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int proj = warp >> 1, lb = warp & 1;
    const int t0 = blockIdx.y * TN;
    const int rb0 = blockIdx.x * 2;
    const int rb = rb0 + lb;
    const bool active = rb < p.row_blocks;
    const ProjView pv = p.proj[proj];
    const int C = G / 2;

    // Group scales (and group sums for fallback rows), coalesced reads, [G][TN] in smem.
    for (int i = threadIdx.x; i < G * TN; i += blockDim.x) {
        const int tok = i / G, gg = i - tok * G;
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
        s_sm[gg * TN + tok] = sv;
        if (FB) zsum_sm[gg * TN + tok] = zs;
    }

    // Stage K chunk kc: activations [TN][kMmaKChunk] and, for each of the 4 warp slots
    // (proj, block), the contiguous code/scale records of chunks kc*4 .. kc*4+3.
    auto stage = [&](int kc, int buf) {
        uint8_t *base = smem + size_t(buf) * stage_bytes;
        constexpr int zv = kMmaKChunk / 16;
        for (int i = threadIdx.x; i < TN * zv; i += blockDim.x) {
            const int tok = i / zv, v = i - tok * zv;
            const bool ok = t0 + tok < T;
            cp_async16(base + tok * kMmaZStride + v * 16,
                       p.z + int64_t(ok ? t0 + tok : 0) * D + kc * kMmaKChunk + v * 16, ok);
        }
        uint8_t *rec_base = base + TN * kMmaZStride;
        constexpr int per_slot = SL::block / 16;
        for (int i = threadIdx.x; i < 4 * per_slot; i += blockDim.x) {
            const int slot = i / per_slot, off = (i - slot * per_slot) * 16;
            const int sp = slot >> 1, sb = rb0 + (slot & 1);
            const bool ok = sb < p.row_blocks;
            const ProjView &q = p.proj[sp];
            // each chunk's 32 records are contiguous; consecutive chunks are a tile apart
            const uint8_t *src;
            if (off < SL::pair) {
                const int cl = off / 512;
                src = reinterpret_cast<const uint8_t *>(q.pair + rec_index(ok ? sb : 0, C, kc * kMmaChunks + cl, 0)) +
                      (off - cl * 512);
            } else if (off < SL::pair + SL::plane) {
                const int o = off - SL::pair, cl = o / 256;
                src = reinterpret_cast<const uint8_t *>(q.plane + rec_index(ok ? sb : 0, C, kc * kMmaChunks + cl, 0)) +
                      (o - cl * 256);
            } else {
                constexpr int rb_ = AHALF ? 4 : 8, cb = 32 * rb_;
                const int o = off - SL::pair - SL::plane, cl = o / cb;
                src = reinterpret_cast<const uint8_t *>(q.alpha) +
                      rec_index(ok ? sb : 0, C, kc * kMmaChunks + cl, 0) * rb_ + (o - cl * cb);
            }
            cp_async16(rec_base + slot * SL::block + off, src, ok);
        }
        cp_async_commit();
    };

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

    const int nk = D / kMmaKChunk;
#pragma unroll
    for (int sgi = 0; sgi < kMmaStages - 1; ++sgi) {
        if (sgi < nk) stage(sgi, sgi);
        else cp_async_commit();
    }
    for (int kc = 0; kc < nk; ++kc) {
        cp_async_wait<kMmaStages - 2>();
        __syncthreads();
        {
            const int nxt = kc + kMmaStages - 1;
            if (nxt < nk) stage(nxt, nxt % kMmaStages);
            else cp_async_commit();
        }
        const uint8_t *base = smem + size_t(kc % kMmaStages) * stage_bytes;
        const int8_t *zb = reinterpret_cast<const int8_t *>(base);
        const uint8_t *mine = base + TN * kMmaZStride + (proj * 2 + lb) * SL::block;
        if (active) {
#pragma unroll 1
            for (int cl = 0; cl < kMmaChunks; ++cl) {
                const int c = kc * kMmaChunks + cl;
                uint4 L[4], H[4];
                uint2 Q[4];
                float a[4][2], b[4][2];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int rec = cl * 32 + g + 8 * i;
                    L[i] = RB != 1 ? reinterpret_cast<const uint4 *>(mine)[rec] : make_uint4(0, 0, 0, 0);
                    Q[i] = RB != 2 ? reinterpret_cast<const uint2 *>(mine + SL::pair)[rec] : make_uint2(0, 0);
                    if (AHALF) {
                        const float2 f = __half22float2(reinterpret_cast<const __half2 *>(mine + SL::pair + SL::plane)[rec]);
                        a[i][0] = f.x;
                        a[i][1] = f.y;
                    } else {
                        const float2 f = reinterpret_cast<const float2 *>(mine + SL::pair + SL::plane)[rec];
                        a[i][0] = f.x;
                        a[i][1] = f.y;
                    }
                    H[i] = make_uint4(0, 0, 0, 0);
                    b[i][0] = b[i][1] = 0.f;
                    if (FB && any_flag) {
                        const int64_t grec = rec_index(rb, C, c, g + 8 * i);
                        if (RB == 1) L[i] = __ldg(pv.pair + grec);
                        H[i] = __ldg(pv.pair_hi + grec);
                        load_scale2<AHALF>(pv.beta, grec, b[i][0], b[i][1]);
                    }
                }
#pragma unroll 1
                for (int j = 0; j < 2; ++j) {  // group 2c + j
                    const int grp = 2 * c + j;
                    uint32_t A[2][4], AF[2][4];
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
#pragma unroll
                        for (int h = 0; h < 2; ++h) {  // h = 0: row g (+16m), h = 1: row g+8 (+16m)
                            const int i = 2 * m + h;
                            const uint32_t lo = j ? L[i].z : L[i].x, hi = j ? L[i].w : L[i].y;
                            const uint32_t pl = j ? Q[i].y : Q[i].x;
                            uint32_t k0, k1;
                            group_codes<RB>(lo, hi, pl, t, k0, k1);
                            A[m][h] = k0;
                            A[m][2 + h] = k1;
                            if (FB && any_flag) {
                                constexpr uint32_t M2 = 0x03030303u;
                                const uint32_t hlo = j ? H[i].z : H[i].x, hhi = j ? H[i].w : H[i].y;
                                AF[m][h] = ((lo >> (2 * t)) & M2) | (((hlo >> (2 * t)) & M2) << 2);
                                AF[m][2 + h] = ((hi >> (2 * t)) & M2) | (((hhi >> (2 * t)) & M2) << 2);
                            } else {
                                AF[m][h] = AF[m][2 + h] = 0;
                            }
                        }
                    }
                    const int kk = cl * 64 + 32 * j;
                    const float ar[4] = {j ? a[0][1] : a[0][0], j ? a[1][1] : a[1][0], j ? a[2][1] : a[2][0],
                                         j ? a[3][1] : a[3][0]};
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
                            const float ar0 = ar[2 * m], ar1 = ar[2 * m + 1];
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
                                const float br0 = j ? b[2 * m][1] : b[2 * m][0];
                                const float br1 = j ? b[2 * m + 1][1] : b[2 * m + 1][0];
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
    }
    cp_async_wait<0>();

    if (p.h_hi == nullptr) {  // residual mode: every warp writes its own projection
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
        return;
    }
    // forward mode: up warps hand their fragments over, gate warps merge and write h
    float *mine_x = xch + lb * (2 * NT * 4 * 32);
    if (proj == 1) {
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) mine_x[((m * NT + n) * 4 + e) * 32 + lane] = acc[m][n][e];
    }
    __syncthreads();
    if (proj == 1 || !active) return;
#pragma unroll
    for (int m = 0; m < 2; ++m) {
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int tk = t0 + n * 8 + 2 * t;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = row[2 * m + (e >> 1)], tok = tk + (e & 1);
                const float uv = mine_x[((m * NT + n) * 4 + e) * 32 + lane];
                if (r < p.F16 && tok < T) store_h(p, tok, r, acc[m][n][e], uv, flag[2 * m + (e >> 1)]);
            }
        }
    }
}

}  // namespace ffnrm
