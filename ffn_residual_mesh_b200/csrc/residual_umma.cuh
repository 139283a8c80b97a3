// Residual contraction for token batches on the 5th-generation tensor cores:
// exact int32 group dots with tcgen05.mma kind::i8 (u8 codes x s8 activations).
//
// Replaces residual_kernel (src/exact_residual_cuda_runner.cu:122-159) for T >= 5
// without fallback tiles.
//
// CTA tile: M = 128 rows = 64 gate rows stacked on the same 64 up rows, N = 16 or 32
// tokens, all of d_model. A 128-code K tile holds 4 groups; one K=32 MMA per group
// writes that group's dots P[row, token] into its own TMEM accumulator, so every MMA
// result is an exact integer group dot and the scale alpha*s is applied afterwards.
//   warp 0 / lane 0  producer: per K tile, the int8 activation tile [N tokens x 128
//                    codes] by 2-D TMA (128-byte swizzle) plus 1-D bulk copies of the
//                    four 32-row blocks' code records and alpha, into a 3-stage ring.
//   warp 1 / lane 0  MMA: 4 x tcgen05.mma kind::i8 per K tile into TMEM buffer it%2
//                    (2 buffers x 4 groups x N int32 columns).
//   warps 2-9        two warps per TMEM lane quadrant (a warp reaches only the lanes of
//                    quadrant warp%4), one tile row per thread. Half h of the pair
//                    unpacks record chunk h of K tile it into the swizzled A tile
//                    ((w >> 2i) & 0x03030303 is codes 4i..4i+3 in natural order) and
//                    drains token columns [h*N/2, (h+1)*N/2) of K tile it-1.
// The accumulators start at 0x4B400000, so an int32 sum 0x4B400000 + P has the bit
// pattern of the float 12582912 + P (|P| < 2^22): the drain turns it into P with one
// packed subtract, applies alpha[row,g]*s[t,g] with packed multiply / FMA, and writes
// 0x4B400000 back before releasing the buffer. Padded token columns hold zero
// activations and zero scales, so the drain runs without per-token branches. The up
// rows hand their totals to the gate rows through shared memory; the gate rows merge
// with the base sums and write h = SiLU(g)*u (fp16 hi + lo). Every mbarrier wait is
// bounded.
#pragma once

#include <cuda_fp16.h>

#include "ffnrm_common.cuh"
#include "residual_dp4a.cuh"
#include "sm100.cuh"

namespace ffnrm {

constexpr int kResTileRows = 64;  // rows of each projection per CTA
constexpr int kResKTile = 128;    // codes per K tile (4 groups, 2 record chunks)
constexpr int kResThreads = 320;  // producer warp, MMA warp, 8 unpack/drain warps
constexpr uint32_t kMagicBits = 0x4B400000u;
constexpr float kMagic = 12582912.0f;

// Shared-memory plan of one pipeline stage. Slot q = 2*proj + (32-row half) holds the
// records of one 32-row block for the stage's two chunks, in their HBM order.
template <int RB, int N, bool AHALF>
struct ResUmmaCfg {
    static constexpr int stages = 3;
    static constexpr int a_bytes = 128 * kResKTile;
    static constexpr int b_bytes = N * kResKTile;
    static constexpr int pair_slot = RB != 1 ? 2 * 32 * 16 : 0;
    static constexpr int plane_slot = RB != 2 ? 2 * 32 * 8 : 0;
    static constexpr int alpha_slot = 2 * 32 * 2 * (AHALF ? 2 : 4);
    static constexpr int slot_bytes = pair_slot + plane_slot + alpha_slot;
    static constexpr int pair_off = a_bytes + b_bytes;
    static constexpr int plane_off = pair_off + 4 * pair_slot;
    static constexpr int alpha_off = plane_off + 4 * plane_slot;
    static constexpr int stage_bytes = (alpha_off + 4 * alpha_slot + 1023) / 1024 * 1024;
    static constexpr int tmem_cols = 8 * N;
    static constexpr int xch_stride = N + 1;
    static size_t smem(int G) {
        return 1024 + size_t(stages) * stage_bytes + size_t(G) * N * 4 + size_t(kResTileRows) * xch_stride * 4 + 256;
    }
};

template <int RB, int N, bool AHALF, bool DOTS>
__global__ void __launch_bounds__(kResThreads, 2) residual_umma_kernel(const __grid_constant__ CUtensorMap tm_z,
                                                                       const ResidualParams p) {
    using Cfg = ResUmmaCfg<RB, N, AHALF>;
    constexpr int S = Cfg::stages;
    constexpr int NH = N / 2;  // token columns drained per warp
    constexpr int kEpi = kResThreads - 64;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *tiles = smem;
    float *s_sm = reinterpret_cast<float *>(smem + S * Cfg::stage_bytes);  // [G][N]
    float *xch = s_sm + p.G * N;                                          // [64][N+1] up totals
    uint64_t *b_full = reinterpret_cast<uint64_t *>(xch + kResTileRows * Cfg::xch_stride + 1);
    b_full = reinterpret_cast<uint64_t *>((reinterpret_cast<uintptr_t>(b_full) + 7) & ~uintptr_t(7));
    uint64_t *a_full = b_full + S;
    uint64_t *st_empty = a_full + S;
    uint64_t *acc_full = st_empty + S;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.G, C = G / 2;
    const int rt = blockIdx.x;  // 64-row tile of each projection
    const int t0 = blockIdx.y * N;
    const int nkt = p.D / kResKTile;
    const int nvalid = min(N, p.T - t0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            sm100::mbar_init(b_full + s, 1);
            sm100::mbar_init(a_full + s, kEpi);
            sm100::mbar_init(st_empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            sm100::mbar_init(acc_full + b, 1);
            sm100::mbar_init(acc_empty + b, kEpi);
        }
        sm100::mbar_init(done, 1);
        sm100::fence_barrier_init();
    }
    if (warp == 1) sm100::tmem_alloc(tmem_slot, Cfg::tmem_cols);
    for (int i = threadIdx.x; i < G * N; i += blockDim.x) {
        const int tok = i / G, g = i - tok * G;
        s_sm[g * N + tok] = t0 + tok < p.T ? p.s[int64_t(t0 + tok) * G + g] : 0.f;
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Row role of warps 2-9: tile row m = TMEM lane; slot q = warp & 3 = 2*proj + half.
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;  // chunk unpacked / column half drained
    const int m = 32 * q + lane;
    const int proj = q >> 1;
    const int row = rt * kResTileRows + 32 * (q & 1) + lane;
    const bool row_ok = 2 * rt + (q & 1) < p.row_blocks;
    const int cbase = h * NH;
    const bool drains = cbase < nvalid;  // warp-uniform
    const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16) + uint32_t(cbase);
    if (warp >= 2) {
#pragma unroll
        for (int c = 0; c < 8; ++c) sm100::tmem_fill<NH>(lane_base + uint32_t(c * N), kMagicBits);
        sm100::tmem_wait_st();
        sm100::tc_fence_before();
    }
    __syncthreads();
    sm100::tc_fence_after();

    if (warp == 0) {
        if (lane == 0) {  // producer
            const int halves = (2 * rt + 1 < p.row_blocks) ? 2 : 1;
            const uint32_t tx = Cfg::b_bytes + 2 * halves * Cfg::slot_bytes;
            constexpr int asz = AHALF ? 2 : 4;
            int issued = 0;
            for (int it = 0; it < nkt; ++it) {
                const int s = it % S;
                if (!sm100::mbar_wait(st_empty + s, ((it / S) & 1) ^ 1, p.err, sm100::kErrWaitEmpty)) break;
                uint8_t *st = tiles + s * Cfg::stage_bytes;
                sm100::mbar_arrive_expect_tx(b_full + s, tx);
                sm100::tma_load_2d(st + Cfg::a_bytes, &tm_z, it * kResKTile, t0, b_full + s);
                for (int qq = 0; qq < 4; ++qq) {
                    if ((qq & 1) >= halves) continue;
                    const ProjView &pv = (qq >> 1) ? p.proj[1] : p.proj[0];
                    const int64_t rec = (int64_t(2 * rt + (qq & 1)) * C + 2 * it) * 32;
                    if (RB != 1)
                        sm100::bulk_load(st + Cfg::pair_off + qq * Cfg::pair_slot, pv.pair + rec, Cfg::pair_slot, b_full + s);
                    if (RB != 2)
                        sm100::bulk_load(st + Cfg::plane_off + qq * Cfg::plane_slot, pv.plane + rec, Cfg::plane_slot,
                                         b_full + s);
                    sm100::bulk_load(st + Cfg::alpha_off + qq * Cfg::alpha_slot,
                                     static_cast<const uint8_t *>(pv.alpha) + rec * 2 * asz, Cfg::alpha_slot, b_full + s);
                }
                ++issued;
            }
            for (int it = max(0, issued - S); it < issued; ++it)
                sm100::mbar_wait(b_full + it % S, (it / S) & 1, p.err, sm100::kErrWaitFull);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = sm100::umma_idesc_u8s8_s32(128, N);
            for (int it = 0; it < nkt; ++it) {
                const int s = it % S, b = it & 1;
                if (!sm100::mbar_wait(b_full + s, (it / S) & 1, p.err, sm100::kErrWaitFull)) break;
                if (!sm100::mbar_wait(a_full + s, (it / S) & 1, p.err, sm100::kErrWaitFull)) break;
                if (!sm100::mbar_wait(acc_empty + b, ((it >> 1) & 1) ^ 1, p.err, sm100::kErrWaitEmpty)) break;
                sm100::tc_fence_after();
                const uint32_t a = sm100::smem_u32(tiles + s * Cfg::stage_bytes), bz = a + Cfg::a_bytes;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    sm100::umma_i8(tmem + uint32_t(b * 4 * N + j * N), sm100::umma_desc_sw128(a + 32 * j),
                                   sm100::umma_desc_sw128(bz + 32 * j), idesc, 1);
                sm100::umma_commit(st_empty + s);
                sm100::umma_commit(acc_full + b);
            }
            sm100::umma_commit(done);
        }
    } else {
        float2 acc[NH / 2];
#pragma unroll
        for (int k = 0; k < NH / 2; ++k) acc[k] = make_float2(0.f, 0.f);
        float alpha_prev[4] = {0.f, 0.f, 0.f, 0.f};
        bool ok = true;
        for (int it = 0; it <= nkt; ++it) {
            float alpha_cur[4] = {0.f, 0.f, 0.f, 0.f};
            if (it < nkt) {
                const int s = it % S;
                ok = __all_sync(0xffffffffu, sm100::mbar_wait(b_full + s, (it / S) & 1, p.err, sm100::kErrWaitFull));
                if (!ok) break;
                const uint8_t *st = tiles + s * Cfg::stage_bytes;
                uint4 wp = make_uint4(0, 0, 0, 0);
                uint2 wq = make_uint2(0, 0);
                if (row_ok) {
                    const int r = h * 32 + lane;
                    if (RB != 1) wp = reinterpret_cast<const uint4 *>(st + Cfg::pair_off + q * Cfg::pair_slot)[r];
                    if (RB != 2) wq = reinterpret_cast<const uint2 *>(st + Cfg::plane_off + q * Cfg::plane_slot)[r];
                    const uint8_t *al = st + Cfg::alpha_off + q * Cfg::alpha_slot;
                    load_scale2_shared<AHALF>(al, lane, alpha_cur[0], alpha_cur[1]);
                    load_scale2_shared<AHALF>(al, 32 + lane, alpha_cur[2], alpha_cur[3]);
                }
                const uint32_t pw[4] = {wp.x, wp.y, wp.z, wp.w};
                uint8_t *arow = tiles + s * Cfg::stage_bytes + m * 128;
#pragma unroll
                for (int j = 0; j < 4; ++j) {  // 16 codes: group 2h + (j>>1) of the tile, half j&1
                    const uint32_t qw = (j >> 1) ? wq.y : wq.x;
                    const int hh = j & 1;
                    uint32_t o[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint32_t v;
                        if (RB == 1) {
                            v = (qw >> (4 * hh + i)) & 0x01010101u;
                        } else {
                            v = (pw[j] >> (2 * i)) & 0x03030303u;
                            if (RB == 3) v |= ((qw >> (4 * hh + i)) & 0x01010101u) << 2;
                        }
                        o[i] = v;
                    }
                    const int piece = 4 * h + j;
                    *reinterpret_cast<uint4 *>(arow + ((piece ^ (m & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                }
                sm100::fence_proxy_async_smem();
                sm100::mbar_arrive(a_full + s);
            }
            if (it >= 1) {
                const int e = it - 1, b = e & 1;
                ok = __all_sync(0xffffffffu, sm100::mbar_wait(acc_full + b, (e >> 1) & 1, p.err, sm100::kErrWaitFull));
                if (!ok) break;
                if (drains) {
                    sm100::tc_fence_after();
                    constexpr int GB = 16 / NH;  // groups per TMEM batch (16 registers)
#pragma unroll
                    for (int j0 = 0; j0 < 4; j0 += GB) {
                        uint32_t r[GB][NH];
#pragma unroll
                        for (int j = 0; j < GB; ++j) sm100::tmem_ld<NH>(lane_base + uint32_t(b * 4 * N + (j0 + j) * N), r[j]);
                        sm100::tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < GB; ++j) sm100::tmem_fill<NH>(lane_base + uint32_t(b * 4 * N + (j0 + j) * N), kMagicBits);
#pragma unroll
                        for (int j = 0; j < GB; ++j) {
                            const int g = 4 * e + j0 + j;
                            const float2 a2 = make_float2(alpha_prev[j0 + j], alpha_prev[j0 + j]);
                            const float2 m2 = make_float2(-kMagic, -kMagic);
                            const float4 *sg = reinterpret_cast<const float4 *>(s_sm + g * N + cbase);
#pragma unroll
                            for (int k4 = 0; k4 < NH / 4; ++k4) {
                                const float4 sv = sg[k4];
                                const float2 x0 = sm100::fadd2(make_float2(__uint_as_float(r[j][4 * k4]),
                                                                           __uint_as_float(r[j][4 * k4 + 1])), m2);
                                const float2 x1 = sm100::fadd2(make_float2(__uint_as_float(r[j][4 * k4 + 2]),
                                                                           __uint_as_float(r[j][4 * k4 + 3])), m2);
                                acc[2 * k4] = sm100::ffma2(x0, sm100::fmul2(make_float2(sv.x, sv.y), a2), acc[2 * k4]);
                                acc[2 * k4 + 1] = sm100::ffma2(x1, sm100::fmul2(make_float2(sv.z, sv.w), a2), acc[2 * k4 + 1]);
                                if constexpr (DOTS) {
                                    if (row < p.F) {
                                        int32_t *dp = p.dots + int64_t(proj) * p.T * p.F * G;
                                        const float xs[4] = {x0.x, x0.y, x1.x, x1.y};
#pragma unroll
                                        for (int i = 0; i < 4; ++i) {
                                            const int t = cbase + 4 * k4 + i;
                                            if (t < nvalid) dp[(int64_t(t0 + t) * p.F + row) * G + g] = int(xs[i]);
                                        }
                                    }
                                }
                            }
                        }
                    }
                    sm100::tmem_wait_st();
                    sm100::tc_fence_before();
                }
                sm100::mbar_arrive(acc_empty + b);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) alpha_prev[j] = alpha_cur[j];
        }
        // Up rows hand their totals to the gate rows (named barrier over warps 2-9).
        if (proj == 1 && drains) {
#pragma unroll
            for (int k = 0; k < NH / 2; ++k) {
                xch[(m - 64) * Cfg::xch_stride + cbase + 2 * k] = acc[k].x;
                xch[(m - 64) * Cfg::xch_stride + cbase + 2 * k + 1] = acc[k].y;
            }
        }
        asm volatile("bar.sync 1, %0;\n" ::"r"(kEpi) : "memory");
        if (ok && drains) {
            const int nt = min(NH, nvalid - cbase);
            if (p.h_hi != nullptr) {
                if (proj == 0 && row < p.F16) {
#pragma unroll
                    for (int k = 0; k < NH / 2; ++k) {
                        if (2 * k < nt)
                            store_h(p, t0 + cbase + 2 * k, row, acc[k].x, xch[m * Cfg::xch_stride + cbase + 2 * k], false);
                        if (2 * k + 1 < nt)
                            store_h(p, t0 + cbase + 2 * k + 1, row, acc[k].y,
                                    xch[m * Cfg::xch_stride + cbase + 2 * k + 1], false);
                    }
                }
            } else if (row < p.F) {
                float *out = proj ? p.out[1] : p.out[0];
#pragma unroll
                for (int k = 0; k < NH / 2; ++k) {
                    if (2 * k < nt) out[int64_t(t0 + cbase + 2 * k) * p.F + row] = acc[k].x;
                    if (2 * k + 1 < nt) out[int64_t(t0 + cbase + 2 * k + 1) * p.F + row] = acc[k].y;
                }
            }
        }
    }
    __syncwarp();
    sm100::mbar_wait(done, 0, p.err, sm100::kErrWaitDone);
    sm100::tc_fence_after();
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 1) sm100::tmem_dealloc(tmem, Cfg::tmem_cols);
}

}  // namespace ffnrm
