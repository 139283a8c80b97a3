// Residual contraction for token batches on the 5th-generation tensor cores:
// exact int32 group dots with tcgen05.mma kind::i8 (u8 codes x s8 activations).
//
// Replaces residual_kernel (src/exact_residual_cuda_runner.cu:122-159) for batches of
// 3 or more tokens (the GEMV keeps 1-2) without fallback tiles.
//
// The A operand is the layer's low codes as one byte per code, stored at load time
// row-tiled: rows [128*rt, 128*rt+64) are gate rows 64*rt.. and the next 64 the up rows
// of the same tile, so a CTA's M = 128 MMA rows are 64 gate rows stacked on the same 64
// up rows and one 2-D TMA (128-byte swizzle) brings a 128 x 128-code K tile. No unpack
// step: every operand arrives by TMA.
//
// CTA tile: M = 128 rows, N = 16 or 32 tokens, all of d_model. A 128-code K tile holds 4
// groups; one K=32 MMA per group writes that group's dots P[row, token] into its own
// TMEM accumulator, so every MMA result is an exact integer group dot and the scale
// alpha*s is applied afterwards.
// Warp roles (10 warps):
//   warp 0     producer: per K tile the A tile and the activation tile [N tokens x 128
//              codes] into a `stages`-deep operand ring (released when the K tile's
//              MMAs complete), and the tile's alpha (1-D bulk copy) into a deeper alpha
//              ring (released by the drain). A thread's copies run one after another,
//              so K tiles are issued in batches with one copy per lane.
//   warp 1     lane 0 issues 4 x tcgen05.mma per K tile into TMEM buffer it%2 (2 buffers
//              x 4 groups x N int32 columns), each writing its group's dots P afresh.
//   warps 2-9  drain: two warps per TMEM lane quadrant (a warp reaches only the lanes of
//              quadrant warp%4), one tile row per thread, token columns [h*N/2,
//              (h+1)*N/2) for warp half h.
// The drain converts each exact int32 dot P to float (exact, |P| < 2^24), multiplies by
// s[t,g] and adds alpha[row,g] times that into the accumulator (packed fp32 pairs, two
// tokens per instruction; s comes from a per-CTA [G][N] table). Padded token columns
// hold zero
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

constexpr int kTcTileRows = 64;  // rows of each projection per CTA
constexpr int kTcKTile = 128;    // codes per K tile (4 groups, 2 record chunks)
constexpr int kTcThreads = 320;  // producer, MMA, 8 drain warps
constexpr int kTcDrain = 256;    // drain threads
constexpr int kTcMaxStages = 8;

// Shared memory: [operand ring of `stages`][alpha ring of 2*stages][s [G][N+4] f32]
// [barriers]. Operand stage: A tile [128][128 B],
// activation tile [N][128 B] (both 128-byte swizzled). Alpha slot: the K tile's two
// chunks in HBM order, (chunk cc, tile row m) at cc*128 + m, 2 values each.
template <int N, bool AHALF>
struct ResTcCfg {
    static constexpr int a_bytes = 128 * kTcKTile;
    static constexpr int b_bytes = N * kTcKTile;
    static constexpr int alpha_bytes = 2 * 128 * 2 * (AHALF ? 2 : 4);
    static constexpr int b_off = a_bytes;
    static constexpr int stage_bytes = a_bytes + b_bytes;  // multiple of 1024
    static constexpr int tx_bytes = stage_bytes + alpha_bytes;
    static constexpr int tmem_cols = 8 * N;
    static constexpr int xch_stride = N + 1;  // up totals [64][N+1], aliased on stage 0 at the end
    static constexpr int s_stride = N + 4;    // padded [G][N] scale table rows (16-byte aligned)
    static_assert(a_bytes >= kTcTileRows * xch_stride * 4, "exchange fits a stage");
    static size_t smem(int G, int stages) {
        return 1024 + size_t(stages) * (stage_bytes + 2 * alpha_bytes) + size_t(G) * s_stride * 4 + 768;
    }
    // Deepest input ring (2..8 stages) that keeps two CTAs per SM, else two stages.
    static int stages_for(int G) {
        for (int s = kTcMaxStages; s > 2; --s)
            if (smem(G, s) <= 113 * 1024) return s;
        return 2;
    }
};

template <int N, bool AHALF, bool DOTS>
__global__ void __launch_bounds__(kTcThreads, 2)
    residual_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_z,
                       const ResidualParams p, const int S) {
    using Cfg = ResTcCfg<N, AHALF>;
    constexpr int NH = N / 2;  // token columns drained per warp
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem;
    uint8_t *aring = ring + S * Cfg::stage_bytes;                                 // [2S] alpha slots
    float *s_sm = reinterpret_cast<float *>(aring + 2 * S * Cfg::alpha_bytes);  // [G][N+4]
    uint64_t *in_full = reinterpret_cast<uint64_t *>(s_sm + p.G * Cfg::s_stride);
    uint64_t *in_empty = in_full + kTcMaxStages;
    uint64_t *al_empty = in_empty + kTcMaxStages;  // [2S]
    uint64_t *acc_full = al_empty + 2 * kTcMaxStages;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    float *xch = reinterpret_cast<float *>(ring);  // after the main loop only

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.G, C = G / 2;
    const int rt = blockIdx.y;  // 64-row tile of each projection (token tiles of a row tile
    const int t0 = blockIdx.x * N;  // run back to back and share its A tiles through L2)
    const int nkt = p.D / kTcKTile;
    const int nvalid = min(N, p.T - t0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            sm100::mbar_init(in_full + s, 1);
            sm100::mbar_init(in_empty + s, 1);
        }
        for (int s = 0; s < 2 * S; ++s) sm100::mbar_init(al_empty + s, kTcDrain);
        for (int b = 0; b < 2; ++b) {
            sm100::mbar_init(acc_full + b, 1);
            sm100::mbar_init(acc_empty + b, kTcDrain);
        }
        sm100::mbar_init(done, 1);
        sm100::fence_barrier_init();
    }
    if (warp == 1) sm100::tmem_alloc(tmem_slot, Cfg::tmem_cols);
    // Everything up to the role split touches only this CTA's shared memory and TMEM. The
    // activations, scales and base sums may come from the preceding kernel of the stream
    // (dependent launch): the producer waits for it after its first weight copies, the
    // drain before it reads anything.
    sm100::trigger_dependents();
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Drain role: tile row m = TMEM lane of quadrant q; column half h.
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    const int m = 32 * q + lane;
    const int proj = q >> 1;
    const int row = rt * kTcTileRows + 32 * (q & 1) + lane;
    const int cbase = h * NH;
    const bool drains = warp >= 2 && cbase < nvalid;  // warp-uniform
    const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16) + uint32_t(cbase);

    if (warp == 0) {
        // Producer warp: batches of B K tiles. Consecutive copies from one thread do not
        // overlap, so each batch uses its own group of 3B lanes (A tiles, activation
        // tiles, alphas), rotating through the warp so several batches are in flight.
        constexpr int asz = AHALF ? 2 : 4;
        const int B = S / 2 > 1 ? (S / 2 < 10 ? S / 2 : 10) : 1;
        const int R = 32 / (3 * B);  // lane groups
        int issued = 0, batch = 0;
        for (int it0 = 0; it0 < nkt; it0 += B, ++batch) {
            const int nb = min(B, nkt - it0);
            const int l = lane - (batch % R) * 3 * B;  // role within this batch's lane group
            const int k = l < 0 ? nb : (l < B ? l : (l < 2 * B ? l - B : l - 2 * B));
            const int it = it0 + k, s = it % S, sa = it % (2 * S);
            bool ok = true;
            if (l >= 0 && l < nb) {
                ok = sm100::mbar_wait(in_empty + s, ((it / S) & 1) ^ 1, p.err, sm100::kErrWaitEmpty) &&
                     sm100::mbar_wait(al_empty + sa, ((it / (2 * S)) & 1) ^ 1, p.err, sm100::kErrWaitEmpty);
                if (ok) sm100::mbar_arrive_expect_tx(in_full + s, Cfg::tx_bytes);
            }
            if (!__all_sync(0xffffffffu, ok)) break;
            uint8_t *st = ring + s * Cfg::stage_bytes;
            if (l >= 0 && l < B && k < nb) sm100::tma_load_2d(st, &tm_a, it * kTcKTile, rt * 128, in_full + s);
            if (l >= 2 * B && l < 3 * B && k < nb) {
                const int64_t rec = rec_index(2 * rt, C, 2 * it, 0);  // the tile's first record
                sm100::bulk_load(aring + sa * Cfg::alpha_bytes,
                                 static_cast<const uint8_t *>(p.proj[0].alpha) + rec * 2 * asz, Cfg::alpha_bytes,
                                 in_full + s);
            }
            // codes and alpha are weights; the activations follow the preceding kernel
            if (batch == 0) sm100::grid_dependency_wait();
            if (l >= B && l < 2 * B && k < nb) sm100::tma_load_2d(st + Cfg::b_off, &tm_z, it * kTcKTile, t0, in_full + s);
            issued = it0 + nb;
        }
        // No copy may still be in flight when the CTA exits.
        if (lane == 0)
            for (int it = max(0, issued - S); it < issued; ++it)
                sm100::mbar_wait(in_full + it % S, (it / S) & 1, p.err, sm100::kErrWaitFull);
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = sm100::umma_idesc_u8s8_s32(128, N);
            int s = 0;  // it mod S and the ring phase, advanced without a division
            uint32_t ph = 0;
            for (int it = 0; it < nkt; ++it, s = s + 1 == S ? 0 : s + 1, ph ^= uint32_t(s == 0)) {
                const int b = it & 1;
                if (!sm100::mbar_wait(in_full + s, ph, p.err, sm100::kErrWaitFull)) break;
                if (!sm100::mbar_wait(acc_empty + b, ((it >> 1) & 1) ^ 1, p.err, sm100::kErrWaitEmpty)) break;
                sm100::tc_fence_after();
                const uint32_t a = sm100::smem_u32(ring + s * Cfg::stage_bytes), bz = a + Cfg::b_off;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    sm100::umma_i8(tmem + uint32_t(b * 4 * N + j * N), sm100::umma_desc_sw128(a + 32 * j),
                                   sm100::umma_desc_sw128(bz + 32 * j), idesc, 0);
                sm100::umma_commit(in_empty + s);
                sm100::umma_commit(acc_full + b);
            }
            sm100::umma_commit(done);
        }
    } else {
        // Drain. Scale table first: coalesced reads of each token's G scales, all issued
        // before the stores (the padded row stride spreads the transposing stores over
        // the banks).
        sm100::grid_dependency_wait();
        {
            constexpr int kU = 8;
            const int dt = threadIdx.x - 64;
            for (int i0 = dt; i0 < G * N; i0 += kU * kTcDrain) {
                float v[kU];
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int i = i0 + u * kTcDrain, tok = i / G, g = i - tok * G;
                    v[u] = i < G * N && t0 + tok < p.T ? __ldg(p.s + int64_t(t0 + tok) * G + g) : 0.f;
                }
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int i = i0 + u * kTcDrain, tok = i / G, g = i - tok * G;
                    if (i < G * N) s_sm[g * Cfg::s_stride + tok] = v[u];
                }
            }
            asm volatile("bar.sync 1, %0;\n" ::"r"(kTcDrain) : "memory");
        }
        float2 acc[NH / 2];
#pragma unroll
        for (int k = 0; k < NH / 2; ++k) acc[k] = make_float2(0.f, 0.f);
        bool ok = true;
        int sa = 0;  // alpha slot of K tile e: e mod 2S, advanced without a division
#pragma unroll 2
        for (int e = 0; e < nkt; ++e, sa = sa + 1 == 2 * S ? 0 : sa + 1) {
            const int b = e & 1;
            ok = __all_sync(0xffffffffu, sm100::mbar_wait(acc_full + b, (e >> 1) & 1, p.err, sm100::kErrWaitFull));
            if (!ok) break;
            if (drains) {
                sm100::tc_fence_after();
                float al[4];
                const uint8_t *as = aring + sa * Cfg::alpha_bytes;
                load_scale2_shared<AHALF>(as, m, al[0], al[1]);
                load_scale2_shared<AHALF>(as, 128 + m, al[2], al[3]);
                constexpr int GB = 16 / NH;  // groups per TMEM batch (16 registers)
#pragma unroll
                for (int j0 = 0; j0 < 4; j0 += GB) {
                    uint32_t r[GB][NH];
#pragma unroll
                    for (int j = 0; j < GB; ++j) sm100::tmem_ld<NH>(lane_base + uint32_t(b * 4 * N + (j0 + j) * N), r[j]);
                    sm100::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < GB; ++j) {
                        const int g = 4 * e + j0 + j;
                        const float2 a2 = make_float2(al[j0 + j], al[j0 + j]);
                        const float4 *sg = reinterpret_cast<const float4 *>(s_sm + g * Cfg::s_stride + cbase);
#pragma unroll
                        for (int k4 = 0; k4 < NH / 4; ++k4) {
                            const float4 sv = sg[k4];
                            const float2 x0 = make_float2(__int2float_rn(int(r[j][4 * k4])), __int2float_rn(int(r[j][4 * k4 + 1])));
                            const float2 x1 =
                                make_float2(__int2float_rn(int(r[j][4 * k4 + 2])), __int2float_rn(int(r[j][4 * k4 + 3])));
                            const float2 u0 = sm100::fmul2(x0, make_float2(sv.x, sv.y));
                            const float2 u1 = sm100::fmul2(x1, make_float2(sv.z, sv.w));
                            acc[2 * k4] = sm100::ffma2(a2, u0, acc[2 * k4]);
                            acc[2 * k4 + 1] = sm100::ffma2(a2, u1, acc[2 * k4 + 1]);
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
                sm100::tc_fence_before();
            }
            sm100::mbar_arrive(acc_empty + b);
            sm100::mbar_arrive(al_empty + sa);
        }
        // Up rows hand their totals to the gate rows (named barrier over the drain warps).
        // The last acc_full wait implies every copy and MMA of the ring has completed.
        if (proj == 1 && drains) {
#pragma unroll
            for (int k = 0; k < NH / 2; ++k) {
                xch[(m - 64) * Cfg::xch_stride + cbase + 2 * k] = acc[k].x;
                xch[(m - 64) * Cfg::xch_stride + cbase + 2 * k + 1] = acc[k].y;
            }
        }
        asm volatile("bar.sync 1, %0;\n" ::"r"(kTcDrain) : "memory");
        if (ok && drains) {
            const int nt = min(NH, nvalid - cbase);
            if (p.h_hi != nullptr) {
                if (proj == 0 && row < p.F16) {
                    // all base sums of this thread's tokens are loaded before any h is stored
                    float gbs[NH], ubs[NH];
#pragma unroll
                    for (int k = 0; k < NH; ++k) {
                        const bool v = k < nt && row < p.F;
                        const int64_t bi = int64_t(t0 + cbase + k) * p.F + row;
                        gbs[k] = v ? __ldg(p.base[0] + bi) : 0.f;
                        ubs[k] = v ? __ldg(p.base[1] + bi) : 0.f;
                    }
#pragma unroll
                    for (int k = 0; k < NH; ++k) {
                        if (k < nt) {
                            const float gv = (k & 1 ? acc[k / 2].y : acc[k / 2].x) + gbs[k];
                            const float uv = xch[m * Cfg::xch_stride + cbase + k] + ubs[k];
                            write_h(p, t0 + cbase + k, row, gv, uv);
                        }
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
