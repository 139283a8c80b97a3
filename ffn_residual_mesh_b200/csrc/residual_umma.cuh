// Residual contraction for token batches on the 5th-generation tensor cores, reading
// the packed 2-bit (and 1-bit plane) code records straight from HBM.
//
// Replaces residual_kernel (src/exact_residual_cuda_runner.cu:122-159,
// src/exact_main_residual_cuda_runner.cu:213-233, src/exact_cpu_base_gpu_full_ffn_runner.cu:195-215)
// for batches of 3 or more tokens, decode and prefill alike, including the rows of
// flagged fallback tiles (src/phone_ffn_loopback.py:155-197), which take the unsplit
// Q4 codes and the beta * sum(z) term.
//
// CTA tile: M = 128 tensor-core rows = 64 gate rows of row tile rt stacked on the same 64
// up rows, N = 16, 32, 64 or 128 tokens, all of d_model. The K loop runs over 128-code
// K tiles (two record chunks, four 32-code groups).
//
// HBM -> shared memory: per K tile the producer warp bulk-copies the row tile's code
// records (2-bit pairs 4 KB, bit planes 2 KB when r != 2, high pairs 4 KB when the tile
// holds fallback rows: each a contiguous run in the row-tiled layout of
// ffnrm_common.cuh) into a source ring, its alphas (betas) into a scale ring, and the
// activation tile [N tokens x 128 codes] by 2-D TMA (128-byte swizzle) into an
// activation ring. So HBM carries r bits per weight plus the fp16 alpha, not a byte.
// Each producer lane owns one stage of one ring and polls it without blocking, so the
// rings - released by different consumers (converters, drain, MMA) - refill
// independently.
//
// Widening: the worker threads turn each 16-byte record (64 codes of one row) of a K tile
// (256 records) into 64 u8 codes - ((w >> 2i) & 0x03030303 already is four codes in natural
// order; r = 1/3 and fallback rows OR in the plane / high bits) - and stores them in the
// K-major 128-byte-swizzled layout the MMA reads (16-byte unit u of row m at m*128 +
// ((u ^ (m & 7)) << 4)), then fences them into the async proxy and arrives on the stage.
// The workers widen K tile kt + S2 - 1 before they drain K tile kt, so the widening of
// one K tile overlaps the MMAs of the previous ones and the drain work.
//
// MMA: one thread issues one tcgen05.mma kind::i8 (u8 codes x s8 activations -> s32,
// K = 32) per group, each into its own TMEM columns, so every result is an exact integer
// group dot P[row, token]. Four accumulator buffers of `gpb` groups each rotate, so the
// MMAs run up to four buffers ahead of the drain and their completion latency is hidden.
//
// Drain (the 8 worker warps, two per TMEM lane quadrant, one token half each): per group,
// acc[t] += alpha[row, g] * (s[t, g] * float(P[t])) in packed fp32 pairs; flagged rows
// also add beta[row, g] * (s[t, g] * sum_i z[t, g, i]). alpha / beta arrive in a
// shared-memory ring (bulk copies by the producer, released by the drain); s (and
// s*zsum) from a double-buffered transposed window of
// 32 groups x N tokens that the drain warps stage themselves. Epilogue: the up rows
// hand their totals to the gate rows through shared memory; the gate rows merge with the
// base sums (not for flagged rows) and write h = SiLU(g)*u (fp16 hi [+ lo]).
//
// Every mbarrier wait is bounded; on timeout the kernel records an error code and winds
// down. No multicast anywhere.
#pragma once

#include <cuda_fp16.h>

#include "ffnrm_common.cuh"
#include "residual_dp4a.cuh"
#include "sm100.cuh"

namespace ffnrm {

constexpr int kUmKTile = 128;    // codes per K tile (two record chunks, four groups)

constexpr int kUmWin = 32;       // groups per staged scale window
constexpr int kUmMaxS1 = 8;      // deepest source ring (code records)
constexpr int kUmMaxS2 = 4;      // deepest widened-code ring
constexpr int kUmMaxS3 = 24;     // deepest scale ring (alpha, beta)
constexpr int kUmMaxSB = 8;      // deepest activation ring

template <int N>
struct UmCfg {
    static constexpr int DW = N >= 64 ? 4 : 2;          // worker warps per TMEM lane quadrant
    static constexpr int workers = 128 * DW;            // worker threads (widen + drain)
    static constexpr int threads = 64 + workers;        // + producer warp + MMA warp
    static constexpr int a_bytes = 128 * kUmKTile;      // widened codes, 16 KB
    static constexpr int b_bytes = N * kUmKTile;        // activations, a multiple of 1024
    static constexpr int nbuf = 4;                      // TMEM accumulator buffers
    static constexpr int gpb = N <= 16 ? 4 : N == 32 ? 2 : N == 64 ? 2 : 1;  // groups per buffer
    static constexpr int tmem_cols = nbuf * gpb * N;    // 256 (two CTAs per SM) or 512
    static constexpr int minb = N <= 32 ? 2 : 1;        // CTAs per SM
    static constexpr int s_stride = N + 4;              // window row (16-byte aligned)
    static constexpr int xch_stride = N + 1;            // up totals [64][N+1] (aliases the code ring)
    static constexpr int NH = N / DW;                   // token columns per worker warp
    static constexpr int win_bytes = kUmWin * s_stride * 4;
};

// Byte offsets of the shared-memory regions (computed on the host, see umma_layout()).
struct UmLayout {
    int S1, S2, S3, SB;                  // ring depths: source, widened codes, scales, activations
    int src_bytes;                       // bytes per source stage
    int off_pair, off_plane, off_hi;     // inside a source stage (-1 = not copied)
    int sc_bytes;                        // bytes per scale stage: alpha [, beta] of one K tile
    int b_off, src_off, sc_off, win_off, bar_off, total;
};

struct UmParams {
    ResidualParams p;
    UmLayout L;
    int has_pair;   // the layer has 2-bit pair records
    int rbits;      // residual bits 1..3
    int alpha_half; // alpha (and beta) stored as fp16
    int fb;         // fallback tiles given (p.fallback_tiles != nullptr)
};

__device__ __forceinline__ uint32_t um_low_bits(uint32_t w, uint32_t pw, int i, int h, int rbits) {
    constexpr uint32_t M2 = 0x03030303u, M1 = 0x01010101u;
    if (rbits == 1) return (pw >> (4 * h + i)) & M1;
    uint32_t v = (w >> (2 * i)) & M2;
    if (rbits == 3) v |= ((pw >> (4 * h + i)) & M1) << 2;
    return v;
}

template <int N, bool DOTS>
__device__ __forceinline__ void residual_umma_body(const CUtensorMap &tm_z, const UmParams &P) {
    using Cfg = UmCfg<N>;
    constexpr int NH = Cfg::NH;
    constexpr int kUmDrain = Cfg::workers;
    const ResidualParams &p = P.p;
    const UmLayout &Ly = P.L;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *a_ring = smem;                 // [S2][128 rows][128 B] widened codes
    uint8_t *b_ring = smem + Ly.b_off;      // [SB][N tokens][128 B] activations
    uint8_t *src_ring = smem + Ly.src_off;  // [S1] code records
    uint8_t *sc_ring = smem + Ly.sc_off;    // [S3][alpha 2 chunks x 128 rows x 2][beta ...]
    float *win = reinterpret_cast<float *>(smem + Ly.win_off);  // [2][kUmWin][N+4] s, then (fallback) s*zsum
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Ly.bar_off);
    uint64_t *src_full = bars, *src_empty = src_full + kUmMaxS1;
    uint64_t *a_full = src_empty + kUmMaxS1, *a_empty = a_full + kUmMaxS2;
    uint64_t *sc_full = a_empty + kUmMaxS2, *sc_empty = sc_full + kUmMaxS3;
    uint64_t *b_full = sc_empty + kUmMaxS3, *b_empty = b_full + kUmMaxSB;
    uint64_t *acc_full = b_empty + kUmMaxSB, *acc_empty = acc_full + Cfg::nbuf;
    uint64_t *done = acc_empty + Cfg::nbuf;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    float *xch = reinterpret_cast<float *>(a_ring);  // after the main loop only (S2 >= 2 stages: 32 KB)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.G, C = G / 2;
    const int rt = blockIdx.y;
    const int t0 = blockIdx.x * N;
    const int nkt = p.D / kUmKTile;
    const int nvalid = min(N, p.T - t0);
    const int S1 = Ly.S1, S2 = Ly.S2, S3 = Ly.S3, SB = Ly.SB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S1; ++s) {
            sm100::mbar_init(src_full + s, 1);
            sm100::mbar_init(src_empty + s, kUmDrain);
        }
        for (int s = 0; s < S2; ++s) {
            sm100::mbar_init(a_full + s, kUmDrain);
            sm100::mbar_init(a_empty + s, 1);
        }
        for (int s = 0; s < S3; ++s) {
            sm100::mbar_init(sc_full + s, 1);
            sm100::mbar_init(sc_empty + s, kUmDrain);
        }
        for (int s = 0; s < SB; ++s) {
            sm100::mbar_init(b_full + s, 1);
            sm100::mbar_init(b_empty + s, 1);
        }
        for (int b = 0; b < Cfg::nbuf; ++b) {
            sm100::mbar_init(acc_full + b, 1);
            sm100::mbar_init(acc_empty + b, kUmDrain);
        }
        sm100::mbar_init(done, 1);
        sm100::fence_barrier_init();
    }
    if (warp == 1) sm100::tmem_alloc(tmem_slot, Cfg::tmem_cols);
    sm100::trigger_dependents();
    // With fallback tiles the flags decide which records to copy: read them (they may come
    // from the preceding work of the stream) only after the dependency wait. Without,
    // the code records and alphas are weights and stream before it.
    if (P.fb) sm100::grid_dependency_wait();
    bool fl = false;
    if (P.fb) {
        const int row = rt * 64 + (threadIdx.x & 63);
        fl = row < p.F && p.fallback_tiles[row / p.tile_rows] != 0;
    }
    sm100::tc_fence_before();
    const bool cta_flagged = __syncthreads_or(fl) != 0;
    sm100::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int off_hi = cta_flagged ? Ly.off_hi : -1;
    // the pair records are needed for r >= 2 and for the full codes of flagged rows
    const int off_pair = (P.rbits != 1 || cta_flagged) ? Ly.off_pair : -1;
    const int off_plane = Ly.off_plane;
    const uint32_t src_tx = (off_pair >= 0 ? 4096u : 0u) + (off_plane >= 0 ? 2048u : 0u) + (off_hi >= 0 ? 4096u : 0u);
    const uint32_t al_bytes = P.alpha_half ? 1024u : 2048u;  // 2 chunks x 128 rows x 2 values
    const uint32_t sc_tx = al_bytes * (cta_flagged ? 2u : 1u);

    if (warp == 0) {
        // Producer. Lane l < S1 owns source stage l (K tiles l, l + S1, ...), the next S3
        // lanes the scale stages, the next SB lanes the activation stages. A lane reuses
        // only its own stage, in order, so each parity test is at most one phase ahead of
        // its barrier; the warp polls with non-blocking tests and stays converged.
        const int64_t rec0 = int64_t(rt) * C * 128;  // first record of the row tile (chunk 0)
        const int role = lane < S1 ? 0 : lane < S1 + S3 ? 1 : lane < S1 + S3 + SB ? 2 : -1;
        const int st = role == 0 ? lane : role == 1 ? lane - S1 : role == 2 ? lane - S1 - S3 : 0;
        const int depth = role == 0 ? S1 : role == 1 ? S3 : SB;
        auto issue = [&](int kt) {
            const int64_t rec = rec0 + int64_t(2 * kt) * 128;  // chunks 2kt, 2kt+1: 256 records
            if (role == 0) {
                uint8_t *src = src_ring + st * Ly.src_bytes;
                sm100::mbar_arrive_expect_tx(src_full + st, src_tx);
                if (off_pair >= 0) sm100::bulk_load(src + off_pair, p.proj[0].pair + rec, 4096, src_full + st);
                if (off_plane >= 0) sm100::bulk_load(src + off_plane, p.proj[0].plane + rec, 2048, src_full + st);
                if (off_hi >= 0) sm100::bulk_load(src + off_hi, p.proj[0].pair_hi + rec, 4096, src_full + st);
            } else if (role == 1) {
                uint8_t *sc = sc_ring + st * Ly.sc_bytes;
                sm100::mbar_arrive_expect_tx(sc_full + st, sc_tx);
                sm100::bulk_load(sc, static_cast<const uint8_t *>(p.proj[0].alpha) + rec * (al_bytes / 256), al_bytes,
                                 sc_full + st);
                if (cta_flagged)
                    sm100::bulk_load(sc + al_bytes, static_cast<const uint8_t *>(p.proj[0].beta) + rec * (al_bytes / 256),
                                     al_bytes, sc_full + st);
            } else {
                sm100::mbar_arrive_expect_tx(b_full + st, Cfg::b_bytes);
                sm100::tma_load_2d(b_ring + st * Cfg::b_bytes, &tm_z, kt * kUmKTile, t0, b_full + st);
            }
        };
        int kt = role >= 0 ? st : nkt;
        // Weights (fresh stages, no wait) go out before the dependency wait; activations,
        // which come from the preceding kernel of the stream, only after it.
        if (role == 0 || role == 1) {
            if (kt < nkt) issue(kt);
            kt += depth;
        }
        if (!P.fb) sm100::grid_dependency_wait();
        uint64_t *empty = role == 0 ? src_empty : role == 1 ? sc_empty : b_empty;
        long long last = clock64();
        while (__any_sync(0xffffffffu, kt < nkt)) {
            const bool ready = kt < nkt && sm100::mbar_test_wait(empty + st, ((kt / depth) & 1) ^ 1);
            if (ready) {
                issue(kt);
                kt += depth;
            }
            if (__any_sync(0xffffffffu, ready)) {
                last = clock64();
            } else if (clock64() - last > sm100::kWaitCycles) {
                if (lane == 0) atomicExch(p.err, sm100::kErrWaitEmpty);
                break;
            } else {
                __nanosleep(64);  // leave the issue slots to the workers sharing this scheduler
            }
        }
        // No copy may still be in flight when the CTA exits: each lane waits for the
        // final use of its stage (earlier uses completed before the stage was refilled).
        if (role >= 0 && st < nkt) {
            const int last_kt = st + (nkt - 1 - st) / depth * depth;
            uint64_t *full = role == 0 ? src_full : role == 1 ? sc_full : b_full;
            sm100::mbar_wait(full + st, (last_kt / depth) & 1, p.err, sm100::kErrWaitFull);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = sm100::umma_idesc_u8s8_s32(128, N);
            bool ok = true;
            for (int kt = 0; kt < nkt && ok; ++kt) {
                const int s2 = kt % S2, sb = kt % SB;
                if (!(ok = sm100::mbar_wait(a_full + s2, (kt / S2) & 1, p.err, sm100::kErrWaitFull) &&
                           sm100::mbar_wait(b_full + sb, (kt / SB) & 1, p.err, sm100::kErrWaitFull)))
                    break;
                sm100::tc_fence_after();
                const uint32_t a = sm100::smem_u32(a_ring + s2 * Cfg::a_bytes);
                const uint32_t bz = sm100::smem_u32(b_ring + sb * Cfg::b_bytes);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int gi = 4 * kt + j, u = gi / Cfg::gpb, b = u % Cfg::nbuf, slot = gi % Cfg::gpb;
                    if (slot == 0) {
                        if (!(ok = sm100::mbar_wait(acc_empty + b, ((u / Cfg::nbuf) & 1) ^ 1, p.err, sm100::kErrWaitEmpty)))
                            break;
                        sm100::tc_fence_after();
                    }
                    sm100::umma_i8(tmem + uint32_t((b * Cfg::gpb + slot) * N), sm100::umma_desc_sw128(a + 32 * j),
                                   sm100::umma_desc_sw128(bz + 32 * j), idesc, 0);
                    if (slot == Cfg::gpb - 1) sm100::umma_commit(acc_full + b);
                }
                sm100::umma_commit(a_empty + s2);
                sm100::umma_commit(b_empty + sb);
            }
            sm100::umma_commit(done);
        }
    } else {
        // Workers. Drain: tile row m = TMEM lane of quadrant q (a warp reaches only the
        // lanes of quadrant warp % 4), token half h. Widening: record dt of each K tile.
        const int q = warp & 3;
        const int h = (warp - 2) >> 2;  // token slice 0 .. DW-1
        const int m = 32 * q + lane;
        const int proj = q >> 1;
        const int row = rt * 64 + 32 * (q & 1) + lane;
        const int cbase = h * NH;
        const bool drains = cbase < nvalid;  // warp-uniform
        const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16) + uint32_t(cbase);
        const int dt = threadIdx.x - 64;  // 0 .. workers-1
        // widening: words [wj0, wj0 + 4 / (DW / 2)) of record wr = (chunk wcc, tile row wm)
        constexpr int WPT = 8 / Cfg::DW;  // 16-code words per thread: 4 (DW = 2) or 2 (DW = 4)
        const int wr = dt / (4 / WPT), wj0 = (dt % (4 / WPT)) * WPT;
        const int wcc = wr >> 7, wm = wr & 127, wrow = rt * 64 + (wm & 63);
        const bool wflag = off_hi >= 0 && wrow < p.F && p.fallback_tiles[wrow / p.tile_rows] != 0;
        const int rbits = P.rbits;
        bool wok = true;
        auto widen = [&](int k) {
            const int s1 = k % S1, s2 = k % S2;
            if (wok)
                wok = __all_sync(0xffffffffu,
                                 sm100::mbar_wait(a_empty + s2, ((k / S2) & 1) ^ 1, p.err, sm100::kErrWaitEmpty) &&
                                     sm100::mbar_wait(src_full + s1, (k / S1) & 1, p.err, sm100::kErrWaitFull));
            if (wok) {
                const uint8_t *src = src_ring + s1 * Ly.src_bytes;
                uint4 w = make_uint4(0, 0, 0, 0), wh = make_uint4(0, 0, 0, 0);
                uint2 pw = make_uint2(0, 0);
                if (off_pair >= 0) w = reinterpret_cast<const uint4 *>(src + off_pair)[wr];
                if (off_plane >= 0) pw = reinterpret_cast<const uint2 *>(src + off_plane)[wr];
                if (wflag) wh = reinterpret_cast<const uint4 *>(src + off_hi)[wr];
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w}, hs[4] = {wh.x, wh.y, wh.z, wh.w};
                uint8_t *A = a_ring + s2 * Cfg::a_bytes + wm * 128;
#pragma unroll
                for (int jj = wj0; jj < wj0 + WPT; ++jj) {
                    const uint32_t pv = jj < 2 ? pw.x : pw.y;
                    uint32_t o[4];
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq) {
                        if (wflag)
                            o[qq] = ((ws[jj] >> (2 * qq)) & 0x03030303u) | (((hs[jj] >> (2 * qq)) & 0x03030303u) << 2);
                        else
                            o[qq] = um_low_bits(ws[jj], pv, qq, jj & 1, rbits);
                    }
                    const int u = 4 * wcc + jj;
                    *reinterpret_cast<uint4 *>(A + ((u ^ (wm & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                }
                sm100::fence_proxy_async_smem();  // generic-proxy stores -> tensor-core operand reads
            }
            sm100::mbar_arrive(a_full + s2);
            sm100::mbar_arrive(src_empty + s1);
        };
        // the code records are weights: the first K tiles widen before the dependency wait
        for (int k = 0; k < S2 - 1 && k < nkt; ++k) widen(k);
        const bool flagged = cta_flagged && row < p.F && p.fallback_tiles[row / p.tile_rows] != 0;
        const int nwin = (G + kUmWin - 1) / kUmWin;
        float *sz_win = win + 2 * kUmWin * Cfg::s_stride;

        // The drain reads activations, scales and base sums: wait for the preceding kernel.
        if (!P.fb) sm100::grid_dependency_wait();

        // Stage scale window w (groups [32w, 32w+32)) transposed into buffer w & 1:
        // s[g][t] and, for fallback rows, s[g][t] * sum_i z[t, g, i].
        auto stage_window = [&](int w) {
            const int g0 = w * kUmWin, ng = min(kUmWin, G - g0);
            float *dst = win + (w & 1) * kUmWin * Cfg::s_stride;
            float *dsz = sz_win + (w & 1) * kUmWin * Cfg::s_stride;
            for (int i = dt; i < ng * N; i += kUmDrain) {
                const int tok = i / ng, g = i - tok * ng;
                if (!cta_flagged) {
                    // s alone: asynchronous copies, waited for at the next window barrier
                    if (t0 + tok < p.T)
                        sm100::cp_async4(dst + g * Cfg::s_stride + tok, p.s + int64_t(t0 + tok) * G + g0 + g);
                    else
                        dst[g * Cfg::s_stride + tok] = 0.f;
                    continue;
                }
                float v = 0.f, vz = 0.f;
                if (t0 + tok < p.T) {
                    v = __ldg(p.s + int64_t(t0 + tok) * G + g0 + g);
                    if (cta_flagged) {
                        const int4 *zr = reinterpret_cast<const int4 *>(p.z + int64_t(t0 + tok) * p.D + int64_t(g0 + g) * kGroup);
                        const int4 a = __ldg(zr), b = __ldg(zr + 1);
                        int zs = 0;
                        zs = __dp4a(a.x, 0x01010101, zs);
                        zs = __dp4a(a.y, 0x01010101, zs);
                        zs = __dp4a(a.z, 0x01010101, zs);
                        zs = __dp4a(a.w, 0x01010101, zs);
                        zs = __dp4a(b.x, 0x01010101, zs);
                        zs = __dp4a(b.y, 0x01010101, zs);
                        zs = __dp4a(b.z, 0x01010101, zs);
                        zs = __dp4a(b.w, 0x01010101, zs);
                        vz = v * float(zs);
                    }
                }
                dst[g * Cfg::s_stride + tok] = v;
                if (cta_flagged) dsz[g * Cfg::s_stride + tok] = vz;
            }
        };
        stage_window(0);

        float2 acc[NH / 2];
#pragma unroll
        for (int k = 0; k < NH / 2; ++k) acc[k] = make_float2(0.f, 0.f);
        // After a timed-out wait a warp stops waiting and computing but keeps looping, so
        // every drain warp reaches the same named barriers.
        bool ok = true;
        for (int kt = 0; kt < nkt; ++kt) {
            if (kt + S2 - 1 < nkt) widen(kt + S2 - 1);
            if (kt % (kUmWin / 4) == 0) {
                // window kt/8 starts: its stores (one window earlier) become visible, and
                // everyone is done with the window before it, whose buffer is refilled now
                sm100::cp_async_wait_all();
                asm volatile("bar.sync 1, %0;\n" ::"r"(kUmDrain) : "memory");
                const int w = kt / (kUmWin / 4);
                if (w + 1 < nwin) stage_window(w + 1);
            }
            // alpha (and beta) of this row for the K tile's four groups stay in the scale ring
            // (read per group; the stage is released after the K tile)
            const int s3 = kt % S3;
            if (ok) ok = __all_sync(0xffffffffu, sm100::mbar_wait(sc_full + s3, (kt / S3) & 1, p.err, sm100::kErrWaitFull));
            const uint8_t *sc = sc_ring + s3 * Ly.sc_bytes;
            // scale of group j (chunk j >> 1, element j & 1) of this thread's row; beta at +al_bytes
            auto scale_of = [&](const uint8_t *base, int j) -> float {
                const int rec = (j >> 1) * 128 + m;
                if (P.alpha_half) {
                    const __half2 v = reinterpret_cast<const __half2 *>(base)[rec];
                    return __half2float((j & 1) ? __high2half(v) : __low2half(v));
                }
                const float2 v = reinterpret_cast<const float2 *>(base)[rec];
                return (j & 1) ? v.y : v.x;
            };
            const float *sw = win + ((kt / (kUmWin / 4)) & 1) * kUmWin * Cfg::s_stride;
            const float *szw = sz_win + ((kt / (kUmWin / 4)) & 1) * kUmWin * Cfg::s_stride;
            const int gw0 = (kt % (kUmWin / 4)) * 4;  // first group of this K tile in the window
#pragma unroll
            // The K tile's accumulators (4 groups x NH columns of this warp) come out of TMEM in
            // chunks of CH columns, software-pipelined: chunk c + 1 is loaded while chunk c is
            // computed, and a buffer is released as soon as its last chunk has landed, so the
            // MMAs refill it while this warp still computes.
            constexpr int UPK = 4 / Cfg::gpb;                 // buffer uses per K tile
            constexpr int CH = NH < 16 ? NH : 16;              // columns per chunk
            constexpr int CPG = NH / CH;                       // chunks per group
            constexpr int NCK = 4 * CPG;                       // chunks per K tile
            constexpr int NC = CH < 16 ? CH : 16;              // columns per TMEM load
            uint32_t rbuf[2][CH];
            auto chunk_load = [&](int c) {
                const int j = c / CPG, c0 = (c % CPG) * CH, ub = j / Cfg::gpb, gg = j % Cfg::gpb;
                const int u = kt * UPK + ub, b = u % Cfg::nbuf;
                if (gg == 0 && c0 == 0 && ok) {  // first chunk of a buffer: wait for its MMAs
                    ok = __all_sync(0xffffffffu,
                                    sm100::mbar_wait(acc_full + b, (u / Cfg::nbuf) & 1, p.err, sm100::kErrWaitFull));
                    sm100::tc_fence_after();
                }
                if (drains && ok) {
#pragma unroll
                    for (int cc = 0; cc < CH; cc += NC)
                        sm100::tmem_ld<NC>(lane_base + uint32_t((b * Cfg::gpb + gg) * N + c0 + cc),
                                           *reinterpret_cast<uint32_t(*)[NC]>(&rbuf[c & 1][cc]));
                }
            };
            chunk_load(0);
#pragma unroll
            for (int c = 0; c < NCK; ++c) {
                const int j = c / CPG, c0 = (c % CPG) * CH, ub = j / Cfg::gpb, gg = j % Cfg::gpb;
                if (drains && ok) sm100::tmem_wait_ld();  // chunk c has landed
                if (gg == Cfg::gpb - 1 && c0 + CH == NH) {  // last chunk of its buffer: release
                    sm100::tc_fence_before();
                    sm100::mbar_arrive(acc_empty + (kt * UPK + ub) % Cfg::nbuf);
                }
                if (c + 1 < NCK) chunk_load(c + 1);
                if (drains && ok) {
                    const uint32_t *r = rbuf[c & 1];
                    const float aj = scale_of(sc, j);
                    const float2 a2 = make_float2(aj, aj);
                    const float *sg = sw + (gw0 + j) * Cfg::s_stride + cbase + c0;
#pragma unroll
                    for (int k4 = 0; k4 < CH / 4; ++k4) {
                        const float4 sv = *reinterpret_cast<const float4 *>(sg + 4 * k4);
                        const float2 x0 = make_float2(__int2float_rn(int(r[4 * k4])), __int2float_rn(int(r[4 * k4 + 1])));
                        const float2 x1 =
                            make_float2(__int2float_rn(int(r[4 * k4 + 2])), __int2float_rn(int(r[4 * k4 + 3])));
                        const float2 u0 = sm100::fmul2(x0, make_float2(sv.x, sv.y));
                        const float2 u1 = sm100::fmul2(x1, make_float2(sv.z, sv.w));
                        const int ka = (c0 + 4 * k4) / 2;
                        acc[ka] = sm100::ffma2(a2, u0, acc[ka]);
                        acc[ka + 1] = sm100::ffma2(a2, u1, acc[ka + 1]);
                        if constexpr (DOTS) {
                            if (row < p.F) {
                                int32_t *dp = p.dots + int64_t(proj) * p.T * p.F * G;
#pragma unroll
                                for (int i = 0; i < 4; ++i) {
                                    const int t = cbase + c0 + 4 * k4 + i;
                                    if (t < nvalid) dp[(int64_t(t0 + t) * p.F + row) * G + 4 * kt + j] = int(r[4 * k4 + i]);
                                }
                            }
                        }
                    }
                    if (flagged) {
                        const float bj = scale_of(sc + al_bytes, j);
                        const float2 b2 = make_float2(bj, bj);
                        const float *szg = szw + (gw0 + j) * Cfg::s_stride + cbase + c0;
#pragma unroll
                        for (int k = 0; k < CH / 2; ++k) {
                            const float2 v = *reinterpret_cast<const float2 *>(szg + 2 * k);
                            acc[c0 / 2 + k] = sm100::ffma2(b2, v, acc[c0 / 2 + k]);
                        }
                    }
                }
            }
            sm100::mbar_arrive(sc_empty + s3);
        }
        // Up rows hand their totals to the gate rows. The last acc_full wait implies that
        // every MMA has completed, so the code ring is no longer read.
        if (proj == 1 && drains) {
#pragma unroll
            for (int k = 0; k < NH / 2; ++k) {
                xch[(m - 64) * Cfg::xch_stride + cbase + 2 * k] = acc[k].x;
                xch[(m - 64) * Cfg::xch_stride + cbase + 2 * k + 1] = acc[k].y;
            }
        }
        asm volatile("bar.sync 1, %0;\n" ::"r"(kUmDrain) : "memory");
        if (ok && drains) {
            const int nt = min(NH, nvalid - cbase);
            if (p.h_hi != nullptr) {
                if (proj == 0 && row < p.F16) {
#pragma unroll
                    for (int k0 = 0; k0 < NH; k0 += 8) {
                        float gbs[8], ubs[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const bool v = k0 + k < nt && row < p.F && !flagged;
                            const int64_t bi = int64_t(t0 + cbase + k0 + k) * p.F + row;
                            gbs[k] = v ? __ldg(p.base[0] + bi) : 0.f;
                            ubs[k] = v ? __ldg(p.base[1] + bi) : 0.f;
                        }
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const int kk = k0 + k;
                            if (kk < nt) {
                                const float gv = (kk & 1 ? acc[kk / 2].y : acc[kk / 2].x) + gbs[k];
                                const float uv = xch[m * Cfg::xch_stride + cbase + kk] + ubs[k];
                                write_h(p, t0 + cbase + kk, row, gv, uv);
                            }
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

// Entry points: two CTAs per SM for N <= 32, one (with more registers) for N >= 64.
template <int N, bool DOTS>
__global__ void __launch_bounds__(UmCfg<N>::threads, 2)
    residual_umma_kernel2(const __grid_constant__ CUtensorMap tm_z, const UmParams P) {
    residual_umma_body<N, DOTS>(tm_z, P);
}
template <int N, bool DOTS>
__global__ void __launch_bounds__(UmCfg<N>::threads, 1)
    residual_umma_kernel1(const __grid_constant__ CUtensorMap tm_z, const UmParams P) {
    residual_umma_body<N, DOTS>(tm_z, P);
}

}  // namespace ffnrm
