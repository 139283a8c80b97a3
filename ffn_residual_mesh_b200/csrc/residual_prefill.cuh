// Residual contraction for prefill-sized token batches on the 5th-generation tensor cores.
//
// Replaces residual_kernel (src/exact_cpu_base_gpu_full_ffn_runner.cu:195-215,
// src/exact_residual_cuda_runner.cu:122-159) for batches of hundreds or thousands of
// tokens without fallback tiles (a 2048-token prefill at d_model 8192 is 30 G
// (row, token, group) dots per layer).
//
// Exact dots in fp16 x fp16 -> fp32: the activations z (|z| <= 128) and the low codes
// (0..7) are exact in fp16, every product is an integer below 2^10 and every partial sum
// of a 32-code group an integer below 2^15, so the tensor cores' fp32 accumulator holds
// the exact integer group dot P whatever its internal order. The TMEM then already holds
// P as a float: the drain needs no int-to-float conversion, only acc += alpha * (s * P)
// (one packed multiply and one packed FMA per two dots), which is what bounds this kernel.
//
// Tile: tokens on the tensor-core M axis and rows on N. A CTA owns 128 tokens (TMEM
// lanes) x one 64-row record tile of both projections: N = 128 = its 64 gate rows, then
// the same 64 up rows. Per 64-code K tile (two groups) two tcgen05.mma kind::f16
// (M = 128, N = 128, K = 16) per group write that group's exact dots P[token, row] into one
// of four 128-column TMEM buffers, so the MMAs run up to three groups ahead of the drain.
//
// Operands: the activations as fp16 [T, D] (converted from z by z_to_f16_kernel just
// before) by 2-D TMA with 128-byte swizzle; the layer's 2-bit (and plane) code records
// by 1-D bulk copies (2 KB per K tile, plus the fp16 alphas), widened to fp16 in shared
// memory by two warps one K tile ahead of the MMA (1024 + c as an fp16 bit pattern,
// minus 1024: exact), in the K-major 128-byte-swizzled layout the MMA reads.
//
// Warp roles (384 threads):
//   warp 0      producer: lane l < S1 owns record stage l (records + alphas), the next SA
//               lanes the activation stages.
//   warp 1      TMEM allocation; lane 0 issues the MMAs.
//   warps 2-3   widen the records into the B tile and write the K tile's alphas as f32
//               [2][128].
//   warps 4-11  drain, one token per thread (warp % 4 = TMEM lane quadrant), warp group
//               h = 0/1 takes rows [32h, 32h+32) of both projections: 64 accumulators,
//               32-column TMEM loads double-buffered. The gate and up totals of a (token,
//               row) meet in the same thread: the epilogue merges them with the base sums
//               and writes h = SiLU(g)*u (fp16 hi + lo).
//
// Every mbarrier wait is bounded; on timeout the kernel records an error code and winds
// down. No multicast anywhere.
#pragma once

#include <cuda_fp16.h>

#include "ffnrm_common.cuh"
#include "residual_dp4a.cuh"
#include "residual_umma.cuh"
#include "sm100.cuh"

namespace ffnrm {

constexpr int kPfTokens = 128;             // tokens per CTA (M, TMEM lanes)
constexpr int kPfRows = 64;                // rows per projection per CTA (N = 2 x 64)
constexpr int kPfN = 2 * kPfRows;          // MMA N
constexpr int kPfKTile = 64;               // codes per K tile: one record chunk, two groups
constexpr int kPfRowBytes = 2 * kPfKTile;  // fp16 bytes per operand row and K tile (128)
constexpr int kPfBufs = 512 / kPfN;        // TMEM accumulator buffers (all 512 columns)
constexpr int kPfDrainWG = 2;              // drain warp groups
constexpr int kPfThreads = 128 * (1 + kPfDrainWG);
constexpr int kPfWiden = 64;               // widening threads (warps 2-3)
constexpr int kPfDrain = 128 * kPfDrainWG;  // drain threads (warps 4..)
constexpr int kPfRpt = kPfRows / kPfDrainWG;  // rows of each projection per drain warp group (32)
constexpr int kPfCh = kPfRpt;              // TMEM columns per drain chunk (one projection)
constexpr int kPfMaxSA = 8, kPfMaxS1 = 8, kPfMaxSW = 4, kPfMaxS4 = 8;

// Shared-memory layout (byte offsets; computed on the host by prefill_layout()).
struct PfLayout {
    int SA, S1, SW, S4;                  // ring depths: activations, records, widened codes, f32 alphas
    int src_bytes;                       // bytes per record stage
    int off_pair, off_plane, off_alpha;  // inside a record stage
    int pair_bytes, plane_bytes, alpha_bytes;  // per K tile (0 = not copied)
    int w_off, src_off, al_off, bar_off, total;
};

struct PfParams {
    ResidualParams p;
    PfLayout L;
    int rbits;       // residual bits 1..3
    int alpha_half;  // alphas stored as fp16
};

// z [n] int8 -> fp16, 16 values per thread (n a multiple of 16; both 16-byte aligned).
__global__ void z_to_f16_kernel(const int8_t *z, __half *z16, int64_t n) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n / 16; i += int64_t(gridDim.x) * blockDim.x) {
        const int4 v = reinterpret_cast<const int4 *>(z)[i];
        const int w[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const __half2 h = __floats2half2_rn(float(int8_t(w[k] >> (16 * e))), float(int8_t(w[k] >> (16 * e + 8))));
                o[2 * k + e] = *reinterpret_cast<const uint32_t *>(&h);
            }
        }
        uint4 *dst = reinterpret_cast<uint4 *>(z16) + 2 * i;
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

// Four codes (bytes 0..3 of v, each < 1024) -> two fp16 pairs (c0, c1), (c2, c3), exactly:
// the byte under 0x64 is the fp16 pattern of 1024 + c; subtracting 1024 leaves c.
__device__ __forceinline__ void codes_to_f16(uint32_t v, uint32_t &lo, uint32_t &hi) {
    const __half2 k1024 = __floats2half2_rn(1024.f, 1024.f);
    const uint32_t a = __byte_perm(v, 0x64646464u, 0x4140), b = __byte_perm(v, 0x64646464u, 0x4342);
    const __half2 ha = __hsub2(*reinterpret_cast<const __half2 *>(&a), k1024);
    const __half2 hb = __hsub2(*reinterpret_cast<const __half2 *>(&b), k1024);
    lo = *reinterpret_cast<const uint32_t *>(&ha);
    hi = *reinterpret_cast<const uint32_t *>(&hb);
}

// TMEM column of drain chunk c (0 = gate, 1 = up) for warp group h: rows [kPfRpt h, kPfRpt (h+1)).
__device__ __forceinline__ constexpr int pf_col(int c, int h) { return kPfRpt * h + kPfRows * c; }

// SiLU(g)*u of two adjacent rows as fp16 hi + lo pairs (rows >= F are padding: zeros).
__device__ __forceinline__ void pf_store_h2(const ResidualParams &p, int tok, int row, float g0, float u0, float g1,
                                            float u1) {
    const int64_t i = (int64_t(tok) * p.F16 + row) >> 1;
    float h0 = g0 / (1.0f + expf(-g0)) * u0, h1 = g1 / (1.0f + expf(-g1)) * u1;
    if (row >= p.F) h0 = 0.f;
    if (row + 1 >= p.F) h1 = 0.f;
    const __half2 hi = __floats2half2_rn(h0, h1);
    const float2 hf = __half22float2(hi);
    reinterpret_cast<__half2 *>(p.h_hi)[i] = hi;
    reinterpret_cast<__half2 *>(p.h_lo)[i] = __floats2half2_rn(h0 - hf.x, h1 - hf.y);
}

// Drain warps (4..11): token 32 (warp % 4) + lane of the CTA's 128, warp group h takes rows
// [32h, 32h+32) of gate and up. Per group two chunks (gate, up) of 32 TMEM columns, each
// loaded one chunk ahead of its arithmetic; a group's buffer is released as soon as its
// last chunk has landed.
template <bool DOTS>
__device__ __forceinline__ void drain_prefill(const ResidualParams &p, const float *al_ring, uint64_t *acc_full,
                                              uint64_t *acc_empty, uint64_t *al_full, uint64_t *al_empty,
                                              uint32_t tmem, int t0, int rt, int nkt, int S4, int warp, int lane) {
    const int q = warp & 3, h = (warp - 4) >> 2;
    const int tok = t0 + 32 * q + lane;
    const bool tv = tok < p.T;
    const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16);
    float2 acc[2][kPfRpt / 2];
#pragma unroll
    for (int pj = 0; pj < 2; ++pj)
#pragma unroll
        for (int k = 0; k < kPfRpt / 2; ++k) acc[pj][k] = make_float2(0.f, 0.f);
    // s and the base sums come from the preceding work of the stream
    sm100::grid_dependency_wait();
    const float2 *srow = reinterpret_cast<const float2 *>(p.s + int64_t(tv ? tok : 0) * p.G);
    float2 s_next = tv ? __ldg(srow) : make_float2(0.f, 0.f);
    bool ok = __all_sync(0xffffffffu, sm100::mbar_wait(acc_full, 0, p.err, sm100::kErrWaitFull));
    uint32_t rb[2][kPfCh];
    sm100::tc_fence_after();
    if (ok) sm100::tmem_ld<kPfCh>(lane_base + uint32_t(pf_col(0, h)), rb[0]);
    for (int kt = 0; kt < nkt; ++kt) {
        const float2 sc = s_next;  // s[tok, 2kt], s[tok, 2kt + 1]
        if (kt + 1 < nkt && tv) s_next = __ldg(srow + kt + 1);
        const int s4 = kt % S4;
        if (ok) ok = __all_sync(0xffffffffu, sm100::mbar_wait(al_full + s4, (kt / S4) & 1, p.err, sm100::kErrWaitFull));
        const float *AL = al_ring + s4 * (2 * kPfN);
#pragma unroll
        for (int st = 0; st < 4; ++st) {
            const int j = st >> 1, c = st & 1;
            const int gi = 2 * kt + j;
            if (ok) sm100::tmem_wait_ld();  // chunk st has landed
            if (c == 1) {                   // last chunk of the group: release its buffer
                sm100::tc_fence_before();
                sm100::mbar_arrive(acc_empty + gi % kPfBufs);
            }
            const int gn = c == 1 ? gi + 1 : gi, cn = c ^ 1;
            if (gn < 2 * nkt && ok) {
                if (cn == 0) {
                    ok = __all_sync(0xffffffffu, sm100::mbar_wait(acc_full + gn % kPfBufs, (gn / kPfBufs) & 1, p.err,
                                                                  sm100::kErrWaitFull));
                    sm100::tc_fence_after();
                }
                if (ok)
                    sm100::tmem_ld<kPfCh>(lane_base + uint32_t((gn % kPfBufs) * kPfN + pf_col(cn, h)), rb[(st + 1) & 1]);
            }
            if (ok) {
                const uint32_t *r = rb[st & 1];
                const float sj = j == 0 ? sc.x : sc.y;
                const float2 s2 = make_float2(sj, sj);
                const float *al = AL + j * kPfN + pf_col(c, h);
#pragma unroll
                for (int k4 = 0; k4 < kPfCh / 4; ++k4) {
                    const float4 a = *reinterpret_cast<const float4 *>(al + 4 * k4);
                    const float2 x0 = make_float2(__uint_as_float(r[4 * k4]), __uint_as_float(r[4 * k4 + 1]));
                    const float2 x1 = make_float2(__uint_as_float(r[4 * k4 + 2]), __uint_as_float(r[4 * k4 + 3]));
                    acc[c][2 * k4] = sm100::ffma2(make_float2(a.x, a.y), sm100::fmul2(x0, s2), acc[c][2 * k4]);
                    acc[c][2 * k4 + 1] = sm100::ffma2(make_float2(a.z, a.w), sm100::fmul2(x1, s2), acc[c][2 * k4 + 1]);
                }
                if constexpr (DOTS) {
                    if (tv) {
                        int32_t *dp = p.dots + (int64_t(c) * p.T + tok) * int64_t(p.F) * p.G;
#pragma unroll
                        for (int k = 0; k < kPfCh; ++k) {
                            const int row = rt * kPfRows + kPfRpt * h + k;
                            if (row < p.F) dp[int64_t(row) * p.G + gi] = int(__uint_as_float(r[k]));
                        }
                    }
                }
            }
        }
        sm100::mbar_arrive(al_empty + s4);
    }
    if (!ok || !tv) return;
    const int row0 = rt * kPfRows + kPfRpt * h;
    if (p.h_hi != nullptr) {
        // merge with the base sums, SiLU(g)*u, fp16 hi + lo; rows F..F16-1 get zeros
        const float *gb = p.base[0] + int64_t(tok) * p.F, *ub = p.base[1] + int64_t(tok) * p.F;
#pragma unroll
        for (int k0 = 0; k0 < kPfRpt / 2; k0 += 4) {
            float gv[8], uv[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int row = row0 + 2 * k0 + k;
                gv[k] = row < p.F ? __ldg(gb + row) : 0.f;
                uv[k] = row < p.F ? __ldg(ub + row) : 0.f;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int row = row0 + 2 * (k0 + k);
                if (row < p.F16)
                    pf_store_h2(p, tok, row, acc[0][k0 + k].x + gv[2 * k], acc[1][k0 + k].x + uv[2 * k],
                                acc[0][k0 + k].y + gv[2 * k + 1], acc[1][k0 + k].y + uv[2 * k + 1]);
            }
        }
    } else {
        float *og = p.out[0] + int64_t(tok) * p.F, *ou = p.out[1] + int64_t(tok) * p.F;
#pragma unroll
        for (int k = 0; k < kPfRpt / 2; ++k) {
            const int row = row0 + 2 * k;
            if (row < p.F) {
                og[row] = acc[0][k].x;
                ou[row] = acc[1][k].x;
            }
            if (row + 1 < p.F) {
                og[row + 1] = acc[0][k].y;
                ou[row + 1] = acc[1][k].y;
            }
        }
    }
}

template <bool DOTS>
__global__ void __launch_bounds__(kPfThreads, 1)
    residual_prefill_kernel(const __grid_constant__ CUtensorMap tm_z16, const PfParams P) {
    const ResidualParams &p = P.p;
    const PfLayout &Ly = P.L;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *a_ring = smem;                 // [SA][128 tokens][128 B] fp16 activations
    uint8_t *w_ring = smem + Ly.w_off;      // [SW][kPfN rows][128 B] fp16 codes
    uint8_t *src_ring = smem + Ly.src_off;  // [S1] records + alphas of the record tile
    float *al_ring = reinterpret_cast<float *>(smem + Ly.al_off);  // [S4][2 groups][kPfN] f32 alphas
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Ly.bar_off);
    uint64_t *a_full = bars, *a_empty = a_full + kPfMaxSA;
    uint64_t *src_full = a_empty + kPfMaxSA, *src_empty = src_full + kPfMaxS1;
    uint64_t *w_full = src_empty + kPfMaxS1, *w_empty = w_full + kPfMaxSW;
    uint64_t *al_full = w_empty + kPfMaxSW, *al_empty = al_full + kPfMaxS4;
    uint64_t *acc_full = al_empty + kPfMaxS4, *acc_empty = acc_full + kPfBufs;
    uint64_t *done = acc_empty + kPfBufs;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int C = p.G / 2;
    const int rt = blockIdx.y, t0 = blockIdx.x * kPfTokens;
    const int nkt = p.D / kPfKTile;  // = C: one record chunk per K tile
    const int SA = Ly.SA, S1 = Ly.S1, SW = Ly.SW, S4 = Ly.S4;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; ++s) {
            sm100::mbar_init(a_full + s, 1);
            sm100::mbar_init(a_empty + s, 1);
        }
        for (int s = 0; s < S1; ++s) {
            sm100::mbar_init(src_full + s, 1);
            sm100::mbar_init(src_empty + s, kPfWiden);
        }
        for (int s = 0; s < SW; ++s) {
            sm100::mbar_init(w_full + s, kPfWiden);
            sm100::mbar_init(w_empty + s, 1);
        }
        for (int s = 0; s < S4; ++s) {
            sm100::mbar_init(al_full + s, kPfWiden);
            sm100::mbar_init(al_empty + s, kPfDrain);
        }
        for (int b = 0; b < kPfBufs; ++b) {
            sm100::mbar_init(acc_full + b, 1);
            sm100::mbar_init(acc_empty + b, kPfDrain);
        }
        sm100::mbar_init(done, 1);
        sm100::fence_barrier_init();
    }
    if (warp == 1) sm100::tmem_alloc(tmem_slot, 512);
    sm100::trigger_dependents();
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= 4) {
        drain_prefill<DOTS>(p, al_ring, acc_full, acc_empty, al_full, al_empty, tmem, t0, rt, nkt, S4, warp, lane);
    } else {
        if (warp == 0) {
            // Producer. A lane reuses only its own stage, in order, so each parity test is at most
            // one phase ahead of its barrier; the warp polls with non-blocking tests.
            const int role = lane < S1 ? 0 : lane < S1 + SA ? 1 : -1;  // 0 records, 1 activations
            const int st = role == 0 ? lane : role == 1 ? lane - S1 : 0;
            const int depth = role == 0 ? S1 : SA;
            const uint32_t src_tx = uint32_t(Ly.pair_bytes + Ly.plane_bytes + Ly.alpha_bytes);
            const int ab = P.alpha_half ? 4 : 8;  // alpha bytes per record
            auto issue = [&](int kt) {
                if (role == 0) {
                    uint8_t *src = src_ring + st * Ly.src_bytes;
                    const int64_t rec = (int64_t(rt) * C + kt) * 128;  // chunk kt of record tile rt
                    sm100::mbar_arrive_expect_tx(src_full + st, src_tx);
                    if (Ly.pair_bytes) sm100::bulk_load(src + Ly.off_pair, p.proj[0].pair + rec, Ly.pair_bytes, src_full + st);
                    if (Ly.plane_bytes)
                        sm100::bulk_load(src + Ly.off_plane, p.proj[0].plane + rec, Ly.plane_bytes, src_full + st);
                    sm100::bulk_load(src + Ly.off_alpha, static_cast<const uint8_t *>(p.proj[0].alpha) + rec * ab,
                                     Ly.alpha_bytes, src_full + st);
                } else {
                    sm100::mbar_arrive_expect_tx(a_full + st, kPfTokens * kPfRowBytes);
                    sm100::tma_load_2d(a_ring + st * (kPfTokens * kPfRowBytes), &tm_z16, kt * kPfKTile, t0, a_full + st);
                }
            };
            int kt = role >= 0 ? st : nkt;
            // Weights (fresh stages) go out before the dependency wait; activations, which come
            // from the preceding kernel of the stream, only after it.
            if (role == 0) {
                if (kt < nkt) issue(kt);
                kt += depth;
            }
            sm100::grid_dependency_wait();
            uint64_t *empty = role == 0 ? src_empty : a_empty;
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
                    __nanosleep(128);
                }
            }
            // No copy may still be in flight when the CTA exits: each lane waits for the final
            // use of its stage (earlier uses completed before the stage was refilled).
            if (role >= 0 && st < nkt) {
                const int last_kt = st + (nkt - 1 - st) / depth * depth;
                sm100::mbar_wait((role == 0 ? src_full : a_full) + st, (last_kt / depth) & 1, p.err, sm100::kErrWaitFull);
            }
        } else if (warp == 1) {
            if (lane == 0) {  // MMA issuer: per group two K = 16 MMAs into its TMEM buffer
                constexpr uint32_t idesc = sm100::umma_idesc_f16_f32(kPfTokens, kPfN);
                bool ok = true;
                for (int kt = 0; kt < nkt && ok; ++kt) {
                    const int sa = kt % SA, sw = kt % SW;
                    if (!(ok = sm100::mbar_wait(a_full + sa, (kt / SA) & 1, p.err, sm100::kErrWaitFull) &&
                               sm100::mbar_wait(w_full + sw, (kt / SW) & 1, p.err, sm100::kErrWaitFull)))
                        break;
                    sm100::tc_fence_after();
                    const uint32_t a = sm100::smem_u32(a_ring + sa * (kPfTokens * kPfRowBytes));
                    const uint32_t w = sm100::smem_u32(w_ring + sw * (kPfN * kPfRowBytes));
    #pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int gi = 2 * kt + j, b = gi % kPfBufs;
                        if (!(ok = sm100::mbar_wait(acc_empty + b, ((gi / kPfBufs) & 1) ^ 1, p.err, sm100::kErrWaitEmpty)))
                            break;
                        sm100::tc_fence_after();
    #pragma unroll
                        for (int k = 0; k < 2; ++k)
                            sm100::umma_f16(tmem + uint32_t(b * kPfN), sm100::umma_desc_sw128(a + 64 * j + 32 * k),
                                            sm100::umma_desc_sw128(w + 64 * j + 32 * k), idesc, k);
                        sm100::umma_commit(acc_full + b);
                    }
                    sm100::umma_commit(a_empty + sa);
                    sm100::umma_commit(w_empty + sw);
                }
                sm100::umma_commit(done);
            }
        } else if (warp < 4) {
            // Widening: thread wt handles records wt and wt + 64 of the K tile's 128 (the
            // [64 gate | 64 up] rows). Record m's 64 codes become fp16 row n = m of the B tile:
            // 16-byte unit u (codes 8u..8u+7) at n*128 + ((u ^ (n & 7)) << 4); its two alphas
            // go to al[0][n], al[1][n].
            const int wt = threadIdx.x - 64;
            const int rbits = P.rbits;
            bool ok = true;
            for (int kt = 0; kt < nkt; ++kt) {
                const int s1 = kt % S1, sw = kt % SW, s4 = kt % S4;
                if (ok)
                    ok = __all_sync(0xffffffffu,
                                    sm100::mbar_wait(src_full + s1, (kt / S1) & 1, p.err, sm100::kErrWaitFull) &&
                                        sm100::mbar_wait(w_empty + sw, ((kt / SW) & 1) ^ 1, p.err, sm100::kErrWaitEmpty) &&
                                        sm100::mbar_wait(al_empty + s4, ((kt / S4) & 1) ^ 1, p.err, sm100::kErrWaitEmpty));
                if (ok) {
                    const uint8_t *src = src_ring + s1 * Ly.src_bytes;
                    uint8_t *W = w_ring + sw * (kPfN * kPfRowBytes);
                    float *AL = al_ring + s4 * (2 * kPfN);
    #pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const int m = wt + 64 * i;
                        uint4 w = make_uint4(0, 0, 0, 0);
                        uint2 pw = make_uint2(0, 0);
                        float a0, a1;
                        if (Ly.pair_bytes) w = reinterpret_cast<const uint4 *>(src + Ly.off_pair)[m];
                        if (Ly.plane_bytes) pw = reinterpret_cast<const uint2 *>(src + Ly.off_plane)[m];
                        if (P.alpha_half)
                            load_scale2_shared<true>(src + Ly.off_alpha, m, a0, a1);
                        else
                            load_scale2_shared<false>(src + Ly.off_alpha, m, a0, a1);
                        AL[m] = a0;
                        AL[kPfN + m] = a1;
                        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
                        uint8_t *row = W + m * kPfRowBytes;
    #pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {  // word jj: codes 16jj .. 16jj + 15
                            const uint32_t pv = jj < 2 ? pw.x : pw.y;
                            uint32_t o[8];
    #pragma unroll
                            for (int qq = 0; qq < 4; ++qq)
                                codes_to_f16(um_low_bits(ws[jj], pv, qq, jj & 1, rbits), o[2 * qq], o[2 * qq + 1]);
                            *reinterpret_cast<uint4 *>(row + (((2 * jj) ^ (m & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                            *reinterpret_cast<uint4 *>(row + (((2 * jj + 1) ^ (m & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
                        }
                    }
                    sm100::fence_proxy_async_smem();  // generic-proxy stores -> tensor-core operand reads
                }
                sm100::mbar_arrive(w_full + sw);
                sm100::mbar_arrive(al_full + s4);
                sm100::mbar_arrive(src_empty + s1);
            }
        }
    }
    __syncwarp();
    sm100::mbar_wait(done, 0, p.err, sm100::kErrWaitDone);
    sm100::tc_fence_after();
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 1) sm100::tmem_dealloc(tmem, 512);
}

}  // namespace ffnrm
