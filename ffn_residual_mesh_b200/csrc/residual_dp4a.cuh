// Decode residual contraction on CUDA cores: exact int32 group dots with __dp4a,
// gate and up of the same rows in one CTA, lane-per-row.
//
// Replaces residual_kernel (src/exact_residual_cuda_runner.cu:122-159), which
// evaluates q*alpha*z*s per element in fp32 with byte loads and a shared-memory
// tree. Here a CTA owns one 32-row block of both projections: lane l owns row
// 32*rb + l; warps 0-3 take the gate rows and 4-7 the up rows, each splitting the
// d_model groups four ways, and every warp-wide load reads 32 consecutive 16-byte
// code records (512 B, fully coalesced). Activations sit in shared memory in natural
// order and are read as broadcasts, so no warp reduction is needed; each group dot is
// exact in int32 before alpha[row,g]*s[t,g] is applied in fp32. Partial sums of the
// warps meet in shared memory in a fixed order. Rows of flagged fallback tiles compute
// sum_g s*(alpha*(P01 + 4 P23) + beta*zsum) instead. In forward mode the CTA then
// merges both projections with the base sums and writes h = SiLU(g)*u for the down
// projection (the merge of src/exact_cpu_base_gpu_full_ffn_runner.cu:225-227).
#pragma once

#include "ffnrm_common.cuh"

namespace ffnrm {

struct ResidualParams {
    ProjView proj[2];
    const int8_t *z;      // [T, D]
    const float *s;       // [T, G]
    float *out[2];        // [T, F] (residual mode) or null
    int32_t *dots;        // [2, T, F, G] or null
    const uint8_t *fallback_tiles;
    // forward mode: merge with the base sums and write h = SiLU(g)*u as fp16 hi + lo
    const float *base[2];  // [T, F]
    __half *h_hi, *h_lo;   // [T, F16], F16 = F rounded up to 16 (padding columns written as 0)
    int F, D, G, T, tile_rows, F16;
    int row_blocks;       // ceil(F / 32)
    int *err;             // pipeline-wait error word (tensor-core kernel), or null
};

// h = g/(1+exp(-g))*u for one (token, row) of merged g and u; rows >= F are padding and
// get zeros. Writes fp16 hi and lo = fp16(h - hi).
__device__ __forceinline__ void write_h(const ResidualParams &p, int tok, int row, float g, float u) {
    const int64_t i = int64_t(tok) * p.F16 + row;
    if (row >= p.F) {
        p.h_hi[i] = __float2half_rn(0.f);
        p.h_lo[i] = __float2half_rn(0.f);
        return;
    }
    const float h = g / (1.0f + expf(-g)) * u;
    const __half hi = __float2half_rn(h);
    p.h_hi[i] = hi;
    p.h_lo[i] = __float2half_rn(h - __half2float(hi));
}

// h = g/(1+exp(-g))*u for one (token, row); flagged rows ignore the base (their g/u
// already are the unsplit projections). Writes fp16 hi and lo = fp16(h - hi).
__device__ __forceinline__ void store_h(const ResidualParams &p, int tok, int row, float g, float u, bool flagged) {
    const int64_t i = int64_t(tok) * p.F16 + row;
    if (row >= p.F) {
        p.h_hi[i] = __float2half_rn(0.f);
        p.h_lo[i] = __float2half_rn(0.f);
        return;
    }
    if (!flagged) {
        g += p.base[0][int64_t(tok) * p.F + row];
        u += p.base[1][int64_t(tok) * p.F + row];
    }
    const float h = g / (1.0f + expf(-g)) * u;
    const __half hi = __float2half_rn(h);
    p.h_hi[i] = hi;
    p.h_lo[i] = __float2half_rn(h - __half2float(hi));
}

constexpr int kResWarps = 4;  // per projection; the CTA runs 2 * kResWarps warps
constexpr int kGemvMaxTokens = 4;  // largest GEMV instance (batches of 3-4 prefer the tensor cores)

// Each warp streams its chunk records through a cp.async ring of kGemvBufs windows of
// kGemvWin chunks, so about kGemvBufs * kGemvWin chunks per lane are in flight while it
// computes.
constexpr int kGemvWin = 4, kGemvBufs = 3;
template <int RB, bool AHALF>
struct GemvStage {
    static constexpr int pair = RB != 1 ? 16 : 0;  // bytes per lane and chunk
    static constexpr int plane = RB != 2 ? 8 : 0;
    static constexpr int alpha = AHALF ? 4 : 8;
    static constexpr int warp_bytes = kGemvBufs * kGemvWin * 32 * (pair + plane + alpha);
};

// Shared memory: [z TT*D int8][s TT*G f32][zsum TT*G f32][red 2*kResWarps*TT*32 f32]
// [per-warp record rings]
template <int RB, bool AHALF>
inline size_t residual_smem_bytes(int TT, int D) {
    const int G = D / 32;
    const size_t head = size_t(TT) * D + size_t(TT) * G * 8 + size_t(2 * kResWarps) * TT * 32 * 4;
    return (head + 15) / 16 * 16 + size_t(2 * kResWarps) * GemvStage<RB, AHALF>::warp_bytes;
}

template <int RB, int TT, bool AHALF>
__global__ void __launch_bounds__(2 * kResWarps * 32, TT == 1 ? 3 : 2) residual_gemv_kernel(const ResidualParams p) {
    using GS = GemvStage<RB, AHALF>;
    extern __shared__ __align__(16) uint8_t smem[];
    const int G = p.G, D = p.D, F = p.F, T = p.T;
    int8_t *z_sm = reinterpret_cast<int8_t *>(smem);
    float *s_sm = reinterpret_cast<float *>(smem + size_t(TT) * D);
    float *zsum_sm = s_sm + TT * G;
    float *red = zsum_sm + TT * G;
    const size_t head = size_t(TT) * D + size_t(TT) * G * 8 + size_t(2 * kResWarps) * TT * 32 * 4;
    uint8_t *rings = smem + (head + 15) / 16 * 16;

    const int rb = blockIdx.x;
    const int t0 = blockIdx.y * TT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int proj = warp / kResWarps, wk = warp - proj * kResWarps;
    const int row = rb * 32 + lane;
    const bool valid = row < F;
    const ProjView pv = p.proj[proj];
    const int C = G / 2;
    const int c_begin = wk * C / kResWarps, c_end = (wk + 1) * C / kResWarps;

    // The warp's chunk records stream through its cp.async ring; each lane reads back only
    // what it copied. The rare fallback rows load their extra data when used. The records
    // and alphas are weights, so the first windows go out before the wait on the preceding
    // kernel of the stream (dependent launch); activations, scales and flags after it.
    uint8_t *ring = rings + size_t(warp) * GS::warp_bytes;
    uint4 *pair_r = reinterpret_cast<uint4 *>(ring);                                          // [bufs][win][32]
    uint2 *plane_r = reinterpret_cast<uint2 *>(ring + kGemvBufs * kGemvWin * 32 * GS::pair);  // [bufs][win][32]
    uint8_t *alpha_r = ring + kGemvBufs * kGemvWin * 32 * (GS::pair + GS::plane);             // [bufs][win][32]
    const int nwin = (c_end - c_begin + kGemvWin - 1) / kGemvWin;
    auto issue = [&](int w) {  // window w into buffer w % kGemvBufs (an empty group past the end)
        if (w < nwin) {
            const int b = w % kGemvBufs;
#pragma unroll
            for (int u = 0; u < kGemvWin; ++u) {
                const int c = c_begin + w * kGemvWin + u;
                if (c < c_end) {
                    const int64_t rec = rec_index(rb, C, c, lane);
                    const int slot = (b * kGemvWin + u) * 32 + lane;
                    if (RB != 1) cp_async16(pair_r + slot, pv.pair + rec, true);
                    if (RB != 2) cp_async_small<8>(plane_r + slot, pv.plane + rec);
                    cp_async_small<GS::alpha>(alpha_r + size_t(slot) * GS::alpha,
                                              static_cast<const uint8_t *>(pv.alpha) + rec * GS::alpha);
                }
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int w = 0; w < kGemvBufs - 1; ++w) issue(w);
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

    // Stage TT tokens of activations (16-byte copies) and their group scales.
    const int zvec = TT * D / 16;
    for (int i = threadIdx.x; i < zvec; i += blockDim.x) {
        const int t = (i * 16) / D;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (t0 + t < T) v = __ldg(reinterpret_cast<const uint4 *>(p.z + int64_t(t0) * D) + i);
        reinterpret_cast<uint4 *>(z_sm)[i] = v;
    }
    for (int i = threadIdx.x; i < TT * G; i += blockDim.x) {
        const int t = i / G;
        float sv = 0.f, zs = 0.f;
        if (t0 + t < T) {
            sv = p.s[int64_t(t0) * G + i];
            if (p.fallback_tiles) {
                const int8_t *zr = p.z + int64_t(t0) * D + int64_t(i) * kGroup;
                int a = 0;
                for (int k = 0; k < kGroup; ++k) a += zr[k];
                zs = float(a);
            }
        }
        s_sm[i] = sv;
        zsum_sm[i] = zs;
    }
    __syncthreads();

    const bool flagged = valid && row_flagged(p.fallback_tiles, row, p.tile_rows);
    float acc[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) acc[t] = 0.f;

    for (int w = 0; w < nwin; ++w) {
        issue(w + kGemvBufs - 1);
        cp_async_wait<kGemvBufs - 1>();  // window w has landed
        const int b = w % kGemvBufs;
#pragma unroll
        for (int u = 0; u < kGemvWin; ++u) {
            const int c = c_begin + w * kGemvWin + u;
            if (c >= c_end) break;
            const int slot = (b * kGemvWin + u) * 32 + lane;
            uint4 wp = RB != 1 ? pair_r[slot] : make_uint4(0, 0, 0, 0), wh = make_uint4(0, 0, 0, 0);
            const uint2 wq = RB != 2 ? plane_r[slot] : make_uint2(0, 0);
            float a0, a1;
            load_scale2_shared<AHALF>(alpha_r, slot, a0, a1);
            float b0 = 0.f, b1 = 0.f;
            if (flagged) {
                const int64_t rec = rec_index(rb, C, c, lane);
                if (RB == 1) wp = __ldg(pv.pair + rec);
                wh = __ldg(pv.pair_hi + rec);
                load_scale2<AHALF>(pv.beta, rec, b0, b1);
            }
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                const uint4 *zv = reinterpret_cast<const uint4 *>(z_sm + t * D + c * 64);
                const uint4 z0 = zv[0], z1 = zv[1], z2 = zv[2], z3 = zv[3];
                int P0, P1;
                if (RB == 1) {
                    P0 = dot_plane(wq.x, z0, z1);
                    P1 = dot_plane(wq.y, z2, z3);
                } else {
                    P0 = dot_pair(wp.x, wp.y, z0, z1);
                    P1 = dot_pair(wp.z, wp.w, z2, z3);
                    if (RB == 3) {
                        P0 += 4 * dot_plane(wq.x, z0, z1);
                        P1 += 4 * dot_plane(wq.y, z2, z3);
                    }
                }
                const float s0 = s_sm[t * G + 2 * c], s1 = s_sm[t * G + 2 * c + 1];
                if (p.dots != nullptr && valid && t0 + t < T)
                    *reinterpret_cast<int2 *>(p.dots + ((int64_t(proj) * T + t0 + t) * F + row) * G + 2 * c) =
                        make_int2(P0, P1);
                if (flagged) {
                    const int F0 = dot_pair(wp.x, wp.y, z0, z1) + 4 * dot_pair(wh.x, wh.y, z0, z1);
                    const int F1 = dot_pair(wp.z, wp.w, z2, z3) + 4 * dot_pair(wh.z, wh.w, z2, z3);
                    const float zs0 = zsum_sm[t * G + 2 * c], zs1 = zsum_sm[t * G + 2 * c + 1];
                    acc[t] += s0 * (a0 * float(F0) + b0 * zs0) + s1 * (a1 * float(F1) + b1 * zs1);
                } else {
                    acc[t] = fmaf(float(P0), a0 * s0, acc[t]);
                    acc[t] = fmaf(float(P1), a1 * s1, acc[t]);
                }
            }
        }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int t = 0; t < TT; ++t) red[(warp * TT + t) * 32 + lane] = acc[t];
    __syncthreads();
    if (p.h_hi != nullptr) {
        // forward mode: warp 0 merges gate and up of its 32 rows and writes h
        if (warp == 0 && row < p.F16) {
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                if (t0 + t >= T) continue;
                float gv = 0.f, uv = 0.f;
#pragma unroll
                for (int w = 0; w < kResWarps; ++w) {
                    gv += red[(w * TT + t) * 32 + lane];
                    uv += red[((kResWarps + w) * TT + t) * 32 + lane];
                }
                store_h(p, t0 + t, row, gv, uv, flagged);
            }
        }
    } else if (wk == 0 && valid) {
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kResWarps; ++w) v += red[((proj * kResWarps + w) * TT + t) * 32 + lane];
            if (t0 + t < T) p.out[proj][int64_t(t0 + t) * F + row] = v;
        }
    }
}

}  // namespace ffnrm
