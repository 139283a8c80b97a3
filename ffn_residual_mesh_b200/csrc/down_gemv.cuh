// Merge + SwiGLU + fp16 down projection on CUDA cores (decode, few tokens).
//
// Replaces swiglu_down_kernel (src/exact_cpu_base_gpu_full_ffn_runner.cu:217-240),
// which recomputes SwiGLU for every output row, and the torch.mm down of
// scripts/benchmark_gpu_full_ffn_density.py:162. Grid = (D/64 output tiles,
// split-K slices of d_ff, token chunks). Each CTA merges g = g_base + g_res and
// u = u_base + u_res for its d_ff slice once into shared memory (rows of flagged
// fallback tiles take the unsplit projection, already in g_res/u_res), applies
// h = g/(1+exp(-g))*u, then every warp streams 8 fp16 down rows with 128-bit loads
// and accumulates in fp32. Split-K partials [splits, T, D] are summed in a fixed
// order by splitk_reduce_kernel, so results are deterministic.
#pragma once

#include "ffnrm_common.cuh"

namespace ffnrm {

struct DownParams {
    const float *gate_res, *up_res;    // [T, F]
    const float *gate_base, *up_base;  // [T, F]
    const uint8_t *fallback_tiles;
    const __half *down;                // [D, F] (ld = F)
    float *partial;                    // [splits, T, D]
    int F, D, T, tile_rows, splits, kc;
};

constexpr int kDownRowsPerWarp = 8;
constexpr int kDownWarps = 8;
constexpr int kDownTileRows = kDownRowsPerWarp * kDownWarps;  // 64 output rows per CTA

template <int TT>
__global__ void __launch_bounds__(256) swiglu_down_kernel(const DownParams p) {
    extern __shared__ __align__(16) float h_sm[];  // [TT][kc]
    const int split = blockIdx.y;
    const int t0 = blockIdx.z * TT;
    const int k0 = split * p.kc;
    const int nk = min(p.kc, p.F - k0);
    if (nk <= 0) return;
    for (int idx = threadIdx.x; idx < TT * p.kc; idx += blockDim.x) {
        const int t = idx / p.kc, k = idx - t * p.kc;
        float hv = 0.f;
        if (k < nk && t0 + t < p.T) {
            const int f = k0 + k;
            const int64_t i = int64_t(t0 + t) * p.F + f;
            float g = p.gate_res[i], u = p.up_res[i];
            if (!row_flagged(p.fallback_tiles, f, p.tile_rows)) {
                g += p.gate_base[i];
                u += p.up_base[i];
            }
            hv = g / (1.0f + expf(-g)) * u;
        }
        h_sm[idx] = hv;
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int o0 = blockIdx.x * kDownTileRows + warp * kDownRowsPerWarp;
    float acc[kDownRowsPerWarp][TT];
#pragma unroll
    for (int j = 0; j < kDownRowsPerWarp; ++j)
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[j][t] = 0.f;

    const int chunks = nk / 8;
    for (int c = lane; c < chunks; c += 32) {
        float hv[TT][8];
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            const float4 *src = reinterpret_cast<const float4 *>(h_sm + t * p.kc + c * 8);
            const float4 lo = src[0], hi = src[1];
            hv[t][0] = lo.x; hv[t][1] = lo.y; hv[t][2] = lo.z; hv[t][3] = lo.w;
            hv[t][4] = hi.x; hv[t][5] = hi.y; hv[t][6] = hi.z; hv[t][7] = hi.w;
        }
#pragma unroll
        for (int j = 0; j < kDownRowsPerWarp; ++j) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(p.down + int64_t(o0 + j) * p.F + k0) + c);
            const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
            float w[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 f = __half22float2(h2[q]);
                w[2 * q] = f.x;
                w[2 * q + 1] = f.y;
            }
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                float a = acc[j][t];
#pragma unroll
                for (int q = 0; q < 8; ++q) a = fmaf(w[q], hv[t][q], a);
                acc[j][t] = a;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kDownRowsPerWarp; ++j) {
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            const float v = warp_sum(acc[j][t]);
            if (lane == 0 && t0 + t < p.T) p.partial[(int64_t(split) * p.T + t0 + t) * p.D + o0 + j] = v;
        }
    }
}

// y[t, o] = sum_s partial[s, t, o] in a fixed order; optional f32 and fp16 outputs.
__global__ void splitk_reduce_kernel(const float *partial, int splits, int64_t n, float *y32, __half *y16) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        float v = 0.f;
        for (int s = 0; s < splits; ++s) v += partial[int64_t(s) * n + i];
        if (y32) y32[i] = v;
        if (y16) y16[i] = __float2half_rn(v);
    }
}

__global__ void cast_f16_kernel(const float *src, __half *dst, int64_t n) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}

}  // namespace ffnrm
