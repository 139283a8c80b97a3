// Merge + SwiGLU + fp16 down projection on CUDA cores (decode, few tokens), lane-per-row.
//
// Replaces swiglu_down_kernel (src/exact_cpu_base_gpu_full_ffn_runner.cu:217-240),
// which recomputes SwiGLU for every output row, and the torch.mm down of
// scripts/benchmark_gpu_full_ffn_density.py:162. Grid = (D/256 output blocks,
// split-K slices of d_ff). A CTA merges g = g_base + g_res and u = u_base + u_res for
// its d_ff slice once into shared memory (rows of flagged fallback tiles take the
// unsplit projection that the residual kernel already wrote into g_res/u_res), applies
// h = g/(1+exp(-g))*u, then each warp streams 32 output rows of the interleaved fp16
// down weight (lane l owns row 32*ob + l, one warp load = 512 contiguous bytes) and
// accumulates in fp32 against broadcast reads of h. Split-K partials [splits, TT, D]
// are summed in a fixed order by splitk_reduce_kernel (deterministic).
#pragma once

#include "ffnrm_common.cuh"

namespace ffnrm {

struct DownParams {
    const float *gate_res, *up_res;    // [T, F]
    const float *gate_base, *up_base;  // [T, F]
    const uint8_t *fallback_tiles;
    const uint4 *down_il;              // [D/32][F/8][32] records of 8 fp16
    float *partial;                    // [splits, TT, D]
    int F, D, T, t0, tile_rows, splits, kc;
};

constexpr int kDownWarps = 8;
constexpr int kDownBlockRows = 32 * kDownWarps;  // 256 output rows per CTA

template <int TT>
__global__ void __launch_bounds__(kDownWarps * 32) down_gemv_kernel(const DownParams p) {
    extern __shared__ __align__(16) float h_sm[];  // [TT][kc]
    const int split = blockIdx.y;
    const int k0 = split * p.kc;
    const int nk = min(p.kc, p.F - k0);
    for (int i = threadIdx.x; i < TT * p.kc; i += blockDim.x) {
        const int t = i / p.kc, k = i - t * p.kc;
        float hv = 0.f;
        if (k < nk && p.t0 + t < p.T) {
            const int f = k0 + k;
            const int64_t x = int64_t(p.t0 + t) * p.F + f;
            float g = p.gate_res[x], u = p.up_res[x];
            if (!row_flagged(p.fallback_tiles, f, p.tile_rows)) {
                g += p.gate_base[x];
                u += p.up_base[x];
            }
            hv = g / (1.0f + expf(-g)) * u;
        }
        h_sm[i] = hv;
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ob = blockIdx.x * kDownWarps + warp;  // 32-row block of outputs
    const int chunks_row = p.F / 8;
    const uint4 *w = p.down_il + (int64_t(ob) * chunks_row + k0 / 8) * 32 + lane;
    float acc[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) acc[t] = 0.f;
    const int nch = nk / 8;
#pragma unroll 4
    for (int c = 0; c < nch; ++c) {
        const uint4 raw = __ldg(w + int64_t(c) * 32);
        const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
        float wf[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 f = __half22float2(h2[q]);
            wf[2 * q] = f.x;
            wf[2 * q + 1] = f.y;
        }
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            const float4 *hv = reinterpret_cast<const float4 *>(h_sm + t * p.kc + c * 8);
            const float4 x0 = hv[0], x1 = hv[1];
            float a = acc[t];
            a = fmaf(wf[0], x0.x, a);
            a = fmaf(wf[1], x0.y, a);
            a = fmaf(wf[2], x0.z, a);
            a = fmaf(wf[3], x0.w, a);
            a = fmaf(wf[4], x1.x, a);
            a = fmaf(wf[5], x1.y, a);
            a = fmaf(wf[6], x1.z, a);
            a = fmaf(wf[7], x1.w, a);
            acc[t] = a;
        }
    }
    const int o = ob * 32 + lane;
#pragma unroll
    for (int t = 0; t < TT; ++t) p.partial[(int64_t(split) * TT + t) * p.D + o] = acc[t];
}

// y[t0 + t, o] = sum_s partial[s, t, o] in a fixed order; optional f32 and fp16 outputs.
__global__ void splitk_reduce_kernel(const float *partial, int splits, int tt, int rows_valid, int D, float *y32,
                                     __half *y16) {
    const int64_t n = int64_t(rows_valid) * D, stride = int64_t(tt) * D;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        float v = 0.f;
        for (int s = 0; s < splits; ++s) v += partial[int64_t(s) * stride + i];
        if (y32) y32[i] = v;
        if (y16) y16[i] = __float2half_rn(v);
    }
}

__global__ void cast_f16_kernel(const float *src, __half *dst, int64_t n) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}

}  // namespace ffnrm
