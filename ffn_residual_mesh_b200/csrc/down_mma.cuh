// Merge + SwiGLU + fp16 down projection on tensor cores (mma.sync m16n8k16, f32 accumulate).
//
// Replaces swiglu_down_kernel (src/exact_cpu_base_gpu_full_ffn_runner.cu:217-240) and
// the torch.mm down of scripts/benchmark_gpu_full_ffn_density.py:162.
//
// Layout: the fp16 down weight is stored fragment-native, [D/16][F16/16][32 lanes][4 words]:
// the 16 bytes a lane loads are exactly its A registers a0..a3 for one 16x16 tile, so a
// warp streams 512 contiguous bytes per tile with one 128-bit load per lane.
// Grid = (D/256 output blocks, split-K slices of d_ff). A CTA walks its d_ff slice in
// chunks: it merges g = g_base + g_res and u = u_base + u_res, applies
// h = g/(1+exp(-g))*u and splits h into fp16 hi + lo parts (h = hi + lo to ~2^-22
// relative) in shared memory; each warp then runs two MMAs per tile (hi and lo) for its
// 32 output rows against all tokens. Rows of flagged fallback tiles take the unsplit
// projection that the residual kernel wrote into g_res/u_res (no base added).
// Split-K partials go to a workspace; the last CTA of each output block (atomic
// ticket) sums them in slice order, so results are deterministic, and writes y.
#pragma once

#include "ffnrm_common.cuh"

namespace ffnrm {

struct DownMmaParams {
    const float *gate_res, *up_res;    // [T, F]
    const float *gate_base, *up_base;  // [T, F]
    const uint8_t *fallback_tiles;
    const uint4 *down_frag;            // [D/16][F16/16][32] records
    float *partial;                    // [splits][Tn][D] with Tn = NT*8
    int *tickets;                      // [D/256] zero-initialised, self-resetting
    float *y32;                        // [T, D] or null
    __half *y16;                       // [T, D] or null
    int F, F16, D, T, t0, tile_rows, splits, kc;
};

constexpr int kDownWarpsMma = 8;
constexpr int kDownRowsCta = kDownWarpsMma * 32;  // 256 output rows
constexpr int kDownKChunk = 128;                  // d_ff rows staged per step
constexpr int kDownHStride = kDownKChunk + 8;     // halves; padded for bank spread

__device__ __forceinline__ void mma_f16(float (&d)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// Shared memory: h hi/lo [2][TN][kDownHStride] fp16 + 1 int ticket flag.
inline size_t down_mma_smem_bytes(int TN) { return size_t(2) * TN * kDownHStride * 2 + 16; }

template <int NT>
__global__ void __launch_bounds__(kDownWarpsMma * 32) down_mma_kernel(const DownMmaParams p) {
    constexpr int TN = NT * 8;
    extern __shared__ __align__(16) uint8_t smem[];
    __half *h_hi = reinterpret_cast<__half *>(smem);
    __half *h_lo = h_hi + TN * kDownHStride;
    int *flag = reinterpret_cast<int *>(h_lo + TN * kDownHStride);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int ob = blockIdx.x;                     // 256-row output block
    const int split = blockIdx.y;
    const int k0 = split * p.kc;
    const int k1 = min(k0 + p.kc, p.F16);
    const int mt0 = ob * (kDownRowsCta / 16) + warp * 2;  // this warp's two 16-row tiles
    const int ksteps_row = p.F16 / 16;

    float acc[2][NT][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[m][n][e] = 0.f;

    for (int kb = k0; kb < k1; kb += kDownKChunk) {
        const int kn = min(kDownKChunk, k1 - kb);  // multiple of 16
        __syncthreads();
        for (int i = threadIdx.x; i < TN * kDownKChunk; i += blockDim.x) {
            const int tok = i / kDownKChunk, k = i - tok * kDownKChunk;
            const int f = kb + k;
            float hv = 0.f;
            if (k < kn && f < p.F && p.t0 + tok < p.T) {
                const int64_t x = int64_t(p.t0 + tok) * p.F + f;
                float gv = p.gate_res[x], uv = p.up_res[x];
                if (!row_flagged(p.fallback_tiles, f, p.tile_rows)) {
                    gv += p.gate_base[x];
                    uv += p.up_base[x];
                }
                hv = gv / (1.0f + expf(-gv)) * uv;
            }
            const __half hi = __float2half_rn(hv);
            h_hi[tok * kDownHStride + k] = hi;
            h_lo[tok * kDownHStride + k] = __float2half_rn(hv - __half2float(hi));
        }
        __syncthreads();
        const int steps = kn / 16;
#pragma unroll 2
        for (int s = 0; s < steps; ++s) {
            const int ks = kb / 16 + s;
            const uint4 a0 = __ldg(p.down_frag + (int64_t(mt0) * ksteps_row + ks) * 32 + lane);
            const uint4 a1 = __ldg(p.down_frag + (int64_t(mt0 + 1) * ksteps_row + ks) * 32 + lane);
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const int off = (n * 8 + g) * kDownHStride + s * 16 + 2 * t;
                const uint32_t bh0 = *reinterpret_cast<const uint32_t *>(h_hi + off);
                const uint32_t bh1 = *reinterpret_cast<const uint32_t *>(h_hi + off + 8);
                const uint32_t bl0 = *reinterpret_cast<const uint32_t *>(h_lo + off);
                const uint32_t bl1 = *reinterpret_cast<const uint32_t *>(h_lo + off + 8);
                mma_f16(acc[0][n], a0, bh0, bh1);
                mma_f16(acc[0][n], a0, bl0, bl1);
                mma_f16(acc[1][n], a1, bh0, bh1);
                mma_f16(acc[1][n], a1, bl0, bl1);
            }
        }
    }

    // Split-K partials: partial[split][tok][row], tok < TN (padding tokens hold zeros).
    const int64_t slice = int64_t(TN) * p.D;
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        const int r0 = (mt0 + m) * 16 + g;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int tk = n * 8 + 2 * t;
            float *pp = p.partial + split * slice;
            pp[int64_t(tk) * p.D + r0] = acc[m][n][0];
            pp[int64_t(tk + 1) * p.D + r0] = acc[m][n][1];
            pp[int64_t(tk) * p.D + r0 + 8] = acc[m][n][2];
            pp[int64_t(tk + 1) * p.D + r0 + 8] = acc[m][n][3];
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int ticket = atomicAdd(p.tickets + ob, 1);
        *flag = ticket == p.splits - 1;
    }
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    // Last CTA of this output block: y[t0 + tok, o] = sum over slices in order.
    const int rows_valid = min(TN, p.T - p.t0);
    for (int i = threadIdx.x; i < rows_valid * kDownRowsCta; i += blockDim.x) {
        const int tok = i / kDownRowsCta, o = ob * kDownRowsCta + (i - tok * kDownRowsCta);
        float v = 0.f;
        for (int sp = 0; sp < p.splits; ++sp) v += __ldcg(p.partial + sp * slice + int64_t(tok) * p.D + o);
        const int64_t yi = int64_t(p.t0 + tok) * p.D + o;
        if (p.y32) p.y32[yi] = v;
        if (p.y16) p.y16[yi] = __float2half_rn(v);
    }
    if (threadIdx.x == 0) p.tickets[ob] = 0;  // ready for the next launch on this stream
}

__global__ void cast_f16_kernel(const float *src, __half *dst, int64_t n) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}

}  // namespace ffnrm
