// fp16 down projection on tensor cores (mma.sync m16n8k16, f32 accumulate).
//
// Replaces swiglu_down_kernel (src/exact_cpu_base_gpu_full_ffn_runner.cu:217-240) and
// the torch.mm down of scripts/benchmark_gpu_full_ffn_density.py:162. The merge and
// SwiGLU already happened in the residual kernel, which wrote h = SiLU(g)*u as two
// fp16 parts (h = hi + lo to ~2^-22 relative), so y keeps fp32-level accuracy.
//
// Layout: the fp16 down weight is fragment-native, [D/16][F16/16][32 lanes][4 words]:
// the 16 bytes a lane loads are its A registers a0..a3 for one 16x16 tile, so a warp
// streams 512 contiguous bytes per tile with one 128-bit load per lane.
// Grid = (D/256 output blocks, split-K slices of d_ff). Each warp owns 32 output rows
// (two M tiles) and all TN tokens; h of the CTA's slice is staged into shared memory by
// cp.async one K chunk ahead. Split-K partials go to a workspace; the last CTA of each
// output block (atomic ticket) sums them in slice order, so the result is
// deterministic, and writes y in f32 and/or fp16.
#pragma once

#include "ffnrm_common.cuh"
#include "residual_mma.cuh"

namespace ffnrm {

struct DownMmaParams {
    const __half *h_hi, *h_lo;  // [T, F16]
    const uint4 *down_frag;     // [D/16][F16/16][32] records
    float *partial;             // [splits][TN][D]
    int *tickets;               // [D/256] zero-initialised, self-resetting
    float *y32;                 // [T, D] or null
    __half *y16;                // [T, D] or null
    int F16, D, T, t0, splits, kc;
};

constexpr int kDownWarpsMma = 8;
constexpr int kDownRowsCta = kDownWarpsMma * 32;  // 256 output rows
constexpr int kDownKChunk = 128;                  // d_ff columns staged per step
constexpr int kDownHStride = kDownKChunk + 8;     // halves; padded for bank spread

__device__ __forceinline__ void mma_f16(float (&d)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// Shared memory: 2 buffers x h hi/lo [TN][kDownHStride] fp16 + the ticket flag.
inline size_t down_mma_smem_bytes(int TN) { return size_t(2) * 2 * TN * kDownHStride * 2 + 16; }

template <int NT>
__global__ void __launch_bounds__(kDownWarpsMma * 32) down_mma_kernel(const DownMmaParams p) {
    constexpr int TN = NT * 8;
    constexpr int buf_halves = 2 * TN * kDownHStride;  // hi then lo
    extern __shared__ __align__(16) uint8_t smem[];
    __half *hbuf = reinterpret_cast<__half *>(smem);
    int *flag = reinterpret_cast<int *>(hbuf + 2 * buf_halves);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int ob = blockIdx.x;
    const int split = blockIdx.y;
    const int k0 = split * p.kc;
    const int k1 = min(k0 + p.kc, p.F16);
    const int mt0 = ob * (kDownRowsCta / 16) + warp * 2;
    const int ksteps_row = p.F16 / 16;

    auto stage = [&](int kb, int buf) {
        __half *dst = hbuf + buf * buf_halves;
        constexpr int vec = kDownKChunk / 8;  // 16-byte copies per token row
        for (int i = threadIdx.x; i < 2 * TN * vec; i += blockDim.x) {
            const int part = i / (TN * vec), r = i - part * TN * vec;
            const int tok = r / vec, v = r - tok * vec;
            const int k = kb + v * 8;
            const bool ok = p.t0 + tok < p.T && k < k1;
            const __half *src = (part ? p.h_lo : p.h_hi) + int64_t(ok ? p.t0 + tok : 0) * p.F16 + (ok ? k : 0);
            cp_async16(dst + part * TN * kDownHStride + tok * kDownHStride + v * 8, src, ok);
        }
        cp_async_commit();
    };

    float acc[2][NT][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[m][n][e] = 0.f;

    if (k0 < k1) stage(k0, 0);
    int buf = 0;
    for (int kb = k0; kb < k1; kb += kDownKChunk, buf ^= 1) {
        if (kb + kDownKChunk < k1) {
            stage(kb + kDownKChunk, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const __half *hh = hbuf + buf * buf_halves;
        const __half *hl = hh + TN * kDownHStride;
        const int steps = min(kDownKChunk, k1 - kb) / 16;
#pragma unroll 2
        for (int s = 0; s < steps; ++s) {
            const int ks = kb / 16 + s;
            const uint4 a0 = __ldg(p.down_frag + (int64_t(mt0) * ksteps_row + ks) * 32 + lane);
            const uint4 a1 = __ldg(p.down_frag + (int64_t(mt0 + 1) * ksteps_row + ks) * 32 + lane);
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const int off = (n * 8 + g) * kDownHStride + s * 16 + 2 * t;
                const uint32_t bh0 = *reinterpret_cast<const uint32_t *>(hh + off);
                const uint32_t bh1 = *reinterpret_cast<const uint32_t *>(hh + off + 8);
                const uint32_t bl0 = *reinterpret_cast<const uint32_t *>(hl + off);
                const uint32_t bl1 = *reinterpret_cast<const uint32_t *>(hl + off + 8);
                mma_f16(acc[0][n], a0, bh0, bh1);
                mma_f16(acc[0][n], a0, bl0, bl1);
                mma_f16(acc[1][n], a1, bh0, bh1);
                mma_f16(acc[1][n], a1, bl0, bl1);
            }
        }
        __syncthreads();  // this buffer is refilled two chunks later
    }

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
    // Last CTA of this output block: y[t0 + tok, o] = sum of the slices in order.
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
