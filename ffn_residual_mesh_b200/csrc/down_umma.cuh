// fp16 down projection on the 5th-generation tensor cores (tcgen05, TMEM accumulator).
//
// Replaces swiglu_down_kernel (src/exact_cpu_base_gpu_full_ffn_runner.cu:217-240) and
// the torch.mm down of scripts/benchmark_gpu_full_ffn_density.py:162. The merge and
// SwiGLU already happened in the residual kernel, which wrote h = SiLU(g)*u as two
// fp16 parts (h = hi + lo to ~2^-22 relative), so y keeps fp32-level accuracy.
//
// y[t, o] = sum_f h[t, f] * Wd[o, f] is a GEMM with M = d_model (down rows), N = tokens,
// K = d_ff. CTA tile: 128 down rows x N tokens x a split-K slice of d_ff.
//   warp 0          : TMA producer. Per 64-column K step it loads the 128x64 fp16 tile of
//                     Wd and the Nx64 tiles of h hi and lo (128-byte swizzle) into a
//                     shared-memory ring, completing on full[s]; a batch of S/2 steps is
//                     issued at once, one copy per lane.
//   warp 1 / lane 0 : MMA issuer. Per stage, 4 K=16 steps x (hi, lo) tcgen05.mma into one
//                     128xN f32 accumulator in tensor memory; tcgen05.commit frees the stage.
//   warps 0-3       : epilogue. Each warp reads its 32 TMEM lanes (down rows) with
//                     tcgen05.ld. One slice: y is written directly. Split-K: the slices
//                     of an output tile run as one thread-block cluster (cluster rank =
//                     slice); every CTA stages its 128xN partial in its own shared memory,
//                     and after a cluster barrier CTA r sums rows [32r/S, 32(r+1)/S) x 4
//                     over the S slices through distributed shared memory, in slice order
//                     (deterministic, no global scratch).
// Every mbarrier wait is bounded; on timeout the kernel records an error code in
// p.err, drains its outstanding copies, frees its TMEM and returns.
#pragma once

#include <cuda_fp16.h>

#include "ffnrm_common.cuh"
#include "sm100.cuh"

namespace ffnrm {

constexpr int kDownMaxSplits = 8;  // portable cluster size

// Output straight into the layer reduction's reduce-scatter slots (d_ff-sharded stack): the
// element e = t*D + o of this rank's partial belongs to rank e / slice and is stored, over
// NVLink, at scatter[owner] + slot(epoch) + rank*stride + (e - owner*slice); when a tile's
// stores are done, every owner it wrote to counts the tile (system-scope atomic on that
// rank's counter of the call's parity).
struct DownScatter {
    float *scatter[8];      // ranks' scatter slot bases (peer addresses), [2][world][stride]
    uint32_t *counter[8];   // ranks' tile counters [2] (peer addresses)
    const uint32_t *epoch;  // this rank's reduction call counter (the call in flight is epoch + 1)
    int64_t slice, stride;
    int world, rank;
};

struct DownUmmaParams {
    float *y32;      // [T, D] or null
    __half *y16;     // [T, D] or null
    int *err;        // error word (bounded waits)
    int D, F16, T, splits, kc;  // kc: d_ff columns per slice, a multiple of 64
    int fused;                   // nonzero: y goes to the reduction's scatter slots `sc` (splits == 1)
    DownScatter sc;
};

constexpr int kUmmaM = 128;
constexpr int kUmmaK = 64;  // d_ff columns per stage (one 128-byte swizzle row)

template <int N>
struct DownUmmaCfg {
    // ring depth within 227 KB: 48 KB stages at N = 128, 64 KB at 192, 80 KB at 256
    static constexpr int stages = N <= 16 ? 5 : (N <= 32 ? 4 : (N <= 64 ? 3 : (N <= 128 ? 4 : (N <= 192 ? 3 : 2))));
    static constexpr int a_bytes = kUmmaM * kUmmaK * 2;  // 16 KB
    static constexpr int b_bytes = N * kUmmaK * 2;       // per part (hi or lo)
    static constexpr int stage_bytes = a_bytes + 2 * b_bytes;
    static constexpr int tmem_cols = N <= 32 ? 32 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256));  // a power of two
    static constexpr size_t smem = size_t(stages) * stage_bytes + 1024 /*align*/ + 256 /*barriers*/;
    static_assert(size_t(stages) * stage_bytes >= size_t(N) * kUmmaM * 4, "partial tile reuses the stage ring");
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// 16 bytes from the shared memory of CTA `rank` of this cluster, at the offset of `local`.
__device__ __forceinline__ float4 ld_dsmem_f4(const void *local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(sm100::smem_u32(local)), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(remote)
                 : "memory");
    return v;
}

template <int N>
__global__ void __launch_bounds__(128, 1) down_umma_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                           const __grid_constant__ CUtensorMap tm_hi,
                                                           const __grid_constant__ CUtensorMap tm_lo,
                                                           const DownUmmaParams p) {
    using Cfg = DownUmmaCfg<N>;
    constexpr int S = Cfg::stages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *tiles = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * Cfg::stage_bytes);
    uint64_t *empty = full + S;
    uint64_t *done = empty + S;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);

    // grid: x = slice (the cluster spans all slices of one output tile), y = row tile,
    // z = token tile
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kUmmaM;
    const int t0 = blockIdx.z * N;
    const int split = blockIdx.x;
    const int k0 = split * p.kc;
    const int k1 = min(k0 + p.kc, p.F16);
    const int nk = (k1 - k0 + kUmmaK - 1) / kUmmaK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            sm100::mbar_init(full + s, 1);
            sm100::mbar_init(empty + s, 1);
        }
        sm100::mbar_init(done, 1);
        sm100::fence_barrier_init();
    }
    if (warp == 0) sm100::tmem_alloc(tmem_slot, Cfg::tmem_cols);
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // TMA producer warp. A thread's copies do not overlap one another, so K steps are
        // issued in batches of max(1, S/2) with one copy per lane (lane 3k + op of the
        // batch's lane group: W, h hi or h lo of its k-th step), and consecutive batches
        // use different lane groups, keeping several batches in flight.
        const int B = S / 2 > 1 ? (S / 2 < 10 ? S / 2 : 10) : 1;
        const int R = 32 / (3 * B);  // lane groups; consecutive batches use different lanes
        int issued = 0, batch = 0;
        for (int it0 = 0; it0 < nk; it0 += B, ++batch) {
            const int nb = min(B, nk - it0);
            const int l = lane - (batch % R) * 3 * B;  // role within this batch's lane group
            const int k = l >= 0 ? l / 3 : nb, op = l - 3 * (l / 3);
            const int it = it0 + k, s = it % S;
            bool ok = true;
            if (l >= 0 && k < nb && op == 0) {
                ok = sm100::mbar_wait(empty + s, ((it / S) & 1) ^ 1, p.err, sm100::kErrWaitEmpty);
                if (ok) sm100::mbar_arrive_expect_tx(full + s, Cfg::stage_bytes);
            }
            if (!__all_sync(0xffffffffu, ok)) break;
            uint8_t *st = tiles + s * Cfg::stage_bytes;
            const int kx = k0 + it * kUmmaK;
            if (batch == 0) {
                // The weight does not depend on the preceding kernel: the first weight tiles
                // load before the dependency wait, h (its output) only after it.
                if (l >= 0 && k < nb && op == 0) sm100::tma_load_2d(st, &tm_w, kx, m0, full + s);
                sm100::grid_dependency_wait();
                sm100::trigger_dependents();
                if (l >= 0 && k < nb && op != 0)
                    sm100::tma_load_2d(st + Cfg::a_bytes + (op - 1) * Cfg::b_bytes, op == 1 ? &tm_hi : &tm_lo, kx, t0,
                                       full + s);
            } else if (l >= 0 && k < nb) {
                const CUtensorMap *map = op == 0 ? &tm_w : op == 1 ? &tm_hi : &tm_lo;
                uint8_t *dst = op == 0 ? st : st + Cfg::a_bytes + (op - 1) * Cfg::b_bytes;
                sm100::tma_load_2d(dst, map, kx, op == 0 ? m0 : t0, full + s);
            }
            issued = it0 + nb;
        }
        // No copy may still be in flight when the CTA exits: wait for the last stages.
        if (lane == 0)
            for (int it = max(0, issued - S); it < issued; ++it)
                sm100::mbar_wait(full + it % S, (it / S) & 1, p.err, sm100::kErrWaitFull);
    } else {
        // The other warps read only what the producer staged; their y writes wait for the
        // preceding kernel like every access to its memory (dependent launch).
        sm100::grid_dependency_wait();
        sm100::trigger_dependents();
    }
    if (warp == 1 && lane == 0) {
        // MMA issuer
        constexpr uint32_t idesc = sm100::umma_idesc_f16_f32(kUmmaM, N);
        for (int it = 0; it < nk; ++it) {
            const int s = it % S;
            if (!sm100::mbar_wait(full + s, (it / S) & 1, p.err, sm100::kErrWaitFull)) break;
            sm100::tc_fence_after();
            const uint32_t a = sm100::smem_u32(tiles + s * Cfg::stage_bytes);
            const uint32_t bh = a + Cfg::a_bytes, bl = bh + Cfg::b_bytes;
#pragma unroll
            for (int k = 0; k < kUmmaK / 16; ++k) {
                const uint64_t ad = sm100::umma_desc_sw128(a + 32 * k);
                sm100::umma_f16(tmem, ad, sm100::umma_desc_sw128(bh + 32 * k), idesc, (it | k) != 0);
                sm100::umma_f16(tmem, ad, sm100::umma_desc_sw128(bl + 32 * k), idesc, 1);
            }
            sm100::umma_commit(empty + s);  // the stage is free once these MMAs finish
        }
        sm100::umma_commit(done);
    }
    __syncwarp();

    // Epilogue: wait for the accumulator, then each warp drains its 32 TMEM lanes.
    const bool ok = sm100::mbar_wait(done, 0, p.err, sm100::kErrWaitDone);
    sm100::tc_fence_after();
    const int row = warp * 32 + lane;
    const int ntok = min(N, p.T - t0);
    if (p.fused) {
        // Fused reduce-scatter: rows of this tile are stored into their owner's slot.
        const DownScatter &q = p.sc;
        const uint32_t ep = *reinterpret_cast<const volatile uint32_t *>(q.epoch) + 1u;
        const int64_t slot = int64_t(ep & 1u) * q.world * q.stride + int64_t(q.rank) * q.stride;
        if (ok) {
            int64_t e = int64_t(t0) * p.D + m0 + row;
            int d = int(e / q.slice);
            int64_t next = int64_t(d + 1) * q.slice;  // first element of the next owner
#pragma unroll 1
            for (int c = 0; c < N; c += 16) {
                if (c >= ntok) break;
                uint32_t r[16];
                sm100::tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + c, r);
                sm100::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    if (c + j >= ntok) break;
                    while (e >= next) {
                        ++d;
                        next += q.slice;
                    }
                    q.scatter[d][slot + (e - (next - q.slice))] = __uint_as_float(r[j]);
                    e += p.D;
                }
            }
        }
        sm100::tc_fence_before();
        __threadfence_system();
        __syncthreads();
        if (warp == 0) sm100::tmem_dealloc(tmem, Cfg::tmem_cols);
        if (threadIdx.x == 0) {
            // every owner between the tile's first and last element saw some of its rows (a
            // slice holds at least two token rows)
            const int d0 = int((int64_t(t0) * p.D + m0) / q.slice);
            const int d1 = int((int64_t(t0 + ntok - 1) * p.D + m0 + kUmmaM - 1) / q.slice);
            for (int d = d0; d <= d1 && d < q.world; ++d) atomicAdd_system(q.counter[d] + (ep & 1u), 1u);
        }
        return;
    }
    if (p.splits == 1) {
        if (ok) {
#pragma unroll
            for (int c = 0; c < N; c += 16) {
                if (c >= ntok) break;
                uint32_t r[16];
                sm100::tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + c, r);
                sm100::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    if (c + j >= ntok) break;
                    const float v = __uint_as_float(r[j]);
                    const int64_t yi = int64_t(t0 + c + j) * p.D + m0 + row;
                    if (p.y32) p.y32[yi] = v;
                    if (p.y16) p.y16[yi] = __float2half_rn(v);
                }
            }
        }
        sm100::tc_fence_before();
        __syncthreads();
        if (warp == 0) sm100::tmem_dealloc(tmem, Cfg::tmem_cols);
        return;
    }

    // Split-K: stage the partial as [N tokens][128 rows] f32 in the (drained) stage ring.
    float *part = reinterpret_cast<float *>(tiles);
    if (ok) {
#pragma unroll
        for (int c = 0; c < N; c += 16) {
            if (c >= ntok) break;
            uint32_t r[16];
            sm100::tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + c, r);
            sm100::tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) part[(c + j) * kUmmaM + row] = __uint_as_float(r[j]);
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 0) sm100::tmem_dealloc(tmem, Cfg::tmem_cols);
    cluster_sync();  // every slice's partial is staged
    // CTA r of the cluster reduces 4-row units [32r/S, 32(r+1)/S) for all tokens.
    const int S_ = p.splits;
    const int rank = int(cluster_ctarank());
    const int u0 = rank * (kUmmaM / 4) / S_, u1 = (rank + 1) * (kUmmaM / 4) / S_;
    const int nu = u1 - u0;
    for (int i = threadIdx.x; i < nu * ntok; i += blockDim.x) {
        const int t = i / nu, u = u0 + (i - t * nu);
        const float *src = part + t * kUmmaM + 4 * u;
        float4 v[kDownMaxSplits];
#pragma unroll
        for (int sp = 0; sp < kDownMaxSplits; ++sp)
            if (sp < S_) v[sp] = ld_dsmem_f4(src, uint32_t(sp));
        float4 a = v[0];
#pragma unroll
        for (int sp = 1; sp < kDownMaxSplits; ++sp)
            if (sp < S_) a.x += v[sp].x, a.y += v[sp].y, a.z += v[sp].z, a.w += v[sp].w;
        const int64_t yi = int64_t(t0 + t) * p.D + m0 + 4 * u;
        if (p.y32) *reinterpret_cast<float4 *>(p.y32 + yi) = a;
        if (p.y16) {
            const __half2 lo = __floats2half2_rn(a.x, a.y), hi = __floats2half2_rn(a.z, a.w);
            uint2 w;
            w.x = *reinterpret_cast<const uint32_t *>(&lo);
            w.y = *reinterpret_cast<const uint32_t *>(&hi);
            *reinterpret_cast<uint2 *>(p.y16 + yi) = w;
        }
    }
    cluster_sync();  // no CTA leaves while a peer still reads its shared memory
}

}  // namespace ffnrm
