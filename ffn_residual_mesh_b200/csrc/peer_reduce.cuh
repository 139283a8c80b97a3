// Layer-output reduction of the d_ff-sharded stack over NVLink, fused with the fp16 cast.
//
// Rank k's down projection leaves a partial y_k [T, D] in its own memory; the layer
// output is y = sum_k y_k on every rank. One kernel per layer and rank does what an
// allreduce followed by a cast would:
//   1. CTA c pushes chunk c of this rank's partial into every rank's receive region
//      (peer memory mapped through CUDA IPC), slot [epoch & 1][this rank];
//   2. after a system-scope fence, it raises flag [this rank][c] on every rank to the
//      call's epoch;
//   3. it waits (bounded) until flag [k][c] of its own region has reached the epoch for
//      every rank k, i.e. chunk c of every partial has landed here;
//   4. it sums the ranks' chunks in rank order (every rank computes the same bits) and
//      writes y as fp16 (and fp32 if asked).
// No CTA waits on another CTA of its own GPU. The epoch lives in device memory and the
// last CTA of a call advances it, so a CUDA graph replays correctly. Two receive slots
// alternate by epoch parity: a rank reaches call e + 2 (which reuses slot e & 1) only
// after every rank has signalled call e + 1, which each does after finishing call e.
// Plain loads and stores only: no multicast, no library kernel on peer memory.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace ffnrm {

constexpr int kPeerMaxRanks = 8;
constexpr int kPeerMaxChunks = 256;
constexpr int kPeerThreads = 256;
constexpr int kPeerUnroll = 4;  // independent 16-byte loads per thread in flight (two-shot copies)
constexpr long long kPeerWaitCycles = 2000000000LL;  // about one second

struct PeerParams {
    float *recv[kPeerMaxRanks];      // rank k's receive region [2][world][max_elems] (peer address)
    uint32_t *flags[kPeerMaxRanks];  // rank k's flags [world][kPeerMaxChunks] (peer address)
    const float *partial;            // this rank's partial [elems]
    __half *y16;                     // [elems] or null
    float *y32;                      // [elems] or null
    uint32_t *epoch;                 // this rank's call counter
    uint32_t *done;                  // CTAs of the current call that have finished
    int *status;                     // set to 1 when a wait gave up
    int64_t elems, max_elems;
    int chunk;  // elements per CTA, a multiple of 4
    int world, rank;
};

__global__ void __launch_bounds__(kPeerThreads) peer_allreduce_kernel(const PeerParams p) {
    __shared__ uint32_t s_ep;
    __shared__ int s_ok;
    const int c = blockIdx.x;
    const int64_t v0 = int64_t(c) * p.chunk / 4, v1 = min(p.elems, int64_t(c + 1) * p.chunk) / 4;  // float4 range
    // Launched as a dependent of the down projection: the partial (and this rank's call
    // counter, last written two kernels earlier) are read only after it has completed.
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    if (threadIdx.x == 0) {
        s_ep = *reinterpret_cast<volatile uint32_t *>(p.epoch) + 1u;
        s_ok = 1;
    }
    __syncthreads();
    const uint32_t ep = s_ep;
    const int64_t slot_off = int64_t(ep & 1u) * p.world * p.max_elems;

    // 1. this rank's chunk into slot [ep & 1][rank] of every rank
    const float4 *src = reinterpret_cast<const float4 *>(p.partial);
    for (int k = 0; k < p.world; ++k) {
        float4 *dst = reinterpret_cast<float4 *>(p.recv[k] + slot_off + int64_t(p.rank) * p.max_elems);
        for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) dst[i] = __ldcg(src + i);
    }
    __threadfence_system();
    __syncthreads();
    // 2. chunk c of this rank has landed everywhere
    if (threadIdx.x < p.world)
        *reinterpret_cast<volatile uint32_t *>(p.flags[threadIdx.x] + p.rank * kPeerMaxChunks + c) = ep;
    // 3. chunk c of every rank has landed here (flags only move forward)
    if (threadIdx.x < p.world) {
        volatile uint32_t *f = p.flags[p.rank] + threadIdx.x * kPeerMaxChunks + c;
        const long long t0 = clock64();
        while (int32_t(*f - ep) < 0) {
            if (clock64() - t0 > kPeerWaitCycles) {
                atomicExch(p.status, 1);
                s_ok = 0;
                break;
            }
        }
    }
    __syncthreads();
    __threadfence();
    // 4. y = sum of the ranks' chunks in rank order
    if (s_ok) {
        const float4 *in = reinterpret_cast<const float4 *>(p.recv[p.rank] + slot_off);
        const int64_t stride = p.max_elems / 4;
        for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
            float4 a = __ldcg(in + i);
            for (int k = 1; k < p.world; ++k) {
                const float4 v = __ldcg(in + int64_t(k) * stride + i);
                a.x += v.x;
                a.y += v.y;
                a.z += v.z;
                a.w += v.w;
            }
            if (p.y32) reinterpret_cast<float4 *>(p.y32)[i] = a;
            if (p.y16) {
                __half2 *o = reinterpret_cast<__half2 *>(p.y16) + 2 * i;
                o[0] = __floats2half2_rn(a.x, a.y);
                o[1] = __floats2half2_rn(a.z, a.w);
            }
        }
    }
    // 5. the last CTA of the call advances the epoch
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.done, 1u) == gridDim.x - 1) {
            *reinterpret_cast<volatile uint32_t *>(p.done) = 0u;
            *reinterpret_cast<volatile uint32_t *>(p.epoch) = ep;
        }
    }
}


// Two-shot variant for large partials (prefill: 2048 x 8192 fp32 = 64 MB per layer).
// Pushing whole partials to every rank moves (world - 1) x the message per rank; here
// rank r owns slice r of the output (elems / world, in chunks of `chunk`):
//   1. CTA c pushes chunk c of every slice d of this rank's partial into rank d's
//      scatter slot [epoch & 1][this rank] and raises scatter flag [this rank][c] there;
//   2. it waits for chunk c of its own slice from every rank, sums them in rank order and
//      pushes the sum (fp32) to every rank's gather slot [epoch & 1][this rank], raising
//      gather flag [this rank][c] there;
//   3. it waits for chunk c of every owner's summed slice and writes it to y (fp16 and/or
//      fp32) at the slice's place.
// Each rank sends (world - 1) / world of the message twice, about 2 x 64 MB x 7/8 at eight
// ranks, instead of 7 x 64 MB. CTA c of one GPU waits only on CTA c of the others; the
// grid fits on the GPU at once, so every CTA a wait depends on is running.
struct PeerTwoShotParams {
    float *scatter[kPeerMaxRanks];    // rank k's scatter slots [2][world][slice] (peer address)
    float *gather[kPeerMaxRanks];     // rank k's gather slots [2][world][slice]
    uint32_t *sflags[kPeerMaxRanks];  // rank k's scatter flags [world][kPeerMaxChunks]
    uint32_t *gflags[kPeerMaxRanks];  // rank k's gather flags [world][kPeerMaxChunks]
    const float *partial;
    __half *y16;
    float *y32;
    uint32_t *epoch, *done;
    int *status;
    uint32_t *tiles;       // this rank's tile counters [2] (fused mode), or null
    uint32_t tiles_expected;  // fused mode: down-projection tiles (all ranks) that write this rank's slice
    int64_t elems, slice;  // slice: elements per rank (a multiple of 4); the last rank's may be shorter
    int64_t stride;        // elements between ranks' slots (the largest slice the region holds)
    int chunk;             // elements per CTA within a slice, a multiple of 4
    int world, rank;
};

__device__ __forceinline__ uint2 pack_half4(const float4 a) {
    const __half2 lo = __floats2half2_rn(a.x, a.y), hi = __floats2half2_rn(a.z, a.w);
    uint2 w;
    w.x = *reinterpret_cast<const uint32_t *>(&lo);
    w.y = *reinterpret_cast<const uint32_t *>(&hi);
    return w;
}

__device__ __forceinline__ bool peer_wait_flag(volatile uint32_t *f, uint32_t ep, int *status) {
    const long long t0 = clock64();
    while (int32_t(*f - ep) < 0) {
        if (clock64() - t0 > kPeerWaitCycles) {
            atomicExch(status, 1);
            return false;
        }
    }
    return true;
}

__global__ void __launch_bounds__(kPeerThreads) peer_two_shot_kernel(const PeerTwoShotParams p) {
    __shared__ uint32_t s_ep;
    __shared__ int s_ok;
    const int c = blockIdx.x;
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    if (threadIdx.x == 0) {
        s_ep = *reinterpret_cast<volatile uint32_t *>(p.epoch) + 1u;
        s_ok = 1;
    }
    __syncthreads();
    const uint32_t ep = s_ep;
    const int64_t slot = int64_t(ep & 1u) * p.world * p.stride;  // elements
    // chunk c of slice d: [d*slice + c*chunk, min(...)) as float4 indices, relative to the slice
    auto range = [&](int d, int64_t &b, int64_t &e) {
        const int64_t s0 = int64_t(d) * p.slice, len = max(int64_t(0), min(p.elems, s0 + p.slice) - s0);
        b = min(len, int64_t(c) * p.chunk) / 4;
        e = min(len, int64_t(c + 1) * p.chunk) / 4;
    };
    // 1. scatter: chunk c of every slice d to rank d (done already, tile by tile, by the down
    //    projection of every rank in fused mode: wait for all of their tiles instead)
    const float4 *src = reinterpret_cast<const float4 *>(p.partial);
    for (int d = 0; d < (p.tiles ? 0 : p.world); ++d) {
        int64_t b, e;
        range(d, b, e);
        float4 *dst = reinterpret_cast<float4 *>(p.scatter[d] + slot + int64_t(p.rank) * p.stride);
        const float4 *sd = src + int64_t(d) * p.slice / 4;
        // four independent loads per thread in flight before their (posted) peer stores
        for (int64_t i0 = b + threadIdx.x; i0 < e; i0 += kPeerUnroll * blockDim.x) {
            float4 v[kPeerUnroll];
#pragma unroll
            for (int u = 0; u < kPeerUnroll; ++u)
                if (i0 + u * blockDim.x < e) v[u] = __ldcg(sd + i0 + u * blockDim.x);
#pragma unroll
            for (int u = 0; u < kPeerUnroll; ++u)
                if (i0 + u * blockDim.x < e) dst[i0 + u * blockDim.x] = v[u];
        }
    }
    __threadfence_system();
    __syncthreads();
    if (p.tiles) {
        if (threadIdx.x == 0) {
            const volatile uint32_t *cnt = p.tiles + (ep & 1u);
            const long long t0 = clock64();
            while (*cnt < p.tiles_expected) {
                if (clock64() - t0 > kPeerWaitCycles) {
                    atomicExch(p.status, 1);
                    s_ok = 0;
                    break;
                }
            }
        }
    } else {
        if (threadIdx.x < p.world)
            *reinterpret_cast<volatile uint32_t *>(p.sflags[threadIdx.x] + p.rank * kPeerMaxChunks + c) = ep;
        // 2. reduce chunk c of this rank's slice in rank order, push the sum to every rank
        if (threadIdx.x < p.world && !peer_wait_flag(p.sflags[p.rank] + threadIdx.x * kPeerMaxChunks + c, ep, p.status))
            s_ok = 0;
    }
    __syncthreads();
    __threadfence();
    {
        int64_t b, e;
        range(p.rank, b, e);
        const float4 *in = reinterpret_cast<const float4 *>(p.scatter[p.rank] + slot);
        const int64_t stride = p.stride / 4;
        if (s_ok) {
            // two elements per thread per pass, each summed over the ranks in rank order
            for (int64_t i0 = b + threadIdx.x; i0 < e; i0 += 2 * blockDim.x) {
                const int64_t i1 = i0 + blockDim.x;
                const bool two = i1 < e;
                float4 a = __ldcg(in + i0), a1 = two ? __ldcg(in + i1) : make_float4(0.f, 0.f, 0.f, 0.f);
                for (int k = 1; k < p.world; ++k) {
                    const float4 v = __ldcg(in + int64_t(k) * stride + i0);
                    const float4 v1 = two ? __ldcg(in + int64_t(k) * stride + i1) : make_float4(0.f, 0.f, 0.f, 0.f);
                    a.x += v.x;
                    a.y += v.y;
                    a.z += v.z;
                    a.w += v.w;
                    a1.x += v1.x;
                    a1.y += v1.y;
                    a1.z += v1.z;
                    a1.w += v1.w;
                }
                if (p.y32) {
                    for (int k = 0; k < p.world; ++k) {
                        float4 *g = reinterpret_cast<float4 *>(p.gather[k] + slot + int64_t(p.rank) * p.stride);
                        g[i0] = a;
                        if (two) g[i1] = a1;
                    }
                } else {
                    // fp16 output only: round the sum here, once, and move half the bytes over
                    // NVLink (the same bits as rounding after the gather)
                    const uint2 h0 = pack_half4(a), h1 = pack_half4(a1);
                    for (int k = 0; k < p.world; ++k) {
                        uint2 *g = reinterpret_cast<uint2 *>(p.gather[k] + slot + int64_t(p.rank) * p.stride);
                        g[i0] = h0;
                        if (two) g[i1] = h1;
                    }
                }
            }
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < p.world)
        *reinterpret_cast<volatile uint32_t *>(p.gflags[threadIdx.x] + p.rank * kPeerMaxChunks + c) = ep;
    // 3. gather: chunk c of every owner's sum into y
    if (threadIdx.x < p.world && !peer_wait_flag(p.gflags[p.rank] + threadIdx.x * kPeerMaxChunks + c, ep, p.status))
        s_ok = 0;
    __syncthreads();
    __threadfence();
    if (s_ok) {
        for (int d = 0; d < p.world; ++d) {
            int64_t b, e;
            range(d, b, e);
            const float4 *g = reinterpret_cast<const float4 *>(p.gather[p.rank] + slot + int64_t(d) * p.stride);
            const int64_t off = int64_t(d) * p.slice / 4;
            if (!p.y32) {  // fp16 sums, already rounded by their owner
                const uint2 *gh = reinterpret_cast<const uint2 *>(g);
                uint2 *yh = reinterpret_cast<uint2 *>(p.y16) + off;
                for (int64_t i0 = b + threadIdx.x; i0 < e; i0 += kPeerUnroll * blockDim.x) {
                    uint2 v[kPeerUnroll];
#pragma unroll
                    for (int u = 0; u < kPeerUnroll; ++u)
                        if (i0 + u * blockDim.x < e) v[u] = __ldcg(gh + i0 + u * blockDim.x);
#pragma unroll
                    for (int u = 0; u < kPeerUnroll; ++u)
                        if (i0 + u * blockDim.x < e) yh[i0 + u * blockDim.x] = v[u];
                }
                continue;
            }
            for (int64_t i0 = b + threadIdx.x; i0 < e; i0 += kPeerUnroll * blockDim.x) {
                float4 v[kPeerUnroll];
#pragma unroll
                for (int u = 0; u < kPeerUnroll; ++u)
                    if (i0 + u * blockDim.x < e) v[u] = __ldcg(g + i0 + u * blockDim.x);
#pragma unroll
                for (int u = 0; u < kPeerUnroll; ++u) {
                    const int64_t i = i0 + u * blockDim.x;
                    if (i >= e) break;
                    if (p.y32) reinterpret_cast<float4 *>(p.y32)[off + i] = v[u];
                    if (p.y16) {
                        __half2 *o = reinterpret_cast<__half2 *>(p.y16) + 2 * (off + i);
                        o[0] = __floats2half2_rn(v[u].x, v[u].y);
                        o[1] = __floats2half2_rn(v[u].z, v[u].w);
                    }
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.done, 1u) == gridDim.x - 1) {
            *reinterpret_cast<volatile uint32_t *>(p.done) = 0u;
            // no tile of this parity arrives before this rank's next call has run
            if (p.tiles) *reinterpret_cast<volatile uint32_t *>(p.tiles + (ep & 1u)) = 0u;
            *reinterpret_cast<volatile uint32_t *>(p.epoch) = ep;
        }
    }
}

}  // namespace ffnrm
