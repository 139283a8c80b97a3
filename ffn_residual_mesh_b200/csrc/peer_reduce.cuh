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
constexpr int kPeerMaxChunks = 128;
constexpr int kPeerThreads = 256;
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

}  // namespace ffnrm
