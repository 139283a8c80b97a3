/*
 * ffnrm.h — C ABI of the B200 exact integer-domain gated-FFN base/residual split.
 *
 * The path: every Q4 weight code is split exactly as q = 2^r * q_hi + q_lo. The host
 * supplies the "base" partial sums  s*(alpha*2^r*dot(q_hi, z) + beta*sum(z))  per
 * token and d_ff row; the GPU computes the "residual"  s*alpha*dot(q_lo, z)  from
 * exact int32 group dots, merges g = g_base + g_res and u = u_base + u_res before
 * SiLU(g)*u, and runs the fp16 down projection.
 *
 * The reference ships this path as three standalone CUDA runners and Python/Triton
 * twins, with no library ABI. Each entry point below names the reference code it
 * replaces (paths relative to the reference project root).
 *
 * Conventions
 *   - Plain pointers and sizes only. "device" pointers are CUDA device addresses
 *     on the context's device; "host" pointers are ordinary (preferably pinned)
 *     host memory. `stream` is a cudaStream_t passed as void* (NULL = legacy
 *     default stream). All compute calls are stream-ordered and asynchronous.
 *   - Shapes: T tokens, D = d_model (reference "hidden"), F = d_ff rows held by
 *     this context (a shard of the full d_ff in multi-GPU runs), G = D/32.
 *     Activations z are int8 [T, D] row-major, their per-group scales s are
 *     f32 [T, G]; base sums and residual outputs are f32 [T, F]; y is [T, D].
 *   - Return value: FFNRM_OK or an error code; ffnrm_last_error() gives the
 *     message of the last failing call on the calling thread. Argument errors
 *     correspond to the reference's ValueError / `error: ...` exit 1 paths.
 *   - One context per device per host thread at a time; contexts are not
 *     internally locked.
 */
#ifndef FFNRM_H
#define FFNRM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FFNRM_OK 0
#define FFNRM_ERR_ARG 1     /* shape / argument error (reference: ValueError) */
#define FFNRM_ERR_CUDA 2    /* CUDA runtime error */
#define FFNRM_ERR_STATE 3   /* e.g. layer not loaded, fallback data missing */
#define FFNRM_ERR_NOMEM 4   /* device or pinned allocation failed */
#define FFNRM_ERR_TIMEOUT 5 /* a kernel's bounded pipeline wait expired (reported by ffnrm_check_device_error) */

/* Residual code formats accepted by ffnrm_load_layer. */
#define FFNRM_CODES_Q4_BYTES 0       /* full Q4 codes, one byte per code [F, D], values 0..15 */
#define FFNRM_CODES_QLO2_ROWPACKED 1 /* r = 2 low codes, row-packed [F, D/4]
                                        (scripts/export_cuda_residual_artifact_v2.py:13-24) */
#define FFNRM_CODES_BITPLANES 2      /* r low-code bit planes, plane-major, each F*D/8 bytes
                                        (scripts/compile_q4k_host_base_gpu_residual.py:17-26) */

typedef struct ffnrm_ctx ffnrm_ctx;

typedef struct {
    int32_t d_model;        /* D, a multiple of 256 (Q4_K super-block) */
    int32_t d_ff;           /* F rows held by this context, a multiple of 8 */
    int32_t residual_bits;  /* r in {1, 2, 3} */
    int32_t n_layers;       /* layers this context can hold */
    int32_t max_tokens;     /* largest T of any call (sizes the workspace) */
    int32_t base_tile_rows; /* rows per base tile / fallback tile (reference TILE_ROWS) */
} ffnrm_config;

typedef struct {
    int32_t codes_format;          /* FFNRM_CODES_* */
    const uint8_t *gate_codes;     /* Q4_BYTES: full codes; otherwise the residual low codes */
    const uint8_t *up_codes;
    const uint8_t *gate_high;      /* BITPLANES / QLO2: optional (4-r) high-code bit planes
                                      (compile_q4k_host_base_gpu_residual.py:66); NULL = no fallback */
    const uint8_t *up_high;
    const float *gate_alpha;       /* [F, G] per-group weight scale */
    const float *up_alpha;
    const float *gate_beta;        /* [F, G] per-group weight min term; NULL = no fallback */
    const float *up_beta;
    const uint16_t *down;          /* fp16 down weight, row o at down + o*down_ld, F columns;
                                      NULL loads a residual-only layer (ffnrm_residual only) */
    int64_t down_ld;               /* leading dimension of `down` in elements (>= F) */
    int32_t keep_fallback;         /* Q4_BYTES only: also keep the high codes for fallback tiles */
} ffnrm_layer_weights;

/* Create a context on `device`. Replaces the per-runner setup of
 * src/exact_cpu_base_gpu_full_ffn_runner.cu:375-397 (device buffers, streams). */
int ffnrm_create(ffnrm_ctx **out, int device, const ffnrm_config *cfg);
int ffnrm_destroy(ffnrm_ctx *ctx);

/* Copy one layer's weights into HBM. Each array may be host memory or device memory of
 * the context's device (borrowed for the call); host arrays are copied to the device
 * first, and the artifact formats are decoded and packed into the device layouts by
 * kernels. Synchronous: the call returns when the layer is ready.
 * Replaces load_projection (src/exact_residual_cuda_runner.cu:88-120) and the
 * resident fp16 down upload (src/exact_cpu_base_gpu_full_ffn_runner.cu:375-387).
 * alpha/beta are kept as fp16 on the device when every value is fp16-exact
 * (lossless), else as f32. Q4 codes above 15 are rejected (FFNRM_ERR_ARG). */
int ffnrm_load_layer(ffnrm_ctx *ctx, int layer, const ffnrm_layer_weights *w);

/* Residual gate/up contraction. Replaces residual_kernel
 * (src/exact_residual_cuda_runner.cu:122-159, and its copies in
 * exact_main_residual_cuda_runner.cu:213-233 and
 * exact_cpu_base_gpu_full_ffn_runner.cu:195-215) for both projections in one launch.
 * Device pointers: z [T,D] i8, s [T,G] f32, gate_res/up_res [T,F] f32.
 * group_dots (optional, device, NULL to skip): [2, T, F, G] int32, the exact
 * residual group dots sum_i q_lo*z (gate then up).
 * fallback_tiles (optional, device): rows of flagged tiles receive the unsplit
 * exact projection sum_g s*(alpha*dot(q,z) + beta*sum(z)) instead of the residual
 * (the "center-GPU exact FFN" fallback, src/phone_ffn_loopback.py:155-197). */
int ffnrm_residual(ffnrm_ctx *ctx, int layer, const int8_t *z, const float *s, int tokens,
                   float *gate_res, float *up_res, int32_t *group_dots, const uint8_t *fallback_tiles,
                   void *stream);

/* Full split FFN, HBM-resident base mode. Replaces enqueue_tile + swiglu_down_kernel
 * (src/exact_cpu_base_gpu_full_ffn_runner.cu:217-289) and the validated Python
 * chain (scripts/benchmark_cpu_base_gpu_full_ffn.py:228-337).
 * Device pointers: z, s as above; gate_base/up_base [T,F] f32; fallback_tiles
 * (device, optional) one byte per base tile, nonzero = recompute those rows on
 * the unsplit exact path (needs fallback data loaded; the base of those rows is
 * ignored); y_f32 (optional, 16-byte aligned) [T,D] f32 partial sum over this
 * context's rows; y_f16 (optional, 8-byte aligned) [T,D] fp16. */
int ffnrm_ffn_forward(ffnrm_ctx *ctx, int layer, const int8_t *z, const float *s, int tokens,
                      const float *gate_base, const float *up_base, const uint8_t *fallback_tiles,
                      float *y_f32, uint16_t *y_f16, void *stream);

/* Full split FFN, host-streamed base mode (the end-to-end call). All data
 * pointers are HOST pointers (pinned for full overlap): z [T,D], s [T,G],
 * gate_base/up_base [T,F], fallback_tiles (optional) [ceil(F/base_tile_rows)],
 * y_f16 [T,D]. z and s are uploaded on `stream`; the base sums are uploaded on the
 * context's copy stream into one of two device slots (alternating per call, so the
 * upload for the next layer overlaps this layer's kernels) while the residual
 * contraction runs on `stream`; the merge waits for the upload by event. This is
 * the double-buffered copy/compute pipeline of
 * src/exact_cpu_base_gpu_full_ffn_runner.cu:315-345, with one transfer per
 * projection instead of one per tile because the base arrives complete. A y_f16 in
 * page-locked, device-mapped memory (cudaHostAlloc, or cudaHostRegister with mapping;
 * 8-byte aligned) is written by the down projection directly over PCIe; any other y is
 * copied back on `stream`. Host buffers must stay valid until `stream` completes. */
int ffnrm_ffn_forward_host(ffnrm_ctx *ctx, int layer, const int8_t *z, const float *s, int tokens,
                           const float *gate_base, const float *up_base, const uint8_t *fallback_tiles,
                           uint16_t *y_f16, void *stream);

/* The same host-streamed call for one shard of a d_ff-split stack: inputs are HOST
 * pointers as above, and the output is this shard's fp32 partial y_f32 [T,D] in DEVICE
 * memory, which the caller then sums over the shards (ffnrm_peer_allreduce). The base
 * upload runs on the copy stream into the alternating slots exactly as above, so it
 * overlaps the previous layer's kernels. No counterpart in the one-device reference. */
int ffnrm_ffn_forward_host_partial(ffnrm_ctx *ctx, int layer, const int8_t *z, const float *s, int tokens,
                                   const float *gate_base, const float *up_base, const uint8_t *fallback_tiles,
                                   float *y_f32, void *stream);

/* Page-lock an existing host range for async copies (cudaHostRegister) and undo it.
 * Replaces the runners' cudaMallocHost packet staging. */
int ffnrm_host_register(void *ptr, size_t bytes);
int ffnrm_host_unregister(void *ptr);

/* Convert f32 [n] -> fp16 [n] on `stream` (used after a cross-GPU allreduce of y_f32). */
int ffnrm_cast_f16(const float *src, uint16_t *dst, int64_t n, void *stream);

/* ---- Layer-output reduction of the d_ff-sharded stack over NVLink -------------------
 * No counterpart in the reference, which runs on one device; it replaces the NCCL
 * allreduce of the fp32 partial y_k plus ffnrm_cast_f16 in the sharded stack. One process
 * per GPU on one node, 2..8 ranks. Each rank creates its peer object (a receive region
 * shared through CUDA IPC), exchanges the FFNRM_IPC_HANDLE_BYTES handle with the other
 * ranks (any host channel), and connects with all handles in rank order. Per layer,
 * every rank calls ffnrm_peer_allreduce in the same order on its stream: one kernel
 * pushes this rank's partial [elems] f32 to every rank, raises per-chunk flags, waits
 * (bounded, about a second) for every rank's chunk, and writes y = sum in rank order as
 * fp16 y16 and/or f32 y32 (identical on every rank). The call counter lives on the
 * device, so the calls may be captured in a CUDA graph and replayed. elems: a positive
 * multiple of 4 up to max_elems; partial and y32 16-byte aligned, y16 8-byte aligned.
 * ffnrm_peer_check synchronises `stream` and reports FFNRM_ERR_TIMEOUT if a wait gave up
 * (a rank stopped calling). Destroy only after every rank has finished its calls. */
#define FFNRM_IPC_HANDLE_BYTES 64
typedef struct ffnrm_peer ffnrm_peer;
int ffnrm_peer_create(ffnrm_peer **out, int device, int world, int rank, int64_t max_elems, void *ipc_handle);
int ffnrm_peer_connect(ffnrm_peer *peer, const void *ipc_handles);
int ffnrm_peer_allreduce(ffnrm_peer *peer, const float *partial, int64_t elems, uint16_t *y16, float *y32,
                         void *stream);
int ffnrm_peer_check(ffnrm_peer *peer, void *stream);
int ffnrm_peer_destroy(ffnrm_peer *peer);
/* Full split FFN of one d_ff shard with the layer-output reduction fused in: device buffers
 * as ffnrm_ffn_forward, y_f16 [T, D] the summed layer output (the same on every rank). For
 * messages above the one-shot limit the down projection stores each output tile straight into
 * its owner rank's reduce-scatter slot over NVLink and counts the tile there, so the reduction
 * kernel only sums its slice and all-gathers (fp16); smaller messages take the down projection
 * into a partial plus ffnrm_peer_allreduce. Every rank makes the same calls in the same order.
 * No reference counterpart (the reference runs on one device). */
int ffnrm_ffn_forward_reduced(ffnrm_ctx *ctx, ffnrm_peer *peer, int layer, const int8_t *z, const float *s, int tokens,
                              const float *gate_base, const float *up_base, const uint8_t *fallback_tiles,
                              uint16_t *y_f16, void *stream);

/* Device bytes held by loaded weights / workspace (for the bench's byte accounting). */
int ffnrm_layer_bytes(ffnrm_ctx *ctx, int layer, int64_t *residual_bytes, int64_t *down_bytes);

/* Allocation-free fp16 down projection y[t, o] = sum_f (h_hi + h_lo)[t, f] * down[o, f].
 * No counterpart in the reference: it exists for callers that cannot allocate device
 * memory -- code running while a CUDA graph is being captured or inside a graph node,
 * allocators that forbid cudaMalloc on the serving path, or processes whose memory pool
 * is fully reserved. It needs no context and calls no cudaMalloc/cudaFree: split-K
 * partial sums are reduced across a thread-block cluster in shared memory, and its only
 * scratch, the default status word, is a file-scope device variable of this library,
 * which every GPU that loads the library holds until the process exits.
 * Device pointers: down fp16 [d_model][down_ld] row-major (d_ff used columns), h_hi and
 * h_lo fp16 [tokens][h_ld] whose sum is h (pass zeros as h_lo for plain fp16 h), outputs
 * y_f32 [tokens][d_model] (16-byte aligned) and/or y_f16 (8-byte aligned); status
 * (optional, 1 int) receives a nonzero code if the kernel gave up on a bounded pipeline
 * wait. Limits (the largest tile grid the call launches): tokens <= 256, d_model a
 * multiple of 128 up to 16384; down/h 16-byte aligned, down_ld and h_ld multiples of 8 and
 * >= d_ff; other requests return FFNRM_ERR_ARG.
 * The status word's device address is looked up (cudaGetSymbolAddress) on the first call
 * on a device, and again after the device's context changed; make that first call before
 * any stream capture. Calls with status = NULL share the default status word and clear it
 * when they start, so such calls that overlap on the GPU (different streams, or another
 * thread) race on it: serialise them, or pass a status word per call. A caller that passes
 * NULL reads (and clears) the default word with ffnrm_noalloc_status. */
int ffnrm_down_project_noalloc(const uint16_t *down, int64_t down_ld, const uint16_t *h_hi, const uint16_t *h_lo,
                               int64_t h_ld, int d_model, int d_ff, int tokens, float *y_f32, uint16_t *y_f16,
                               int32_t *status, void *stream);

/* Copies the current device's default status word of ffnrm_down_project_noalloc (nonzero:
 * a call with status = NULL gave up on a bounded wait) to *out and clears it, ordered on
 * `stream`, and synchronises `stream`. Allocates nothing. */
int ffnrm_noalloc_status(int32_t *out, void *stream);

/* Synchronises `stream` and reports whether any kernel of this context gave up on a
 * bounded pipeline wait since the last check (FFNRM_ERR_TIMEOUT, error word cleared). */
int ffnrm_check_device_error(ffnrm_ctx *ctx, void *stream);

/* Kernel launches issued by this context since creation (the bench's launch count). */
int64_t ffnrm_launch_count(ffnrm_ctx *ctx);

/* Live per-kernel timing with CUDA events recorded on the launching stream around
 * each of this context's kernel launches (off by default; enabling clears the
 * records). Kinds: FFNRM_KERNEL_RESIDUAL, FFNRM_KERNEL_DOWN, FFNRM_KERNEL_REDUCE.
 * ffnrm_profile_read waits for the recorded events and returns the summed device
 * time and launch count of that kind over the records; records are kept, so calls
 * captured into a CUDA graph with profiling on can be read after every replay. */
#define FFNRM_KERNEL_RESIDUAL 0
#define FFNRM_KERNEL_DOWN 1
#define FFNRM_KERNEL_REDUCE 2
int ffnrm_profile_enable(ffnrm_ctx *ctx, int enable);
int ffnrm_profile_read(ffnrm_ctx *ctx, int kind, double *total_ms, int64_t *launches);

/* ---- Host base producer (no GPU) ----------------------------------------------------
 * The exact base sums of the split computed on the host's cores from the reference's
 * radix table artifact (scripts/export_radix_table_artifact.py:17-80):
 *   base[t, f] = sum_g s[t,g] * (alpha[f,g] * (multiplier * P_hi[t,f,g]) + beta[f,g] * zsum[t,g])
 * with P_hi = sum_d 4^d sum_b table[b, state_d(b), f] - 128 * high_sum[f, g], exact in
 * integers (multiplier = 2^r, 4 for the radix-4 tables). Replaces cpu_eval
 * (src/exact_main_residual_cuda_runner.cu:144-187,
 * src/exact_cpu_base_gpu_full_ffn_runner.cu:134-169) and the AVX2 fused evaluator
 * (src/radix_cpu_kernels.h:143-217). Rows are produced in tiles of tile_rows by a
 * pool of `threads` threads that claim tiles dynamically; the fp32 sum runs over the
 * groups in order. */
typedef struct ffnrm_base_producer ffnrm_base_producer;
typedef struct {
    int32_t rows;               /* F */
    int32_t hidden;             /* D, a multiple of 32 */
    int32_t block_size;         /* 2, 4 or 8 */
    const uint8_t *table;       /* [hidden/block_size, 4^block_size, rows] */
    const int16_t *high_sum;    /* [rows, hidden/32] */
    const float *alpha, *beta;  /* [rows, hidden/32] */
} ffnrm_radix_table;
int ffnrm_base_producer_create(ffnrm_base_producer **out, int threads);
int ffnrm_base_producer_destroy(ffnrm_base_producer *p);
/* z [tokens, hidden] int8, s [tokens, hidden/32] f32, base [tokens, rows] f32 (host).
 * tile_ready (optional) [tokens, ceil(rows/tile_rows)]: each entry is set to 1 (release
 * store) when that tile's base values are written, so a consumer thread can stream
 * finished tiles. deadline_ns > 0: tiles that finish later than that after the call
 * started are flagged in late_tiles [ceil(rows/tile_rows)] (required then) for the
 * exact GPU fallback path (ffnrm_ffn_forward's fallback_tiles), the deadline rule of
 * src/phone_ffn_loopback.py:155-197; their values are still written. */
int ffnrm_base_from_table(ffnrm_base_producer *p, const ffnrm_radix_table *table, const int8_t *z, const float *s,
                          int tokens, int multiplier, float *base, int tile_rows, uint32_t *tile_ready,
                          int64_t deadline_ns, uint8_t *late_tiles);
/* The exact integer dots P_hi [rows, hidden/32] of one token (verification). */
int ffnrm_table_dots(const ffnrm_radix_table *table, const int8_t *z, int32_t *dots);

const char *ffnrm_last_error(void);
const char *ffnrm_version(void);

#ifdef __cplusplus
}
#endif
#endif /* FFNRM_H */
