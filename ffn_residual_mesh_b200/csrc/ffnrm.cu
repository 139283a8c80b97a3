// C ABI of the B200 exact base/residual split (see include/ffnrm.h).
//
// One context per device: owns each layer's device weights (codes in the layouts of
// ffnrm_common.cuh, alpha/beta, fp16 down), a workspace sized for max_tokens, and a
// non-blocking copy stream plus events for the host-streamed base pipeline.
#include "ffnrm.h"

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <utility>
#include <vector>

#include "down_umma.cuh"
#include "ffnrm_common.cuh"
#include "residual_dp4a.cuh"
#include "residual_mma.cuh"
#include "pack.cuh"
#include "peer_reduce.cuh"
#include "residual_tc.cuh"
#include "residual_umma.cuh"
#include "residual_prefill.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

#define FFNRM_CUDA(expr)                                                                          \
    do {                                                                                          \
        cudaError_t _e = (expr);                                                                  \
        if (_e != cudaSuccess)                                                                    \
            return fail(FFNRM_ERR_CUDA, "%s failed at %s:%d: %s", #expr, __FILE__, __LINE__,      \
                        cudaGetErrorString(_e));                                                  \
    } while (0)

struct DevBuf {
    void *ptr = nullptr;
    size_t bytes = 0;
};

struct LayerDev {
    bool loaded = false;
    bool scales_half = true;
    bool has_fallback = false;
    // code records, bit-plane records, fallback high pairs and scales of both projections
    // in the row-tiled layout of ffnrm_common.cuh (a projection's view starts 64 records in
    // for up)
    DevBuf pair, plane, pair_hi, alpha, beta, down;
    // low codes, one byte each, rows [128*rt, 128*rt+64) gate rows of tile rt then its up
    // rows: the tensor-core A operand (built when batches larger than the GEMV's fit)
    DevBuf codes8;
    CUtensorMap codes8_map;  // box 128 codes x 128 rows, 128-byte swizzle
    CUtensorMap down_map;    // TMA view of down [D][F16] fp16, box 64 x 128, 128-byte swizzle
};

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            ptr = nullptr;
        return reinterpret_cast<EncodeTiledFn>(ptr);
    }();
    return fn;
}

// 2-D fp16 tensor [rows][cols] (row stride ld elements) viewed in boxes of 64 columns x box_rows
// rows with 128-byte swizzle; out-of-range elements read as zero.
bool make_fp16_map(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D int8 activations [tokens][d_model] viewed in boxes of 128 codes x box_rows tokens
// with 128-byte swizzle; tokens past the end read as zero.
bool make_z_map(CUtensorMap *map, const void *z, uint64_t d_model, uint64_t tokens, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[2] = {d_model, tokens};
    const cuuint64_t strides[1] = {d_model};
    const cuuint32_t box[2] = {128, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(z), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Launches `kern`, when `dependent`, as a programmatic dependent of the preceding kernel of
// the stream (its launch overlaps that kernel's tail; the kernel waits for it with
// griddepcontrol.wait before touching its outputs), optionally as clusters of `cluster_x`
// CTAs along x. The residual kernels launch as dependents; the down projection's clusters
// do not (launched early they wait on SM space held by the residual and measured slower),
// but it triggers its dependents so the next residual launch overlaps its tail.
template <typename... Params, typename... Args>
cudaError_t launch_dependent(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             bool dependent, unsigned cluster_x, Args &&...args) {
    cudaLaunchConfig_t lc{};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    if (dependent) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster_x > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster_x;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    lc.attrs = attr;
    lc.numAttrs = n;
    return cudaLaunchKernelEx(&lc, kern, std::forward<Args>(args)...);
}

}  // namespace

struct ffnrm_ctx {
    int device = 0;
    ffnrm_config cfg{};
    int G = 0;
    std::vector<LayerDev> layers;
    DevBuf scratch;  // load-time decode scratch (grown on demand, kept for later layers)
    // workspace
    int *err = nullptr;                  // device error word written by bounded waits
    // T >= 3 residual: 1 = tcgen05 on byte codes where possible, packed records otherwise
    // (default); 0 = packed records only (no byte codes are built); 2 = mma.sync tiles
    // (FFNRM_RESIDUAL_KERNEL=bytes|packed|mma)
    int res_kernel = 1;
    int prefill_tokens = 0;  // batches of at least this many tokens (no fallback tiles) take the prefill residual (0 = off)
    CUtensorMap h_map[6][2];             // h hi/lo views for token tiles 16, 32, 64, 128, 192, 256
    int down_wide = -1;                  // token tile of the down GEMM above 128 tokens: 192 or 256;
                                         // 0 keeps 128; -1 (default) takes 192 from 1024 tokens
    __half *h_hi = nullptr, *h_lo = nullptr;  // [Tm, F16] h = SiLU(g)*u as fp16 hi + lo
    // host-streamed mode staging, double-buffered per call
    int8_t *z_dev[2] = {nullptr, nullptr};
    float *s_dev[2] = {nullptr, nullptr};
    float *base_dev[2][2] = {{nullptr, nullptr}, {nullptr, nullptr}};  // [slot][proj] [Tm, F]
    uint8_t *tiles_dev[2] = {nullptr, nullptr};
    uint16_t *y16_dev = nullptr;
    void *z16 = nullptr;  // [Tm, D] fp16 activations for the prefill residual
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t base_ready[2] = {nullptr, nullptr}, slot_free[2] = {nullptr, nullptr};
    int slot = 0;
    unsigned long long capture_id = 0;  // stream capture the slot events below belong to
    bool slot_in_capture[2] = {false, false};
    int64_t launches = 0;
    int num_sms = 148;
    int gemv_tokens = 2;  // FFNRM_GEMV_TOKENS: largest batch for the dp4a GEMV (measured crossover)
    // live profiling: event pairs around launches, resolved by ffnrm_profile_read
    bool prof = false;
    std::vector<cudaEvent_t> prof_pool;
    size_t prof_used = 0;
    std::vector<int> prof_kind;
};

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int dev_alloc(DevBuf &b, size_t bytes) {
    if (bytes == 0) return FFNRM_OK;
    if (cudaMalloc(&b.ptr, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(FFNRM_ERR_NOMEM, "cudaMalloc of %zu bytes failed", bytes);
    }
    b.bytes = bytes;
    return FFNRM_OK;
}

void dev_free(DevBuf &b) {
    if (b.ptr) cudaFree(b.ptr);
    b.ptr = nullptr;
    b.bytes = 0;
}

// Grid of a grid-stride load-time kernel over n outputs.
unsigned pack_blocks(int64_t n) { return unsigned(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16))); }

// Device view of one input array of ffnrm_load_layer: the caller's pointer when it is
// device memory of the context's device, else a device copy of the host data (owned).
struct Staged {
    const void *dev = nullptr;
    void *owned = nullptr;
    ~Staged() {
        if (owned) cudaFree(owned);
    }
};

int stage_in(int device, const void *src, size_t bytes, Staged &out) {
    if (!src || !bytes) return FFNRM_OK;
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, src) == cudaSuccess &&
        (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged)) {
        if (a.type == cudaMemoryTypeDevice && a.device != device)
            return fail(FFNRM_ERR_ARG, "a weight array lives on device %d, the context on device %d", a.device, device);
        out.dev = src;
        return FFNRM_OK;
    }
    cudaGetLastError();
    if (cudaMalloc(&out.owned, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(FFNRM_ERR_NOMEM, "cudaMalloc of %zu staging bytes failed", bytes);
    }
    FFNRM_CUDA(cudaMemcpy(out.owned, src, bytes, cudaMemcpyHostToDevice));
    out.dev = out.owned;
    return FFNRM_OK;
}

// 2-D u8 tensor [rows][cols] in boxes of 128 x box_rows with 128-byte swizzle.
bool make_u8_map(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols};
    const cuuint32_t box[2] = {128, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void free_layer(LayerDev &L) {
    {
        dev_free(L.pair);
        dev_free(L.plane);
        dev_free(L.pair_hi);
        dev_free(L.alpha);
        dev_free(L.beta);
        dev_free(L.codes8);
    }
    dev_free(L.down);
    L.loaded = false;
}

int check_ctx(ffnrm_ctx *ctx, int layer) {
    if (!ctx) return fail(FFNRM_ERR_ARG, "null context");
    if (layer < 0 || layer >= ctx->cfg.n_layers) return fail(FFNRM_ERR_ARG, "layer %d out of range [0, %d)", layer, ctx->cfg.n_layers);
    if (!ctx->layers[size_t(layer)].loaded) return fail(FFNRM_ERR_STATE, "layer %d is not loaded", layer);
    return FFNRM_OK;
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_tokens(ffnrm_ctx *ctx, int tokens) {
    if (tokens < 0 || tokens > ctx->cfg.max_tokens)
        return fail(FFNRM_ERR_ARG, "tokens=%d outside [0, max_tokens=%d]", tokens, ctx->cfg.max_tokens);
    return FFNRM_OK;
}

cudaEvent_t prof_event(ffnrm_ctx *ctx) {
    if (ctx->prof_used == ctx->prof_pool.size()) {
        cudaEvent_t e = nullptr;
        if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
        ctx->prof_pool.push_back(e);
    }
    return ctx->prof_pool[ctx->prof_used++];
}

// Brackets one kernel launch with events when profiling is on.
struct ProfScope {
    ffnrm_ctx *ctx;
    cudaStream_t st;
    int kind;
    bool on;
    // Inside a stream capture the events become external event-record nodes of the graph,
    // so they can be read after each replay.
    static void record(cudaEvent_t e, cudaStream_t st) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(st, &cap);
        if (cap == cudaStreamCaptureStatusActive)
            cudaEventRecordWithFlags(e, st, cudaEventRecordExternal);
        else
            cudaEventRecord(e, st);
    }
    ProfScope(ffnrm_ctx *c, cudaStream_t s, int k) : ctx(c), st(s), kind(k), on(c->prof) {
        if (on) {
            cudaEvent_t e = prof_event(ctx);
            if (!e) { on = false; return; }
            record(e, st);
        }
    }
    ~ProfScope() {
        if (!on) return;
        cudaEvent_t e = prof_event(ctx);
        if (!e) { ctx->prof_used--; return; }
        record(e, st);
        ctx->prof_kind.push_back(kind);
    }
};

// ---------------------------------------------------------------------------
// Kernel launchers
// ---------------------------------------------------------------------------
template <int RB, int TT, bool AH>
int launch_residual_t(ffnrm_ctx *ctx, ffnrm::ResidualParams &p, cudaStream_t st) {
    const size_t smem = ffnrm::residual_smem_bytes<RB, AH>(TT, p.D);
    auto kern = ffnrm::residual_gemv_kernel<RB, TT, AH>;
    if (smem > 48 * 1024) FFNRM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    p.row_blocks = (p.F + 31) / 32;
    dim3 grid(unsigned(p.row_blocks), unsigned((p.T + TT - 1) / TT));
    ProfScope prof(ctx, st, FFNRM_KERNEL_RESIDUAL);
    FFNRM_CUDA(launch_dependent(kern, grid, dim3(2 * ffnrm::kResWarps * 32), smem, st, true, 1, p));
    ctx->launches++;
    return FFNRM_OK;
}

template <int RB, int TT>
int launch_residual_tt(ffnrm_ctx *ctx, ffnrm::ResidualParams &p, bool half, cudaStream_t st) {
    return half ? launch_residual_t<RB, TT, true>(ctx, p, st) : launch_residual_t<RB, TT, false>(ctx, p, st);
}

template <int RB, int NT, bool AH, bool FB>
int launch_residual_mma_t(ffnrm_ctx *ctx, ffnrm::ResidualParams &p, cudaStream_t st) {
    constexpr int TN = NT * 8;
    const size_t smem = ffnrm::residual_mma_smem_bytes<RB, AH>(TN, p.G, FB);
    auto kern = ffnrm::residual_mma_kernel<RB, NT, AH, FB>;
    if (smem > 48 * 1024) FFNRM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    p.row_blocks = (p.F + 31) / 32;
    dim3 grid(unsigned((p.row_blocks + 1) / 2), unsigned((p.T + TN - 1) / TN));
    ProfScope prof(ctx, st, FFNRM_KERNEL_RESIDUAL);
    kern<<<grid, 128, smem, st>>>(p);
    ctx->launches++;
    FFNRM_CUDA(cudaGetLastError());
    return FFNRM_OK;
}

template <int RB, int NT>
int launch_residual_mma_nt(ffnrm_ctx *ctx, ffnrm::ResidualParams &p, bool half, cudaStream_t st) {
    const bool fb = p.fallback_tiles != nullptr;
    if (half) return fb ? launch_residual_mma_t<RB, NT, true, true>(ctx, p, st) : launch_residual_mma_t<RB, NT, true, false>(ctx, p, st);
    return fb ? launch_residual_mma_t<RB, NT, false, true>(ctx, p, st) : launch_residual_mma_t<RB, NT, false, false>(ctx, p, st);
}

template <int N, bool AH>
int launch_residual_tc_t(ffnrm_ctx *ctx, const LayerDev &L, ffnrm::ResidualParams &p, cudaStream_t st) {
    using Cfg = ffnrm::ResTcCfg<N, AH>;
    const int stages = Cfg::stages_for(p.G);
    const size_t smem = Cfg::smem(p.G, stages);
    CUtensorMap zm;
    if (!make_z_map(&zm, p.z, uint64_t(p.D), uint64_t(p.T), N))
        return fail(FFNRM_ERR_CUDA, "cuTensorMapEncodeTiled rejected the activations");
    auto kern = p.dots ? ffnrm::residual_tc_kernel<N, AH, true> : ffnrm::residual_tc_kernel<N, AH, false>;
    FFNRM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    p.row_blocks = (p.F + 31) / 32;
    p.err = ctx->err;
    dim3 grid(unsigned((p.T + N - 1) / N), unsigned((p.F + ffnrm::kTcTileRows - 1) / ffnrm::kTcTileRows));
    ProfScope prof(ctx, st, FFNRM_KERNEL_RESIDUAL);
    FFNRM_CUDA(launch_dependent(kern, grid, dim3(ffnrm::kTcThreads), smem, st, true, 1, L.codes8_map, zm, p, stages));
    ctx->launches++;
    return FFNRM_OK;
}

// Shared-memory layout of the packed-record tcgen05 residual for token tile N within
// `budget` bytes. Ring depths (S1 + S3 + SB <= 32 producer lanes) are chosen by a score
// of what each ring has to cover: code records (S1) one HBM round trip (~8 K tiles at the
// decode streaming rate), scales (S3) that plus the converter/MMA/drain lag (~16), the
// activation tiles (SB) an L2 round trip (~4), widened codes (S2) 2-3. The epilogue's
// up-row exchange [64][N+1] f32 reuses the code and activation rings.
ffnrm::UmLayout umma_layout(int N, bool has_pair, bool has_plane, bool has_hi, bool alpha_half, bool fb,
                            size_t budget) {
    const int a = 128 * ffnrm::kUmKTile, b = N * ffnrm::kUmKTile;
    ffnrm::UmLayout L{}, best{};
    int off = 0;
    L.off_pair = has_pair ? off : -1;
    off += has_pair ? 4096 : 0;
    L.off_plane = has_plane ? off : -1;
    off += has_plane ? 2048 : 0;
    L.off_hi = has_hi ? off : -1;
    off += has_hi ? 4096 : 0;
    L.src_bytes = std::max(off, 16);
    L.sc_bytes = (alpha_half ? 1024 : 2048) * (fb ? 2 : 1);
    const int win = 2 * ffnrm::kUmWin * (N + 4) * 4 * (fb ? 2 : 1);
    const int bars = (2 * (ffnrm::kUmMaxS1 + ffnrm::kUmMaxS2 + ffnrm::kUmMaxS3 + ffnrm::kUmMaxSB) + 2 * 4 + 1) * 8 + 16;
    const int xch = 64 * (N + 1) * 4;
    best.total = -1;
    int best_score = -1;
    for (int S2 = 2; S2 <= 3; ++S2)
        for (int SB = 2; SB <= ffnrm::kUmMaxSB; ++SB)
            for (int S1 = 3; S1 <= ffnrm::kUmMaxS1; ++S1)
                for (int S3 = 4; S3 <= std::min(ffnrm::kUmMaxS3, 32 - S1 - SB); ++S3) {
                    L.S1 = S1;
                    L.S2 = S2;
                    L.S3 = S3;
                    L.SB = SB;
                    L.b_off = S2 * a;
                    L.src_off = L.b_off + SB * b;
                    L.sc_off = L.src_off + S1 * L.src_bytes;
                    L.win_off = L.sc_off + S3 * L.sc_bytes;
                    L.bar_off = (L.win_off + win + 7) / 8 * 8;
                    L.total = L.bar_off + bars;
                    if (size_t(L.total) + 1024 > budget || L.src_off < xch) continue;
                    const int score = 4 * std::min(S1, 8) + 2 * std::min(S3, 16) + 4 * std::min(SB, 4) + 3 * S2 +
                                      std::min(S3, 24) / 4 + std::min(SB, 8) / 4;
                    if (score > best_score || (score == best_score && L.total < best.total)) {
                        best_score = score;
                        best = L;
                    }
                }
    return best;
}

template <int N>
int launch_residual_umma_t(ffnrm_ctx *ctx, const LayerDev &L, ffnrm::ResidualParams &p, cudaStream_t st) {
    using Cfg = ffnrm::UmCfg<N>;
    ffnrm::UmParams P{};
    P.rbits = ctx->cfg.residual_bits;
    P.has_pair = L.pair.ptr != nullptr;
    P.alpha_half = L.scales_half ? 1 : 0;
    P.fb = p.fallback_tiles != nullptr;
    const size_t budget = Cfg::minb == 2 ? 113 * 1024 : 227 * 1024;
    P.L = umma_layout(N, P.has_pair, P.rbits != 2, P.fb && L.pair_hi.ptr, L.scales_half, P.fb, budget);
    if (P.L.total < 0) return fail(FFNRM_ERR_ARG, "no shared-memory layout for the tensor-core residual (N=%d)", N);
    const size_t smem = size_t(P.L.total) + 1024;
    CUtensorMap zm;
    if (!make_z_map(&zm, p.z, uint64_t(p.D), uint64_t(p.T), N))
        return fail(FFNRM_ERR_CUDA, "cuTensorMapEncodeTiled rejected the activations");
    void (*kern)(const CUtensorMap, const ffnrm::UmParams);
    if constexpr (Cfg::minb == 2)
        kern = p.dots ? ffnrm::residual_umma_kernel2<N, true> : ffnrm::residual_umma_kernel2<N, false>;
    else
        kern = p.dots ? ffnrm::residual_umma_kernel1<N, true> : ffnrm::residual_umma_kernel1<N, false>;
    FFNRM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    p.row_blocks = (p.F + 31) / 32;
    p.err = ctx->err;
    P.p = p;
    dim3 grid(unsigned((p.T + N - 1) / N), unsigned((p.F + 63) / 64));
    ProfScope prof(ctx, st, FFNRM_KERNEL_RESIDUAL);
    FFNRM_CUDA(launch_dependent(kern, grid, dim3(Cfg::threads), smem, st, true, 1, zm, P));
    ctx->launches++;
    return FFNRM_OK;
}

// Shared-memory layout of the prefill residual: ring depths chosen to fit one CTA per SM.
// Activations (SA) and code records (S1) cover the L2/HBM latency (several K tiles each),
// widened codes (SW) the widening ahead of the MMA, f32 alphas (S4) the lag of the drain
// behind the widening (the MMAs run up to kPfBufs groups ahead of the drain).
ffnrm::PfLayout prefill_layout(bool has_pair, bool has_plane, bool alpha_half, size_t budget) {
    using namespace ffnrm;
    PfLayout L{}, best{};
    L.pair_bytes = has_pair ? 128 * 16 : 0;  // one chunk of 128 records
    L.plane_bytes = has_plane ? 128 * 8 : 0;
    L.alpha_bytes = 128 * (alpha_half ? 4 : 8);
    L.off_pair = 0;
    L.off_plane = L.pair_bytes;
    L.off_alpha = L.off_plane + L.plane_bytes;
    L.src_bytes = L.off_alpha + L.alpha_bytes;
    const int a = kPfTokens * kPfRowBytes, w = kPfN * kPfRowBytes, al = 2 * kPfN * 4;
    const int bars = (2 * (kPfMaxSA + kPfMaxS1 + kPfMaxSW + kPfMaxS4) + 2 * kPfBufs + 1) * 8 + 16;
    best.total = -1;
    int best_score = -1;
    for (int SW = 2; SW <= kPfMaxSW; ++SW)
        for (int SA = 2; SA <= kPfMaxSA; ++SA)
            for (int S1 = 2; S1 <= kPfMaxS1; ++S1)
                for (int S4 = 2; S4 <= kPfMaxS4; ++S4) {
                    L.SA = SA;
                    L.S1 = S1;
                    L.SW = SW;
                    L.S4 = S4;
                    L.w_off = SA * a;
                    L.src_off = L.w_off + SW * w;
                    L.al_off = L.src_off + S1 * L.src_bytes;
                    L.bar_off = (L.al_off + S4 * al + 7) / 8 * 8;
                    L.total = L.bar_off + bars;
                    if (size_t(L.total) + 1024 > budget) continue;
                    const int score = 4 * std::min(SA, 6) + 4 * std::min(S1, 6) + 3 * std::min(S4, 6) + 3 * std::min(SW, 3) +
                                      SA + S1 + S4 / 2;
                    if (score > best_score || (score == best_score && L.total < best.total)) {
                        best_score = score;
                        best = L;
                    }
                }
    return best;
}

template <bool DOTS>
int launch_residual_prefill_t(ffnrm_ctx *ctx, const LayerDev &L, ffnrm::ResidualParams &p, cudaStream_t st) {
    using namespace ffnrm;
    PfParams P{};
    P.rbits = ctx->cfg.residual_bits;
    P.alpha_half = L.scales_half ? 1 : 0;
    const bool has_pair = P.rbits != 1;
    if ((has_pair && !L.pair.ptr) || (P.rbits != 2 && !L.plane.ptr))
        return fail(FFNRM_ERR_STATE, "layer lacks the code records the prefill residual reads");
    if (!ctx->z16) return fail(FFNRM_ERR_STATE, "no fp16 activation workspace");
    P.L = prefill_layout(has_pair, P.rbits != 2, L.scales_half, 227 * 1024);
    if (P.L.total < 0) return fail(FFNRM_ERR_ARG, "no shared-memory layout for the prefill residual");
    const size_t smem = size_t(P.L.total) + 1024;
    auto kern = residual_prefill_kernel<DOTS>;
    CUtensorMap zm;
    if (!make_fp16_map(&zm, ctx->z16, uint64_t(p.D), uint64_t(p.T), uint64_t(p.D), kPfTokens))
        return fail(FFNRM_ERR_CUDA, "cuTensorMapEncodeTiled rejected the fp16 activations");
    FFNRM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    // z -> fp16 (exact) into the workspace, then the residual as its dependent
    const int64_t n = int64_t(p.T) * p.D;
    const int cblocks = int(std::min<int64_t>((n / 16 + 255) / 256, int64_t(ctx->num_sms) * 8));
    FFNRM_CUDA(launch_dependent(z_to_f16_kernel, dim3(unsigned(cblocks)), dim3(256), 0, st, false, 1, p.z,
                                static_cast<__half *>(ctx->z16), n));
    ctx->launches++;
    p.row_blocks = (p.F + 31) / 32;
    p.err = ctx->err;
    P.p = p;
    dim3 grid(unsigned((p.T + kPfTokens - 1) / kPfTokens), unsigned((p.F + kPfRows - 1) / kPfRows));
    ProfScope prof(ctx, st, FFNRM_KERNEL_RESIDUAL);
    FFNRM_CUDA(launch_dependent(kern, grid, dim3(kPfThreads), smem, st, true, 1, zm, P));
    ctx->launches++;
    return FFNRM_OK;
}

// T <= 2 (FFNRM_GEMV_TOKENS): dp4a GEMV on the packed records. Larger batches: tcgen05
// kind::i8 tiles - on the byte codes (token tiles of 16 or 32) when the layer has them and
// no fallback tile is flagged; otherwise, fallback tiles included, on the packed records
// widened to bytes in shared memory (token tiles of 16, 32, 64, 128). The mma.sync tiles
// remain selectable for comparison (FFNRM_RESIDUAL_KERNEL=mma).
template <int RB>
int launch_residual_rb(ffnrm_ctx *ctx, const LayerDev &L, ffnrm::ResidualParams &p, bool half, cudaStream_t st) {
    if (p.T <= std::min(ctx->gemv_tokens, ffnrm::kGemvMaxTokens)) {
        if (p.T == 1) return launch_residual_tt<RB, 1>(ctx, p, half, st);
        if (p.T == 2) return launch_residual_tt<RB, 2>(ctx, p, half, st);
        return launch_residual_tt<RB, 4>(ctx, p, half, st);
    }
    if (ctx->res_kernel == 2) {
        if (p.T <= ffnrm::kGemvMaxTokens) return launch_residual_tt<RB, 4>(ctx, p, half, st);
        if (p.T <= 8) return launch_residual_mma_nt<RB, 1>(ctx, p, half, st);
        if (p.T <= 16) return launch_residual_mma_nt<RB, 2>(ctx, p, half, st);
        return launch_residual_mma_nt<RB, 4>(ctx, p, half, st);  // 32-token tiles (64 would spill)
    }
    if (p.fallback_tiles == nullptr && ctx->prefill_tokens > 0 && p.T >= ctx->prefill_tokens &&
        (reinterpret_cast<uintptr_t>(p.s) & 7) == 0 && (reinterpret_cast<uintptr_t>(p.z) & 15) == 0)
        return p.dots ? launch_residual_prefill_t<true>(ctx, L, p, st) : launch_residual_prefill_t<false>(ctx, L, p, st);
    if (ctx->res_kernel == 1 && p.fallback_tiles == nullptr && L.codes8.ptr &&
        ffnrm::ResTcCfg<32, false>::smem(p.G, 2) <= 227 * 1024) {
        // 16-token tiles when 32-token ones would leave SMs idle (a d_ff shard's few row tiles at
        // decode sizes): twice the CTAs, each A tile read twice, mostly from L2.
        const int row_tiles = (p.F + ffnrm::kTcTileRows - 1) / ffnrm::kTcTileRows;
        const bool narrow = p.T <= 16 || (p.T <= 64 && row_tiles * ((p.T + 31) / 32) < ctx->num_sms);
        if (narrow) return half ? launch_residual_tc_t<16, true>(ctx, L, p, st) : launch_residual_tc_t<16, false>(ctx, L, p, st);
        return half ? launch_residual_tc_t<32, true>(ctx, L, p, st) : launch_residual_tc_t<32, false>(ctx, L, p, st);
    }
    if (p.T <= 16) return launch_residual_umma_t<16>(ctx, L, p, st);
    if (p.T <= 32) return launch_residual_umma_t<32>(ctx, L, p, st);
    if (p.T <= 64) return launch_residual_umma_t<64>(ctx, L, p, st);
    return launch_residual_umma_t<128>(ctx, L, p, st);
}

// Residual contraction of both projections. Residual mode (gate_base == nullptr): writes
// gate_res/up_res. Forward mode: merges with the base sums and writes h into the workspace.
int enqueue_residual(ffnrm_ctx *ctx, int layer, const int8_t *z, const float *s, int T, float *gate_res,
                     float *up_res, int32_t *dots, const uint8_t *tiles, const float *gate_base,
                     const float *up_base, cudaStream_t st) {
    LayerDev &L = ctx->layers[size_t(layer)];
    if (tiles && !L.has_fallback)
        return fail(FFNRM_ERR_STATE, "fallback tiles given but layer %d was loaded without fallback data", layer);
    ffnrm::ResidualParams p{};
    for (int q = 0; q < 2; ++q) {
        // a projection's view starts 64 records into each tile's run (0 for gate, 64 for up)
        const int64_t o = 64 * q, sb = L.scales_half ? 4 : 8;
        auto at = [](const DevBuf &b, int64_t bytes) -> const void * {
            return b.ptr ? static_cast<const uint8_t *>(b.ptr) + bytes : nullptr;
        };
        p.proj[q] = ffnrm::ProjView{static_cast<const uint4 *>(at(L.pair, o * 16)), static_cast<const uint2 *>(at(L.plane, o * 8)),
                                    static_cast<const uint4 *>(at(L.pair_hi, o * 16)), at(L.alpha, o * sb),
                                    at(L.beta, o * sb)};
    }
    p.z = z;
    p.s = s;
    p.out[0] = gate_res;
    p.out[1] = up_res;
    p.dots = dots;
    p.base[0] = gate_base;
    p.base[1] = up_base;
    p.h_hi = gate_base ? ctx->h_hi : nullptr;
    p.h_lo = gate_base ? ctx->h_lo : nullptr;
    p.F16 = (ctx->cfg.d_ff + 15) / 16 * 16;
    p.fallback_tiles = tiles;
    p.F = ctx->cfg.d_ff;
    p.D = ctx->cfg.d_model;
    p.G = ctx->G;
    p.T = T;
    p.tile_rows = ctx->cfg.base_tile_rows;
    const int r = ctx->cfg.residual_bits;
    switch (r) {
        case 1: return launch_residual_rb<1>(ctx, L, p, L.scales_half, st);
        case 2: return launch_residual_rb<2>(ctx, L, p, L.scales_half, st);
        default: return launch_residual_rb<3>(ctx, L, p, L.scales_half, st);
    }
}

// Launches the down GEMM: split-K slices of one output tile form a thread-block cluster
// (at most 8) sized so that about two CTAs per SM are busy.
template <int N>
int launch_down_cluster(const CUtensorMap &wm, const CUtensorMap &hm, const CUtensorMap &lm, ffnrm::DownUmmaParams &p,
                        int num_sms, cudaStream_t st) {
    using Cfg = ffnrm::DownUmmaCfg<N>;
    auto kern = ffnrm::down_umma_kernel<N>;
    FFNRM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg::smem)));
    const int occ = Cfg::smem <= 113 * 1024 ? 2 : 1;
    const int mt = p.D / ffnrm::kUmmaM, ntile = (p.T + N - 1) / N;
    const int ksteps = (p.F16 + ffnrm::kUmmaK - 1) / ffnrm::kUmmaK;
    int splits = p.fused ? 1 : std::max(1, std::min({ksteps, ffnrm::kDownMaxSplits, occ * num_sms / (mt * ntile)}));
    const int kc_steps = (ksteps + splits - 1) / splits;
    splits = (ksteps + kc_steps - 1) / kc_steps;
    p.splits = splits;
    p.kc = kc_steps * ffnrm::kUmmaK;
    FFNRM_CUDA(launch_dependent(kern, dim3(unsigned(splits), unsigned(mt), unsigned(ntile)), dim3(128), Cfg::smem, st,
                                false, unsigned(splits), wm, hm, lm, p));
    return FFNRM_OK;
}

template <int N>
int launch_down_t(ffnrm_ctx *ctx, const CUtensorMap &wmap, int map_idx, ffnrm::DownUmmaParams &p, cudaStream_t st) {
    ProfScope prof(ctx, st, FFNRM_KERNEL_DOWN);
    const int rc = launch_down_cluster<N>(wmap, ctx->h_map[map_idx][0], ctx->h_map[map_idx][1], p, ctx->num_sms, st);
    ctx->launches++;
    return rc;
}

// Token tile of the down GEMM for a batch of T tokens. 192-token tiles give each MMA 1.5x the
// work of 128-token ones (measured c4 layer at T = 2048: 1.67 ms vs 1.96 ms) but leave fewer,
// larger tiles: below about 1024 tokens the 128-token grid is faster (T = 512: 0.54 vs 0.60 ms).
static int down_token_tile(const ffnrm_ctx *ctx, int T) {
    if (T <= 16) return 16;
    if (T <= 32) return 32;
    if (T <= 64) return 64;
    const int wide = ctx->down_wide < 0 ? (T >= 1024 ? 192 : 0) : ctx->down_wide;
    return T <= 128 || wide == 0 ? 128 : wide;
}

// `sc` non-null: the output tiles go straight into the layer reduction's scatter slots.
int enqueue_down(ffnrm_ctx *ctx, int layer, int T, float *y32, uint16_t *y16, cudaStream_t st,
                 const ffnrm::DownScatter *sc = nullptr) {
    LayerDev &L = ctx->layers[size_t(layer)];
    if (!L.down.ptr) return fail(FFNRM_ERR_STATE, "layer %d was loaded without a down projection", layer);
    ffnrm::DownUmmaParams p{};
    p.y32 = y32;
    p.y16 = reinterpret_cast<__half *>(y16);
    p.err = ctx->err;
    p.D = ctx->cfg.d_model;
    p.F16 = (ctx->cfg.d_ff + 15) / 16 * 16;
    p.T = T;
    if (sc) {
        p.fused = 1;
        p.sc = *sc;
    }
    switch (down_token_tile(ctx, T)) {
        case 16: return launch_down_t<16>(ctx, L.down_map, 0, p, st);
        case 32: return launch_down_t<32>(ctx, L.down_map, 1, p, st);
        case 64: return launch_down_t<64>(ctx, L.down_map, 2, p, st);
        case 128: return launch_down_t<128>(ctx, L.down_map, 3, p, st);
        case 192: return launch_down_t<192>(ctx, L.down_map, 4, p, st);
        default: return launch_down_t<256>(ctx, L.down_map, 5, p, st);
    }
}

// ---------------------------------------------------------------------------
// Allocation-free down projection: its only scratch is a file-scope device word
// ---------------------------------------------------------------------------
constexpr int kNoAllocMaxTokens = 256;     // largest token-tile grid the call launches
constexpr int kNoAllocMaxDModel = 16384;   // largest d_model (output row tiles) it accepts
constexpr int kNoAllocMaxDevices = 64;

// The default status word of calls that pass status = NULL. Every GPU that loads this
// library holds its own copy until the process exits.
__device__ __align__(256) int g_noalloc_status;

using CtxGetCurrentFn = CUresult (*)(CUcontext *);

CUcontext current_context() {
    static CtxGetCurrentFn fn = [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            ptr = nullptr;
        return reinterpret_cast<CtxGetCurrentFn>(ptr);
    }();
    CUcontext c = nullptr;
    if (fn) fn(&c);
    return c;
}

struct NoAllocScratch {
    int *status = nullptr;
    CUcontext ctx = nullptr;  // the context the address belongs to
};
std::mutex g_noalloc_mutex;
NoAllocScratch g_noalloc[kNoAllocMaxDevices];

// Device address of the status word on `dev` (the current device). It is looked up with
// cudaGetSymbolAddress the first time and again whenever the device's context changed (a
// reset or a new primary context), so no stale address is ever used.
int noalloc_scratch(int dev, NoAllocScratch &out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoAllocScratch &s = g_noalloc[dev];
    const CUcontext c = current_context();
    if (!s.status || s.ctx != c) {
        NoAllocScratch t;
        FFNRM_CUDA(cudaGetSymbolAddress(reinterpret_cast<void **>(&t.status), g_noalloc_status));
        t.ctx = c;
        s = t;
    }
    out = s;
    return FFNRM_OK;
}

template <int N>
int launch_down_noalloc(const uint16_t *down, int64_t down_ld, const uint16_t *h_hi, const uint16_t *h_lo,
                        int64_t h_ld, int D, int F, int T, float *y32, uint16_t *y16, int32_t *status,
                        const NoAllocScratch &scr, cudaStream_t st) {
    CUtensorMap wm, hm, lm;
    if (!make_fp16_map(&wm, down, uint64_t(F), uint64_t(D), uint64_t(down_ld), 128) ||
        !make_fp16_map(&hm, h_hi, uint64_t(F), uint64_t(T), uint64_t(h_ld), N) ||
        !make_fp16_map(&lm, h_lo, uint64_t(F), uint64_t(T), uint64_t(h_ld), N))
        return fail(FFNRM_ERR_CUDA, "cuTensorMapEncodeTiled rejected the down weight or h");
    int dev = 0, sms = 148;
    FFNRM_CUDA(cudaGetDevice(&dev));
    FFNRM_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    ffnrm::DownUmmaParams p{};
    p.y32 = y32;
    p.y16 = reinterpret_cast<__half *>(y16);
    p.err = status ? status : scr.status;
    p.D = D;
    p.F16 = (F + 15) / 16 * 16;
    p.T = T;
    // The status word keeps the previous call's value: it must start at zero.
    FFNRM_CUDA(cudaMemsetAsync(p.err, 0, sizeof(int), st));
    return launch_down_cluster<N>(wm, hm, lm, p, sms, st);
}

}  // namespace

// Sets the calling thread's last error (used by the host-side translation units).
int ffnrm_set_error(int code, const char *msg) { return fail(code, "%s", msg); }

extern "C" {

const char *ffnrm_last_error(void) { return g_last_error.c_str(); }
const char *ffnrm_version(void) { return "ffnrm 0.1 (sm_100a)"; }

int ffnrm_create(ffnrm_ctx **out, int device, const ffnrm_config *cfg) {
    if (!out || !cfg) return fail(FFNRM_ERR_ARG, "null argument");
    *out = nullptr;
    const ffnrm_config c = *cfg;
    if (c.d_model <= 0 || c.d_model % 256) return fail(FFNRM_ERR_ARG, "d_model=%d must be a positive multiple of 256", c.d_model);
    if (c.d_ff <= 0) return fail(FFNRM_ERR_ARG, "d_ff=%d must be positive", c.d_ff);
    if (c.residual_bits < 1 || c.residual_bits > 3) return fail(FFNRM_ERR_ARG, "residual_bits=%d must be 1, 2 or 3", c.residual_bits);
    if (c.n_layers <= 0 || c.max_tokens <= 0) return fail(FFNRM_ERR_ARG, "n_layers and max_tokens must be positive");
    if (c.base_tile_rows <= 0) return fail(FFNRM_ERR_ARG, "base_tile_rows must be positive");
    int count = 0;
    FFNRM_CUDA(cudaGetDeviceCount(&count));
    if (device < 0 || device >= count) return fail(FFNRM_ERR_ARG, "device %d not present (%d devices)", device, count);
    DeviceGuard guard(device);
    auto *ctx = new (std::nothrow) ffnrm_ctx;
    if (!ctx) return fail(FFNRM_ERR_NOMEM, "host allocation failed");
    ctx->device = device;
    ctx->cfg = c;
    ctx->G = c.d_model / 32;
    ctx->layers.resize(size_t(c.n_layers));
    if (const char *e = std::getenv("FFNRM_RESIDUAL_KERNEL"))
        ctx->res_kernel = std::strcmp(e, "packed") == 0 ? 0 : std::strcmp(e, "mma") == 0 ? 2 : 1;
    if (const char *e = std::getenv("FFNRM_GEMV_TOKENS")) ctx->gemv_tokens = std::max(1, std::atoi(e));
    if (const char *e = std::getenv("FFNRM_PREFILL_TOKENS")) ctx->prefill_tokens = std::max(0, std::atoi(e));
    if (const char *e = std::getenv("FFNRM_DOWN_WIDE")) {
        const int w = std::atoi(e);
        ctx->down_wide = w == 192 || w == 256 ? w : (w == 0 && e[0] == '0' ? 0 : -1);
    }
    cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
    const size_t TF = size_t(c.max_tokens) * c.d_ff, TD = size_t(c.max_tokens) * c.d_model;
    const size_t F16 = (size_t(c.d_ff) + 15) / 16 * 16;
    const int ntiles = (c.d_ff + c.base_tile_rows - 1) / c.base_tile_rows;
    bool ok = cudaMalloc(&ctx->err, sizeof(int)) == cudaSuccess && cudaMemset(ctx->err, 0, sizeof(int)) == cudaSuccess &&
              cudaMalloc(&ctx->h_hi, size_t(c.max_tokens) * F16 * 2) == cudaSuccess &&
              cudaMalloc(&ctx->h_lo, size_t(c.max_tokens) * F16 * 2) == cudaSuccess &&
              cudaMalloc(&ctx->y16_dev, TD * 2) == cudaSuccess && cudaMalloc(&ctx->z16, TD * 2) == cudaSuccess;
    for (int sl = 0; sl < 2 && ok; ++sl) {
        ok = cudaMalloc(&ctx->base_dev[sl][0], TF * 4) == cudaSuccess && cudaMalloc(&ctx->base_dev[sl][1], TF * 4) == cudaSuccess &&
             cudaMalloc(&ctx->tiles_dev[sl], size_t(ntiles)) == cudaSuccess &&
             cudaMalloc(&ctx->z_dev[sl], TD) == cudaSuccess &&
             cudaMalloc(&ctx->s_dev[sl], size_t(c.max_tokens) * ctx->G * 4) == cudaSuccess;
    }
    ok = ok && cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking) == cudaSuccess;
    for (int sl = 0; sl < 2 && ok; ++sl)
        ok = cudaEventCreateWithFlags(&ctx->base_ready[sl], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&ctx->slot_free[sl], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        ffnrm_destroy(ctx);
        return fail(FFNRM_ERR_NOMEM, "workspace allocation failed (max_tokens=%d, d_ff=%d)", c.max_tokens, c.d_ff);
    }
    const uint32_t tiles[6] = {16, 32, 64, 128, 192, 256};
    for (int i = 0; i < (c.max_tokens > 128 ? 6 : 4); ++i)  // the wide tiles serve batches above 128
        if (!make_fp16_map(&ctx->h_map[i][0], ctx->h_hi, F16, size_t(c.max_tokens), F16, tiles[i]) ||
            !make_fp16_map(&ctx->h_map[i][1], ctx->h_lo, F16, size_t(c.max_tokens), F16, tiles[i])) {
            ffnrm_destroy(ctx);
            return fail(FFNRM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable or rejected the h buffers");
        }
    *out = ctx;
    return FFNRM_OK;
}

int ffnrm_destroy(ffnrm_ctx *ctx) {
    if (!ctx) return FFNRM_OK;
    DeviceGuard guard(ctx->device);
    cudaDeviceSynchronize();
    for (auto &L : ctx->layers) free_layer(L);
    dev_free(ctx->scratch);
    cudaFree(ctx->err);
    cudaFree(ctx->h_hi);
    cudaFree(ctx->h_lo);
    cudaFree(ctx->y16_dev);
    cudaFree(ctx->z16);
    for (int sl = 0; sl < 2; ++sl) {
        cudaFree(ctx->base_dev[sl][0]);
        cudaFree(ctx->base_dev[sl][1]);
        cudaFree(ctx->tiles_dev[sl]);
        cudaFree(ctx->z_dev[sl]);
        cudaFree(ctx->s_dev[sl]);
        if (ctx->base_ready[sl]) cudaEventDestroy(ctx->base_ready[sl]);
        if (ctx->slot_free[sl]) cudaEventDestroy(ctx->slot_free[sl]);
    }
    if (ctx->copy_stream) cudaStreamDestroy(ctx->copy_stream);
    for (cudaEvent_t e : ctx->prof_pool) cudaEventDestroy(e);
    delete ctx;
    return FFNRM_OK;
}

int ffnrm_load_layer(ffnrm_ctx *ctx, int layer, const ffnrm_layer_weights *w) {
    if (!ctx || !w) return fail(FFNRM_ERR_ARG, "null argument");
    if (layer < 0 || layer >= ctx->cfg.n_layers) return fail(FFNRM_ERR_ARG, "layer %d out of range", layer);
    if (!w->gate_codes || !w->up_codes || !w->gate_alpha || !w->up_alpha)
        return fail(FFNRM_ERR_ARG, "codes and alpha are required");
    const int64_t F = ctx->cfg.d_ff, D = ctx->cfg.d_model, G = ctx->G, n = F * D;
    const int r = ctx->cfg.residual_bits;
    const int fmt = w->codes_format;
    if (w->down && w->down_ld < F) return fail(FFNRM_ERR_ARG, "down_ld=%lld must be >= d_ff=%lld", (long long)w->down_ld, (long long)F);
    if (fmt != FFNRM_CODES_Q4_BYTES && fmt != FFNRM_CODES_QLO2_ROWPACKED && fmt != FFNRM_CODES_BITPLANES)
        return fail(FFNRM_ERR_ARG, "unknown codes_format %d", fmt);
    if (fmt == FFNRM_CODES_QLO2_ROWPACKED && r != 2)
        return fail(FFNRM_ERR_ARG, "QLO2 row-packed codes require residual_bits == 2");
    const bool want_hi = fmt == FFNRM_CODES_Q4_BYTES ? w->keep_fallback != 0 : (w->gate_high && w->up_high);
    const bool have_beta = w->gate_beta && w->up_beta;
    if (want_hi && !have_beta) return fail(FFNRM_ERR_ARG, "fallback high codes need gate_beta and up_beta");
    DeviceGuard guard(ctx->device);
    LayerDev &L = ctx->layers[size_t(layer)];
    free_layer(L);
    L.has_fallback = want_hi && have_beta;
    const size_t code_bytes = fmt == FFNRM_CODES_Q4_BYTES ? size_t(n) : fmt == FFNRM_CODES_QLO2_ROWPACKED ? size_t(n / 4)
                                                                                                           : size_t(r * n / 8);
    // Stage every input on the device, then decode and pack there.
    Staged codes[2], high[2], alpha[2], beta[2];
    const uint8_t *cin[2] = {w->gate_codes, w->up_codes}, *hin[2] = {w->gate_high, w->up_high};
    const float *ain[2] = {w->gate_alpha, w->up_alpha}, *bin[2] = {w->gate_beta, w->up_beta};
    int rc = FFNRM_OK;
    for (int q = 0; q < 2 && rc == FFNRM_OK; ++q) {
        rc = stage_in(ctx->device, cin[q], code_bytes, codes[q]);
        if (rc == FFNRM_OK && L.has_fallback && fmt != FFNRM_CODES_Q4_BYTES)
            rc = stage_in(ctx->device, hin[q], size_t((4 - r) * n / 8), high[q]);
        if (rc == FFNRM_OK) rc = stage_in(ctx->device, ain[q], size_t(F * G) * 4, alpha[q]);
        if (rc == FFNRM_OK && L.has_fallback) rc = stage_in(ctx->device, bin[q], size_t(F * G) * 4, beta[q]);
    }
    if (rc) return rc;
    // scratch: low codes [2][n], full codes [2][n] (fallback, unless given as Q4 bytes), two flags
    const bool full_scratch = L.has_fallback && fmt != FFNRM_CODES_Q4_BYTES;
    const size_t need = size_t(n) * (full_scratch ? 4 : 2) + 16;
    if (ctx->scratch.bytes < need) {
        dev_free(ctx->scratch);
        if ((rc = dev_alloc(ctx->scratch, need))) return rc;
    }
    uint8_t *lo[2] = {static_cast<uint8_t *>(ctx->scratch.ptr), static_cast<uint8_t *>(ctx->scratch.ptr) + n};
    const uint8_t *full[2] = {nullptr, nullptr};
    if (L.has_fallback)
        for (int q = 0; q < 2; ++q)
            full[q] = fmt == FFNRM_CODES_Q4_BYTES ? static_cast<const uint8_t *>(codes[q].dev)
                                                  : static_cast<uint8_t *>(ctx->scratch.ptr) + (2 + q) * n;
    int *flags = reinterpret_cast<int *>(static_cast<uint8_t *>(ctx->scratch.ptr) + size_t(n) * (full_scratch ? 4 : 2));
    FFNRM_CUDA(cudaMemset(flags, 0, 2 * sizeof(int)));
    for (int q = 0; q < 2; ++q)
        ffnrm::decode_codes_kernel<<<pack_blocks(n), 256>>>(fmt, static_cast<const uint8_t *>(codes[q].dev),
                                                           static_cast<const uint8_t *>(high[q].dev), r, n, lo[q],
                                                           full_scratch ? const_cast<uint8_t *>(full[q]) : nullptr, flags);
    for (int q = 0; q < 2; ++q) {
        ffnrm::half_exact_kernel<<<pack_blocks(F * G), 256>>>(static_cast<const float *>(alpha[q].dev), F * G, flags + 1);
        if (L.has_fallback)
            ffnrm::half_exact_kernel<<<pack_blocks(F * G), 256>>>(static_cast<const float *>(beta[q].dev), F * G,
                                                                  flags + 1);
    }
    FFNRM_CUDA(cudaGetLastError());
    int hflags[2] = {0, 0};
    FFNRM_CUDA(cudaMemcpy(hflags, flags, sizeof(hflags), cudaMemcpyDeviceToHost));
    if (hflags[0]) return fail(FFNRM_ERR_ARG, "Q4 codes must be in [0, 15]");
    L.scales_half = hflags[1] == 0;
    const int64_t F64 = (F + 63) / 64, C = D / 64, recs = F64 * C * 128;
    if ((r != 1 || L.has_fallback) && (rc = dev_alloc(L.pair, size_t(recs) * 16)) == FFNRM_OK) {
        // bits 0-1 of the full code equal the low two residual bits for r >= 2
        const uint8_t *s0 = L.has_fallback ? full[0] : lo[0], *s1 = L.has_fallback ? full[1] : lo[1];
        ffnrm::pack_pair_kernel<<<pack_blocks(recs), 256>>>(s0, s1, 0, F, D, static_cast<uint4 *>(L.pair.ptr));
    }
    if (rc == FFNRM_OK && r != 2 && (rc = dev_alloc(L.plane, size_t(recs) * 8)) == FFNRM_OK)
        ffnrm::pack_plane_kernel<<<pack_blocks(recs), 256>>>(lo[0], lo[1], r == 1 ? 0 : 2, F, D,
                                                             static_cast<uint2 *>(L.plane.ptr));
    if (rc == FFNRM_OK && L.has_fallback && (rc = dev_alloc(L.pair_hi, size_t(recs) * 16)) == FFNRM_OK)
        ffnrm::pack_pair_kernel<<<pack_blocks(recs), 256>>>(full[0], full[1], 2, F, D, static_cast<uint4 *>(L.pair_hi.ptr));
    const size_t sbytes = size_t(recs) * (L.scales_half ? 4 : 8);
    if (rc == FFNRM_OK && (rc = dev_alloc(L.alpha, sbytes)) == FFNRM_OK)
        ffnrm::pack_scales_kernel<<<pack_blocks(recs), 256>>>(static_cast<const float *>(alpha[0].dev),
                                                              static_cast<const float *>(alpha[1].dev), F, G,
                                                              L.scales_half, L.alpha.ptr);
    if (rc == FFNRM_OK && L.has_fallback && (rc = dev_alloc(L.beta, sbytes)) == FFNRM_OK)
        ffnrm::pack_scales_kernel<<<pack_blocks(recs), 256>>>(static_cast<const float *>(beta[0].dev),
                                                              static_cast<const float *>(beta[1].dev), F, G,
                                                              L.scales_half, L.beta.ptr);
    if (rc == FFNRM_OK && ctx->res_kernel == 1 && ctx->cfg.max_tokens > std::min(ctx->gemv_tokens, ffnrm::kGemvMaxTokens) &&
        (rc = dev_alloc(L.codes8, size_t(F64) * 128 * D)) == FFNRM_OK) {
        ffnrm::pack_codes8_kernel<<<pack_blocks(F64 * 128 * D / 16), 256>>>(lo[0], lo[1], F, D,
                                                                             static_cast<uint4 *>(L.codes8.ptr));
        if (!make_u8_map(&L.codes8_map, L.codes8.ptr, uint64_t(D), uint64_t(F64 * 128), 128))
            rc = fail(FFNRM_ERR_CUDA, "cuTensorMapEncodeTiled rejected the byte codes");
    }
    // fp16 down [D, ld] (F used columns) -> row-major [D][F16] with zero columns F..F16-1
    const int64_t F16 = (F + 15) / 16 * 16;
    if (rc == FFNRM_OK && w->down && (rc = dev_alloc(L.down, size_t(D * F16) * 2)) == FFNRM_OK) {
        FFNRM_CUDA(cudaMemset(L.down.ptr, 0, L.down.bytes));
        FFNRM_CUDA(cudaMemcpy2D(L.down.ptr, size_t(F16) * 2, w->down, size_t(w->down_ld) * 2, size_t(F) * 2, size_t(D),
                                cudaMemcpyDefault));
    }
    if (rc == FFNRM_OK && w->down && !make_fp16_map(&L.down_map, L.down.ptr, uint64_t(F16), uint64_t(D), uint64_t(F16), 128))
        rc = fail(FFNRM_ERR_CUDA, "cuTensorMapEncodeTiled rejected the down weight");
    if (rc == FFNRM_OK) {
        const cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) rc = fail(FFNRM_ERR_CUDA, "layer packing failed: %s", cudaGetErrorString(e));
    }
    if (rc) {
        free_layer(L);
        return rc;
    }
    L.loaded = true;
    return FFNRM_OK;
}

int ffnrm_residual(ffnrm_ctx *ctx, int layer, const int8_t *z, const float *s, int tokens, float *gate_res,
                   float *up_res, int32_t *group_dots, const uint8_t *fallback_tiles, void *stream) {
    int rc = check_ctx(ctx, layer);
    if (rc) return rc;
    if ((rc = check_tokens(ctx, tokens))) return rc;
    if (tokens == 0) return FFNRM_OK;  // empty batch
    if (!z || !s || !gate_res || !up_res) return fail(FFNRM_ERR_ARG, "null device pointer");
    if (!aligned(z, 16) || !aligned(s, 4) || !aligned(gate_res, 4) || !aligned(up_res, 4) || !aligned(group_dots, 8))
        return fail(FFNRM_ERR_ARG, "z must be 16-byte aligned and s/outputs 4-byte aligned (dots 8-byte)");
    DeviceGuard guard(ctx->device);
    return enqueue_residual(ctx, layer, z, s, tokens, gate_res, up_res, group_dots, fallback_tiles, nullptr,
                            nullptr, static_cast<cudaStream_t>(stream));
}

int ffnrm_ffn_forward(ffnrm_ctx *ctx, int layer, const int8_t *z, const float *s, int tokens, const float *gate_base,
                      const float *up_base, const uint8_t *fallback_tiles, float *y_f32, uint16_t *y_f16,
                      void *stream) {
    int rc = check_ctx(ctx, layer);
    if (rc) return rc;
    if ((rc = check_tokens(ctx, tokens))) return rc;
    if (tokens == 0) return FFNRM_OK;  // empty batch
    if (!z || !s || !gate_base || !up_base) return fail(FFNRM_ERR_ARG, "null device pointer");
    if (!y_f32 && !y_f16) return fail(FFNRM_ERR_ARG, "no output requested");
    if (!ctx->layers[size_t(layer)].down.ptr)
        return fail(FFNRM_ERR_STATE, "layer %d was loaded without a down projection", layer);
    if (!aligned(z, 16) || !aligned(s, 4) || !aligned(gate_base, 4) || !aligned(up_base, 4) || !aligned(y_f32, 16) ||
        !aligned(y_f16, 8))
        return fail(FFNRM_ERR_ARG, "z and y_f32 must be 16-byte aligned, y_f16 8-byte, s and base sums 4-byte");
    DeviceGuard guard(ctx->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((rc = enqueue_residual(ctx, layer, z, s, tokens, nullptr, nullptr, nullptr, fallback_tiles, gate_base, up_base,
                               st)))
        return rc;
    return enqueue_down(ctx, layer, tokens, y_f32, y_f16, st);
}

// Host-streamed forward; y goes to host fp16 `y_f16` or, for a shard of a d_ff-split
// stack, to the device fp32 partial `y32_dev`.
static int forward_host_impl(ffnrm_ctx *ctx, int layer, const int8_t *z, const float *s, int tokens,
                             const float *gate_base, const float *up_base, const uint8_t *fallback_tiles,
                             uint16_t *y_f16, float *y32_dev, void *stream) {
    int rc = check_ctx(ctx, layer);
    if (rc) return rc;
    if ((rc = check_tokens(ctx, tokens))) return rc;
    if (tokens == 0) return FFNRM_OK;  // empty batch
    if (!z || !s || !gate_base || !up_base || (!y_f16 && !y32_dev)) return fail(FFNRM_ERR_ARG, "null host pointer");
    if (!ctx->layers[size_t(layer)].down.ptr)
        return fail(FFNRM_ERR_STATE, "layer %d was loaded without a down projection", layer);
    DeviceGuard guard(ctx->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int F = ctx->cfg.d_ff, D = ctx->cfg.d_model, G = ctx->G;
    const int sl = ctx->slot;
    ctx->slot ^= 1;
    const size_t tf_bytes = size_t(tokens) * F * 4;
    cudaStream_t cs = ctx->copy_stream;
    // Inside a CUDA graph capture the copy stream may only wait on events recorded in the
    // same capture: the first use of each slot in a capture forks from `stream` here.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    unsigned long long cap_id = 0;
    FFNRM_CUDA(cudaStreamGetCaptureInfo(st, &cap, &cap_id));
    if (cap == cudaStreamCaptureStatusActive) {
        if (cap_id != ctx->capture_id) {
            ctx->capture_id = cap_id;
            ctx->slot_in_capture[0] = ctx->slot_in_capture[1] = false;
        }
        if (!ctx->slot_in_capture[sl]) {
            FFNRM_CUDA(cudaEventRecord(ctx->slot_free[sl], st));
            ctx->slot_in_capture[sl] = true;
        }
    } else if (ctx->capture_id != 0) {
        // The slot events were last recorded as nodes of a capture, which an eager wait
        // may not reference: record them again on `stream`.
        for (int i = 0; i < 2; ++i) FFNRM_CUDA(cudaEventRecord(ctx->slot_free[i], st));
        ctx->capture_id = 0;
        ctx->slot_in_capture[0] = ctx->slot_in_capture[1] = false;
    }
    // Every upload goes on the copy stream into slot `sl`, which the call before the
    // previous one has released; the next layer's upload thus overlaps this layer's kernels.
    FFNRM_CUDA(cudaStreamWaitEvent(cs, ctx->slot_free[sl], 0));
    FFNRM_CUDA(cudaMemcpyAsync(ctx->z_dev[sl], z, size_t(tokens) * D, cudaMemcpyHostToDevice, cs));
    FFNRM_CUDA(cudaMemcpyAsync(ctx->s_dev[sl], s, size_t(tokens) * G * 4, cudaMemcpyHostToDevice, cs));
    const uint8_t *tiles_dev = nullptr;
    if (fallback_tiles) {
        const int ntiles = (F + ctx->cfg.base_tile_rows - 1) / ctx->cfg.base_tile_rows;
        FFNRM_CUDA(cudaMemcpyAsync(ctx->tiles_dev[sl], fallback_tiles, size_t(ntiles), cudaMemcpyHostToDevice, cs));
        tiles_dev = ctx->tiles_dev[sl];
    }
    FFNRM_CUDA(cudaMemcpyAsync(ctx->base_dev[sl][0], gate_base, tf_bytes, cudaMemcpyHostToDevice, cs));
    FFNRM_CUDA(cudaMemcpyAsync(ctx->base_dev[sl][1], up_base, tf_bytes, cudaMemcpyHostToDevice, cs));
    FFNRM_CUDA(cudaEventRecord(ctx->base_ready[sl], cs));
    FFNRM_CUDA(cudaStreamWaitEvent(st, ctx->base_ready[sl], 0));
    if ((rc = enqueue_residual(ctx, layer, ctx->z_dev[sl], ctx->s_dev[sl], tokens, nullptr, nullptr, nullptr, tiles_dev,
                               ctx->base_dev[sl][0], ctx->base_dev[sl][1], st)))
        return rc;
    if (y32_dev) {
        if ((rc = enqueue_down(ctx, layer, tokens, y32_dev, nullptr, st))) return rc;
        FFNRM_CUDA(cudaEventRecord(ctx->slot_free[sl], st));
        return FFNRM_OK;
    }
    // A page-locked, device-mapped y (cudaHostAlloc, or cudaHostRegister with mapping) is
    // written by the down projection itself over PCIe; otherwise y goes through device
    // staging and one copy back.
    uint16_t *y_mapped = nullptr;
    {
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, y_f16) == cudaSuccess && a.type == cudaMemoryTypeHost && a.devicePointer &&
            aligned(a.devicePointer, 8))
            y_mapped = static_cast<uint16_t *>(a.devicePointer);
        cudaGetLastError();
    }
    if ((rc = enqueue_down(ctx, layer, tokens, nullptr, y_mapped ? y_mapped : ctx->y16_dev, st))) return rc;
    FFNRM_CUDA(cudaEventRecord(ctx->slot_free[sl], st));
    if (!y_mapped) FFNRM_CUDA(cudaMemcpyAsync(y_f16, ctx->y16_dev, size_t(tokens) * D * 2, cudaMemcpyDeviceToHost, st));
    return FFNRM_OK;
}

int ffnrm_ffn_forward_host(ffnrm_ctx *ctx, int layer, const int8_t *z, const float *s, int tokens,
                           const float *gate_base, const float *up_base, const uint8_t *fallback_tiles,
                           uint16_t *y_f16, void *stream) {
    if (!y_f16) return fail(FFNRM_ERR_ARG, "null host pointer");
    return forward_host_impl(ctx, layer, z, s, tokens, gate_base, up_base, fallback_tiles, y_f16, nullptr, stream);
}

int ffnrm_ffn_forward_host_partial(ffnrm_ctx *ctx, int layer, const int8_t *z, const float *s, int tokens,
                                   const float *gate_base, const float *up_base, const uint8_t *fallback_tiles,
                                   float *y_f32, void *stream) {
    if (!y_f32) return fail(FFNRM_ERR_ARG, "null device pointer");
    return forward_host_impl(ctx, layer, z, s, tokens, gate_base, up_base, fallback_tiles, nullptr, y_f32, stream);
}

int ffnrm_host_register(void *ptr, size_t bytes) {
    if (!ptr || !bytes) return fail(FFNRM_ERR_ARG, "null or empty range");
    FFNRM_CUDA(cudaHostRegister(ptr, bytes, cudaHostRegisterPortable));
    return FFNRM_OK;
}

int ffnrm_host_unregister(void *ptr) {
    FFNRM_CUDA(cudaHostUnregister(ptr));
    return FFNRM_OK;
}

int ffnrm_cast_f16(const float *src, uint16_t *dst, int64_t n, void *stream) {
    if (!src || !dst || n < 0) return fail(FFNRM_ERR_ARG, "bad cast arguments");
    if (n == 0) return FFNRM_OK;
    const int blocks = int(std::min<int64_t>((n + 255) / 256, 1024));
    ffnrm::cast_f16_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(src, reinterpret_cast<__half *>(dst), n);
    FFNRM_CUDA(cudaGetLastError());
    return FFNRM_OK;
}

// ---------------------------------------------------------------------------
// Peer reduction of the sharded stack's layer output (NVLink, CUDA IPC)
// ---------------------------------------------------------------------------
struct ffnrm_peer {
    int device = 0, world = 1, rank = 0;
    int64_t max_elems = 0;
    // Region (CUDA IPC shared): one-shot receive slots [2][world][one_max] f32, one-shot
    // flags [world][chunks] u32; then, when max_elems > one_max, the two-shot scatter and
    // gather slots [2][world][stride] f32 each and their flags [world][chunks] u32 each.
    void *region = nullptr;
    int64_t one_max = 0, stride = 0;  // largest one-shot message; two-shot slice stride
    size_t recv_bytes = 0, two_off = 0, region_bytes = 0;
    void *mapped[ffnrm::kPeerMaxRanks] = {};  // peers' regions opened here (own: region)
    uint32_t *counters = nullptr;              // epoch, done
    int *status = nullptr;
    float *partial = nullptr;                  // [max_elems] f32: the fused call's partial when it does not fuse
    bool connected = false;
};

int ffnrm_peer_create(ffnrm_peer **out, int device, int world, int rank, int64_t max_elems, void *ipc_handle) {
    if (!out || !ipc_handle) return fail(FFNRM_ERR_ARG, "null argument");
    *out = nullptr;
    if (world < 2 || world > ffnrm::kPeerMaxRanks || rank < 0 || rank >= world)
        return fail(FFNRM_ERR_ARG, "world=%d rank=%d: 2..%d ranks", world, rank, ffnrm::kPeerMaxRanks);
    if (max_elems <= 0 || max_elems % 4)
        return fail(FFNRM_ERR_ARG, "max_elems=%lld must be a positive multiple of 4", (long long)max_elems);
    DeviceGuard guard(device);
    auto *pr = new (std::nothrow) ffnrm_peer;
    if (!pr) return fail(FFNRM_ERR_NOMEM, "host allocation failed");
    pr->device = device;
    pr->world = world;
    pr->rank = rank;
    pr->max_elems = max_elems;
    // Messages above FFNRM_PEER_TWO_SHOT elements (default 2^20; 0 = never) take the
    // two-shot reduce-scatter + all-gather, which needs far less receive space.
    int64_t two_shot = int64_t(1) << 20;
    if (const char *e = std::getenv("FFNRM_PEER_TWO_SHOT")) two_shot = std::atoll(e);
    pr->one_max = two_shot > 0 ? std::min(max_elems, (two_shot + 3) / 4 * 4) : max_elems;
    pr->recv_bytes = size_t(2) * world * size_t(pr->one_max) * 4;
    const size_t flag_bytes = size_t(world) * ffnrm::kPeerMaxChunks * 4;
    pr->two_off = pr->recv_bytes + flag_bytes;
    pr->region_bytes = pr->two_off;
    if (max_elems > pr->one_max) {
        // scatter and gather slots, their flags, and the fused call's tile counters [2]
        pr->stride = ((max_elems + world - 1) / world + 3) / 4 * 4;
        pr->region_bytes += size_t(4) * world * size_t(pr->stride) * 4 + 2 * flag_bytes + 256;
    }
    cudaIpcMemHandle_t h;
    const bool ok = cudaMalloc(&pr->region, pr->region_bytes) == cudaSuccess &&
                    cudaMemset(pr->region, 0, pr->region_bytes) == cudaSuccess &&
                    cudaMalloc(&pr->counters, 2 * sizeof(uint32_t)) == cudaSuccess &&
                    cudaMemset(pr->counters, 0, 2 * sizeof(uint32_t)) == cudaSuccess &&
                    cudaMalloc(&pr->status, sizeof(int)) == cudaSuccess &&
                    cudaMemset(pr->status, 0, sizeof(int)) == cudaSuccess &&
                    cudaMalloc(&pr->partial, size_t(max_elems) * 4) == cudaSuccess &&
                    cudaIpcGetMemHandle(&h, pr->region) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
    if (!ok) {
        const cudaError_t e = cudaGetLastError();
        ffnrm_peer_destroy(pr);
        return fail(FFNRM_ERR_CUDA, "peer region set-up failed: %s", cudaGetErrorString(e));
    }
    std::memcpy(ipc_handle, &h, sizeof(h));
    pr->mapped[rank] = pr->region;
    *out = pr;
    return FFNRM_OK;
}

int ffnrm_peer_connect(ffnrm_peer *pr, const void *ipc_handles) {
    if (!pr || !ipc_handles) return fail(FFNRM_ERR_ARG, "null argument");
    if (pr->connected) return fail(FFNRM_ERR_STATE, "already connected");
    DeviceGuard guard(pr->device);
    for (int k = 0; k < pr->world; ++k) {
        if (k == pr->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t *>(ipc_handles) + size_t(k) * sizeof(h), sizeof(h));
        const cudaError_t e = cudaIpcOpenMemHandle(&pr->mapped[k], h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            cudaGetLastError();
            pr->mapped[k] = nullptr;
            return fail(FFNRM_ERR_CUDA, "cannot map rank %d's region: %s", k, cudaGetErrorString(e));
        }
    }
    pr->connected = true;
    return FFNRM_OK;
}

// The two-shot reduction of `elems` (> one_max) elements. tiles_expected > 0: fused mode —
// every rank's down projection has already stored its tiles into the scatter slots and counts
// them on the owner; the kernel waits for that count instead of scattering `partial`.
static int launch_two_shot(ffnrm_peer *pr, const float *partial, int64_t elems, uint16_t *y16, float *y32,
                           uint32_t tiles_expected, cudaStream_t stream) {
    ffnrm::PeerTwoShotParams q{};
    const size_t slot_bytes = size_t(2) * pr->world * size_t(pr->stride) * 4;
    const size_t flag_bytes = size_t(pr->world) * ffnrm::kPeerMaxChunks * 4;
    for (int k = 0; k < pr->world; ++k) {
        uint8_t *base = static_cast<uint8_t *>(pr->mapped[k]) + pr->two_off;
        q.scatter[k] = reinterpret_cast<float *>(base);
        q.gather[k] = reinterpret_cast<float *>(base + slot_bytes);
        q.sflags[k] = reinterpret_cast<uint32_t *>(base + 2 * slot_bytes);
        q.gflags[k] = reinterpret_cast<uint32_t *>(base + 2 * slot_bytes + flag_bytes);
    }
    if (tiles_expected) {
        q.tiles = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(pr->region) + pr->two_off + 2 * slot_bytes +
                                               2 * flag_bytes);
        q.tiles_expected = tiles_expected;
    }
    q.partial = partial;
    q.y16 = reinterpret_cast<__half *>(y16);
    q.y32 = y32;
    q.epoch = pr->counters;
    q.done = pr->counters + 1;
    q.status = pr->status;
    q.elems = elems;
    q.slice = ((elems + pr->world - 1) / pr->world + 3) / 4 * 4;
    q.stride = pr->stride;
    q.world = pr->world;
    q.rank = pr->rank;
    const int64_t per = (q.slice + ffnrm::kPeerMaxChunks - 1) / ffnrm::kPeerMaxChunks;
    q.chunk = int(std::max<int64_t>(2048, (per + 3) / 4 * 4));
    const int chunks = int((q.slice + q.chunk - 1) / q.chunk);
    FFNRM_CUDA(launch_dependent(ffnrm::peer_two_shot_kernel, dim3(unsigned(chunks)), dim3(ffnrm::kPeerThreads), 0,
                                stream, true, 1, q));
    return FFNRM_OK;
}

int ffnrm_peer_allreduce(ffnrm_peer *pr, const float *partial, int64_t elems, uint16_t *y16, float *y32,
                         void *stream) {
    if (!pr || !partial || (!y16 && !y32)) return fail(FFNRM_ERR_ARG, "null argument");
    if (!pr->connected) return fail(FFNRM_ERR_STATE, "peer reduction not connected");
    if (elems <= 0 || elems % 4 || elems > pr->max_elems)
        return fail(FFNRM_ERR_ARG, "elems=%lld: a positive multiple of 4 up to %lld", (long long)elems,
                    (long long)pr->max_elems);
    if (!aligned(partial, 16) || (y32 && !aligned(y32, 16)) || (y16 && !aligned(y16, 8)))
        return fail(FFNRM_ERR_ARG, "partial and y32 must be 16-byte aligned, y16 8-byte aligned");
    DeviceGuard guard(pr->device);
    if (elems > pr->one_max) return launch_two_shot(pr, partial, elems, y16, y32, 0, static_cast<cudaStream_t>(stream));
    ffnrm::PeerParams p{};
    for (int k = 0; k < pr->world; ++k) {
        p.recv[k] = static_cast<float *>(pr->mapped[k]);
        p.flags[k] = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(pr->mapped[k]) + pr->recv_bytes);
    }
    p.partial = partial;
    p.y16 = reinterpret_cast<__half *>(y16);
    p.y32 = y32;
    p.epoch = pr->counters;
    p.done = pr->counters + 1;
    p.status = pr->status;
    p.elems = elems;
    p.max_elems = pr->one_max;
    p.world = pr->world;
    p.rank = pr->rank;
    const int64_t per = (elems + ffnrm::kPeerMaxChunks - 1) / ffnrm::kPeerMaxChunks;
    p.chunk = int(std::max<int64_t>(2048, (per + 3) / 4 * 4));
    const int chunks = int((elems + p.chunk - 1) / p.chunk);
    // a dependent launch: its start overlaps the tail of the preceding kernel (the down
    // projection, which releases its dependents early)
    FFNRM_CUDA(launch_dependent(ffnrm::peer_allreduce_kernel, dim3(unsigned(chunks)), dim3(ffnrm::kPeerThreads), 0,
                                static_cast<cudaStream_t>(stream), true, 1, p));
    return FFNRM_OK;
}

int ffnrm_ffn_forward_reduced(ffnrm_ctx *ctx, ffnrm_peer *pr, int layer, const int8_t *z, const float *s, int tokens,
                              const float *gate_base, const float *up_base, const uint8_t *fallback_tiles,
                              uint16_t *y_f16, void *stream) {
    int rc = check_ctx(ctx, layer);
    if (rc) return rc;
    if ((rc = check_tokens(ctx, tokens))) return rc;
    if (!pr || !pr->connected) return fail(FFNRM_ERR_STATE, "peer reduction not connected");
    if (pr->device != ctx->device) return fail(FFNRM_ERR_ARG, "context and peer reduction on different devices");
    if (tokens == 0) return FFNRM_OK;  // empty batch
    if (!z || !s || !gate_base || !up_base || !y_f16) return fail(FFNRM_ERR_ARG, "null device pointer");
    if (!ctx->layers[size_t(layer)].down.ptr)
        return fail(FFNRM_ERR_STATE, "layer %d was loaded without a down projection", layer);
    const int D = ctx->cfg.d_model, W = pr->world;
    const int64_t elems = int64_t(tokens) * D;
    if (elems > pr->max_elems)
        return fail(FFNRM_ERR_ARG, "tokens x d_model = %lld exceeds the reduction's %lld", (long long)elems,
                    (long long)pr->max_elems);
    if (!aligned(z, 16) || !aligned(s, 4) || !aligned(gate_base, 4) || !aligned(up_base, 4) || !aligned(y_f16, 8))
        return fail(FFNRM_ERR_ARG, "z must be 16-byte aligned, y_f16 8-byte, s and base sums 4-byte");
    DeviceGuard guard(ctx->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((rc = enqueue_residual(ctx, layer, z, s, tokens, nullptr, nullptr, nullptr, fallback_tiles, gate_base, up_base,
                               st)))
        return rc;
    const int64_t slice = ((elems + W - 1) / W + 3) / 4 * 4;
    if (elems <= pr->one_max || slice < 2 * int64_t(D)) {
        // small messages (and slices under two token rows): the down projection writes a
        // partial, which the reduction then takes as usual
        if ((rc = enqueue_down(ctx, layer, tokens, pr->partial, nullptr, st))) return rc;
        return ffnrm_peer_allreduce(pr, pr->partial, elems, y_f16, nullptr, stream);
    }
    // Fused: the down projection stores its output tiles into the owners' scatter slots; the
    // owner of slice r expects one count per (rank, tile) whose rows reach slice r.
    ffnrm::DownScatter sc{};
    const size_t slot_bytes = size_t(2) * W * size_t(pr->stride) * 4;
    const size_t flag_bytes = size_t(W) * ffnrm::kPeerMaxChunks * 4;
    for (int k = 0; k < W; ++k) {
        uint8_t *base = static_cast<uint8_t *>(pr->mapped[k]) + pr->two_off;
        sc.scatter[k] = reinterpret_cast<float *>(base);
        sc.counter[k] = reinterpret_cast<uint32_t *>(base + 2 * slot_bytes + 2 * flag_bytes);
    }
    sc.epoch = pr->counters;
    sc.slice = slice;
    sc.stride = pr->stride;
    sc.world = W;
    sc.rank = pr->rank;
    const int N = down_token_tile(ctx, tokens);
    uint32_t expected = 0;
    for (int t0 = 0; t0 < tokens; t0 += N)
        for (int m0 = 0; m0 < D; m0 += ffnrm::kUmmaM) {
            const int ntok = std::min(N, tokens - t0);
            const int64_t d0 = (int64_t(t0) * D + m0) / slice;
            const int64_t d1 = (int64_t(t0 + ntok - 1) * D + m0 + ffnrm::kUmmaM - 1) / slice;
            if (d0 <= pr->rank && pr->rank <= d1) expected += uint32_t(W);
        }
    if ((rc = enqueue_down(ctx, layer, tokens, nullptr, nullptr, st, &sc))) return rc;
    return launch_two_shot(pr, nullptr, elems, y_f16, nullptr, expected, st);
}

int ffnrm_peer_check(ffnrm_peer *pr, void *stream) {
    if (!pr) return fail(FFNRM_ERR_ARG, "null argument");
    DeviceGuard guard(pr->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int code = 0;
    FFNRM_CUDA(cudaMemcpyAsync(&code, pr->status, sizeof(int), cudaMemcpyDeviceToHost, st));
    FFNRM_CUDA(cudaStreamSynchronize(st));
    if (code) {
        FFNRM_CUDA(cudaMemsetAsync(pr->status, 0, sizeof(int), st));
        FFNRM_CUDA(cudaStreamSynchronize(st));
        return fail(FFNRM_ERR_TIMEOUT, "the peer reduction gave up waiting for another rank");
    }
    return FFNRM_OK;
}

int ffnrm_peer_destroy(ffnrm_peer *pr) {
    if (!pr) return FFNRM_OK;
    DeviceGuard guard(pr->device);
    cudaDeviceSynchronize();
    for (int k = 0; k < pr->world; ++k)
        if (k != pr->rank && pr->mapped[k]) cudaIpcCloseMemHandle(pr->mapped[k]);
    cudaFree(pr->region);
    cudaFree(pr->counters);
    cudaFree(pr->status);
    cudaGetLastError();
    delete pr;
    return FFNRM_OK;
}

int ffnrm_layer_bytes(ffnrm_ctx *ctx, int layer, int64_t *residual_bytes, int64_t *down_bytes) {
    int rc = check_ctx(ctx, layer);
    if (rc) return rc;
    const LayerDev &L = ctx->layers[size_t(layer)];
    int64_t res = 0;
    res += int64_t(L.alpha.bytes);
    const int r = ctx->cfg.residual_bits;
    if (r != 1) res += int64_t(L.pair.bytes);
    if (r != 2) res += int64_t(L.plane.bytes);
    if (residual_bytes) *residual_bytes = res;
    if (down_bytes) *down_bytes = int64_t(L.down.bytes);
    return FFNRM_OK;
}

int64_t ffnrm_launch_count(ffnrm_ctx *ctx) { return ctx ? ctx->launches : -1; }

int ffnrm_down_project_noalloc(const uint16_t *down, int64_t down_ld, const uint16_t *h_hi, const uint16_t *h_lo,
                               int64_t h_ld, int d_model, int d_ff, int tokens, float *y_f32, uint16_t *y_f16,
                               int32_t *status, void *stream) {
    if (tokens < 0 || tokens > kNoAllocMaxTokens)
        return fail(FFNRM_ERR_ARG, "tokens=%d outside [0, %d], the largest token-tile grid this call launches", tokens,
                    kNoAllocMaxTokens);
    if (d_model <= 0 || d_model % 128 || d_model > kNoAllocMaxDModel)
        return fail(FFNRM_ERR_ARG, "d_model=%d must be a positive multiple of 128 up to %d", d_model,
                    kNoAllocMaxDModel);
    if (d_ff <= 0) return fail(FFNRM_ERR_ARG, "d_ff=%d must be positive", d_ff);
    if (!down || !h_hi || !h_lo || (!y_f32 && !y_f16)) return fail(FFNRM_ERR_ARG, "null device pointer");
    if (down_ld < d_ff || h_ld < d_ff || down_ld % 8 || h_ld % 8)
        return fail(FFNRM_ERR_ARG, "down_ld and h_ld must be >= d_ff and multiples of 8");
    if (!aligned(down, 16) || !aligned(h_hi, 16) || !aligned(h_lo, 16) || !aligned(y_f32, 16) || !aligned(y_f16, 8) ||
        !aligned(status, 4))
        return fail(FFNRM_ERR_ARG, "down, h_hi, h_lo and y_f32 must be 16-byte aligned, y_f16 8-byte");
    if (tokens == 0) return FFNRM_OK;
    int dev = 0;
    FFNRM_CUDA(cudaGetDevice(&dev));
    if (dev >= kNoAllocMaxDevices) return fail(FFNRM_ERR_ARG, "device %d beyond the supported %d", dev, kNoAllocMaxDevices);
    NoAllocScratch scr;
    int rc = noalloc_scratch(dev, scr);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (tokens <= 16) return launch_down_noalloc<16>(down, down_ld, h_hi, h_lo, h_ld, d_model, d_ff, tokens, y_f32, y_f16, status, scr, st);
    if (tokens <= 32) return launch_down_noalloc<32>(down, down_ld, h_hi, h_lo, h_ld, d_model, d_ff, tokens, y_f32, y_f16, status, scr, st);
    if (tokens <= 64) return launch_down_noalloc<64>(down, down_ld, h_hi, h_lo, h_ld, d_model, d_ff, tokens, y_f32, y_f16, status, scr, st);
    return launch_down_noalloc<128>(down, down_ld, h_hi, h_lo, h_ld, d_model, d_ff, tokens, y_f32, y_f16, status, scr, st);
}

int ffnrm_noalloc_status(int32_t *out, void *stream) {
    if (!out) return fail(FFNRM_ERR_ARG, "null argument");
    int dev = 0;
    FFNRM_CUDA(cudaGetDevice(&dev));
    if (dev >= kNoAllocMaxDevices) return fail(FFNRM_ERR_ARG, "device %d beyond the supported %d", dev, kNoAllocMaxDevices);
    NoAllocScratch scr;
    int rc = noalloc_scratch(dev, scr);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    FFNRM_CUDA(cudaMemcpyAsync(out, scr.status, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    FFNRM_CUDA(cudaMemsetAsync(scr.status, 0, sizeof(int32_t), st));
    FFNRM_CUDA(cudaStreamSynchronize(st));
    return FFNRM_OK;
}

int ffnrm_check_device_error(ffnrm_ctx *ctx, void *stream) {
    if (!ctx) return fail(FFNRM_ERR_ARG, "null context");
    DeviceGuard guard(ctx->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int code = 0;
    FFNRM_CUDA(cudaMemcpyAsync(&code, ctx->err, sizeof(int), cudaMemcpyDeviceToHost, st));
    FFNRM_CUDA(cudaStreamSynchronize(st));
    if (code) {
        FFNRM_CUDA(cudaMemsetAsync(ctx->err, 0, sizeof(int), st));
        FFNRM_CUDA(cudaStreamSynchronize(st));
        return fail(FFNRM_ERR_TIMEOUT, "a kernel gave up waiting on a pipeline barrier (code %d)", code);
    }
    return FFNRM_OK;
}

int ffnrm_profile_enable(ffnrm_ctx *ctx, int enable) {
    if (!ctx) return fail(FFNRM_ERR_ARG, "null context");
    DeviceGuard guard(ctx->device);
    if (ctx->prof_used) FFNRM_CUDA(cudaDeviceSynchronize());
    ctx->prof = enable != 0;
    ctx->prof_used = 0;
    ctx->prof_kind.clear();
    return FFNRM_OK;
}

// Sums the device time of the recorded launch pairs of `kind`. The records stay, so a
// CUDA graph captured with profiling on can be replayed and read again after each replay.
int ffnrm_profile_read(ffnrm_ctx *ctx, int kind, double *total_ms, int64_t *launches) {
    if (!ctx || kind < 0 || kind > 2) return fail(FFNRM_ERR_ARG, "bad profile arguments");
    DeviceGuard guard(ctx->device);
    double ms_sum = 0;
    int64_t n = 0;
    for (size_t i = 0; i < ctx->prof_kind.size(); ++i) {
        if (ctx->prof_kind[i] != kind) continue;
        cudaEvent_t a = ctx->prof_pool[2 * i], b = ctx->prof_pool[2 * i + 1];
        FFNRM_CUDA(cudaEventSynchronize(b));
        float ms = 0.f;
        FFNRM_CUDA(cudaEventElapsedTime(&ms, a, b));
        ms_sum += ms;
        ++n;
    }
    if (total_ms) *total_ms = ms_sum;
    if (launches) *launches = n;
    return FFNRM_OK;
}

}  // extern "C"
