// Host base producer: the exact "base" partial sums of the split, computed on the CPU
// from the reference's radix table artifact while the GPU runs the residual.
//
// For one token with activation codes z and per-group scales s, row f of a projection
// gets
//     base[f] = sum_g s[g] * (alpha[f,g] * (2^r * P_hi[f,g]) + beta[f,g] * zsum[g])
// with the exact integer dot P_hi[f,g] = sum_i q_hi[f,g,i] * z[g,i], which the table
// yields without multiplications: writing u = z + 128 in base 4 (digit d of block b
// selects state_d(b)), P_hi = sum_d 4^d sum_b table[b, state_d(b), f] - 128 * high_sum[f,g]
// (scripts/benchmark_exact_radix_split_pipeline.py:50-109; the runners' cpu_eval,
// src/exact_main_residual_cuda_runner.cu:144-187; the fused AVX2 evaluator,
// src/radix_cpu_kernels.h:143-217). The fp32 sum runs over groups in order, as there.
//
// Design: rows are cut into tiles (256 rows by default); a pool of threads claims tiles
// from an atomic counter, so fast threads take more tiles and the caller's thread works
// too. A tile accumulates its dots in int16 ([groups][tile rows], exact: every partial
// sum is at most 85 * 3 * 32 = 8160 in magnitude) with 16-lane AVX2 adds of the widened
// table bytes, then applies the scales. A per-tile callback reports each finished tile,
// so a consumer can stream tiles to the GPU as they complete.
#pragma once

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#if defined(__AVX2__)
#include <immintrin.h>
#endif

namespace ffnrm_host {

// A fixed set of worker threads that execute `fn(task)` for task in [0, n) per run(),
// claiming tasks dynamically. run() returns when every task has finished.
class TilePool {
public:
    explicit TilePool(int threads) : nthreads_(std::max(1, threads)) {
        for (int i = 1; i < nthreads_; ++i) workers_.emplace_back([this] { loop(); });
    }
    ~TilePool() {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
            ++epoch_;
        }
        cv_.notify_all();
        for (auto &t : workers_) t.join();
    }
    TilePool(const TilePool &) = delete;
    TilePool &operator=(const TilePool &) = delete;
    int threads() const { return nthreads_; }

    void run(int n, const std::function<void(int)> &fn) {
        if (n <= 0) return;
        if (nthreads_ == 1) {
            for (int i = 0; i < n; ++i) fn(i);
            return;
        }
        {
            std::lock_guard<std::mutex> lk(mu_);
            fn_ = &fn;
            ntasks_ = n;
            next_.store(0);
            active_ = nthreads_ - 1;
            ++epoch_;
        }
        cv_.notify_all();
        work();
        std::unique_lock<std::mutex> lk(mu_);
        done_cv_.wait(lk, [this] { return active_ == 0; });
        fn_ = nullptr;
    }

private:
    void work() {
        for (;;) {
            const int t = next_.fetch_add(1);
            if (t >= ntasks_) return;
            (*fn_)(t);
        }
    }
    void loop() {
        uint64_t seen = 0;
        for (;;) {
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return epoch_ != seen; });
                seen = epoch_;
                if (stop_) return;
            }
            work();
            std::lock_guard<std::mutex> lk(mu_);
            if (--active_ == 0) done_cv_.notify_all();
        }
    }
    int nthreads_;
    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_, done_cv_;
    uint64_t epoch_ = 0;
    bool stop_ = false;
    const std::function<void(int)> *fn_ = nullptr;
    int ntasks_ = 0;
    int active_ = 0;
    std::atomic<int> next_{0};
};

// Base-4 digit streams of u = z + 128: states[d * blocks + b] =
// sum_j digit_d(u[b*bs + j]) * 4^j (scripts/benchmark_exact_radix_split_pipeline.py:67-79).
inline void encode_states(const int8_t *z, int hidden, int block_size, uint16_t *states) {
    const int blocks = hidden / block_size;
    for (int d = 0; d < 4; ++d)
        for (int b = 0; b < blocks; ++b) {
            uint32_t st = 0;
            for (int j = 0; j < block_size; ++j) {
                const uint32_t u = uint32_t(int(z[b * block_size + j]) + 128);
                st |= ((u >> (2 * d)) & 3u) << (2 * j);
            }
            states[size_t(d) * blocks + b] = uint16_t(st);
        }
}

struct TableView {
    int rows, hidden, groups, block_size, blocks, state_count;
    const uint8_t *table;     // [blocks, state_count, rows]
    const int16_t *high_sum;  // [rows, groups]
    const float *alpha, *beta;
};

// dst[r] += (int16)src[r] << shift for r < n.
inline void add_shifted(int16_t *dst, const uint8_t *src, int n, int shift) {
    int r = 0;
#if defined(__AVX2__)
    const __m128i sh = _mm_cvtsi32_si128(shift);
    for (; r + 16 <= n; r += 16) {
        const __m256i v = _mm256_cvtepu8_epi16(_mm_loadu_si128(reinterpret_cast<const __m128i *>(src + r)));
        __m256i a = _mm256_loadu_si256(reinterpret_cast<const __m256i *>(dst + r));
        a = _mm256_add_epi16(a, _mm256_sll_epi16(v, sh));
        _mm256_storeu_si256(reinterpret_cast<__m256i *>(dst + r), a);
    }
#endif
    for (; r < n; ++r) dst[r] = int16_t(dst[r] + (int16_t(src[r]) << shift));
}

// Exact P_hi for rows [r0, r0 + n) of one token into acc [groups][n] (int16).
inline void table_dots_tile(const TableView &T, const uint16_t *states, int r0, int n, int16_t *acc) {
    std::fill(acc, acc + size_t(T.groups) * n, int16_t(0));
    const int bpg = 32 / T.block_size;
    for (int d = 0; d < 4; ++d)
        for (int b = 0; b < T.blocks; ++b) {
            const uint8_t *e = T.table + (size_t(b) * T.state_count + states[size_t(d) * T.blocks + b]) * T.rows + r0;
            add_shifted(acc + size_t(b / bpg) * n, e, n, 2 * d);
        }
    for (int g = 0; g < T.groups; ++g) {
        int16_t *a = acc + size_t(g) * n;
        for (int i = 0; i < n; ++i) a[i] = int16_t(a[i] - 128 * T.high_sum[size_t(r0 + i) * T.groups + g]);
    }
}

// base[r] for rows [r0, r0 + n) from their exact dots (fp32, groups in order).
inline void base_from_dots(const TableView &T, const int16_t *acc, int r0, int n, const float *s, const int32_t *zsum,
                           int mult, float *out) {
    for (int i = 0; i < n; ++i) {
        const size_t row = size_t(r0 + i);
        const float *al = T.alpha + row * T.groups, *be = T.beta + row * T.groups;
        float v = 0.0f;
        for (int g = 0; g < T.groups; ++g)
            v += s[g] * (al[g] * float(mult * int(acc[size_t(g) * n + i])) + be[g] * float(zsum[g]));
        out[i] = v;
    }
}

// Base sums of one projection for `tokens` tokens: z [tokens, hidden], s [tokens, groups],
// out [tokens, rows]. `on_tile(token, tile)` (optional) is called from the worker thread
// as each row tile of a token completes.
inline void table_base(TilePool &pool, const TableView &T, const int8_t *z, const float *s, int tokens, int mult,
                       float *out, int tile_rows = 256, const std::function<void(int, int)> *on_tile = nullptr) {
    const int ntile = (T.rows + tile_rows - 1) / tile_rows;
    std::vector<uint16_t> states(size_t(tokens) * 4 * T.blocks);
    std::vector<int32_t> zsum(size_t(tokens) * T.groups, 0);
    for (int t = 0; t < tokens; ++t) {
        encode_states(z + size_t(t) * T.hidden, T.hidden, T.block_size, states.data() + size_t(t) * 4 * T.blocks);
        for (int g = 0; g < T.groups; ++g)
            for (int i = 0; i < 32; ++i) zsum[size_t(t) * T.groups + g] += z[size_t(t) * T.hidden + g * 32 + i];
    }
    pool.run(tokens * ntile, [&](int task) {
        const int t = task / ntile, tile = task % ntile;
        const int r0 = tile * tile_rows, n = std::min(tile_rows, T.rows - r0);
        thread_local std::vector<int16_t> acc;
        acc.resize(size_t(T.groups) * tile_rows);
        table_dots_tile(T, states.data() + size_t(t) * 4 * T.blocks, r0, n, acc.data());
        base_from_dots(T, acc.data(), r0, n, s + size_t(t) * T.groups, zsum.data() + size_t(t) * T.groups, mult,
                       out + size_t(t) * T.rows + r0);
        if (on_tile) (*on_tile)(t, tile);
    });
}

}  // namespace ffnrm_host
