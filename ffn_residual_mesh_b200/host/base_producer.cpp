// C ABI of the host base producer (declared in include/ffnrm.h): exact base sums of the
// split from the reference's radix table artifact, on the host's cores, tile by tile,
// with optional per-tile readiness flags and a deadline after which unfinished tiles are
// handed to the GPU's exact fallback path instead (the deadline rule of
// src/phone_ffn_loopback.py:155-197). No GPU is involved.
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <exception>
#include <new>
#include <string>

#include "ffnrm.h"
#include "radix_base.hpp"

// The library's last-error slot (ffnrm.cu).
int ffnrm_set_error(int code, const char *msg);

struct ffnrm_base_producer {
    ffnrm_host::TilePool pool;
    explicit ffnrm_base_producer(int threads) : pool(threads) {}
};

namespace {

int check_table(const ffnrm_radix_table *t, ffnrm_host::TableView &v) {
    if (!t || !t->table || !t->high_sum || !t->alpha || !t->beta) return ffnrm_set_error(FFNRM_ERR_ARG, "null table array");
    if (t->rows <= 0 || t->hidden <= 0 || t->hidden % 32)
        return ffnrm_set_error(FFNRM_ERR_ARG, "table rows must be positive and hidden a positive multiple of 32");
    if (t->block_size != 2 && t->block_size != 4 && t->block_size != 8)
        return ffnrm_set_error(FFNRM_ERR_ARG, "block_size must be 2, 4 or 8");
    v.rows = t->rows;
    v.hidden = t->hidden;
    v.groups = t->hidden / 32;
    v.block_size = t->block_size;
    v.blocks = t->hidden / t->block_size;
    v.state_count = 1 << (2 * t->block_size);
    v.table = t->table;
    v.high_sum = t->high_sum;
    v.alpha = t->alpha;
    v.beta = t->beta;
    return FFNRM_OK;
}

}  // namespace

extern "C" {

int ffnrm_base_producer_create(ffnrm_base_producer **out, int threads) {
    if (!out) return ffnrm_set_error(FFNRM_ERR_ARG, "null argument");
    if (threads <= 0) return ffnrm_set_error(FFNRM_ERR_ARG, "threads must be positive");
    try {
        *out = new ffnrm_base_producer(threads);
    } catch (const std::exception &e) {
        return ffnrm_set_error(FFNRM_ERR_NOMEM, e.what());
    }
    return FFNRM_OK;
}

int ffnrm_base_producer_destroy(ffnrm_base_producer *p) {
    delete p;
    return FFNRM_OK;
}

int ffnrm_table_dots(const ffnrm_radix_table *tbl, const int8_t *z, int32_t *dots) {
    ffnrm_host::TableView v{};
    int rc = check_table(tbl, v);
    if (rc) return rc;
    if (!z || !dots) return ffnrm_set_error(FFNRM_ERR_ARG, "null argument");
    std::vector<uint16_t> st(size_t(4) * v.blocks);
    ffnrm_host::encode_states(z, v.hidden, v.block_size, st.data());
    const int tile = 256;
    std::vector<int16_t> acc(size_t(v.groups) * tile);
    for (int r0 = 0; r0 < v.rows; r0 += tile) {
        const int n = std::min(tile, v.rows - r0);
        ffnrm_host::table_dots_tile(v, st.data(), r0, n, acc.data());
        for (int i = 0; i < n; ++i)
            for (int g = 0; g < v.groups; ++g) dots[size_t(r0 + i) * v.groups + g] = acc[size_t(g) * n + i];
    }
    return FFNRM_OK;
}

int ffnrm_base_from_table(ffnrm_base_producer *p, const ffnrm_radix_table *tbl, const int8_t *z, const float *s,
                          int tokens, int multiplier, float *base, int tile_rows, uint32_t *tile_ready,
                          int64_t deadline_ns, uint8_t *late_tiles) {
    if (!p) return ffnrm_set_error(FFNRM_ERR_ARG, "null producer");
    ffnrm_host::TableView v{};
    int rc = check_table(tbl, v);
    if (rc) return rc;
    if (tokens < 0) return ffnrm_set_error(FFNRM_ERR_ARG, "tokens must be >= 0");
    if (tokens == 0) return FFNRM_OK;
    if (!z || !s || !base) return ffnrm_set_error(FFNRM_ERR_ARG, "null argument");
    if (tile_rows <= 0) return ffnrm_set_error(FFNRM_ERR_ARG, "tile_rows must be positive");
    if (deadline_ns > 0 && !late_tiles) return ffnrm_set_error(FFNRM_ERR_ARG, "a deadline needs late_tiles");
    const int ntile = (v.rows + tile_rows - 1) / tile_rows;
    if (late_tiles) std::memset(late_tiles, 0, size_t(ntile));
    const auto t0 = std::chrono::steady_clock::now();
    // A tile that finishes after the deadline is reported late (flagged for the exact
    // GPU fallback); its base values are still written, and its readiness flag raised.
    std::function<void(int, int)> on_tile = [&](int tok, int tile) {
        if (deadline_ns > 0) {
            const int64_t el =
                std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
            if (el > deadline_ns) reinterpret_cast<std::atomic<uint8_t> *>(late_tiles)[tile].store(1, std::memory_order_relaxed);
        }
        if (tile_ready)
            reinterpret_cast<std::atomic<uint32_t> *>(tile_ready)[size_t(tok) * ntile + tile].store(
                1u, std::memory_order_release);
    };
    try {
        ffnrm_host::table_base(p->pool, v, z, s, tokens, multiplier, base, tile_rows,
                               (tile_ready || deadline_ns > 0) ? &on_tile : nullptr);
    } catch (const std::exception &e) {
        return ffnrm_set_error(FFNRM_ERR_NOMEM, e.what());
    }
    return FFNRM_OK;
}

}  // extern "C"
