// CPU reference driver (TEST INFRASTRUCTURE / CPU BASELINE ONLY).
//
// Exposes the reference's own AVX2 CPU evaluator (src/radix_cpu_kernels.h,
// compiled from the reference source where it lies, see oracle/Makefile) through a
// small C ABI so tests can pin the numpy oracle against it and bench.py can time it
// as the CPU baseline. Only tests/, __graft_entry__.smoke() and bench.py's CPU leg
// load this library.
//
// What is the reference's code and what is not:
//   * gate/up projections: residual_mesh::direct_q4 (radix_cpu_kernels.h:228-248),
//     the reference's unsplit packed-Q4 AVX2 kernel, run on its CpuPool
//     (radix_cpu_kernels.h:16-65) with its row_range partition (:250-254);
//   * the radix-table base: residual_mesh::fused_base (radix_cpu_kernels.h:143-217);
//   * SwiGLU + fp16 down: the reference has only numpy for this step
//     (scripts/benchmark_cpu_base_gpu_full_ffn.py:369-370); the loop below is a
//     port of that formula, blocked so each fp16 row of the down weight is read
//     once for all tokens.
#include "radix_cpu_kernels.h"

#include <immintrin.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <vector>

using namespace residual_mesh;

namespace {

// Cold-start repack used by the reference bench (radix_cpu_bench.cpp:65-67):
// per 32-code group, byte i holds code i in the low nibble and code i+16 high.
void repack_q4(const std::uint8_t *q, std::size_t count, std::uint8_t *packed) {
    for (std::size_t g = 0; g < count / 32; ++g)
        for (int i = 0; i < 16; ++i)
            packed[g * 16 + i] = static_cast<std::uint8_t>(q[g * 32 + i] | (q[g * 32 + i + 16] << 4));
}

struct Projection {
    Shape shape{0, 0, 4};
    std::vector<std::uint8_t> packed;
    std::vector<float> alpha, beta;
};

struct RefFfn {
    int rows = 0, hidden = 0, threads = 1;
    Projection gate, up;
    std::vector<std::uint16_t> down;  // [hidden, rows] fp16 bits
    std::unique_ptr<CpuPool> pool;
    Activation act;
    std::vector<float> g, u, h;
};

void project(RefFfn &m, const Projection &p, const std::int8_t *z, const float *s, float *out,
             int *dots) {
    m.act.prepare(p.shape, z, false);
    m.pool->run([&](int id) {
        int begin, end;
        row_range(p.shape, id, m.threads, begin, end);
        direct_q4(p.shape, p.packed.data(), p.alpha.data(), p.beta.data(), z, s, m.act, out, begin, end,
                  dots);
    });
}

}  // namespace

extern "C" {

// Create a CPU FFN over Q4 codes [rows, hidden] (one byte per code, values 0..15),
// alpha/beta [rows, hidden/32] f32 and down fp16 [hidden, rows].
void *ref_ffn_create(int rows, int hidden, int threads, const std::uint8_t *gate_q, const std::uint8_t *up_q,
                     const float *gate_alpha, const float *up_alpha, const float *gate_beta,
                     const float *up_beta, const std::uint16_t *down) {
    auto *m = new RefFfn;
    m->rows = rows;
    m->hidden = hidden;
    m->threads = threads;
    const std::size_t n = std::size_t(rows) * hidden, ng = n / 32;
    for (auto *p : {&m->gate, &m->up}) {
        p->shape = Shape{rows, hidden, 4};
        p->packed.resize(n / 2);
    }
    repack_q4(gate_q, n, m->gate.packed.data());
    repack_q4(up_q, n, m->up.packed.data());
    m->gate.alpha.assign(gate_alpha, gate_alpha + ng);
    m->gate.beta.assign(gate_beta, gate_beta + ng);
    m->up.alpha.assign(up_alpha, up_alpha + ng);
    m->up.beta.assign(up_beta, up_beta + ng);
    if (down) m->down.assign(down, down + n);
    m->pool = std::make_unique<CpuPool>(threads);
    m->act.resize(m->gate.shape);
    m->g.resize(rows);
    m->u.resize(rows);
    return m;
}

void ref_ffn_destroy(void *handle) { delete static_cast<RefFfn *>(handle); }

// Unsplit gate/up projections for T tokens (reference direct_q4, one token at a
// time as the reference evaluates it). gate_out/up_out: [T, rows]; dots (optional):
// [2, T, rows, groups] exact int32 group dots from the reference's verified_dots.
void ref_ffn_gate_up(void *handle, const std::int8_t *z, const float *s, int tokens, float *gate_out,
                     float *up_out, int *dots) {
    auto &m = *static_cast<RefFfn *>(handle);
    const std::size_t stride = std::size_t(m.rows) * (m.hidden / 32);
    for (int t = 0; t < tokens; ++t) {
        const auto *zt = z + std::size_t(t) * m.hidden;
        const auto *st = s + std::size_t(t) * (m.hidden / 32);
        project(m, m.gate, zt, st, gate_out + std::size_t(t) * m.rows, dots ? dots + t * stride : nullptr);
        project(m, m.up, zt, st, up_out + std::size_t(t) * m.rows,
                dots ? dots + (std::size_t(tokens) + t) * stride : nullptr);
    }
}

// Full CPU FFN for T tokens: direct_q4 gate/up, SwiGLU, fp16 down with fp32
// accumulation. y: [T, hidden] f32.
void ref_ffn_forward(void *handle, const std::int8_t *z, const float *s, int tokens, float *y) {
    auto &m = *static_cast<RefFfn *>(handle);
    m.h.resize(std::size_t(tokens) * m.rows);
    std::vector<float> gate(std::size_t(tokens) * m.rows), up(gate.size());
    ref_ffn_gate_up(handle, z, s, tokens, gate.data(), up.data(), nullptr);
    for (std::size_t i = 0; i < gate.size(); ++i)
        m.h[i] = gate[i] / (1.0f + std::exp(-gate[i])) * up[i];
    const int rows = m.rows, hidden = m.hidden, threads = m.threads;
    m.pool->run([&](int id) {
        const int begin = int(std::int64_t(hidden) * id / threads);
        const int end = int(std::int64_t(hidden) * (id + 1) / threads);
        std::vector<float> w(rows);
        for (int o = begin; o < end; ++o) {
            const std::uint16_t *row = m.down.data() + std::size_t(o) * rows;
            int f = 0;
            for (; f + 8 <= rows; f += 8)
                _mm256_storeu_ps(w.data() + f,
                                 _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i *>(row + f))));
            for (; f < rows; ++f) w[f] = _cvtsh_ss(row[f]);
            for (int t = 0; t < tokens; ++t) {
                const float *ht = m.h.data() + std::size_t(t) * rows;
                __m256 acc = _mm256_setzero_ps();
                int k = 0;
                for (; k + 8 <= rows; k += 8)
                    acc = _mm256_add_ps(acc, _mm256_mul_ps(_mm256_loadu_ps(w.data() + k), _mm256_loadu_ps(ht + k)));
                alignas(32) float lanes[8];
                _mm256_store_ps(lanes, acc);
                float sum = 0;
                for (float v : lanes) sum += v;
                for (; k < rows; ++k) sum += w[k] * ht[k];
                y[std::size_t(t) * hidden + o] = sum;
            }
        }
    });
}

// Radix-table base (reference fused_base, r = 2 only) for one token.
// table [hidden/block, 4**block, rows] u8; high_sum/alpha/beta [rows, groups].
// out [rows] f32; dots (optional) [rows, groups] exact int32 P_hi.
int ref_fused_base(int rows, int hidden, int block, int threads, int prefetch, const std::uint8_t *table,
                   const std::int16_t *high_sum, const float *alpha, const float *beta, const std::int8_t *z,
                   const float *s, float *out, int *dots) {
    try {
        Shape shape{rows, hidden, block};
        shape.validate();
        const int groups = shape.groups();
        std::vector<std::int16_t> hs(std::size_t(rows) * groups);
        std::vector<float> a(hs.size()), b(hs.size());
        for (int r = 0; r < rows; ++r)
            for (int g = 0; g < groups; ++g) {
                hs[std::size_t(g) * rows + r] = high_sum[std::size_t(r) * groups + g];
                a[std::size_t(g) * rows + r] = alpha[std::size_t(r) * groups + g];
                b[std::size_t(g) * rows + r] = beta[std::size_t(r) * groups + g];
            }
        BaseView view{table, hs.data(), a.data(), b.data()};
        Activation act;
        act.resize(shape);
        act.prepare(shape, z, true);
        CpuPool pool(threads);
        pool.run([&](int id) {
            int begin, end;
            row_range(shape, id, threads, begin, end);
            fused_base(shape, view, act, s, out, begin, end, prefetch, dots);
        });
        return 0;
    } catch (...) {
        return 1;
    }
}

}  // extern "C"
