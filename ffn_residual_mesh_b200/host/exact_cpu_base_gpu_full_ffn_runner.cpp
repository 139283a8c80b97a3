// Drop-in for src/exact_cpu_base_gpu_full_ffn_runner.cu: same argv, exit codes and JSON keys.
//
//   exact_cpu_base_gpu_full_ffn_runner TABLE_DIR RESIDUAL_DIR DOWN_FP16 OUTPUT_JSON BLOCK_SIZE TILE_ROWS REPEATS THREADS
//
// The CPU produces the exact base sums of gate and up from the radix table artifact
// (radix_base.hpp, THREADS threads); the GPU runs residual + merge + SwiGLU + fp16 down
// through ffnrm_ffn_forward_host with the base in page-locked host memory. Reported as
// the reference does (serial CPU + GPU, the GPU alone with the residual payload uploaded
// in series and with the weights HBM-resident, the max(cpu, gpu) lower bound), plus
// "cpu_gpu_pipelined_ms": the measured time per call when the CPU produces the next
// call's base while the GPU runs the current one (two pinned base slots). "correctness"
// compares y with a double-precision evaluation of the same split on the host (exact
// table dots + residual dots, SwiGLU, down), which the reference leaves to Python.
// Usage errors exit 2; failures exit 1.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <fstream>
#include <future>
#include <iomanip>
#include <iostream>

#include "artifacts.hpp"
#include "ffnrm.h"
#include "radix_base.hpp"
#include "runner_common.hpp"

using namespace ffnrm_host;

namespace {

TableView view_of(const TableProjection &P) {
    return TableView{P.rows, P.hidden, P.groups, P.block_size, P.blocks, P.state_count,
                     P.table.data(), P.high_sum.data(), P.alpha.data(), P.beta.data()};
}

double half_to_double(uint16_t h) {
    const int sign = h >> 15, exp = (h >> 10) & 31, man = h & 1023;
    double v;
    if (exp == 0)
        v = std::ldexp(double(man), -24);
    else if (exp == 31)
        v = man ? NAN : INFINITY;
    else
        v = std::ldexp(double(man | 1024), exp - 25);
    return sign ? -v : v;
}

// Exact split projection of one row in double: base from the table's integer dots plus
// the residual from the row-packed low codes.
void exact_projection(const TableView &V, const ResidualProjection &Rp, const int8_t *z, const float *s,
                      std::vector<double> &out) {
    const int rows = V.rows, G = V.groups, tile = 256;
    std::vector<uint16_t> st(size_t(4) * V.blocks);
    encode_states(z, V.hidden, V.block_size, st.data());
    std::vector<int32_t> zsum(size_t(G), 0);
    for (int g = 0; g < G; ++g)
        for (int i = 0; i < 32; ++i) zsum[size_t(g)] += z[g * 32 + i];
    std::vector<int16_t> acc(size_t(G) * tile);
    out.assign(size_t(rows), 0.0);
    for (int r0 = 0; r0 < rows; r0 += tile) {
        const int n = std::min(tile, rows - r0);
        table_dots_tile(V, st.data(), r0, n, acc.data());
        for (int i = 0; i < n; ++i) {
            const size_t row = size_t(r0 + i);
            double v = 0.0;
            for (int g = 0; g < G; ++g)
                v += double(s[g]) * (double(V.alpha[row * G + g]) * 4.0 * double(acc[size_t(g) * n + i]) +
                                     double(V.beta[row * G + g]) * double(zsum[size_t(g)]));
            out[row] = v + residual_row_f64(Rp.codes.data() + row * size_t(V.hidden / 4), Rp.alpha.data() + row * G, z, s,
                                            V.hidden);
        }
    }
}

}  // namespace

int main(int argc, char **argv) {
    try {
        if (argc != 9) {
            std::cerr << "usage: exact_cpu_base_gpu_full_ffn_runner TABLE_DIR RESIDUAL_DIR DOWN_FP16 OUTPUT_JSON BLOCK_SIZE "
                         "TILE_ROWS REPEATS THREADS\n";
            return 2;
        }
        const std::string table_dir = argv[1], residual_dir = argv[2], down_path = argv[3], out_path = argv[4];
        const int block_size = parse_int(argv[5], "BLOCK_SIZE");
        const int tile_rows = parse_int(argv[6], "TILE_ROWS");
        const int repeats = parse_int(argv[7], "REPEATS");
        const int threads = parse_int(argv[8], "THREADS");
        if (block_size != 2 && block_size != 4) throw std::runtime_error("block size must be 2 or 4");
        if (tile_rows <= 0 || repeats <= 0 || threads <= 0) throw std::runtime_error("invalid tile/repeat arguments");

        const TableArtifact T = read_table_artifact(table_dir, block_size);
        const ResidualArtifact R = read_residual_artifact(residual_dir);
        const int rows = T.proj[0].rows, hidden = T.proj[0].hidden, groups = T.proj[0].groups;
        if (R.proj[0].rows != rows || R.proj[0].hidden != hidden)
            throw std::runtime_error("table and residual artifacts have different shapes");
        if (rows % tile_rows != 0) throw std::runtime_error("invalid tile/repeat arguments");
        const std::vector<uint16_t> down = read_down_fp16(down_path, hidden, rows);

        RUNNER_CUDA(cudaSetDevice(0));
        cudaDeviceProp prop{};
        RUNNER_CUDA(cudaGetDeviceProperties(&prop, 0));
        ffnrm_config cfg{hidden, rows, 2, 1, 1, tile_rows};
        ffnrm_ctx *ctx = nullptr;
        RUNNER_FFNRM(ffnrm_create(&ctx, 0, &cfg));
        struct CtxGuard {
            ffnrm_ctx *c;
            ~CtxGuard() { ffnrm_destroy(c); }
        } guard{ctx};
        const size_t code_bytes = R.proj[0].codes.size(), alpha_bytes = R.proj[0].alpha.size() * 4;
        const size_t payload = code_bytes + alpha_bytes;
        Pinned host[2] = {Pinned(payload), Pinned(payload)};
        for (int q = 0; q < 2; ++q) {
            std::memcpy(host[q].as<uint8_t>(), R.proj[q].codes.data(), code_bytes);
            std::memcpy(host[q].as<uint8_t>() + code_bytes, R.proj[q].alpha.data(), alpha_bytes);
        }
        ffnrm_layer_weights w{};
        w.codes_format = FFNRM_CODES_QLO2_ROWPACKED;
        w.gate_codes = host[0].as<uint8_t>();
        w.up_codes = host[1].as<uint8_t>();
        w.gate_alpha = reinterpret_cast<const float *>(host[0].as<uint8_t>() + code_bytes);
        w.up_alpha = reinterpret_cast<const float *>(host[1].as<uint8_t>() + code_bytes);
        w.down = down.data();
        w.down_ld = rows;
        RUNNER_FFNRM(ffnrm_load_layer(ctx, 0, &w));

        // pinned activations, two base slots (gate | up rows each), device-mapped y
        Pinned hz{size_t(hidden)}, hs{size_t(groups) * 4}, hbase[2] = {Pinned(size_t(rows) * 8), Pinned(size_t(rows) * 8)};
        std::memcpy(hz.as<void>(), T.act.z.data(), size_t(hidden));
        std::memcpy(hs.as<void>(), T.act.s.data(), size_t(groups) * 4);
        uint16_t *y16 = nullptr;
        RUNNER_CUDA(cudaHostAlloc(reinterpret_cast<void **>(&y16), size_t(hidden) * 2, cudaHostAllocMapped));
        struct YGuard {
            uint16_t *p;
            ~YGuard() { cudaFreeHost(p); }
        } yguard{y16};
        DevMem dpay{payload};
        cudaStream_t st;
        RUNNER_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));

        TilePool pool(threads);
        const TableView V[2] = {view_of(T.proj[0]), view_of(T.proj[1])};
        auto cpu_base = [&](int slot) {
            const auto t0 = std::chrono::steady_clock::now();
            float *b = hbase[slot].as<float>();
            table_base(pool, V[0], T.act.z.data(), T.act.s.data(), 1, 4, b, 256);
            table_base(pool, V[1], T.act.z.data(), T.act.s.data(), 1, 4, b + rows, 256);
            return ms_since(t0);
        };
        auto gpu_forward = [&](int slot) {
            const float *b = hbase[slot].as<float>();
            RUNNER_FFNRM(ffnrm_ffn_forward_host(ctx, 0, hz.as<int8_t>(), hs.as<float>(), 1, b, b + rows, nullptr, y16, st));
        };
        auto upload_payload = [&] {
            for (int q = 0; q < 2; ++q)
                RUNNER_CUDA(cudaMemcpyAsync(dpay.as<void>(), host[q].as<void>(), payload, cudaMemcpyHostToDevice, st));
        };
        for (int i = 0; i < 2; ++i) {  // warm-up
            cpu_base(0);
            gpu_forward(0);
            RUNNER_CUDA(cudaStreamSynchronize(st));
        }
        RUNNER_FFNRM(ffnrm_check_device_error(ctx, st));

        // correctness of y against the double-precision split
        std::vector<double> g, u;
        exact_projection(V[0], R.proj[0], T.act.z.data(), T.act.s.data(), g);
        exact_projection(V[1], R.proj[1], T.act.z.data(), T.act.s.data(), u);
        std::vector<double> h(static_cast<size_t>(rows)), yref(static_cast<size_t>(hidden), 0.0);
        for (int f = 0; f < rows; ++f) h[size_t(f)] = g[size_t(f)] / (1.0 + std::exp(-g[size_t(f)])) * u[size_t(f)];
        for (int o = 0; o < hidden; ++o) {
            double acc = 0.0;
            const uint16_t *dr = down.data() + size_t(o) * rows;
            for (int f = 0; f < rows; ++f) acc += half_to_double(dr[f]) * h[size_t(f)];
            yref[size_t(o)] = acc;
        }
        std::vector<float> ygpu(static_cast<size_t>(hidden));
        for (int o = 0; o < hidden; ++o) ygpu[size_t(o)] = float(half_to_double(y16[o]));
        const ErrStats yerr = compare(yref, ygpu.data(), size_t(hidden));

        std::vector<double> cpu_t, gser_t, ser_t, gov_t;
        double unused = 0;
        for (int i = 0; i < repeats; ++i) {
            const double c = cpu_base(0);
            cpu_t.push_back(c);
            double gs = 0, go = 0;
            time_gpu(1, st, [&] { upload_payload(); gpu_forward(0); }, gs, unused);
            time_gpu(1, st, [&] { gpu_forward(0); }, go, unused);
            gser_t.push_back(gs);
            ser_t.push_back(c + gs);
            gov_t.push_back(go);
        }
        // pipelined: the CPU fills slot (i+1)&1 while the GPU consumes slot i&1
        cpu_base(0);
        RUNNER_CUDA(cudaStreamSynchronize(st));
        const auto tp = std::chrono::steady_clock::now();
        for (int i = 0; i < repeats; ++i) {
            gpu_forward(i & 1);
            cpu_base((i + 1) & 1);
            RUNNER_CUDA(cudaStreamSynchronize(st));
        }
        const double pipelined = ms_since(tp) / repeats;
        RUNNER_FFNRM(ffnrm_check_device_error(ctx, st));
        cudaStreamDestroy(st);

        const double cpu_ms = median(cpu_t), gser = median(gser_t), gov = median(gov_t), ser = median(ser_t);
        const double lb = std::max(cpu_ms, gov);
        std::ofstream out(out_path, std::ios::trunc);
        if (!out) throw std::runtime_error("cannot write " + out_path);
        out << std::setprecision(8) << "{\n";
        out << "  \"experiment\": \"cpu_base_gpu_residual_swiglu_down_v1\",\n";
        out << "  \"gpu\": ";
        json_string(out, prop.name);
        out << ",\n";
        out << "  \"shape\": {\"rows\": " << rows << ", \"hidden\": " << hidden << ", \"tile_rows\": " << tile_rows
            << ", \"tile_count\": " << rows / tile_rows << ", \"cpu_threads\": " << threads << "},\n";
        out << "  \"cpu_base_gate_up_ms\": " << cpu_ms << ",\n";
        out << "  \"gpu_serial_copy_compute_ms\": " << gser << ",\n";
        out << "  \"serial_cpu_plus_gpu_ms\": " << ser << ",\n";
        out << "  \"gpu_double_buffer_overlap_ms\": " << gov << ",\n";
        out << "  \"gpu_overlap_speedup_vs_gpu_serial\": " << gser / std::max(gov, 1.0e-12) << ",\n";
        out << "  \"cpu_gpu_critical_lower_bound_ms\": " << lb << ",\n";
        out << "  \"serial_to_cpu_gpu_lower_bound_speedup\": " << ser / std::max(lb, 1.0e-12) << ",\n";
        out << "  \"cpu_gpu_pipelined_ms\": " << pipelined << ",\n";
        out << "  \"h2d\": {\"residual_gate_up_bytes\": " << 2 * payload
            << ", \"base_gate_up_bytes\": " << size_t(2) * rows * sizeof(float)
            << ", \"resident_down_bytes\": " << down.size() * sizeof(uint16_t) << "},\n";
        out << "  \"correctness\": {\"status\": \"y compared with a double-precision evaluation of the exact split\", "
               "\"y_max_abs\": "
            << yerr.max_abs << ", \"y_rel_l2\": " << yerr.rel_l2 << "}\n";
        out << "}\n";
        std::cout << "wrote " << out_path << '\n';
        return 0;
    } catch (const std::exception &e) {
        std::cerr << "error: " << e.what() << '\n';
        return 1;
    }
}
