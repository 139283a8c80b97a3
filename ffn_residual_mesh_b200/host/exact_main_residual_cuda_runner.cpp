// Drop-in for src/exact_main_residual_cuda_runner.cu: same argv, exit codes and JSON keys.
//
//   exact_main_residual_cuda_runner TABLE_DIR RESIDUAL_DIR OUTPUT_JSON BLOCK_SIZE TILE_ROWS REPEATS THREADS
//
// The CPU evaluates the exact base ("main") term of each projection from the radix table
// artifact with THREADS threads (the host base producer of radix_base.hpp) while the GPU
// computes the residual through the C ABI; shapes come from the manifests (the reference
// fixes them at 6144 x 2048). Per projection it reports the CPU time, the GPU time with
// the payload upload in series and with the weights HBM-resident, the serial sum, and
// the wall time of the CPU evaluation and the GPU residual running concurrently
// (src/exact_main_residual_cuda_runner.cu:396-406). Gate and up run as one fused GPU
// launch; each projection reports half of it. Usage errors exit 2; failures exit 1.
#include <cuda_runtime.h>

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

void check_states(const TableArtifact &T) {
    std::vector<uint16_t> st(T.states.size());
    encode_states(T.act.z.data(), T.act.hidden, T.block_size, st.data());
    if (st != T.states) throw std::runtime_error("states.u16.bin does not encode the artifact's activation");
}

}  // namespace

int main(int argc, char **argv) {
    try {
        if (argc != 8) {
            std::cerr << "usage: exact_main_residual_cuda_runner TABLE_DIR RESIDUAL_DIR OUTPUT_JSON BLOCK_SIZE TILE_ROWS "
                         "REPEATS THREADS\n";
            return 2;
        }
        const std::string table_dir = argv[1], residual_dir = argv[2], out_path = argv[3];
        const int block_size = parse_int(argv[4], "BLOCK_SIZE");
        const int tile_rows = parse_int(argv[5], "TILE_ROWS");
        const int repeats = parse_int(argv[6], "REPEATS");
        const int threads = parse_int(argv[7], "THREADS");
        if (block_size != 2 && block_size != 4 && block_size != 8) throw std::runtime_error("block size must be 2, 4, or 8");
        if (tile_rows <= 0 || repeats <= 0 || threads <= 0) throw std::runtime_error("invalid tile/repeat arguments");

        const TableArtifact T = read_table_artifact(table_dir, block_size);
        const ResidualArtifact R = read_residual_artifact(residual_dir);
        const int rows = T.proj[0].rows, hidden = T.proj[0].hidden, groups = T.proj[0].groups;
        if (R.proj[0].rows != rows || R.proj[0].hidden != hidden)
            throw std::runtime_error("table and residual artifacts have different shapes");
        if (rows % tile_rows != 0) throw std::runtime_error("invalid tile/repeat arguments");
        check_states(T);

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
        RUNNER_FFNRM(ffnrm_load_layer(ctx, 0, &w));

        DevMem dz{size_t(hidden)}, ds{size_t(groups) * 4}, dres{size_t(rows) * 8}, dpay{payload};
        RUNNER_CUDA(cudaMemcpy(dz.as<void>(), T.act.z.data(), size_t(hidden), cudaMemcpyHostToDevice));
        RUNNER_CUDA(cudaMemcpy(ds.as<void>(), T.act.s.data(), size_t(groups) * 4, cudaMemcpyHostToDevice));
        float *g_res = dres.as<float>(), *u_res = g_res + rows;
        cudaStream_t st;
        RUNNER_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        auto residual = [&] {
            RUNNER_FFNRM(ffnrm_residual(ctx, 0, dz.as<int8_t>(), ds.as<float>(), 1, g_res, u_res, nullptr, nullptr, st));
        };
        residual();
        RUNNER_CUDA(cudaStreamSynchronize(st));
        RUNNER_FFNRM(ffnrm_check_device_error(ctx, st));
        std::vector<float> gpu(static_cast<size_t>(rows) * 2);
        RUNNER_CUDA(cudaMemcpy(gpu.data(), g_res, gpu.size() * 4, cudaMemcpyDeviceToHost));

        TilePool pool(threads);
        struct Row {
            double cpu = 0, gpu_serial = 0, gpu_overlap = 0, serial = 0, concurrent = 0;
            ErrStats val;
        } res[2];
        double pair_kernel = 0, pair_kernel_host = 0;
        time_gpu(repeats, st, residual, pair_kernel, pair_kernel_host);
        for (int q = 0; q < 2; ++q) {
            const TableView V = view_of(T.proj[q]);
            std::vector<float> base(static_cast<size_t>(rows));
            auto cpu_eval = [&] {
                const auto t0 = std::chrono::steady_clock::now();
                table_base(pool, V, T.act.z.data(), T.act.s.data(), 1, 4, base.data(), 256);
                return ms_since(t0);
            };
            std::vector<double> want(static_cast<size_t>(tile_rows));
            for (int r = 0; r < tile_rows; ++r)
                want[size_t(r)] = residual_row_f64(R.proj[q].codes.data() + size_t(r) * (hidden / 4),
                                                   R.proj[q].alpha.data() + size_t(r) * groups, T.act.z.data(),
                                                   T.act.s.data(), hidden);
            res[q].val = compare(want, gpu.data() + size_t(q) * rows, size_t(tile_rows));
            const void *src = host[q].as<void>();
            double copy = 0, copy_host = 0;
            time_gpu(repeats, st, [&] { RUNNER_CUDA(cudaMemcpyAsync(dpay.as<void>(), src, payload, cudaMemcpyHostToDevice, st)); },
                     copy, copy_host);
            for (int i = 0; i < 2; ++i) cpu_eval();  // warm-up
            std::vector<double> cpu_t, ser_t, conc_t;
            for (int i = 0; i < repeats; ++i) {
                const double c = cpu_eval();
                cpu_t.push_back(c);
                ser_t.push_back(c + copy + 0.5 * pair_kernel);
                RUNNER_CUDA(cudaStreamSynchronize(st));
                const auto t0 = std::chrono::steady_clock::now();
                RUNNER_CUDA(cudaMemcpyAsync(dpay.as<void>(), src, payload, cudaMemcpyHostToDevice, st));
                residual();
                cpu_eval();
                RUNNER_CUDA(cudaStreamSynchronize(st));
                conc_t.push_back(ms_since(t0));
            }
            res[q].cpu = median(cpu_t);
            res[q].gpu_serial = copy + 0.5 * pair_kernel;
            res[q].gpu_overlap = 0.5 * pair_kernel;
            res[q].serial = median(ser_t);
            res[q].concurrent = median(conc_t);
        }
        RUNNER_FFNRM(ffnrm_check_device_error(ctx, st));
        cudaStreamDestroy(st);

        std::ofstream out(out_path, std::ios::trunc);
        if (!out) throw std::runtime_error("cannot write " + out_path);
        out << std::setprecision(8) << "{\n";
        out << "  \"experiment\": \"cuda_cpu_main_plus_exact_residual_v1\",\n";
        out << "  \"gpu\": ";
        json_string(out, prop.name);
        out << ",\n";
        out << "  \"shape\": {\"rows\": " << rows << ", \"hidden\": " << hidden << ", \"tile_rows\": " << tile_rows
            << ", \"cpu_threads\": " << threads << "},\n";
        out << "  \"projections\": {\n";
        for (int q = 0; q < 2; ++q) {
            const Row &r = res[q];
            out << "    \"" << (q == 0 ? "gate" : "up") << "\": {\"cpu_main_ms\": " << r.cpu
                << ", \"gpu_serial_copy_compute_ms\": " << r.gpu_serial << ", \"gpu_overlap_ms\": " << r.gpu_overlap
                << ", \"residual_validation_max_abs\": " << r.val.max_abs
                << ", \"residual_validation_rel_l2\": " << r.val.rel_l2 << ", \"serial_cpu_plus_gpu_ms\": " << r.serial
                << ", \"cpu_gpu_concurrent_wall_ms\": " << r.concurrent
                << ", \"serial_to_concurrent_speedup\": " << r.serial / std::max(r.concurrent, 1.0e-12) << "}"
                << (q == 0 ? ",\n" : "\n");
        }
        out << "  },\n";
        const double ps = res[0].serial + res[1].serial, pc = res[0].concurrent + res[1].concurrent;
        out << "  \"pair\": {\"serial_cpu_plus_gpu_ms\": " << ps << ", \"concurrent_wall_ms\": " << pc
            << ", \"speedup\": " << ps / std::max(pc, 1.0e-12) << "}\n";
        out << "}\n";
        std::cout << "wrote " << out_path << '\n';
        return 0;
    } catch (const std::exception &e) {
        std::cerr << "error: " << e.what() << '\n';
        return 1;
    }
}
