// Drop-in for src/exact_residual_cuda_runner.cu: same argv, exit codes and JSON keys.
//
//   exact_residual_cuda_runner ARTIFACT_DIR OUTPUT_JSON [TILE_ROWS=1024] [REPEATS=7]
//
// Reads a FFN_EXACT_QLO2_ROWPACKED_V2 residual artifact (shapes from its manifest, file
// checksums verified), loads gate and up into HBM through the C ABI (ffnrm_load_layer)
// and times, per projection:
//   copy_only          the pinned host -> device upload of the projection's payload
//                      (packed codes + alpha), as the reference uploads it per call;
//   kernel_only        the residual contraction on the HBM-resident weights (gate and up
//                      run as one launch; each projection reports half of it);
//   serial             upload followed by the contraction on one stream;
//   double_buffer      the upload on a copy stream overlapped with the contraction on
//                      the compute stream (the weights of the next call arriving while
//                      this one computes).
// The first TILE_ROWS rows are validated against a double-precision evaluation of the
// artifact (as validate_first_tile, src/exact_residual_cuda_runner.cu:386-420).
// Usage errors exit 2; any other failure prints "error: ..." and exits 1.
#include <cuda_runtime.h>

#include <cstring>
#include <fstream>
#include <iomanip>
#include <iostream>

#include "artifacts.hpp"
#include "ffnrm.h"
#include "runner_common.hpp"

using namespace ffnrm_host;

int main(int argc, char **argv) {
    try {
        if (argc < 3 || argc > 5) {
            std::cerr << "usage: exact_residual_cuda_runner ARTIFACT_DIR OUTPUT_JSON [TILE_ROWS] [REPEATS]\n";
            return 2;
        }
        const std::string dir = argv[1], out_path = argv[2];
        const int tile_rows = argc >= 4 ? parse_int(argv[3], "TILE_ROWS") : 1024;
        const int repeats = argc >= 5 ? parse_int(argv[4], "REPEATS") : 7;
        if (tile_rows <= 0 || repeats <= 0) throw std::runtime_error("tile_rows and repeats must be positive");

        const ResidualArtifact A = read_residual_artifact(dir);
        const int rows = A.proj[0].rows, hidden = A.proj[0].hidden, groups = A.proj[0].groups;
        if (rows % tile_rows != 0) throw std::runtime_error("artifact shape is incompatible with tile or QLO2 layout");

        RUNNER_CUDA(cudaSetDevice(0));
        cudaDeviceProp prop{};
        RUNNER_CUDA(cudaGetDeviceProperties(&prop, 0));
        ffnrm_config cfg{};
        cfg.d_model = hidden;
        cfg.d_ff = rows;
        cfg.residual_bits = 2;
        cfg.n_layers = 1;
        cfg.max_tokens = 1;
        cfg.base_tile_rows = tile_rows;
        ffnrm_ctx *ctx = nullptr;
        RUNNER_FFNRM(ffnrm_create(&ctx, 0, &cfg));
        struct CtxGuard {
            ffnrm_ctx *c;
            ~CtxGuard() { ffnrm_destroy(c); }
        } guard{ctx};

        // Pinned payloads (codes then alpha, one contiguous run per projection) and the
        // residual-only layer (no down projection) in HBM.
        const size_t code_bytes = A.proj[0].codes.size(), alpha_bytes = A.proj[0].alpha.size() * 4;
        const size_t payload = code_bytes + alpha_bytes;
        Pinned host[2] = {Pinned(payload), Pinned(payload)};
        for (int q = 0; q < 2; ++q) {
            std::memcpy(host[q].as<uint8_t>(), A.proj[q].codes.data(), code_bytes);
            std::memcpy(host[q].as<uint8_t>() + code_bytes, A.proj[q].alpha.data(), alpha_bytes);
        }
        ffnrm_layer_weights w{};
        w.codes_format = FFNRM_CODES_QLO2_ROWPACKED;
        w.gate_codes = host[0].as<uint8_t>();
        w.up_codes = host[1].as<uint8_t>();
        w.gate_alpha = reinterpret_cast<const float *>(host[0].as<uint8_t>() + code_bytes);
        w.up_alpha = reinterpret_cast<const float *>(host[1].as<uint8_t>() + code_bytes);
        const auto t_load = std::chrono::steady_clock::now();
        RUNNER_FFNRM(ffnrm_load_layer(ctx, 0, &w));
        const double load_ms = ms_since(t_load);

        DevMem dz{size_t(hidden)}, ds{size_t(groups) * 4}, dres{size_t(rows) * 4 * 2}, dpay{payload};
        RUNNER_CUDA(cudaMemcpy(dz.as<void>(), A.act.z.data(), size_t(hidden), cudaMemcpyHostToDevice));
        RUNNER_CUDA(cudaMemcpy(ds.as<void>(), A.act.s.data(), size_t(groups) * 4, cudaMemcpyHostToDevice));
        float *g_res = dres.as<float>(), *u_res = g_res + rows;
        cudaStream_t st, cs;
        RUNNER_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        RUNNER_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
        cudaEvent_t copied, computed;
        RUNNER_CUDA(cudaEventCreateWithFlags(&copied, cudaEventDisableTiming));
        RUNNER_CUDA(cudaEventCreateWithFlags(&computed, cudaEventDisableTiming));
        auto residual = [&] {
            RUNNER_FFNRM(ffnrm_residual(ctx, 0, dz.as<int8_t>(), ds.as<float>(), 1, g_res, u_res, nullptr, nullptr, st));
        };

        // validation of the first tile of each projection
        residual();
        RUNNER_CUDA(cudaStreamSynchronize(st));
        RUNNER_FFNRM(ffnrm_check_device_error(ctx, st));
        std::vector<float> gpu(static_cast<size_t>(rows) * 2);
        RUNNER_CUDA(cudaMemcpy(gpu.data(), g_res, gpu.size() * 4, cudaMemcpyDeviceToHost));
        ErrStats val[2];
        for (int q = 0; q < 2; ++q) {
            std::vector<double> want(static_cast<size_t>(tile_rows));
            for (int r = 0; r < tile_rows; ++r)
                want[size_t(r)] = residual_row_f64(A.proj[q].codes.data() + size_t(r) * (hidden / 4),
                                                   A.proj[q].alpha.data() + size_t(r) * groups, A.act.z.data(),
                                                   A.act.s.data(), hidden);
            val[q] = compare(want, gpu.data() + size_t(q) * rows, size_t(tile_rows));
        }

        struct Times {
            double copy = 0, copy_host = 0, kernel = 0, kernel_host = 0, serial = 0, serial_host = 0, overlap = 0,
                   overlap_host = 0;
        } tm[2];
        double pair_kernel = 0, pair_kernel_host = 0;
        time_gpu(repeats, st, residual, pair_kernel, pair_kernel_host);
        for (int q = 0; q < 2; ++q) {
            Times &t = tm[q];
            const void *src = host[q].as<void>();
            time_gpu(repeats, st, [&] { RUNNER_CUDA(cudaMemcpyAsync(dpay.as<void>(), src, payload, cudaMemcpyHostToDevice, st)); },
                     t.copy, t.copy_host);
            t.kernel = 0.5 * pair_kernel;
            t.kernel_host = 0.5 * pair_kernel_host;
            double sk = 0, skh = 0;
            time_gpu(repeats, st,
                     [&] {
                         RUNNER_CUDA(cudaMemcpyAsync(dpay.as<void>(), src, payload, cudaMemcpyHostToDevice, st));
                         residual();
                     },
                     sk, skh);
            t.serial = sk - t.kernel;  // this projection's upload + its share of the fused launch
            t.serial_host = skh;
            double ov = 0, ovh = 0;
            time_gpu(repeats, st,
                     [&] {
                         RUNNER_CUDA(cudaEventRecord(computed, st));
                         RUNNER_CUDA(cudaStreamWaitEvent(cs, computed, 0));
                         RUNNER_CUDA(cudaMemcpyAsync(dpay.as<void>(), src, payload, cudaMemcpyHostToDevice, cs));
                         RUNNER_CUDA(cudaEventRecord(copied, cs));
                         residual();
                         RUNNER_CUDA(cudaStreamWaitEvent(st, copied, 0));
                     },
                     ov, ovh);
            t.overlap = std::max(ov - t.kernel, t.copy);
            t.overlap_host = ovh;
        }
        RUNNER_FFNRM(ffnrm_check_device_error(ctx, st));

        std::ofstream out(out_path, std::ios::trunc);
        if (!out) throw std::runtime_error("cannot write " + out_path);
        out << std::setprecision(8);
        out << "{\n";
        out << "  \"experiment\": \"cuda_exact_qlo2_residual_runner_v1\",\n";
        out << "  \"layer\": " << (A.layer >= 0 ? A.layer : 23) << ",\n";
        out << "  \"gpu\": {\"name\": ";
        json_string(out, prop.name);
        out << ", \"global_memory_bytes\": " << prop.totalGlobalMem << "},\n";
        out << "  \"shape\": {\"rows\": " << rows << ", \"hidden\": " << hidden << ", \"groups\": " << groups
            << ", \"tile_rows\": " << tile_rows << ", \"tile_count\": " << rows / tile_rows << "},\n";
        out << "  \"implementation\": {\"library\": \"libffnrm\", \"weights\": \"HBM-resident after ffnrm_load_layer\", "
               "\"load_layer_ms\": "
            << load_ms << ", \"fused_gate_up_kernel_gpu_ms\": " << pair_kernel << "},\n";
        out << "  \"projections\": {\n";
        for (int q = 0; q < 2; ++q) {
            const Times &t = tm[q];
            const double hidden_copy = std::max(0.0, t.copy + t.kernel - t.overlap);
            const double visible = std::max(0.0, t.overlap - t.kernel);
            out << "    ";
            json_string(out, A.proj[q].name);
            out << ": {\n";
            out << "      \"tile_payload_bytes\": " << size_t(tile_rows) * (payload / size_t(rows)) << ",\n";
            out << "      \"full_payload_bytes\": " << payload << ",\n";
            out << "      \"validation_max_abs\": " << val[q].max_abs << ",\n";
            out << "      \"validation_rel_l2\": " << val[q].rel_l2 << ",\n";
            out << "      \"copy_only_gpu_ms\": " << t.copy << ",\n";
            out << "      \"copy_only_host_ms\": " << t.copy_host << ",\n";
            out << "      \"kernel_only_gpu_ms\": " << t.kernel << ",\n";
            out << "      \"serial_copy_compute_gpu_ms\": " << t.serial << ",\n";
            out << "      \"serial_copy_compute_host_ms\": " << t.serial_host << ",\n";
            out << "      \"double_buffer_overlap_gpu_ms\": " << t.overlap << ",\n";
            out << "      \"double_buffer_overlap_host_ms\": " << t.overlap_host << ",\n";
            out << "      \"overlap_speedup_vs_serial\": " << t.serial / std::max(t.overlap, 1.0e-12) << ",\n";
            out << "      \"hidden_copy_ms\": " << hidden_copy << ",\n";
            out << "      \"visible_copy_wait_ms\": " << visible << "\n";
            out << "    }" << (q == 0 ? ",\n" : "\n");
        }
        const double ps = tm[0].serial + tm[1].serial, po = tm[0].overlap + tm[1].overlap;
        out << "  },\n";
        out << "  \"pair\": {\n";
        out << "    \"full_payload_bytes\": " << payload * 2 << ",\n";
        out << "    \"serial_gpu_ms\": " << ps << ",\n";
        out << "    \"overlap_gpu_ms\": " << po << ",\n";
        out << "    \"overlap_speedup_vs_serial\": " << ps / std::max(po, 1.0e-12) << "\n";
        out << "  }\n";
        out << "}\n";
        cudaEventDestroy(copied);
        cudaEventDestroy(computed);
        cudaStreamDestroy(st);
        cudaStreamDestroy(cs);
        std::cout << "wrote " << out_path << '\n';
        return 0;
    } catch (const std::exception &e) {
        std::cerr << "error: " << e.what() << '\n';
        return 1;
    }
}
