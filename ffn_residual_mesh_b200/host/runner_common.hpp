// Shared pieces of the drop-in runners: CUDA/C-ABI error checks that throw (the runners
// turn exceptions into "error: ..." and exit status 1, a usage error into status 2, as
// src/exact_residual_cuda_runner.cu:460-464,591-594 does), pinned host buffers, event
// timing, medians and JSON string output.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <ostream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "ffnrm.h"

namespace ffnrm_host {

inline void cuda_check(cudaError_t e, const char *expr, const char *file, int line) {
    if (e != cudaSuccess) {
        std::ostringstream m;
        m << expr << " failed at " << file << ':' << line << ": " << cudaGetErrorString(e);
        throw std::runtime_error(m.str());
    }
}
#define RUNNER_CUDA(expr) ::ffnrm_host::cuda_check((expr), #expr, __FILE__, __LINE__)

inline void ffnrm_check(int rc, const char *expr) {
    if (rc != FFNRM_OK) {
        const char *msg = ffnrm_last_error();
        throw std::runtime_error(std::string(expr) + ": " + (msg ? msg : "ffnrm error " + std::to_string(rc)));
    }
}
#define RUNNER_FFNRM(expr) ::ffnrm_host::ffnrm_check((expr), #expr)

inline int parse_int(const char *s, const char *what) {
    try {
        size_t used = 0;
        const int v = std::stoi(s, &used);
        if (used != std::string(s).size()) throw std::invalid_argument(s);
        return v;
    } catch (const std::exception &) {
        throw std::runtime_error(std::string("invalid ") + what + ": " + s);
    }
}

inline double median(std::vector<double> v) {
    if (v.empty()) return 0.0;
    std::sort(v.begin(), v.end());
    const size_t m = v.size() / 2;
    return v.size() % 2 ? v[m] : 0.5 * (v[m - 1] + v[m]);
}

inline double ms_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

// Page-locked host copy of a byte range (cudaMallocHost), freed on destruction.
class Pinned {
public:
    Pinned() = default;
    explicit Pinned(size_t bytes) : bytes_(bytes) { RUNNER_CUDA(cudaMallocHost(&p_, std::max<size_t>(bytes, 16))); }
    ~Pinned() {
        if (p_) cudaFreeHost(p_);
    }
    Pinned(const Pinned &) = delete;
    Pinned &operator=(const Pinned &) = delete;
    Pinned(Pinned &&o) noexcept : p_(o.p_), bytes_(o.bytes_) { o.p_ = nullptr; }
    template <typename T>
    T *as() const { return static_cast<T *>(p_); }
    size_t bytes() const { return bytes_; }

private:
    void *p_ = nullptr;
    size_t bytes_ = 0;
};

// Device buffer freed on destruction.
class DevMem {
public:
    DevMem() = default;
    explicit DevMem(size_t bytes) { RUNNER_CUDA(cudaMalloc(&p_, std::max<size_t>(bytes, 16))); }
    ~DevMem() {
        if (p_) cudaFree(p_);
    }
    DevMem(const DevMem &) = delete;
    DevMem &operator=(const DevMem &) = delete;
    template <typename T>
    T *as() const { return static_cast<T *>(p_); }

private:
    void *p_ = nullptr;
};

// Median over `repeats` of the GPU time (CUDA events on `st`) and of the host wall time of
// `enqueue()`, which issues work on `st`.
template <typename F>
void time_gpu(int repeats, cudaStream_t st, F &&enqueue, double &gpu_ms, double &host_ms) {
    cudaEvent_t a, b;
    RUNNER_CUDA(cudaEventCreate(&a));
    RUNNER_CUDA(cudaEventCreate(&b));
    std::vector<double> g, h;
    for (int i = 0; i < repeats; ++i) {
        RUNNER_CUDA(cudaStreamSynchronize(st));
        RUNNER_CUDA(cudaEventRecord(a, st));
        const auto t0 = std::chrono::steady_clock::now();
        enqueue();
        RUNNER_CUDA(cudaEventRecord(b, st));
        RUNNER_CUDA(cudaEventSynchronize(b));
        h.push_back(ms_since(t0));
        float ms = 0.f;
        RUNNER_CUDA(cudaEventElapsedTime(&ms, a, b));
        g.push_back(ms);
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    gpu_ms = median(g);
    host_ms = median(h);
}

inline void json_string(std::ostream &out, const std::string &v) {
    out << '"';
    for (const char c : v) {
        if (c == '\\' || c == '"') out << '\\';
        out << c;
    }
    out << '"';
}

// Residual of one row from QLO2 row-packed codes in double precision:
// sum_k q[k] * alpha[k/32] * z[k] * s[k/32] (the reference's validate_first_tile target,
// src/exact_residual_cuda_runner.cu:405-413).
inline double residual_row_f64(const uint8_t *code_row, const float *alpha_row, const int8_t *z, const float *s,
                               int hidden) {
    double acc = 0.0;
    for (int k = 0; k < hidden; ++k) {
        const int q = (code_row[k >> 2] >> ((k & 3) * 2)) & 3;
        acc += double(q) * alpha_row[k >> 5] * double(z[k]) * double(s[k >> 5]);
    }
    return acc;
}

struct ErrStats {
    double max_abs = 0.0, rel_l2 = 0.0;
};

inline ErrStats compare(const std::vector<double> &want, const float *got, size_t n) {
    double e2 = 0.0, t2 = 0.0, mx = 0.0;
    for (size_t i = 0; i < n; ++i) {
        const double e = double(got[i]) - want[i];
        e2 += e * e;
        t2 += want[i] * want[i];
        mx = std::max(mx, std::abs(e));
    }
    return {mx, std::sqrt(e2) / std::max(std::sqrt(t2), 1.0e-12)};
}

}  // namespace ffnrm_host
