// Readers for the reference's on-disk artifact contract (read unchanged):
//
//   residual dir  (scripts/export_cuda_residual_artifact_v2.py:56-125, format
//                 FFN_EXACT_QLO2_ROWPACKED_V2): {gate,up}.qlo2.rowpacked.bin u8 [F, D/4],
//                 {gate,up}.alpha.f32.bin f32 [F, G], activation.z.i8.bin [D],
//                 activation.scale.f32.bin [G], manifest.json (rows, hidden, file names,
//                 sha256 of the code and alpha files)
//   table dir     (scripts/export_radix_table_artifact.py:17-80, format
//                 FFN_RADIX_TABLE_ARTIFACT_V1): {p}.table.u8.bin [blocks, 4^bs, F],
//                 {p}.high_sum.i16.bin [F, G], {p}.alpha.f32.bin, {p}.beta.f32.bin,
//                 states.u16.bin [4, blocks], the same activation files, manifest.json
//   down          raw fp16 [D, F] (scripts/export_down_fp16.py:19-21)
//
// Shapes come from the manifests (the reference runners read rows/hidden by string
// search, src/exact_residual_cuda_runner.cu:50-69, or fix them at 6144 x 2048,
// src/exact_main_residual_cuda_runner.cu:47-56); every file size is checked against them
// and a checksum listed in the manifest is verified. Failures throw std::runtime_error.
#pragma once

#include <cstdint>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "json.hpp"
#include "sha256.hpp"

namespace ffnrm_host {

inline std::vector<uint8_t> read_file(const std::string &path) {
    std::ifstream in(path, std::ios::binary | std::ios::ate);
    if (!in) throw std::runtime_error("cannot open " + path);
    const std::streamsize n = in.tellg();
    if (n < 0) throw std::runtime_error("cannot size " + path);
    in.seekg(0, std::ios::beg);
    std::vector<uint8_t> data(static_cast<size_t>(n));
    if (n > 0 && !in.read(reinterpret_cast<char *>(data.data()), n)) throw std::runtime_error("cannot read " + path);
    return data;
}

template <typename T>
std::vector<T> read_array(const std::string &path, size_t count, const std::string &what) {
    const std::vector<uint8_t> raw = read_file(path);
    if (raw.size() != count * sizeof(T))
        throw std::runtime_error(what + " size does not match manifest (" + std::to_string(raw.size()) + " bytes, expected " +
                                 std::to_string(count * sizeof(T)) + ")");
    std::vector<T> out(count);
    if (!raw.empty()) std::memcpy(out.data(), raw.data(), raw.size());
    return out;
}

inline Json read_manifest(const std::string &dir) {
    const std::vector<uint8_t> raw = read_file(dir + "/manifest.json");
    return Json::parse(std::string(raw.begin(), raw.end()));
}

inline std::string file_or(const Json &j, const char *key, const std::string &fallback) {
    return j.has(key) ? j.at(key).text() : fallback;
}

// Verifies `bytes` against manifest key `sha_key` when the manifest lists it.
inline void check_sha(const Json &j, const char *sha_key, const std::vector<uint8_t> &bytes, const std::string &what) {
    if (!j.has(sha_key)) return;
    const std::string want = j.at(sha_key).text();
    const std::string got = sha256_hex(bytes.data(), bytes.size());
    if (got != want) throw std::runtime_error(what + " sha256 mismatch (manifest " + want + ", file " + got + ")");
}

struct Activation {
    int hidden = 0, groups = 0;
    std::vector<int8_t> z;  // [hidden]
    std::vector<float> s;   // [groups]
};

struct ResidualProjection {
    std::string name;
    int rows = 0, hidden = 0, groups = 0, residual_bits = 2, packed_row_bytes = 0;
    std::vector<uint8_t> codes;  // QLO2 row-packed [rows, hidden/4]
    std::vector<float> alpha;    // [rows, groups]
};

struct ResidualArtifact {
    std::string dir, format;
    int layer = -1;
    ResidualProjection proj[2];  // gate, up
    Activation act;
};

inline Activation read_activation(const std::string &dir, const std::string &zfile, const std::string &sfile, int hidden) {
    Activation a;
    a.hidden = hidden;
    a.groups = hidden / 32;
    a.z = read_array<int8_t>(dir + "/" + zfile, size_t(hidden), "activation z");
    a.s = read_array<float>(dir + "/" + sfile, size_t(a.groups), "activation scale");
    return a;
}

inline ResidualArtifact read_residual_artifact(const std::string &dir, bool verify = true) {
    ResidualArtifact A;
    A.dir = dir;
    const Json m = read_manifest(dir);
    A.format = m.has("format") ? m.at("format").text() : "";
    if (m.has("layer")) A.layer = int(m.at("layer").integer());
    const Json &projs = m.at("projections");
    const char *names[2] = {"gate", "up"};
    for (int q = 0; q < 2; ++q) {
        const Json &pj = projs.at(names[q]);
        ResidualProjection &P = A.proj[q];
        P.name = names[q];
        P.rows = int(pj.at("rows").integer());
        P.hidden = int(pj.at("hidden").integer());
        P.residual_bits = pj.has("residual_bits") ? int(pj.at("residual_bits").integer()) : 2;
        if (P.rows <= 0 || P.hidden <= 0 || P.hidden % 32) throw std::runtime_error("artifact shape is incompatible with the QLO2 layout");
        if (P.residual_bits != 2) throw std::runtime_error("QLO2 row-packed artifacts hold 2-bit residuals");
        P.groups = P.hidden / 32;
        P.packed_row_bytes = pj.has("packed_row_bytes") ? int(pj.at("packed_row_bytes").integer()) : P.hidden / 4;
        if (P.packed_row_bytes != P.hidden / 4) throw std::runtime_error("packed_row_bytes does not match hidden / 4");
        const std::string cf = file_or(pj, "packed_code_file", P.name + ".qlo2.rowpacked.bin");
        const std::string af = file_or(pj, "alpha_file", P.name + ".alpha.f32.bin");
        std::vector<uint8_t> codes = read_file(dir + "/" + cf);
        if (codes.size() != size_t(P.rows) * size_t(P.packed_row_bytes))
            throw std::runtime_error(P.name + " packed code size does not match manifest");
        std::vector<uint8_t> alpha = read_file(dir + "/" + af);
        if (alpha.size() != size_t(P.rows) * size_t(P.groups) * 4)
            throw std::runtime_error(P.name + " alpha size does not match manifest");
        if (verify) {
            check_sha(pj, "packed_code_sha256", codes, P.name + " packed codes");
            check_sha(pj, "alpha_sha256", alpha, P.name + " alpha");
        }
        P.codes = std::move(codes);
        P.alpha.resize(alpha.size() / 4);
        std::memcpy(P.alpha.data(), alpha.data(), alpha.size());
    }
    if (A.proj[0].rows != A.proj[1].rows || A.proj[0].hidden != A.proj[1].hidden)
        throw std::runtime_error("gate and up shapes differ");
    std::string zf = "activation.z.i8.bin", sf = "activation.scale.f32.bin";
    if (m.has("activation")) {
        zf = file_or(m.at("activation"), "z_file", zf);
        sf = file_or(m.at("activation"), "scale_file", sf);
    }
    A.act = read_activation(dir, zf, sf, A.proj[0].hidden);
    return A;
}

struct TableProjection {
    std::string name;
    int rows = 0, hidden = 0, groups = 0, block_size = 4, blocks = 0, state_count = 0;
    std::vector<uint8_t> table;     // [blocks, state_count, rows]
    std::vector<int16_t> high_sum;  // [rows, groups]
    std::vector<float> alpha, beta; // [rows, groups]
};

struct TableArtifact {
    std::string dir, format;
    int block_size = 4;
    TableProjection proj[2];
    std::vector<uint16_t> states;  // [4, blocks] for the artifact's activation
    Activation act;
};

// block_size: the value the caller passes (the runners' BLOCK_SIZE argument); it must
// match the manifest's.
inline TableArtifact read_table_artifact(const std::string &dir, int block_size) {
    TableArtifact A;
    A.dir = dir;
    const Json m = read_manifest(dir);
    A.format = m.has("format") ? m.at("format").text() : "";
    A.block_size = m.has("block_size") ? int(m.at("block_size").integer()) : block_size;
    if (A.block_size != block_size)
        throw std::runtime_error("BLOCK_SIZE " + std::to_string(block_size) + " does not match the table artifact's " +
                                 std::to_string(A.block_size));
    const Json &projs = m.at("projections");
    const char *names[2] = {"gate", "up"};
    for (int q = 0; q < 2; ++q) {
        const Json &pj = projs.at(names[q]);
        TableProjection &P = A.proj[q];
        P.name = names[q];
        P.rows = int(pj.at("rows").integer());
        P.hidden = int(pj.at("hidden").integer());
        P.groups = P.hidden / 32;
        P.block_size = block_size;
        if (P.rows <= 0 || P.hidden <= 0 || P.hidden % 32) throw std::runtime_error("table artifact shape is invalid");
        P.blocks = P.hidden / block_size;
        P.state_count = 1 << (2 * block_size);
        if (pj.has("blocks") && pj.at("blocks").integer() != P.blocks)
            throw std::runtime_error("table blocks do not match hidden / block_size");
        Json files;
        if (pj.has("files")) files = pj.at("files");
        const std::string base = dir + "/";
        P.table = read_array<uint8_t>(base + file_or(files, "table", P.name + ".table.u8.bin"),
                                      size_t(P.blocks) * P.state_count * P.rows, P.name + " table");
        P.high_sum = read_array<int16_t>(base + file_or(files, "high_sum", P.name + ".high_sum.i16.bin"),
                                         size_t(P.rows) * P.groups, P.name + " high_sum");
        P.alpha = read_array<float>(base + file_or(files, "alpha", P.name + ".alpha.f32.bin"), size_t(P.rows) * P.groups,
                                    P.name + " alpha");
        P.beta = read_array<float>(base + file_or(files, "beta", P.name + ".beta.f32.bin"), size_t(P.rows) * P.groups,
                                   P.name + " beta");
    }
    if (A.proj[0].rows != A.proj[1].rows || A.proj[0].hidden != A.proj[1].hidden)
        throw std::runtime_error("gate and up shapes differ");
    std::string zf = "activation.z.i8.bin", sf = "activation.scale.f32.bin", stf = "states.u16.bin";
    if (m.has("activation") && m.at("activation").has("files")) {
        const Json &f = m.at("activation").at("files");
        zf = file_or(f, "z", zf);
        sf = file_or(f, "scale", sf);
        stf = file_or(f, "states", stf);
    }
    A.act = read_activation(dir, zf, sf, A.proj[0].hidden);
    A.states = read_array<uint16_t>(dir + "/" + stf, size_t(4) * A.proj[0].blocks, "states");
    return A;
}

inline std::vector<uint16_t> read_down_fp16(const std::string &path, int hidden, int rows) {
    return read_array<uint16_t>(path, size_t(hidden) * size_t(rows), "down fp16");
}

}  // namespace ffnrm_host
