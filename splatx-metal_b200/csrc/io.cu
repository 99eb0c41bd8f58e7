// io.cu — INRIA 3DGS PLY files and the export filter (host code; replaces
// Sources/SplatXCore/PlyIO.cpp and its header's contract, PlyIO.h:1-60).
//
// Layout: `binary_little_endian 1.0`, one `vertex` element of float properties
//   x y z nx ny nz f_dc_0..2 f_rest_0..(3K'-1) opacity scale_0..2 rot_0..3
// with normals 0, f_rest channel-major (all of red's coefficients, then green's, then blue's —
// the in-memory shN is coefficient-major [N, K, 3]) and, when padding, every channel's block
// zero-padded from K to 15 coefficients for viewers that require all 45 (degree 0 is never padded).
// The reader takes the properties by name, rejects non-float properties and other encodings, and
// infers the SH degree from the f_rest count. The export filter drops rows with a non-finite
// value, then rows with sigmoid(opacity) <= min_opacity (strict `>` keeps), in that order.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

struct File {
    FILE* f = nullptr;
    File(const char* path, const char* mode) : f(std::fopen(path, mode)) {}
    ~File() {
        if (f) std::fclose(f);
    }
};

inline int rest_coeffs(int degree) { return (degree + 1) * (degree + 1) - 1; }

// sigmoid_f32 (Trainer.cpp:430): float std::exp, as the reference's filter evaluates it.
inline float sigmoid_host(float x) { return 1.0f / (1.0f + std::exp(-x)); }

}  // namespace

void ply_write(const SxCloud& c, const char* path, bool pad_sh_full) {
    if (!path) throw_invalid("ply_write", "null path");
    if (c.count < 0) throw_invalid("ply_write", "negative count");
    if (c.sh_degree < 0 || c.sh_degree > 3) throw_invalid("ply_write", "sh_degree must be in [0,3]");
    const int K = rest_coeffs(c.sh_degree);
    if (c.count > 0 && (!c.means || !c.scales || !c.quats || !c.opacities || !c.sh0 || (K && !c.shN)))
        throw_invalid("ply_write", "null cloud array");
    const int Kw = (pad_sh_full && K > 0 && K < 15) ? 15 : K;
    File f(path, "wb");
    if (!f.f) throw RuntimeError(std::string("ply: cannot write ") + path);
    std::string h = "ply\nformat binary_little_endian 1.0\nelement vertex " +
                    std::to_string(c.count) + "\n";
    auto prop = [&](const std::string& n) { h += "property float " + n + "\n"; };
    for (const char* n : {"x", "y", "z", "nx", "ny", "nz"}) prop(n);
    for (int i = 0; i < 3; ++i) prop("f_dc_" + std::to_string(i));
    for (int i = 0; i < 3 * Kw; ++i) prop("f_rest_" + std::to_string(i));
    prop("opacity");
    for (int i = 0; i < 3; ++i) prop("scale_" + std::to_string(i));
    for (int i = 0; i < 4; ++i) prop("rot_" + std::to_string(i));
    h += "end_header\n";
    if (std::fwrite(h.data(), 1, h.size(), f.f) != h.size()) throw RuntimeError("ply: write failed");
    const size_t row_floats = 6 + 3 + 3 * static_cast<size_t>(Kw) + 1 + 3 + 4;
    // rows in chunks: one fwrite per 16K rows
    constexpr int64_t kChunk = 1 << 14;
    std::vector<float> buf(row_floats * kChunk);
    for (int64_t r0 = 0; r0 < c.count; r0 += kChunk) {
        const int64_t n = std::min<int64_t>(kChunk, c.count - r0);
        for (int64_t j = 0; j < n; ++j) {
            const int64_t i = r0 + j;
            float* row = buf.data() + j * row_floats;
            size_t p = 0;
            for (int k = 0; k < 3; ++k) row[p++] = c.means[i * 3 + k];
            for (int k = 0; k < 3; ++k) row[p++] = 0.0f;
            for (int k = 0; k < 3; ++k) row[p++] = c.sh0[i * 3 + k];
            for (int ch = 0; ch < 3; ++ch)
                for (int k = 0; k < Kw; ++k) row[p++] = k < K ? c.shN[(i * K + k) * 3 + ch] : 0.0f;
            row[p++] = c.opacities[i];
            for (int k = 0; k < 3; ++k) row[p++] = c.scales[i * 3 + k];
            for (int k = 0; k < 4; ++k) row[p++] = c.quats[i * 4 + k];
        }
        const size_t nf = row_floats * static_cast<size_t>(n);
        if (std::fwrite(buf.data(), 4, nf, f.f) != nf) throw RuntimeError("ply: write failed");
    }
}

namespace {

struct PlyHeader {
    int64_t count = 0;
    int degree = 0;
    std::vector<std::string> props;
    long body = 0;  // byte offset of the first row
};

PlyHeader ply_header(FILE* f) {
    PlyHeader ph;
    char line[512];
    bool binary_le = false;
    for (;;) {
        if (!std::fgets(line, sizeof(line), f)) throw RuntimeError("ply: bad header");
        std::string s(line);
        while (!s.empty() && (s.back() == '\n' || s.back() == '\r')) s.pop_back();
        if (s == "end_header") break;
        if (s.rfind("format ", 0) == 0) {
            binary_le = s == "format binary_little_endian 1.0";
        } else if (s.rfind("element vertex ", 0) == 0) {
            ph.count = std::stoll(s.substr(15));
        } else if (s.rfind("property float ", 0) == 0) {
            ph.props.push_back(s.substr(15));
        } else if (s.rfind("property ", 0) == 0) {
            throw RuntimeError("ply: only float properties supported (found: " + s + ")");
        }
    }
    if (!binary_le) throw RuntimeError("ply: only binary_little_endian supported");
    if (ph.count < 0) throw RuntimeError("ply: negative vertex count");
    int rest = 0;
    std::map<std::string, size_t> idx;
    for (size_t i = 0; i < ph.props.size(); ++i) idx[ph.props[i]] = i;
    while (idx.count("f_rest_" + std::to_string(rest))) ++rest;
    if (rest % 3 != 0) throw RuntimeError("ply: f_rest not divisible by 3");
    ph.degree = -1;
    for (int d = 0; d <= 4; ++d)
        if (rest_coeffs(d) == rest / 3) ph.degree = d;
    if (ph.degree < 0) throw RuntimeError("ply: unsupported f_rest count " + std::to_string(rest));
    ph.body = std::ftell(f);
    return ph;
}

}  // namespace

void ply_info(const char* path, int64_t* count, int32_t* degree) {
    if (!path) throw_invalid("ply_info", "null path");
    File f(path, "rb");
    if (!f.f) throw RuntimeError(std::string("ply: cannot open ") + path);
    const PlyHeader ph = ply_header(f.f);
    if (count) *count = ph.count;
    if (degree) *degree = ph.degree;
}

void ply_read(const char* path, const SxCloud& out) {
    if (!path) throw_invalid("ply_read", "null path");
    File f(path, "rb");
    if (!f.f) throw RuntimeError(std::string("ply: cannot open ") + path);
    const PlyHeader ph = ply_header(f.f);
    if (ph.degree > 3) throw RuntimeError("ply: SH degree 4 is outside the training path (0..3)");
    if (out.count != ph.count || out.sh_degree != ph.degree)
        throw_invalid("ply_read", "cloud buffers sized for another count / degree (ply_info first)");
    const int K = rest_coeffs(ph.degree);
    if (ph.count > 0 && (!out.means || !out.scales || !out.quats || !out.opacities || !out.sh0 ||
                         (K && !out.shN)))
        throw_invalid("ply_read", "null cloud array");
    std::map<std::string, size_t> idx;
    for (size_t i = 0; i < ph.props.size(); ++i) idx[ph.props[i]] = i;
    auto col = [&](const std::string& n) -> size_t {
        auto it = idx.find(n);
        if (it == idx.end()) throw RuntimeError("ply: missing property " + n);
        return it->second;
    };
    size_t cm[3], cdc[3], csc[3], crot[4];
    for (int k = 0; k < 3; ++k) {
        cm[k] = col(k == 0 ? "x" : k == 1 ? "y" : "z");
        cdc[k] = col("f_dc_" + std::to_string(k));
        csc[k] = col("scale_" + std::to_string(k));
    }
    for (int k = 0; k < 4; ++k) crot[k] = col("rot_" + std::to_string(k));
    const size_t cop = col("opacity");
    std::vector<size_t> crest(static_cast<size_t>(3 * K));
    for (int ch = 0; ch < 3; ++ch)
        for (int k = 0; k < K; ++k) crest[ch * K + k] = col("f_rest_" + std::to_string(ch * K + k));
    const size_t nprop = ph.props.size();
    constexpr int64_t kChunk = 1 << 14;
    std::vector<float> buf(nprop * kChunk);
    for (int64_t r0 = 0; r0 < ph.count; r0 += kChunk) {
        const int64_t n = std::min<int64_t>(kChunk, ph.count - r0);
        const size_t nf = nprop * static_cast<size_t>(n);
        if (std::fread(buf.data(), 4, nf, f.f) != nf) throw RuntimeError("ply: truncated body");
        for (int64_t j = 0; j < n; ++j) {
            const int64_t i = r0 + j;
            const float* row = buf.data() + j * nprop;
            for (int k = 0; k < 3; ++k) {
                out.means[i * 3 + k] = row[cm[k]];
                out.sh0[i * 3 + k] = row[cdc[k]];
                out.scales[i * 3 + k] = row[csc[k]];
            }
            for (int ch = 0; ch < 3; ++ch)
                for (int k = 0; k < K; ++k) out.shN[(i * K + k) * 3 + ch] = row[crest[ch * K + k]];
            out.opacities[i] = row[cop];
            for (int k = 0; k < 4; ++k) out.quats[i * 4 + k] = row[crot[k]];
        }
    }
}

void filter_for_export(const SxCloud& c, float min_opacity, uint8_t* keep, SxExportFilterStats& st) {
    if (c.count < 0) throw_invalid("filter_for_export", "negative count");
    const int64_t K3 = 3 * static_cast<int64_t>(rest_coeffs(c.sh_degree));
    if (c.count > 0 && (!c.means || !c.scales || !c.quats || !c.opacities || !c.sh0 ||
                        (K3 && !c.shN) || !keep))
        throw_invalid("filter_for_export", "null cloud array / keep mask");
    st = SxExportFilterStats{};
    st.input = c.count;
    for (int64_t i = 0; i < c.count; ++i) {
        bool finite = true;
        for (int k = 0; k < 3 && finite; ++k)
            finite = std::isfinite(c.means[i * 3 + k]) && std::isfinite(c.scales[i * 3 + k]) &&
                     std::isfinite(c.sh0[i * 3 + k]);
        for (int k = 0; k < 4 && finite; ++k) finite = std::isfinite(c.quats[i * 4 + k]);
        finite = finite && std::isfinite(c.opacities[i]);
        for (int64_t k = 0; k < K3 && finite; ++k) finite = std::isfinite(c.shN[i * K3 + k]);
        if (!finite) {
            keep[i] = 0;
            ++st.removed_nonfinite;
        } else if (!(sigmoid_host(c.opacities[i]) > min_opacity)) {
            keep[i] = 0;
            ++st.removed_low_opacity;
        } else {
            keep[i] = 1;
            ++st.kept;
        }
    }
}

}  // namespace sx
