// spz.cu — Niantic SPZ files (host code; replaces save_spz / load_spz, Sources/SplatXCore/SpzIO.cpp,
// which wrap the vendored spz library v2.1.0, ThirdParty/spz/src/cc/load-spz.cc).
//
// The format (version 3 written; 1..3 read): a gzip stream (zlib deflate, default level, window
// 15 + gzip wrapper, memLevel 9) of a 16-byte header {magic "NGSP" as u32 0x5053474e, version,
// point count (u32), SH degree, fractional bits (12), flags (bit 0 antialiased), reserved} and the
// planar attribute blocks in the order positions, alphas, colours, scales, rotations, SH:
//   position   24-bit two's-complement fixed point, round(v * 2^12)        (v1: half floats)
//   alpha      u8 round(sigmoid(logit) * 255)
//   colour     u8 round(sh0 * 0.15 * 255 + 127.5)
//   scale      u8 round((log_scale + 10) * 16)
//   rotation   32-bit "smallest three": index of the largest |component| in the top 2 bits, the
//              other three as sign + 9-bit magnitude of |q| / sqrt(1/2) in [0, 511], largest made
//              positive                                                  (v1, v2: u8 x, y, z)
//   SH         u8 round(x * 128) + 128 snapped to buckets of 8 (degree 1) or 16 (higher bands)
// all u8 values clamped to [0, 255]. The training world is the PLY's right-down-front frame and the
// file stores right-up-back: y and z of positions, the quaternion's x-axis-preserving flips and
// the SH coefficients whose basis functions are odd in y or z change sign. Loading inverts every
// step; the opacity logits of the saturated bytes 0 / 255 are clamped to +-ln(509). Saving applies
// the export filter first (non-finite rows, then sigmoid(opacity) <= min_opacity).
#include <zlib.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

constexpr uint32_t kMagic = 0x5053474e;
constexpr float kColorScale = 0.15f;
constexpr float kSqrt1_2 = 0.707106781186547524401f;
constexpr float kOpacityLogitLimit = 6.2324481f;  // ln(509)

// right-down-front <-> right-up-back: x kept, y and z flipped
constexpr float kFlipP[3] = {1.0f, -1.0f, -1.0f};
constexpr float kFlipQ[3] = {1.0f, -1.0f, -1.0f};  // (y z, x z, x y)
// SH basis functions in degree order: sign of each under (x, -y, -z)
constexpr float kFlipSh[15] = {-1.0f, -1.0f, 1.0f, -1.0f, 1.0f, 1.0f, -1.0f, 1.0f,
                               -1.0f, 1.0f,  -1.0f, -1.0f, 1.0f, -1.0f, 1.0f};

int sh_dim(int degree) { return degree == 1 ? 3 : degree == 2 ? 8 : degree == 3 ? 15 : 0; }

uint8_t to_u8(float x) { return static_cast<uint8_t>(std::min(std::max(std::round(x), 0.0f), 255.0f)); }

uint8_t quantize_sh(float x, int bucket) {
    int q = static_cast<int>(std::round(x * 128.0f) + 128.0f);
    q = (q + bucket / 2) / bucket * bucket;
    return static_cast<uint8_t>(std::min(std::max(q, 0), 255));
}

// q = (x, y, z, w)
void pack_rotation(uint8_t out[4], const float q_in[4]) {
    const float n = std::sqrt(q_in[0] * q_in[0] + q_in[1] * q_in[1] + q_in[2] * q_in[2] + q_in[3] * q_in[3]);
    float q[4] = {q_in[0] / n, q_in[1] / n, q_in[2] / n, q_in[3] / n};
    for (int i = 0; i < 3; ++i) q[i] *= kFlipQ[i];
    unsigned big = 0;
    for (unsigned i = 1; i < 4; ++i)
        if (std::fabs(q[i]) > std::fabs(q[big])) big = i;
    const unsigned negate = q[big] < 0;
    uint32_t comp = big;
    for (unsigned i = 0; i < 4; ++i) {
        if (i == big) continue;
        const uint32_t neg = (q[i] < 0) ^ negate;
        const uint32_t mag = static_cast<uint32_t>(511.0f * (std::fabs(q[i]) / kSqrt1_2) + 0.5f);
        comp = (comp << 10u) | (neg << 9u) | mag;
    }
    for (int b = 0; b < 4; ++b) out[b] = static_cast<uint8_t>((comp >> (8 * b)) & 0xff);
}

void unpack_rotation3(float r[4], const uint8_t b[4]) {  // (x, y, z, w)
    uint32_t comp = b[0] + (b[1] << 8) + (b[2] << 16) + (static_cast<uint32_t>(b[3]) << 24);
    const uint32_t mask = 511u;
    const int big = static_cast<int>(comp >> 30);
    float ss = 0.0f;
    for (int i = 3; i >= 0; --i) {
        if (i == big) continue;
        const uint32_t mag = comp & mask, neg = (comp >> 9u) & 1u;
        comp >>= 10u;
        r[i] = kSqrt1_2 * static_cast<float>(mag) / static_cast<float>(mask);
        if (neg) r[i] = -r[i];
        ss += r[i] * r[i];
    }
    r[big] = std::sqrt(1.0f - ss);
}

void unpack_rotation_first3(float r[4], const uint8_t b[3]) {
    float ss = 0.0f;
    for (int i = 0; i < 3; ++i) {
        r[i] = static_cast<float>(b[i]) * (1.0f / 127.5f) + -1.0f;
        ss += r[i] * r[i];
    }
    r[3] = std::sqrt(std::max(0.0f, 1.0f - ss));
}

float half_to_float(uint16_t h) {
    const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    float v;
    if (exp == 0) v = std::ldexp(static_cast<float>(man), -24);
    else if (exp == 31) v = man ? NAN : INFINITY;
    else v = std::ldexp(static_cast<float>(man | 0x400u), static_cast<int>(exp) - 25);
    return sign ? -v : v;
}

std::vector<uint8_t> gzip(const std::vector<uint8_t>& in) {
    z_stream s{};
    if (deflateInit2(&s, Z_DEFAULT_COMPRESSION, Z_DEFLATED, 16 + MAX_WBITS, 9, Z_DEFAULT_STRATEGY) != Z_OK)
        throw RuntimeError("spz: deflate init failed");
    std::vector<uint8_t> out, buf(8192);
    out.reserve(in.size() / 4);
    s.next_in = const_cast<Bytef*>(in.data());
    s.avail_in = static_cast<uInt>(in.size());
    for (;;) {
        s.next_out = buf.data();
        s.avail_out = static_cast<uInt>(buf.size());
        const int r = deflate(&s, Z_FINISH);
        if (r != Z_OK && r != Z_STREAM_END) {
            deflateEnd(&s);
            throw RuntimeError("spz: deflate failed");
        }
        out.insert(out.end(), buf.data(), buf.data() + (buf.size() - s.avail_out));
        if (r == Z_STREAM_END) break;
    }
    deflateEnd(&s);
    return out;
}

std::vector<uint8_t> gunzip(const std::vector<uint8_t>& in) {
    z_stream s{};
    if (inflateInit2(&s, 16 | MAX_WBITS) != Z_OK) throw RuntimeError("spz: inflate init failed");
    std::vector<uint8_t> out, buf(8192);
    s.next_in = const_cast<Bytef*>(in.data());
    s.avail_in = static_cast<uInt>(in.size());
    for (;;) {
        s.next_out = buf.data();
        s.avail_out = static_cast<uInt>(buf.size());
        const int r = inflate(&s, Z_NO_FLUSH);
        if (r != Z_OK && r != Z_STREAM_END) {
            inflateEnd(&s);
            throw RuntimeError("spz: not a gzip stream or corrupt");
        }
        out.insert(out.end(), buf.data(), buf.data() + (buf.size() - s.avail_out));
        if (r == Z_STREAM_END) break;
        if (s.avail_in == 0 && s.avail_out != 0) {
            inflateEnd(&s);
            throw RuntimeError("spz: truncated gzip stream");
        }
    }
    inflateEnd(&s);
    return out;
}

}  // namespace

void spz_write(const SxCloud& in, const char* path, float min_opacity, bool antialiased,
               SxExportFilterStats& st) {
    if (!path) throw_invalid("spz_write", "null path");
    if (in.sh_degree < 0 || in.sh_degree > 3)
        throw_invalid("spz_write", "unsupported sh_degree " + std::to_string(in.sh_degree) + " (0..3 only)");
    std::vector<uint8_t> keep(static_cast<size_t>(std::max<int64_t>(in.count, 1)));
    filter_for_export(in, min_opacity, keep.data(), st);
    if (st.kept > 0x7fffffff) throw_invalid("spz_write", "count exceeds int32 numPoints limit");
    const int64_t N = st.kept;
    const int K = sh_dim(in.sh_degree);
    const int64_t Kin = (in.sh_degree + 1) * (in.sh_degree + 1) - 1;  // == K for 0..3
    std::vector<uint8_t> raw(16 + N * (9 + 1 + 3 + 3 + 4 + 3 * K));
    const uint32_t hdr[3] = {kMagic, 3u, static_cast<uint32_t>(N)};
    std::memcpy(raw.data(), hdr, 12);
    raw[12] = static_cast<uint8_t>(in.sh_degree);
    raw[13] = 12;
    raw[14] = antialiased ? 1 : 0;
    raw[15] = 0;
    uint8_t* pos = raw.data() + 16;
    uint8_t* alpha = pos + N * 9;
    uint8_t* color = alpha + N;
    uint8_t* scale = color + N * 3;
    uint8_t* rot = scale + N * 3;
    uint8_t* sh = rot + N * 4;
    int64_t j = 0;
    for (int64_t i = 0; i < in.count; ++i) {
        if (!keep[i]) continue;
        for (int k = 0; k < 3; ++k) {
            const int32_t fx = static_cast<int32_t>(std::round(kFlipP[k] * in.means[i * 3 + k] * 4096.0f));
            uint8_t* p = pos + (j * 3 + k) * 3;
            p[0] = fx & 0xff;
            p[1] = (fx >> 8) & 0xff;
            p[2] = (fx >> 16) & 0xff;
            color[j * 3 + k] = to_u8(in.sh0[i * 3 + k] * (kColorScale * 255.0f) + (0.5f * 255.0f));
            scale[j * 3 + k] = to_u8((in.scales[i * 3 + k] + 10.0f) * 16.0f);
        }
        alpha[j] = to_u8(1.0f / (1.0f + std::exp(-in.opacities[i])) * 255.0f);
        const float q[4] = {in.quats[i * 4 + 1], in.quats[i * 4 + 2], in.quats[i * 4 + 3],
                            in.quats[i * 4 + 0]};
        pack_rotation(rot + j * 4, q);
        for (int k = 0; k < K; ++k) {
            const int bucket = k < 3 ? 8 : 16;
            for (int ch = 0; ch < 3; ++ch)
                sh[(j * K + k) * 3 + ch] =
                    quantize_sh(kFlipSh[k] * in.shN[(i * Kin + k) * 3 + ch], bucket);
        }
        ++j;
    }
    const std::vector<uint8_t> z = gzip(raw);
    FILE* f = std::fopen(path, "wb");
    if (!f) throw RuntimeError(std::string("spz: cannot write ") + path);
    const size_t w = std::fwrite(z.data(), 1, z.size(), f);
    const int rc = std::fclose(f);
    if (w != z.size() || rc != 0) throw RuntimeError(std::string("spz: cannot write ") + path);
}

namespace {

struct SpzPacked {
    uint32_t version = 0;
    int64_t n = 0;
    int degree = 0;
    int frac = 0;
    bool antialiased = false;
    std::vector<uint8_t> data;
    size_t pos = 0, alpha = 0, color = 0, scale = 0, rot = 0, sh = 0;
};

SpzPacked spz_parse(const char* path) {
    if (!path) throw_invalid("spz_read", "null path");
    FILE* f = std::fopen(path, "rb");
    if (!f) throw RuntimeError(std::string("spz: cannot load ") + path + " (missing)");
    std::vector<uint8_t> z;
    uint8_t buf[65536];
    size_t got;
    while ((got = std::fread(buf, 1, sizeof(buf), f)) > 0) z.insert(z.end(), buf, buf + got);
    std::fclose(f);
    SpzPacked p;
    p.data = gunzip(z);
    if (p.data.size() < 16) throw RuntimeError(std::string("spz: header not found in ") + path);
    uint32_t h[3];
    std::memcpy(h, p.data.data(), 12);
    if (h[0] != kMagic) throw RuntimeError(std::string("spz: header not found in ") + path);
    if (h[1] < 1 || h[1] > 3) throw RuntimeError("spz: version not supported: " + std::to_string(h[1]));
    if (h[2] > 10000000u) throw RuntimeError("spz: too many points: " + std::to_string(h[2]));
    p.version = h[1];
    p.n = h[2];
    p.degree = p.data[12];
    p.frac = p.data[13];
    p.antialiased = (p.data[14] & 1) != 0;
    if (p.degree > 3) throw RuntimeError("spz: unsupported SH degree " + std::to_string(p.degree));
    const int K = sh_dim(p.degree);
    const size_t pb = p.version == 1 ? 6 : 9, rb = p.version >= 3 ? 4 : 3;
    p.pos = 16;
    p.alpha = p.pos + p.n * pb;
    p.color = p.alpha + p.n;
    p.scale = p.color + p.n * 3;
    p.rot = p.scale + p.n * 3;
    p.sh = p.rot + p.n * rb;
    if (p.data.size() < p.sh + static_cast<size_t>(p.n) * K * 3)
        throw RuntimeError(std::string("spz: read error (truncated) in ") + path);
    if (p.n <= 0) throw RuntimeError(std::string("spz: cannot load ") + path + " (empty)");
    return p;
}

}  // namespace

void spz_info(const char* path, int64_t* count, int32_t* degree, int32_t* antialiased) {
    const SpzPacked p = spz_parse(path);
    if (count) *count = p.n;
    if (degree) *degree = p.degree;
    if (antialiased) *antialiased = p.antialiased ? 1 : 0;
}

void spz_read(const char* path, const SxCloud& out) {
    const SpzPacked p = spz_parse(path);
    if (out.count != p.n || out.sh_degree != p.degree)
        throw_invalid("spz_read", "cloud buffers sized for another count / degree (spz_info first)");
    const int K = sh_dim(p.degree);
    const uint8_t* d = p.data.data();
    const float inv = static_cast<float>(1.0 / (1 << p.frac));
    for (int64_t i = 0; i < p.n; ++i) {
        for (int k = 0; k < 3; ++k) {
            float v;
            if (p.version == 1) {
                uint16_t hb;
                std::memcpy(&hb, d + p.pos + (i * 3 + k) * 2, 2);
                v = half_to_float(hb);
            } else {
                const uint8_t* b = d + p.pos + (i * 3 + k) * 3;
                int32_t fx = b[0] | (b[1] << 8) | (b[2] << 16);
                if (fx & 0x800000) fx |= static_cast<int32_t>(0xff000000u);
                v = static_cast<float>(fx) * inv;
            }
            out.means[i * 3 + k] = v * kFlipP[k];
            out.scales[i * 3 + k] = d[p.scale + i * 3 + k] / 16.0f - 10.0f;
            out.sh0[i * 3 + k] = ((d[p.color + i * 3 + k] / 255.0f) - 0.5f) / kColorScale;
        }
        float r[4];
        if (p.version >= 3) unpack_rotation3(r, d + p.rot + i * 4);
        else unpack_rotation_first3(r, d + p.rot + i * 3);
        out.quats[i * 4 + 0] = r[3];
        for (int k = 0; k < 3; ++k) out.quats[i * 4 + 1 + k] = r[k] * kFlipQ[k];
        const float a = d[p.alpha + i] / 255.0f;
        const float logit = std::log(a / (1.0f - a));
        out.opacities[i] = std::min(std::max(logit, -kOpacityLogitLimit), kOpacityLogitLimit);
        for (int k = 0; k < K; ++k)
            for (int ch = 0; ch < 3; ++ch)
                out.shN[(i * K + k) * 3 + ch] =
                    ((static_cast<float>(d[p.sh + (i * K + k) * 3 + ch]) - 128.0f) / 128.0f) * kFlipSh[k];
    }
}

}  // namespace sx
