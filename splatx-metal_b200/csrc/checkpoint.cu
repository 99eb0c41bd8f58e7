// checkpoint.cu — SXCK checkpoints of the resident arena (replaces the reference's
// save_checkpoint_file / load_checkpoint_file / load_checkpoint_header / verify_checkpoint_config,
// Sources/SplatXCore/Checkpoint.cpp and the format contract in Checkpoint.h:1-60).
//
// Format (little endian): "SXCK", version u32 = 1, flags u32 (bit 0 = fp16); the config
// fingerprint field by field (sh_degree, factor, test_split, total_iters i32; mcmc_enabled,
// antialiased, two reserved zero bytes u8; cap_max i64; mcmc_seed u64; scene_scale, ssim_weight
// f32); iter i32; alive count i64; the mt19937_64 text state (u64 length + bytes); then the six
// parameter groups (D3 order, count rows each, row-major) and per group exp_avg then exp_avg_sq.
// fp16 stores IEEE half (round to nearest even, finite values clamped to +-65504) and exp_avg_sq
// as half(sqrt(v)); loading squares it back and zeroes exp_avg wherever exp_avg_sq came back 0.
// The file is written to path + ".tmp", flushed, fsync'd, renamed over path, and the directory is
// fsync'd (best effort).
//
// B200 shape: rows leave the tiled arena through the 64K-row staging buffer; the fp16 conversion
// (and sqrt / square) runs on the device, so an fp16 checkpoint crosses PCIe at 2 bytes per value.
#include <cuda_fp16.h>
#include <fcntl.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

constexpr char kMagic[4] = {'S', 'X', 'C', 'K'};
constexpr uint32_t kVersion = 1;
constexpr uint32_t kFlagFp16 = 1u;

__global__ void to_half_kernel(const float* __restrict__ in, __half* __restrict__ out, int64_t n,
                               bool sqrt_first) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= n) return;
    float x = in[i];
    if (sqrt_first) x = sqrtf(x);
    if (x > 65504.0f) x = 65504.0f;
    else if (x < -65504.0f) x = -65504.0f;  // NaN passes through
    out[i] = __float2half_rn(x);
}

__global__ void from_half_kernel(const __half* __restrict__ in, float* __restrict__ out, int64_t n,
                                 bool square) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= n) return;
    const float v = __half2float(in[i]);
    out[i] = square ? v * v : v;
}

// exp_avg = 0 wherever exp_avg_sq is 0 (rows [0, n) of one tiled group)
__global__ void pair_zero_kernel(float* __restrict__ m, const float* __restrict__ v, int64_t n_floats) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= n_floats) return;
    if (v[i] == 0.0f) m[i] = 0.0f;
}

struct File {
    FILE* f = nullptr;
    File(const std::string& p, const char* mode) : f(std::fopen(p.c_str(), mode)) {
        if (!f) throw RuntimeError("checkpoint: cannot open " + p);
    }
    ~File() {
        if (f) std::fclose(f);
    }
};

void wbytes(FILE* f, const void* p, size_t n) {
    if (n && std::fwrite(p, 1, n, f) != n) throw RuntimeError("checkpoint: write failed");
}
template <typename T>
void wpod(FILE* f, T v) {
    wbytes(f, &v, sizeof(T));
}
void rbytes(FILE* f, void* p, size_t n) {
    if (n && std::fread(p, 1, n, f) != n) throw RuntimeError("checkpoint: truncated file (short read)");
}
template <typename T>
T rpod(FILE* f) {
    T v;
    rbytes(f, &v, sizeof(T));
    return v;
}

int64_t group_dim(int g, int deg) {
    constexpr int64_t fixed[5] = {3, 4, 3, 1, 3};
    return g < 5 ? fixed[g] : (static_cast<int64_t>(deg) + 1) * (deg + 1) * 3 - 3;
}

struct Pinned {
    void* p = nullptr;
    explicit Pinned(size_t bytes) { cuda_check(cudaMallocHost(&p, bytes), "checkpoint pinned buffer"); }
    ~Pinned() {
        if (p) cudaFreeHost(p);
    }
};

SxCheckpointHeader read_header(FILE* f, const std::string& path) {
    char magic[4];
    rbytes(f, magic, 4);
    if (std::memcmp(magic, kMagic, 4) != 0)
        throw RuntimeError("checkpoint: bad magic (not a splatx checkpoint): " + path);
    SxCheckpointHeader h{};
    h.version = rpod<uint32_t>(f);
    if (h.version != kVersion)
        throw RuntimeError("checkpoint: unsupported version " + std::to_string(h.version) +
                           " (expected " + std::to_string(kVersion) + ")");
    const uint32_t flags = rpod<uint32_t>(f);
    if (flags & ~kFlagFp16) throw RuntimeError("checkpoint: unknown flags");
    h.fp16 = (flags & kFlagFp16) ? 1 : 0;
    SxCheckpointConfig& c = h.config;
    c.sh_degree = rpod<int32_t>(f);
    c.factor = rpod<int32_t>(f);
    c.test_split = rpod<int32_t>(f);
    c.total_iters = rpod<int32_t>(f);
    c.mcmc_enabled = rpod<uint8_t>(f);
    c.antialiased = rpod<uint8_t>(f);
    if (rpod<uint8_t>(f) != 0)
        throw RuntimeError("checkpoint: bilateral grid checkpoints are no longer supported "
                           "(feature removed): " + path);
    (void)rpod<uint8_t>(f);
    c.cap_max = rpod<int64_t>(f);
    c.mcmc_seed = rpod<uint64_t>(f);
    c.scene_scale = rpod<float>(f);
    c.ssim_weight = rpod<float>(f);
    if (c.sh_degree < 0 || c.sh_degree > 3) throw RuntimeError("checkpoint: sh_degree out of [0,3]");
    h.iter = rpod<int32_t>(f);
    if (h.iter < 0) throw RuntimeError("checkpoint: negative iter");
    h.alive_count = rpod<int64_t>(f);
    if (h.alive_count < 1 || h.alive_count > (int64_t{1} << 33))
        throw RuntimeError("checkpoint: invalid count");
    return h;
}

[[noreturn]] void mismatch(const char* field, const std::string& saved, const std::string& cur,
                           const char* extra = nullptr) {
    std::string m = std::string("checkpoint resume: ") + field + " mismatch (saved " + saved +
                    ", current " + cur + ")";
    if (extra) m += std::string(" — ") + extra;
    throw RuntimeError(m);
}

std::string fstr(float v) {
    char b[32];
    std::snprintf(b, sizeof(b), "%.9g", static_cast<double>(v));
    return b;
}

}  // namespace

void checkpoint_verify(const SxCheckpointConfig& s, const SxCheckpointConfig& c) {
    if (s.sh_degree != c.sh_degree)
        mismatch("sh_degree", std::to_string(s.sh_degree), std::to_string(c.sh_degree),
                 "resume enforces fixed SH degree (the SH arrays would misalign)");
    if (s.mcmc_enabled != c.mcmc_enabled)
        mismatch("mcmc", s.mcmc_enabled ? "on" : "off", c.mcmc_enabled ? "on" : "off");
    if (s.cap_max != c.cap_max) mismatch("cap_max", std::to_string(s.cap_max), std::to_string(c.cap_max));
    if (s.mcmc_seed != c.mcmc_seed)
        mismatch("mcmc seed", std::to_string(s.mcmc_seed), std::to_string(c.mcmc_seed),
                 "noise(Philox key)/multinomial stream would diverge");
    if (s.factor != c.factor) mismatch("factor", std::to_string(s.factor), std::to_string(c.factor));
    if (s.test_split != c.test_split)
        mismatch("test_split", std::to_string(s.test_split), std::to_string(c.test_split),
                 "train view stream (it % n_train) would diverge and trained views would leak "
                 "into the test split");
    if (s.total_iters != c.total_iters)
        mismatch("total_iters", std::to_string(s.total_iters), std::to_string(c.total_iters),
                 "ratio schedules (lr decay/SH promotion/refine) are normalized by total_iters — "
                 "resume iter would change meaning");
    if (s.scene_scale != c.scene_scale) mismatch("scene_scale", fstr(s.scene_scale), fstr(c.scene_scale));
    if (s.ssim_weight != c.ssim_weight) mismatch("ssim_weight", fstr(s.ssim_weight), fstr(c.ssim_weight));
    if (s.antialiased != c.antialiased)
        mismatch("antialiased", s.antialiased ? "on" : "off", c.antialiased ? "on" : "off");
}

void checkpoint_header(const char* path, SxCheckpointHeader& out) {
    if (!path) throw_invalid("checkpoint_info", "null path");
    File file(path, "rb");
    out = read_header(file.f, path);
}

void checkpoint_save(const ArenaView& a, float* stage, int64_t stage_rows,
                     const SxCheckpointConfig& cfg, int32_t iter, int64_t count,
                     const std::string& rng_state, const char* path_c, bool fp16) {
    if (!path_c) throw_invalid("save_checkpoint", "null path");
    if (count < 1 || count > a.rows) throw_invalid("save_checkpoint", "count out of [1, arena_rows]");
    if (iter < 0) throw_invalid("save_checkpoint", "negative iter");
    const int deg = cfg.sh_degree;
    if (deg < 0 || deg > 3 || group_dim(5, deg) != a.dims[5])
        throw_invalid("save_checkpoint", "config sh_degree differs from the executor's");
    const std::string path(path_c), tmp = path + ".tmp";
    cudaStream_t s = a.stream;
    Pinned host(static_cast<size_t>(stage_rows) * 45 * sizeof(float));
    __half* half_dev = nullptr;
    if (fp16) cuda_check(cudaMallocAsync(&half_dev, sizeof(__half) * stage_rows * 45, s), "checkpoint");
    try {
        File file(tmp, "wb");
        FILE* f = file.f;
        wbytes(f, kMagic, 4);
        wpod<uint32_t>(f, kVersion);
        wpod<uint32_t>(f, fp16 ? kFlagFp16 : 0u);
        wpod<int32_t>(f, cfg.sh_degree);
        wpod<int32_t>(f, cfg.factor);
        wpod<int32_t>(f, cfg.test_split);
        wpod<int32_t>(f, cfg.total_iters);
        wpod<uint8_t>(f, cfg.mcmc_enabled);
        wpod<uint8_t>(f, cfg.antialiased);
        wpod<uint8_t>(f, 0);
        wpod<uint8_t>(f, 0);
        wpod<int64_t>(f, cfg.cap_max);
        wpod<uint64_t>(f, cfg.mcmc_seed);
        wpod<float>(f, cfg.scene_scale);
        wpod<float>(f, cfg.ssim_weight);
        wpod<int32_t>(f, iter);
        wpod<int64_t>(f, count);
        wpod<uint64_t>(f, static_cast<uint64_t>(rng_state.size()));
        wbytes(f, rng_state.data(), rng_state.size());
        // params x6, then per group exp_avg and exp_avg_sq (sqrt-compressed in fp16)
        auto dump = [&](const float* tiles, int d, bool sqrt_first) {
            for (int64_t r0 = 0; r0 < count; r0 += stage_rows) {
                const int64_t m = std::min<int64_t>(stage_rows, count - r0);
                const int64_t nf = m * d;
                launch_tiles_to_rows(tiles, stage, d, m, r0, s);
                if (fp16) {
                    SX_LAUNCH(to_half_kernel, blocks_for(nf, 256), 256, 0, s, stage, half_dev, nf,
                              sqrt_first);
                    cuda_check(cudaMemcpyAsync(host.p, half_dev, sizeof(__half) * nf,
                                               cudaMemcpyDeviceToHost, s), "checkpoint d2h");
                } else {
                    cuda_check(cudaMemcpyAsync(host.p, stage, sizeof(float) * nf,
                                               cudaMemcpyDeviceToHost, s), "checkpoint d2h");
                }
                cuda_check(cudaStreamSynchronize(s), "checkpoint d2h");
                wbytes(f, host.p, (fp16 ? sizeof(__half) : sizeof(float)) * nf);
            }
        };
        for (int g = 0; g < 6; ++g)
            if (a.dims[g]) dump(a.p[g], a.dims[g], false);
        for (int g = 0; g < 6; ++g)
            if (a.dims[g]) {
                dump(a.m[g], a.dims[g], false);
                dump(a.v[g], a.dims[g], true);
            }
        if (std::fflush(f) != 0) throw RuntimeError("checkpoint: fflush failed for " + tmp);
        if (::fsync(::fileno(f)) != 0) throw RuntimeError("checkpoint: fsync failed for " + tmp);
        const int rc = std::fclose(f);
        file.f = nullptr;
        if (rc != 0) throw RuntimeError("checkpoint: close/flush failed for " + tmp);
    } catch (...) {
        if (half_dev) cudaFreeAsync(half_dev, s);
        std::remove(tmp.c_str());
        throw;
    }
    if (half_dev) cuda_check(cudaFreeAsync(half_dev, s), "checkpoint");
    if (std::rename(tmp.c_str(), path.c_str()) != 0) {
        std::remove(tmp.c_str());
        throw RuntimeError("checkpoint: rename failed: " + tmp + " -> " + path);
    }
    std::string dir = ".";
    const size_t slash = path.find_last_of('/');
    if (slash != std::string::npos) dir = slash == 0 ? "/" : path.substr(0, slash);
    const int dfd = ::open(dir.c_str(), O_RDONLY);
    if (dfd >= 0) {
        (void)::fsync(dfd);
        (void)::close(dfd);
    }
}

void checkpoint_load(const ArenaView& a, float* stage, int64_t stage_rows, const char* path_c,
                     const SxCheckpointConfig* current, SxCheckpointHeader& out,
                     std::string& rng_state) {
    if (!path_c) throw_invalid("load_checkpoint", "null path");
    const std::string path(path_c);
    File file(path, "rb");
    FILE* f = file.f;
    const SxCheckpointHeader h = read_header(f, path);
    if (current) checkpoint_verify(h.config, *current);
    const int deg = h.config.sh_degree;
    if (group_dim(5, deg) != a.dims[5])
        throw_invalid("load_checkpoint", "the checkpoint's SH degree differs from the executor's");
    if (h.alive_count > a.rows)
        throw_invalid("load_checkpoint", "the checkpoint holds more rows than the executor's arena");
    const uint64_t rng_len = rpod<uint64_t>(f);
    if (rng_len > (1u << 20)) throw RuntimeError("checkpoint: rng state too large");
    rng_state.assign(static_cast<size_t>(rng_len), '\0');
    rbytes(f, rng_state.empty() ? nullptr : &rng_state[0], rng_state.size());
    const bool fp16 = h.fp16 != 0;
    const int64_t count = h.alive_count;
    cudaStream_t s = a.stream;
    // The body must be exactly the header's count x (params, exp_avg, exp_avg_sq) of every group:
    // checked against the file size before the arena is touched, so a truncated or padded file
    // fails here and leaves the executor's state as it was.
    {
        int64_t floats_per_row = 0;
        for (int g = 0; g < 6; ++g) floats_per_row += a.dims[g];
        const int64_t want = count * floats_per_row * 3 *
                             static_cast<int64_t>(fp16 ? sizeof(__half) : sizeof(float));
        const long pos = std::ftell(f);
        if (pos < 0 || std::fseek(f, 0, SEEK_END) != 0) throw RuntimeError("checkpoint: seek failed: " + path);
        const long end = std::ftell(f);
        if (end < 0 || std::fseek(f, pos, SEEK_SET) != 0) throw RuntimeError("checkpoint: seek failed: " + path);
        if (static_cast<int64_t>(end - pos) != want)
            throw RuntimeError("checkpoint: body holds " + std::to_string(end - pos) + " bytes, the header implies " +
                               std::to_string(want) + " (truncated or corrupt): " + path);
    }
    // the arena tail (rows >= count) is zero after a load, as in a fresh arena
    const int64_t padded = (a.rows + 31) / 32 * 32;
    for (int g = 0; g < 6; ++g) {
        if (!a.dims[g]) continue;
        const size_t bytes = sizeof(float) * static_cast<size_t>(padded) * a.dims[g];
        cuda_check(cudaMemsetAsync(a.p[g], 0, bytes, s), "checkpoint zero");
        cuda_check(cudaMemsetAsync(a.m[g], 0, bytes, s), "checkpoint zero");
        cuda_check(cudaMemsetAsync(a.v[g], 0, bytes, s), "checkpoint zero");
    }
    Pinned host(static_cast<size_t>(stage_rows) * 45 * sizeof(float));
    __half* half_dev = nullptr;
    if (fp16) cuda_check(cudaMallocAsync(&half_dev, sizeof(__half) * stage_rows * 45, s), "checkpoint");
    try {
        auto fill = [&](float* tiles, int d, bool square) {
            for (int64_t r0 = 0; r0 < count; r0 += stage_rows) {
                const int64_t m = std::min<int64_t>(stage_rows, count - r0);
                const int64_t nf = m * d;
                cuda_check(cudaStreamSynchronize(s), "checkpoint h2d");  // host buffer reuse
                rbytes(f, host.p, (fp16 ? sizeof(__half) : sizeof(float)) * nf);
                if (fp16) {
                    cuda_check(cudaMemcpyAsync(half_dev, host.p, sizeof(__half) * nf,
                                               cudaMemcpyHostToDevice, s), "checkpoint h2d");
                    SX_LAUNCH(from_half_kernel, blocks_for(nf, 256), 256, 0, s, half_dev, stage, nf,
                              square);
                } else {
                    cuda_check(cudaMemcpyAsync(stage, host.p, sizeof(float) * nf,
                                               cudaMemcpyHostToDevice, s), "checkpoint h2d");
                }
                launch_rows_to_tiles(stage, tiles, d, m, r0, s);
            }
        };
        for (int g = 0; g < 6; ++g)
            if (a.dims[g]) fill(a.p[g], a.dims[g], false);
        for (int g = 0; g < 6; ++g) {
            if (!a.dims[g]) continue;
            fill(a.m[g], a.dims[g], false);
            fill(a.v[g], a.dims[g], true);
            if (fp16) {
                const int64_t nf = padded * a.dims[g];
                SX_LAUNCH(pair_zero_kernel, blocks_for(nf, 256), 256, 0, s, a.m[g], a.v[g], nf);
            }
        }
        if (std::fgetc(f) != EOF) throw RuntimeError("checkpoint: trailing bytes (corrupt or size mismatch)");
        cuda_check(cudaStreamSynchronize(s), "checkpoint load");
    } catch (...) {
        cudaStreamSynchronize(s);
        if (half_dev) cudaFreeAsync(half_dev, s);
        throw;
    }
    if (half_dev) cuda_check(cudaFreeAsync(half_dev, s), "checkpoint");
    cuda_check(cudaStreamSynchronize(s), "checkpoint load");
    out = h;
}

}  // namespace sx
