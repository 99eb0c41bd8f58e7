// mcmc.cu — MCMC refine on the device-resident arena (Trainer::mcmc_refine,
// Sources/SplatXCore/Trainer.cpp:1273-1435) without the reference's full parameter round trip
// (sync_host_for_mutation, Trainer.cpp:1275 and :959-967).
//
// Split between host and device:
//   host    the decisions: sigmoid of the opacity logits, dead/alive split, the mt19937_64
//           multinomial over a double CDF, bincount ratios, and the float exp/log around the
//           relocation kernel — the reference's own arithmetic, so the sampled indices are the
//           reference's indices for the same parameters and seed
//   device  the data: the opacity logits and the sampled rows' log-scales are read back (N + 3n
//           floats), the relocation kernel runs on the device, and the row surgery (source
//           updates, dead <- source and tail <- source row copies of all six groups, Adam row
//           zeroing) happens in place on the tiled arena.
// Per refine the host moves 4·N bytes of logits plus a few floats per sampled row, instead of
// downloading and re-uploading parameters and both moments (3 × 236 B per row at SH degree 3).
#include <algorithm>
#include <cmath>
#include <locale>
#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

// kMcmcNMax (Trainer.cpp:27): the upper bound of the relocation ratio and the binoms LUT side.
constexpr int kNMax = 51;

// sigmoid_f32 / logit_f32 (Trainer.cpp:430-436): float std::exp and std::log, as the reference.
inline float sigmoid_f32(float x) { return 1.0f / (1.0f + std::exp(-x)); }
inline float logit_f32(float p) {
    if (!(p > 0.0f && p < 1.0f)) throw std::invalid_argument("logit_f32: p must be in (0,1)");
    return std::log(p / (1.0f - p));
}

template <typename T>
struct Pinned {
    T* p = nullptr;
    size_t n = 0;
    void ensure(size_t c) {
        if (c <= n) return;
        if (p) cudaFreeHost(p);
        p = nullptr;
        n = 0;
        cuda_check(cudaMallocHost(&p, std::max<size_t>(c, 1) * sizeof(T)), "mcmc pinned buffer");
        n = c;
    }
    ~Pinned() {
        if (p) cudaFreeHost(p);
    }
};

template <typename T>
struct DevBuf {
    T* p = nullptr;
    size_t n = 0;
    void ensure(size_t c) {
        if (c <= n) return;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        cuda_check(cudaMalloc(&p, std::max<size_t>(c, 1) * sizeof(T)), "mcmc device buffer");
        n = c;
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
};

// Elementwise sigmoid over the logits on the host cores (deterministic: each value alone).
void sigmoid_all(const float* x, float* y, int64_t n) {
    const int64_t kMinPerThread = 1 << 16;
    const int hw = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
    const int T = static_cast<int>(std::min<int64_t>(std::min(hw, 16), (n + kMinPerThread - 1) / kMinPerThread));
    if (T <= 1) {
        for (int64_t i = 0; i < n; ++i) y[i] = sigmoid_f32(x[i]);
        return;
    }
    std::vector<std::thread> th;
    const int64_t chunk = (n + T - 1) / T;
    for (int t = 0; t < T; ++t) {
        const int64_t b = t * chunk, e = std::min(n, b + chunk);
        th.emplace_back([=] {
            for (int64_t i = b; i < e; ++i) y[i] = sigmoid_f32(x[i]);
        });
    }
    for (auto& t : th) t.join();
}

// multinomial_with_replacement (Trainer.cpp:1199-1217): torch.multinomial(replacement=True)
// semantics with a standard-fixed engine — a double CDF accumulated in index order, one draw
// u = (rng() >> 11) · 2^-53 · total per sample, the first CDF entry above u (an upper bound, so a
// zero weight is never chosen), clamped to the last index.
void multinomial(const float* w, int64_t n, int64_t n_samples, std::mt19937_64& rng,
                 std::vector<double>& cdf, std::vector<int64_t>& out) {
    cdf.resize(static_cast<size_t>(n));
    double acc = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        const float x = w[i];
        if (!(x >= 0.0f)) throw std::invalid_argument("multinomial: weights must be >= 0 and finite");
        acc += static_cast<double>(x);
        cdf[static_cast<size_t>(i)] = acc;
    }
    if (!(acc > 0.0)) throw std::invalid_argument("multinomial: weight sum must be > 0");
    out.resize(static_cast<size_t>(n_samples));
    for (int64_t j = 0; j < n_samples; ++j) {
        const double u = static_cast<double>(rng() >> 11) * 0x1.0p-53 * acc;
        const int64_t idx = std::upper_bound(cdf.begin(), cdf.end(), u) - cdf.begin();
        out[static_cast<size_t>(j)] = std::min(idx, n - 1);
    }
}

}  // namespace

struct McmcRefine {
    std::mt19937_64 rng{42};  // McmcOptions::seed default (Trainer.h:196)
    int device = -1;
    DevBuf<float> lut;  // binoms [kNMax, kNMax]
    DevBuf<int64_t> d_src, d_dst;
    DevBuf<int32_t> d_ratio;
    DevBuf<float> d_gls, d_gop, d_gsc, d_nop, d_nsc, d_logit, d_ls;
    Pinned<float> h_logits, h_gls, h_gop, h_gsc, h_nop, h_nsc, h_logit, h_ls;
    Pinned<int64_t> h_src, h_dst;
    Pinned<int32_t> h_ratio;
    std::vector<float> op_act;
    std::vector<double> cdf;
    std::vector<int32_t> counts;  // bincount scratch, all zero between uses
    std::vector<int64_t> dead, alive, local, sampled;
    std::vector<float> probs;

    void ensure_lut(int dev, cudaStream_t s) {
        if (lut.p && device == dev) return;
        device = dev;
        std::vector<float> h(static_cast<size_t>(kNMax) * kNMax);
        // Pascal's rows in exact 64-bit integers, one float cast each (make_binoms_lut,
        // CpuKernels.cpp:906-917)
        std::vector<uint64_t> row(kNMax, 0);
        for (int n = 0; n < kNMax; ++n) {
            for (int k = n; k >= 1; --k) row[k] += row[k - 1];
            row[0] = 1;
            for (int k = 0; k < kNMax; ++k)
                h[static_cast<size_t>(n) * kNMax + k] = k <= n ? static_cast<float>(row[k]) : 0.0f;
        }
        lut.n = 0;
        if (lut.p) cudaFree(lut.p);
        lut.p = nullptr;
        lut.ensure(h.size());
        cuda_check(cudaMemcpyAsync(lut.p, h.data(), h.size() * 4, cudaMemcpyHostToDevice, s), "lut");
        cuda_check(cudaStreamSynchronize(s), "lut");
    }

    void ensure_rows(size_t n) {
        d_src.ensure(n);
        d_dst.ensure(n);
        d_ratio.ensure(n);
        d_gls.ensure(n * 3);
        d_gop.ensure(n);
        d_gsc.ensure(n * 3);
        d_nop.ensure(n);
        d_nsc.ensure(n * 3);
        d_logit.ensure(n);
        d_ls.ensure(n * 3);
        h_gls.ensure(n * 3);
        h_gop.ensure(n);
        h_gsc.ensure(n * 3);
        h_nop.ensure(n);
        h_nsc.ensure(n * 3);
        h_logit.ensure(n);
        h_ls.ensure(n * 3);
        h_src.ensure(n);
        h_dst.ensure(n);
        h_ratio.ensure(n);
    }

    // run_relocation_for + the source update (Trainer.cpp:1231-1257 and :1313-1323 / :1365-1375):
    // ratios = min(bincount(sampled)[s] + 1, kNMax); the relocation kernel on the sources' post-
    // sigmoid opacities and exp(log-scales); the sources' logit and log-scales replaced by
    // logit_f32(new_opacity) and log(new_scale). Leaves the sampled rows in d_src and updates the
    // host mirror op_act of the sources.
    void relocate_sources(const ArenaView& a, const std::vector<int64_t>& src, float min_opacity,
                          const char* who) {
        const size_t n = src.size();
        ensure_rows(n);
        cudaStream_t s = a.stream;
        for (int64_t r : src) counts[static_cast<size_t>(r)]++;
        for (size_t j = 0; j < n; ++j) {
            const int64_t r = src[j];
            h_src.p[j] = r;
            h_gop.p[j] = op_act[static_cast<size_t>(r)];
            h_ratio.p[j] = std::min(counts[static_cast<size_t>(r)] + 1, kNMax);
        }
        for (int64_t r : src) counts[static_cast<size_t>(r)] = 0;
        cuda_check(cudaMemcpyAsync(d_src.p, h_src.p, n * 8, cudaMemcpyHostToDevice, s), "mcmc src");
        launch_gather_log_scales(a.p[2], d_src.p, static_cast<int64_t>(n), d_gls.p, s);
        cuda_check(cudaMemcpyAsync(h_gls.p, d_gls.p, n * 12, cudaMemcpyDeviceToHost, s), "mcmc gls");
        cuda_check(cudaStreamSynchronize(s), "mcmc gather");
        for (size_t j = 0; j < n * 3; ++j) h_gsc.p[j] = std::exp(h_gls.p[j]);
        cuda_check(cudaMemcpyAsync(d_gop.p, h_gop.p, n * 4, cudaMemcpyHostToDevice, s), "mcmc op");
        cuda_check(cudaMemcpyAsync(d_gsc.p, h_gsc.p, n * 12, cudaMemcpyHostToDevice, s), "mcmc sc");
        cuda_check(cudaMemcpyAsync(d_ratio.p, h_ratio.p, n * 4, cudaMemcpyHostToDevice, s),
                   "mcmc ratios");
        SxRelocationInputs rin{};
        rin.opacities = d_gop.p;
        rin.scales = d_gsc.p;
        rin.ratios = d_ratio.p;
        rin.binoms = lut.p;
        rin.N = static_cast<int64_t>(n);
        rin.n_max = kNMax;
        rin.min_opacity = min_opacity;
        launch_relocation(rin, d_nop.p, d_nsc.p, s);
        cuda_check(cudaMemcpyAsync(h_nop.p, d_nop.p, n * 4, cudaMemcpyDeviceToHost, s), "mcmc nop");
        cuda_check(cudaMemcpyAsync(h_nsc.p, d_nsc.p, n * 12, cudaMemcpyDeviceToHost, s), "mcmc nsc");
        cuda_check(cudaStreamSynchronize(s), "mcmc relocation");
        for (size_t j = 0; j < n; ++j) {
            h_logit.p[j] = logit_f32(h_nop.p[j]);
            for (int k = 0; k < 3; ++k) {
                const float ns = h_nsc.p[j * 3 + k];
                if (!(ns > 0.0f))
                    throw std::logic_error(std::string(who) + ": non-positive new_scale");
                h_ls.p[j * 3 + k] = std::log(ns);
            }
        }
        cuda_check(cudaMemcpyAsync(d_logit.p, h_logit.p, n * 4, cudaMemcpyHostToDevice, s),
                   "mcmc logits");
        cuda_check(cudaMemcpyAsync(d_ls.p, h_ls.p, n * 12, cudaMemcpyHostToDevice, s), "mcmc ls");
        launch_write_sources(a.p[3], a.p[2], d_src.p, d_logit.p, d_ls.p, static_cast<int64_t>(n), s);
        for (size_t j = 0; j < n; ++j) op_act[static_cast<size_t>(src[j])] = sigmoid_f32(h_logit.p[j]);
    }

    void refine(const ArenaView& a, int64_t count, int64_t cap_max, float min_opacity,
                McmcRefineOut& out) {
        const char* w = "mcmc_refine";
        if (count < 1 || count > a.rows) throw_invalid(w, "count out of [1, arena_rows]");
        if (cap_max < count) throw_invalid(w, "cap_max must be >= count");
        if (cap_max > a.rows) throw_invalid(w, "cap_max exceeds the executor's arena_rows");
        if (!(min_opacity > 0.0f && min_opacity < 1.0f))
            throw_invalid(w, "min_opacity must be in (0,1)");
        cudaStream_t s = a.stream;
        ensure_lut(a.device, s);
        if (counts.size() < static_cast<size_t>(a.rows)) counts.assign(static_cast<size_t>(a.rows), 0);
        out = McmcRefineOut{};
        const int64_t N = count;

        // activated opacities of the alive rows (the opacity group's tiled layout is the identity)
        h_logits.ensure(static_cast<size_t>(N));
        cuda_check(cudaMemcpyAsync(h_logits.p, a.p[3], static_cast<size_t>(N) * 4,
                                   cudaMemcpyDeviceToHost, s),
                   "mcmc logits");
        cuda_check(cudaStreamSynchronize(s), "mcmc logits");
        op_act.resize(static_cast<size_t>(N));
        sigmoid_all(h_logits.p, op_act.data(), N);

        // relocate (Trainer.cpp:1284-1340): dead = sigmoid(op) <= min_opacity; sources drawn from
        // the alive rows in proportion to opacity; dead row <- updated source row in every group;
        // Adam moments of the SOURCE rows zeroed (the dead rows keep theirs)
        dead.clear();
        alive.clear();
        for (int64_t i = 0; i < N; ++i)
            (op_act[static_cast<size_t>(i)] <= min_opacity ? dead : alive).push_back(i);
        if (!dead.empty() && !alive.empty()) {
            probs.resize(alive.size());
            for (size_t j = 0; j < alive.size(); ++j) probs[j] = op_act[static_cast<size_t>(alive[j])];
            multinomial(probs.data(), static_cast<int64_t>(alive.size()),
                        static_cast<int64_t>(dead.size()), rng, cdf, local);
            sampled.resize(dead.size());
            for (size_t j = 0; j < dead.size(); ++j) sampled[j] = alive[static_cast<size_t>(local[j])];
            relocate_sources(a, sampled, min_opacity, "mcmc_relocate");
            const size_t n = dead.size();
            for (size_t j = 0; j < n; ++j) h_dst.p[j] = dead[j];
            cuda_check(cudaMemcpyAsync(d_dst.p, h_dst.p, n * 8, cudaMemcpyHostToDevice, s), "mcmc dst");
            RowCopyArgs ca{};
            MomentRowsArgs ma{};
            for (int g = 0; g < 6; ++g) {
                ca.p[g] = a.p[g];
                ca.dims[g] = a.dims[g];
                ma.m[g] = a.m[g];
                ma.v[g] = a.v[g];
                ma.dims[g] = a.dims[g];
            }
            launch_copy_rows(ca, d_dst.p, d_src.p, static_cast<int64_t>(n), s);
            launch_zero_moment_rows(ma, d_src.p, static_cast<int64_t>(n), s);
            for (size_t j = 0; j < n; ++j)
                op_act[static_cast<size_t>(dead[j])] = op_act[static_cast<size_t>(sampled[j])];
            out.relocated_dead = dead;
            out.relocation_src = sampled;
        }

        // add (Trainer.cpp:1342-1394): grow to min(cap_max, ceil(1.05 N)) = (21N + 19) / 20; sources
        // drawn from ALL rows in proportion to opacity; new row N+j <- updated source row; Adam
        // moments of the NEW rows zeroed (the sources keep theirs)
        const int64_t target = std::min(cap_max, (N * 21 + 19) / 20);
        const int64_t n_add = target - N;
        if (n_add > 0) {
            multinomial(op_act.data(), N, n_add, rng, cdf, sampled);
            relocate_sources(a, sampled, min_opacity, "mcmc_add");
            for (int64_t j = 0; j < n_add; ++j) h_dst.p[j] = N + j;
            cuda_check(cudaMemcpyAsync(d_dst.p, h_dst.p, static_cast<size_t>(n_add) * 8,
                                       cudaMemcpyHostToDevice, s),
                       "mcmc dst");
            RowCopyArgs ca{};
            MomentRowsArgs ma{};
            for (int g = 0; g < 6; ++g) {
                ca.p[g] = a.p[g];
                ca.dims[g] = a.dims[g];
                ma.m[g] = a.m[g];
                ma.v[g] = a.v[g];
                ma.dims[g] = a.dims[g];
            }
            launch_copy_rows(ca, d_dst.p, d_src.p, n_add, s);
            launch_zero_moment_rows(ma, d_dst.p, n_add, s);
            out.added_src = sampled;
        }
        out.count = N + std::max<int64_t>(n_add, 0);
        cuda_check(cudaStreamSynchronize(s), "mcmc refine");
    }
};

McmcRefine* mcmc_new() { return new McmcRefine(); }
void mcmc_delete(McmcRefine* m) { delete m; }
void mcmc_seed(McmcRefine* m, uint64_t seed) { m->rng.seed(seed); }

// The engine's state as text in the classic locale (Trainer.cpp:1506-1509 / :1559-1563).
std::string mcmc_rng_state(const McmcRefine* m) {
    std::ostringstream oss;
    oss.imbue(std::locale::classic());
    oss << m->rng;
    return oss.str();
}
void mcmc_set_rng_state(McmcRefine* m, const std::string& text) {
    std::istringstream iss(text);
    iss.imbue(std::locale::classic());
    std::mt19937_64 r;
    iss >> r;
    if (!iss) throw_invalid("mcmc_set_rng_state", "corrupt rng state");
    m->rng = r;
}

void mcmc_refine(McmcRefine* m, const ArenaView& a, int64_t count, int64_t cap_max,
                 float min_opacity, McmcRefineOut& out) {
    m->refine(a, count, cap_max, min_opacity, out);
}

}  // namespace sx
