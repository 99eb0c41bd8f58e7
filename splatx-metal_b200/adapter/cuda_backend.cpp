// cuda_backend.cpp — splatx::KernelBackend and splatx::TrainStepExecutor over libsplatx_cuda.
//
// Each method follows one pattern: upload the host inputs into device buffers owned by a per-call
// Scratch, call the C-ABI entry point on the backend's stream, download the outputs into the
// result vectors, synchronise. Sizes come from the reference's struct fields (the same ones its
// validators check, Validate.h); a negative size uploads nothing, so the C-ABI's own checks report
// the violation with the reference's exception type.
#include "cuda_backend.h"

#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/splatx_cuda.h"

namespace splatx {
namespace {

void check(int32_t rc) {
    if (rc == SXCUDA_OK) return;
    const std::string msg = sxcuda_last_error();
    if (rc == SXCUDA_EINVAL) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

void cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        throw std::runtime_error(std::string("cuda backend: ") + what + ": " + cudaGetErrorString(e));
}

size_t count(int64_t n) { return n > 0 ? static_cast<size_t>(n) : 0; }

// Device buffers of one call, freed when the call returns (after the stream has drained).
class Scratch {
public:
    explicit Scratch(cudaStream_t s) : s_(s) {}
    ~Scratch() {
        cudaStreamSynchronize(s_);
        for (void* p : bufs_) cudaFree(p);
    }
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;

    // A zeroed device buffer of n elements (nullptr when n == 0).
    template <class T>
    T* alloc(size_t n) {
        if (n == 0) return nullptr;
        void* p = nullptr;
        cuda(cudaMalloc(&p, n * sizeof(T)), "cudaMalloc");
        bufs_.push_back(p);
        cuda(cudaMemsetAsync(p, 0, n * sizeof(T), s_), "cudaMemsetAsync");
        return static_cast<T*>(p);
    }
    // A device copy of host[0..n) (nullptr for a null host pointer or n == 0).
    template <class T>
    T* up(const T* host, size_t n) {
        if (!host || n == 0) return nullptr;
        void* p = nullptr;
        cuda(cudaMalloc(&p, n * sizeof(T)), "cudaMalloc");
        bufs_.push_back(p);
        cuda(cudaMemcpyAsync(p, host, n * sizeof(T), cudaMemcpyHostToDevice, s_), "upload");
        return static_cast<T*>(p);
    }
    // The device buffer's first n elements as a host vector.
    template <class T>
    std::vector<T> down(const T* dev, size_t n) {
        std::vector<T> v(n);
        if (n && dev) {
            cuda(cudaMemcpyAsync(v.data(), dev, n * sizeof(T), cudaMemcpyDeviceToHost, s_), "download");
            cuda(cudaStreamSynchronize(s_), "download");
        }
        return v;
    }
    template <class T>
    void down_into(T* host, const T* dev, size_t n) {
        if (!n || !dev || !host) return;
        cuda(cudaMemcpyAsync(host, dev, n * sizeof(T), cudaMemcpyDeviceToHost, s_), "download");
        cuda(cudaStreamSynchronize(s_), "download");
    }
    // Workspace of a query-protocol entry point: `call(ws, &bytes)` with ws == nullptr fills
    // bytes; the buffer is never null, so the second call cannot be mistaken for a query.
    template <class F>
    void with_workspace(F call) {
        size_t bytes = 0;
        check(call(nullptr, &bytes));
        void* ws = alloc<unsigned char>(bytes > 0 ? bytes : 1);
        check(call(ws, &bytes));
    }

private:
    cudaStream_t s_;
    std::vector<void*> bufs_;
};

// ---------------------------------------------------------------- resident executor
class CudaTrainStepExecutor final : public TrainStepExecutor {
public:
    CudaTrainStepExecutor(const TrainStepExecutorDesc& d, int device) {
        SxTrainStepExecutorDesc c{};
        c.arena_rows = d.arena_rows;
        c.sh_degree = d.sh_degree;
        c.eps2d = d.eps2d;
        c.near_plane = d.near_plane;
        c.far_plane = d.far_plane;
        c.radius_clip = d.radius_clip;
        c.b1 = d.b1;
        c.b2 = d.b2;
        c.eps = d.eps;
        c.ssim_weight = d.ssim_weight;
        c.antialiased = d.antialiased ? 1 : 0;
        check(sxcuda_executor_create(&c, device, &ex_));
    }
    ~CudaTrainStepExecutor() override { sxcuda_executor_destroy(ex_); }

    void upload_params(const ResidentParamSync& s) override {
        const SxResidentParamSync c = sync(s);
        check(sxcuda_executor_upload_params(ex_, &c));
    }
    void download_params(const ResidentParamSync& s) override {
        const SxResidentParamSync c = sync(s);
        check(sxcuda_executor_download_params(ex_, &c));
    }
    ResidentStepOutputs step(const ResidentStepInputs& in) override {
        SxResidentStepInputs c{};
        c.viewmat = in.viewmat;
        c.K = in.K;
        c.width = in.width;
        c.height = in.height;
        c.gt_rgb = in.gt_rgb;
        c.count = in.count;
        c.degrees_to_use = in.degrees_to_use;
        for (int g = 0; g < 6; ++g) c.lr[g] = in.lr[g];
        c.opacity_reg_w = in.opacity_reg_w;
        c.scale_reg_w = in.scale_reg_w;
        c.forward_only = in.forward_only ? 1 : 0;
        c.want_render = in.want_render ? 1 : 0;
        c.inject_noise = in.inject_noise ? 1 : 0;
        c.noise_seed = in.noise_seed;
        c.noise_offset = in.noise_offset;
        c.noise_scale = in.noise_scale;
        c.gt_on_device = 0;
        ResidentStepOutputs out;
        if (in.want_render && in.width > 0 && in.height > 0)
            out.render_colors.resize(static_cast<size_t>(in.width) * in.height * 3);
        SxResidentStepOutputs o{};
        o.render_colors = out.render_colors.empty() ? nullptr : out.render_colors.data();
        check(sxcuda_executor_step(ex_, &c, &o));
        out.loss = o.loss;
        out.n_isects = o.n_isects;
        return out;
    }

private:
    static SxResidentParamSync sync(const ResidentParamSync& s) {
        SxResidentParamSync c{};
        for (int g = 0; g < 6; ++g) {
            c.params[g] = s.params[g];
            c.exp_avg[g] = s.exp_avg[g];
            c.exp_avg_sq[g] = s.exp_avg_sq[g];
        }
        c.rows = s.rows;
        return c;
    }
    SxExecutor* ex_ = nullptr;
};

// ---------------------------------------------------------------- per-kernel backend
class CudaBackend final : public KernelBackend {
public:
    explicit CudaBackend(int device) : device_(device) {
        int n = 0;
        cuda(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
        if (device < 0 || device >= n)
            throw std::runtime_error("make_cuda_backend: no CUDA device " + std::to_string(device));
        cuda(cudaSetDevice(device), "cudaSetDevice");
        cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    }
    ~CudaBackend() override {
        if (stream_) {
            cudaStreamSynchronize(stream_);
            cudaStreamDestroy(stream_);
        }
    }

    const char* name() const override { return "cuda(sm_100a)"; }

    // The reference's Metal backend has no projection_ewa_fwd either (MetalBackend.cpp:233-235):
    // it is the CPU-only torch-semantics projection.
    ProjectionOutputs projection_ewa_fwd(const ProjectionInputs&) override {
        throw std::runtime_error("projection_ewa_fwd: unimplemented on cuda backend");
    }

    void fused_adam(const AdamInputs& in) override {
        Scratch sc = scratch();
        const size_t n = count(in.n_elems);
        SxAdamInputs a{};
        a.param = sc.up(in.param, n);
        a.grad = sc.up(in.grad, n);
        a.exp_avg = sc.up(in.exp_avg, n);
        a.exp_avg_sq = sc.up(in.exp_avg_sq, n);
        a.valid = sc.up(in.valid, count(in.n_gauss));
        a.n_elems = in.n_elems;
        a.n_gauss = in.n_gauss;
        a.lr = in.lr;
        a.b1 = in.b1;
        a.b2 = in.b2;
        a.eps = in.eps;
        check(sxcuda_fused_adam(&a, stream_));
        sc.down_into(in.param, a.param, n);
        sc.down_into(in.exp_avg, a.exp_avg, n);
        sc.down_into(in.exp_avg_sq, a.exp_avg_sq, n);
    }

    ProjectionFusedOutputs projection_fused_fwd(const ProjectionFusedInputs& in) override {
        Scratch sc = scratch();
        const SxProjectionFusedInputs p = proj_inputs(sc, in);
        const size_t cn = count(in.C) * count(in.N);
        SxProjectionFusedOutputs o{};
        o.radii = sc.alloc<int32_t>(cn * 2);
        o.means2d = sc.alloc<float>(cn * 2);
        o.depths = sc.alloc<float>(cn);
        o.conics = sc.alloc<float>(cn * 3);
        o.compensations = in.calc_compensations ? sc.alloc<float>(cn) : nullptr;
        check(sxcuda_projection_fused_fwd(&p, &o, stream_));
        ProjectionFusedOutputs out;
        out.radii = sc.down(o.radii, cn * 2);
        out.means2d = sc.down(o.means2d, cn * 2);
        out.depths = sc.down(o.depths, cn);
        out.conics = sc.down(o.conics, cn * 3);
        if (in.calc_compensations) out.compensations = sc.down(o.compensations, cn);
        return out;
    }

    ProjectionFusedGrads projection_fused_bwd(const ProjectionFusedInputs& in,
                                              const ProjectionFusedGradsIn& g) override {
        Scratch sc = scratch();
        const SxProjectionFusedInputs p = proj_inputs(sc, in);
        const size_t n = count(in.N), cn = count(in.C) * n;
        SxProjectionFusedGradsIn gi{};
        gi.radii = sc.up(g.radii, cn * 2);
        gi.conics = sc.up(g.conics, cn * 3);
        gi.compensations = sc.up(g.compensations, cn);
        gi.v_means2d = sc.up(g.v_means2d, cn * 2);
        gi.v_depths = sc.up(g.v_depths, cn);
        gi.v_conics = sc.up(g.v_conics, cn * 3);
        gi.v_compensations = sc.up(g.v_compensations, cn);
        gi.viewmats_grad = g.viewmats_grad ? 1 : 0;
        const bool covars = in.covars != nullptr;
        SxProjectionFusedGrads o{};
        o.v_means = sc.alloc<float>(n * 3);
        o.v_covars = covars ? sc.alloc<float>(n * 6) : nullptr;
        o.v_quats = covars ? nullptr : sc.alloc<float>(n * 4);
        o.v_scales = covars ? nullptr : sc.alloc<float>(n * 3);
        o.v_viewmats = g.viewmats_grad ? sc.alloc<float>(count(in.C) * 16) : nullptr;
        check(sxcuda_projection_fused_bwd(&p, &gi, &o, stream_));
        ProjectionFusedGrads out;
        out.v_means = sc.down(o.v_means, n * 3);
        if (covars) {
            out.v_covars = sc.down(o.v_covars, n * 6);
        } else {
            out.v_quats = sc.down(o.v_quats, n * 4);
            out.v_scales = sc.down(o.v_scales, n * 3);
        }
        if (g.viewmats_grad) out.v_viewmats = sc.down(o.v_viewmats, count(in.C) * 16);
        return out;
    }

    ShOutputs sh_fwd(const ShInputs& in) override {
        Scratch sc = scratch();
        const SxShInputs s = sh_inputs(sc, in);
        const size_t m = count(in.B) * count(in.N) * in.D;
        float* colors = sc.alloc<float>(m);
        check(sxcuda_sh_fwd(&s, colors, stream_));
        ShOutputs out;
        out.colors = sc.down(colors, m);
        return out;
    }

    ShGrads sh_bwd(const ShInputs& in, const float* v_colors) override {
        Scratch sc = scratch();
        const SxShInputs s = sh_inputs(sc, in);
        const size_t bn = count(in.B) * count(in.N);
        const size_t nk = count(in.N) * count(in.K) * in.D;
        const float* vc = sc.up(v_colors, bn * in.D);
        float* v_coeffs = sc.alloc<float>(nk);
        float* v_dirs = in.compute_v_dirs ? sc.alloc<float>(bn * 3) : nullptr;
        check(sxcuda_sh_bwd(&s, vc, v_coeffs, v_dirs, stream_));
        ShGrads out;
        out.v_coeffs = sc.down(v_coeffs, nk);
        if (in.compute_v_dirs) out.v_dirs = sc.down(v_dirs, bn * 3);
        return out;
    }

    IsectTilesOutputs isect_tiles(const IsectTilesInputs& in) override {
        Scratch sc = scratch();
        const size_t n = count(in.I) * count(in.N);
        SxIsectTilesInputs t{};
        t.means2d = sc.up(in.means2d, n * 2);
        t.radii = sc.up(in.radii, n * 2);
        t.depths = sc.up(in.depths, n);
        t.conics = sc.up(in.conics, n * 3);
        t.opacities = sc.up(in.opacities, n);
        t.I = in.I;
        t.N = in.N;
        t.tile_size = in.tile_size;
        t.tile_width = in.tile_width;
        t.tile_height = in.tile_height;
        int32_t* tiles = sc.alloc<int32_t>(n);
        int64_t* cum = sc.alloc<int64_t>(n);
        int64_t n_isects = 0;
        sc.with_workspace([&](void* w, size_t* b) {
            return sxcuda_isect_tile_count(&t, tiles, cum, &n_isects, w, b, stream_);
        });
        const size_t ni = count(n_isects);
        uint64_t* ids = sc.alloc<uint64_t>(ni);
        int32_t* flat = sc.alloc<int32_t>(ni);
        if (ni > 0) check(sxcuda_isect_tile_emit(&t, cum, ids, flat, stream_));
        IsectTilesOutputs out;
        out.tiles_per_gauss = sc.down(tiles, n);
        out.isect_ids = sc.down(ids, ni);
        out.flatten_ids = sc.down(flat, ni);
        out.n_isects = n_isects;
        out.tile_n_bits = sxcuda_bits_for_count(static_cast<int64_t>(in.tile_width) * in.tile_height);
        out.image_n_bits = sxcuda_bits_for_count(in.I);
        return out;
    }

    std::vector<int64_t> prefix_scan_i64(const int32_t* v, int64_t n) override {
        Scratch sc = scratch();
        const int32_t* d_in = sc.up(v, count(n));
        int64_t* d_out = sc.alloc<int64_t>(count(n));
        sc.with_workspace([&](void* w, size_t* b) {
            return sxcuda_prefix_scan_i64(d_in, d_out, n, w, b, stream_);
        });
        return sc.down(d_out, count(n));
    }

    SortIsectOutputs sort_isect(const SortIsectInputs& in) override {
        Scratch sc = scratch();
        const size_t n = count(in.n);
        const uint64_t* k = sc.up(in.keys, n);
        const int32_t* v = sc.up(in.values, n);
        uint64_t* ko = sc.alloc<uint64_t>(n);
        int32_t* vo = sc.alloc<int32_t>(n);
        sc.with_workspace([&](void* w, size_t* b) {
            return sxcuda_sort_isect(k, v, ko, vo, in.n, in.key_n_bits, w, b, stream_);
        });
        SortIsectOutputs out;
        out.keys_sorted = sc.down(ko, n);
        out.values_sorted = sc.down(vo, n);
        return out;
    }

    std::vector<int32_t> isect_offset_encode(const IsectOffsetInputs& in) override {
        Scratch sc = scratch();
        const size_t total = count(in.I) * in.tile_width * in.tile_height;
        const uint64_t* ids = sc.up(in.isect_ids, count(in.n_isects));
        int32_t* off = sc.alloc<int32_t>(total);
        check(sxcuda_isect_offset_encode(ids, in.n_isects, in.I, in.tile_width, in.tile_height, off,
                                         stream_));
        return sc.down(off, total);
    }

    RasterizeFwdOutputs rasterize_fwd(const RasterizeFwdInputs& in) override {
        Scratch sc = scratch();
        const SxRasterizeFwdInputs r = raster_inputs(sc, in);
        const size_t px = count(in.I) * in.image_width * in.image_height;
        float* rc = sc.alloc<float>(px * 3);
        float* ra = sc.alloc<float>(px);
        int32_t* li = sc.alloc<int32_t>(px);
        check(sxcuda_rasterize_fwd(&r, rc, ra, li, stream_));
        RasterizeFwdOutputs out;
        out.render_colors = sc.down(rc, px * 3);
        out.render_alphas = sc.down(ra, px);
        out.last_ids = sc.down(li, px);
        return out;
    }

    RasterizeBwdGrads rasterize_bwd(const RasterizeFwdInputs& in,
                                    const RasterizeBwdGradsIn& g) override {
        Scratch sc = scratch();
        const SxRasterizeFwdInputs r = raster_inputs(sc, in);
        const size_t px = count(in.I) * in.image_width * in.image_height;
        const size_t in_ = count(in.I) * count(in.N);
        SxRasterizeBwdGradsIn gi{};
        gi.render_alphas = sc.up(g.render_alphas, px);
        gi.last_ids = sc.up(g.last_ids, px);
        gi.v_render_colors = sc.up(g.v_render_colors, px * 3);
        gi.v_render_alphas = sc.up(g.v_render_alphas, px);
        gi.absgrad = g.absgrad ? 1 : 0;
        SxRasterizeBwdGrads o{};
        o.v_means2d = sc.alloc<float>(in_ * 2);
        o.v_conics = sc.alloc<float>(in_ * 3);
        o.v_colors = sc.alloc<float>(in_ * 3);
        o.v_opacities = sc.alloc<float>(in_);
        o.v_means2d_abs = g.absgrad ? sc.alloc<float>(in_ * 2) : nullptr;
        check(sxcuda_rasterize_bwd(&r, &gi, &o, stream_));
        RasterizeBwdGrads out;
        out.v_means2d = sc.down(o.v_means2d, in_ * 2);
        out.v_conics = sc.down(o.v_conics, in_ * 3);
        out.v_colors = sc.down(o.v_colors, in_ * 3);
        out.v_opacities = sc.down(o.v_opacities, in_);
        if (g.absgrad) out.v_means2d_abs = sc.down(o.v_means2d_abs, in_ * 2);
        return out;
    }

    std::vector<float> rng_normal_f32(const RngNormalInputs& in) override {
        Scratch sc = scratch();
        float* out = sc.alloc<float>(count(in.count));
        check(sxcuda_rng_normal_f32(in.seed, in.offset, in.count, out, stream_));
        return sc.down(out, count(in.count));
    }

    std::vector<uint32_t> rng_philox_u32(const RngNormalInputs& in) override {
        Scratch sc = scratch();
        uint32_t* out = sc.alloc<uint32_t>(count(in.count));
        check(sxcuda_rng_philox_u32(in.seed, in.offset, in.count, out, stream_));
        return sc.down(out, count(in.count));
    }

    RelocationOutputs mcmc_relocation(const RelocationInputs& in) override {
        Scratch sc = scratch();
        const size_t n = count(in.N);
        SxRelocationInputs r{};
        r.opacities = sc.up(in.opacities, n);
        r.scales = sc.up(in.scales, n * 3);
        r.ratios = sc.up(in.ratios, n);
        r.binoms = sc.up(in.binoms, count(in.n_max) * count(in.n_max));
        r.N = in.N;
        r.n_max = in.n_max;
        r.min_opacity = in.min_opacity;
        float* no = sc.alloc<float>(n);
        float* ns = sc.alloc<float>(n * 3);
        check(sxcuda_mcmc_relocation(&r, no, ns, stream_));
        RelocationOutputs out;
        out.new_opacities = sc.down(no, n);
        out.new_scales = sc.down(ns, n * 3);
        return out;
    }

    void mcmc_perturb_positions(const PerturbInputs& in) override {
        Scratch sc = scratch();
        const size_t n = count(in.N);
        SxPerturbInputs p{};
        p.positions = sc.up(in.positions, n * 3);
        p.quats = sc.up(in.quats, n * 4);
        p.scales_log = sc.up(in.scales_log, n * 3);
        p.opacities_logit = sc.up(in.opacities_logit, n);
        p.noise = sc.up(in.noise, n * 3);
        p.N = in.N;
        p.noise_scale = in.noise_scale;
        p.t = in.t;
        p.k = in.k;
        check(sxcuda_mcmc_perturb_positions(&p, stream_));
        sc.down_into(in.positions, p.positions, n * 3);
    }

    SsimFwdOutputs ssim_fwd(const SsimInputs& in) override {
        Scratch sc = scratch();
        const SxSsimInputs s = ssim_inputs(sc, in);
        const size_t m = count(in.I) * count(in.H - 10) * count(in.W - 10) * count(in.C);
        float* map = sc.alloc<float>(m);
        float* cmu = in.need_coeffs ? sc.alloc<float>(m) : nullptr;
        float* csg = in.need_coeffs ? sc.alloc<float>(m) : nullptr;
        float* ccr = in.need_coeffs ? sc.alloc<float>(m) : nullptr;
        double* mean = sc.alloc<double>(1);
        sc.with_workspace([&](void* w, size_t* b) {
            return sxcuda_ssim_fwd(&s, map, cmu, csg, ccr, mean, w, b, stream_);
        });
        SsimFwdOutputs out;
        out.ssim = sc.down(mean, 1)[0];
        out.ssim_map = sc.down(map, m);
        if (in.need_coeffs) {
            out.coeff_mu = sc.down(cmu, m);
            out.coeff_sigma = sc.down(csg, m);
            out.coeff_cross = sc.down(ccr, m);
        }
        return out;
    }

    std::vector<float> ssim_bwd(const SsimInputs& in, const SsimGradsIn& g) override {
        Scratch sc = scratch();
        const SxSsimInputs s = ssim_inputs(sc, in);
        const size_t m = count(in.I) * count(in.H - 10) * count(in.W - 10) * count(in.C);
        SxSsimGradsIn gi{};
        gi.coeff_mu = sc.up(g.coeff_mu, m);
        gi.coeff_sigma = sc.up(g.coeff_sigma, m);
        gi.coeff_cross = sc.up(g.coeff_cross, m);
        gi.v_loss = g.v_loss;
        const size_t n = count(in.I) * count(in.H) * count(in.W) * count(in.C);
        float* v = sc.alloc<float>(n);
        check(sxcuda_ssim_bwd(&s, &gi, v, stream_));
        return sc.down(v, n);
    }

    std::unique_ptr<TrainStepExecutor> make_train_step_executor(
        const TrainStepExecutorDesc& d) override {
        return std::unique_ptr<TrainStepExecutor>(new CudaTrainStepExecutor(d, device_));
    }

private:
    Scratch scratch() {
        cuda(cudaSetDevice(device_), "cudaSetDevice");
        return Scratch(stream_);
    }

    SxProjectionFusedInputs proj_inputs(Scratch& sc, const ProjectionFusedInputs& in) {
        const size_t n = count(in.N), c = count(in.C);
        SxProjectionFusedInputs p{};
        p.means = sc.up(in.means, n * 3);
        p.covars = sc.up(in.covars, n * 6);
        p.quats = sc.up(in.quats, n * 4);
        p.scales = sc.up(in.scales, n * 3);
        p.opacities = sc.up(in.opacities, n);
        p.viewmats = sc.up(in.viewmats, c * 16);
        p.Ks = sc.up(in.Ks, c * 9);
        p.N = in.N;
        p.C = in.C;
        p.width = in.width;
        p.height = in.height;
        p.eps2d = in.eps2d;
        p.near_plane = in.near_plane;
        p.far_plane = in.far_plane;
        p.radius_clip = in.radius_clip;
        p.camera_model = in.camera_model;
        p.calc_compensations = in.calc_compensations ? 1 : 0;
        return p;
    }

    SxShInputs sh_inputs(Scratch& sc, const ShInputs& in) {
        const size_t bn = count(in.B) * count(in.N);
        SxShInputs s{};
        s.dirs = sc.up(in.dirs, bn * 3);
        s.coeffs = sc.up(in.coeffs, count(in.N) * count(in.K) * in.D);
        s.masks = sc.up(in.masks, bn);
        s.degrees_to_use = in.degrees_to_use;
        s.B = in.B;
        s.N = in.N;
        s.K = in.K;
        s.D = in.D;
        s.compute_v_dirs = in.compute_v_dirs ? 1 : 0;
        return s;
    }

    SxRasterizeFwdInputs raster_inputs(Scratch& sc, const RasterizeFwdInputs& in) {
        const size_t in_ = count(in.I) * count(in.N);
        const size_t tiles = count(in.I) * in.tile_width * in.tile_height;
        SxRasterizeFwdInputs r{};
        r.means2d = sc.up(in.means2d, in_ * 2);
        r.conics = sc.up(in.conics, in_ * 3);
        r.colors = sc.up(in.colors, in_ * 3);
        r.opacities = sc.up(in.opacities, in_);
        r.backgrounds = sc.up(in.backgrounds, count(in.I) * 3);
        r.masks = sc.up(in.masks, tiles);
        r.isect_offsets = sc.up(in.isect_offsets, tiles);
        r.flatten_ids = sc.up(in.flatten_ids, count(in.n_isects));
        r.I = in.I;
        r.N = in.N;
        r.n_isects = in.n_isects;
        r.image_width = in.image_width;
        r.image_height = in.image_height;
        r.tile_size = in.tile_size;
        r.tile_width = in.tile_width;
        r.tile_height = in.tile_height;
        return r;
    }

    SxSsimInputs ssim_inputs(Scratch& sc, const SsimInputs& in) {
        const size_t n = count(in.I) * count(in.H) * count(in.W) * count(in.C);
        SxSsimInputs s{};
        s.img1 = sc.up(in.img1, n);
        s.img2 = sc.up(in.img2, n);
        s.I = in.I;
        s.H = in.H;
        s.W = in.W;
        s.C = in.C;
        s.need_coeffs = in.need_coeffs ? 1 : 0;
        return s;
    }

    int device_ = 0;
    cudaStream_t stream_ = nullptr;
};

}  // namespace

std::unique_ptr<KernelBackend> make_cuda_backend(int device) {
    return std::unique_ptr<KernelBackend>(new CudaBackend(device));
}

}  // namespace splatx
