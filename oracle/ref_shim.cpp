// ref_shim.cpp — extern "C" access to the reference's own CPU kernels (splatx-metal
// Sources/SplatXCore/CpuKernels.cpp, compiled from the reference tree by oracle/Makefile into the
// git-ignored oracle/_ref/). TEST INFRASTRUCTURE: used only to validate the C oracle and to
// generate golden vectors; every function returns 0, or -1 with the reference's exception text in
// sxr_last_error().
#include <cstring>
#include <string>
#include <vector>

#include "splatx/CpuKernels.h"
#include "splatx/KernelBackend.h"
#include "splatx/Checkpoint.h"
#include "splatx/ColmapLoader.h"
#include "splatx/TrainingInput.h"
#include "splatx/PlyIO.h"
#include "splatx/SpzIO.h"
#include "splatx/Trainer.h"

#include <random>

using namespace splatx;

namespace {
thread_local std::string g_err;
template <typename F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}
template <typename T>
void put(T* dst, const std::vector<T>& v) {
    if (dst && !v.empty()) std::memcpy(dst, v.data(), v.size() * sizeof(T));
}
}  // namespace

extern "C" {

const char* sxr_last_error() { return g_err.c_str(); }

int sxr_fused_adam(float* p, const float* g, float* m, float* v, const uint8_t* valid, int64_t n,
                   int64_t n_gauss, float lr, float b1, float b2, float eps) {
    return guarded([&] {
        AdamInputs a;
        a.param = p; a.grad = g; a.exp_avg = m; a.exp_avg_sq = v; a.valid = valid;
        a.n_elems = n; a.n_gauss = n_gauss; a.lr = lr; a.b1 = b1; a.b2 = b2; a.eps = eps;
        fused_adam_cpu(a);
    });
}

int sxr_projection_fused_fwd(const float* means, const float* covars6, const float* quats,
                             const float* scales, const float* opacities, const float* viewmats,
                             const float* Ks, int64_t N, int64_t C, int width, int height,
                             float eps2d, float near_plane, float far_plane, float radius_clip,
                             int calc_comp, int32_t* radii, float* means2d, float* depths,
                             float* conics, float* comps) {
    return guarded([&] {
        ProjectionFusedInputs in;
        in.means = means; in.covars = covars6; in.quats = quats; in.scales = scales;
        in.opacities = opacities; in.viewmats = viewmats; in.Ks = Ks; in.N = N; in.C = C;
        in.width = width; in.height = height; in.eps2d = eps2d; in.near_plane = near_plane;
        in.far_plane = far_plane; in.radius_clip = radius_clip; in.camera_model = 0;
        in.calc_compensations = calc_comp != 0;
        const ProjectionFusedOutputs o = projection_fused_fwd_cpu(in);
        put(radii, o.radii); put(means2d, o.means2d); put(depths, o.depths); put(conics, o.conics);
        put(comps, o.compensations);
    });
}

int sxr_sh_fwd(const float* dirs, const float* coeffs, const uint8_t* masks, uint32_t degree,
               int64_t B, int64_t N, int64_t K, uint32_t D, float* colors) {
    return guarded([&] {
        ShInputs in;
        in.dirs = dirs; in.coeffs = coeffs; in.masks = masks; in.degrees_to_use = degree;
        in.B = B; in.N = N; in.K = K; in.D = D;
        put(colors, sh_fwd_cpu(in).colors);
    });
}

// Runs isect_tiles_cpu; writes tiles_per_gauss, and isect ids/flatten ids when cap >= n_isects.
int sxr_isect_tiles(const float* means2d, const int32_t* radii, const float* depths,
                    const float* conics, const float* opacities, int64_t I, int64_t N,
                    uint32_t tile_size, uint32_t tw, uint32_t th, int32_t* tiles, uint64_t* ids,
                    int32_t* flat, int64_t cap, int64_t* n_isects) {
    return guarded([&] {
        IsectTilesInputs in;
        in.means2d = means2d; in.radii = radii; in.depths = depths; in.conics = conics;
        in.opacities = opacities; in.I = I; in.N = N; in.tile_size = tile_size;
        in.tile_width = tw; in.tile_height = th;
        const IsectTilesOutputs o = isect_tiles_cpu(in);
        put(tiles, o.tiles_per_gauss);
        *n_isects = o.n_isects;
        if (cap >= o.n_isects) {
            put(ids, o.isect_ids);
            put(flat, o.flatten_ids);
        }
    });
}

int sxr_sort_isect(const uint64_t* keys, const int32_t* vals, int64_t n, uint32_t bits,
                   uint64_t* ko, int32_t* vo) {
    return guarded([&] {
        SortIsectInputs in;
        in.keys = keys; in.values = vals; in.n = n; in.key_n_bits = bits;
        const SortIsectOutputs o = sort_isect_cpu(in);
        put(ko, o.keys_sorted);
        put(vo, o.values_sorted);
    });
}

int sxr_isect_offset_encode(const uint64_t* ids, int64_t n, int64_t I, uint32_t tw, uint32_t th,
                            int32_t* offsets) {
    return guarded([&] {
        IsectOffsetInputs in;
        in.isect_ids = ids; in.n_isects = n; in.I = I; in.tile_width = tw; in.tile_height = th;
        put(offsets, isect_offset_encode_cpu(in));
    });
}

int sxr_rasterize_fwd(const float* means2d, const float* conics, const float* colors,
                      const float* opacities, const float* bgs, const int32_t* offsets,
                      const int32_t* flatten_ids, int64_t I, int64_t N, int64_t n_isects,
                      uint32_t W, uint32_t H, uint32_t ts, uint32_t tw, uint32_t th, float* rc,
                      float* ra, int32_t* li) {
    return guarded([&] {
        RasterizeFwdInputs in;
        in.means2d = means2d; in.conics = conics; in.colors = colors; in.opacities = opacities;
        in.backgrounds = bgs; in.isect_offsets = offsets; in.flatten_ids = flatten_ids;
        in.I = I; in.N = N; in.n_isects = n_isects; in.image_width = W; in.image_height = H;
        in.tile_size = ts; in.tile_width = tw; in.tile_height = th;
        const RasterizeFwdOutputs o = rasterize_fwd_cpu(in);
        put(rc, o.render_colors); put(ra, o.render_alphas); put(li, o.last_ids);
    });
}

int sxr_ssim_fwd(const float* img1, const float* img2, int64_t I, int64_t H, int64_t W, int64_t C,
                 int need, float* map, float* cmu, float* csg, float* ccr, double* mean) {
    return guarded([&] {
        SsimInputs in;
        in.img1 = img1; in.img2 = img2; in.I = I; in.H = H; in.W = W; in.C = C;
        in.need_coeffs = need != 0;
        const SsimFwdOutputs o = ssim_fwd_cpu(in);
        put(map, o.ssim_map); put(cmu, o.coeff_mu); put(csg, o.coeff_sigma); put(ccr, o.coeff_cross);
        *mean = o.ssim;
    });
}

int sxr_rng_philox_u32(uint64_t seed, uint64_t offset, int64_t count, uint32_t* out) {
    return guarded([&] {
        RngNormalInputs in;
        in.seed = seed; in.offset = offset; in.count = count;
        put(out, rng_philox_u32_cpu(in));
    });
}

int sxr_rng_normal_f32(uint64_t seed, uint64_t offset, int64_t count, float* out) {
    return guarded([&] {
        RngNormalInputs in;
        in.seed = seed; in.offset = offset; in.count = count;
        put(out, rng_normal_f32_cpu(in));
    });
}

int sxr_make_binoms_lut(int n_max, float* lut) {
    return guarded([&] { put(lut, make_binoms_lut(n_max)); });
}

int sxr_mcmc_relocation(const float* op, const float* sc, const int32_t* ratios,
                        const float* binoms, int64_t N, int n_max, float min_op, float* new_op,
                        float* new_sc) {
    return guarded([&] {
        RelocationInputs in;
        in.opacities = op; in.scales = sc; in.ratios = ratios; in.binoms = binoms; in.N = N;
        in.n_max = n_max; in.min_opacity = min_op;
        const RelocationOutputs o = mcmc_relocation_cpu(in);
        put(new_op, o.new_opacities);
        put(new_sc, o.new_scales);
    });
}

int sxr_mcmc_perturb_positions(float* pos, const float* quats, const float* scales_log,
                               const float* op_logit, const float* noise, int64_t N,
                               float noise_scale, float t, float k) {
    return guarded([&] {
        PerturbInputs in;
        in.positions = pos; in.quats = quats; in.scales_log = scales_log;
        in.opacities_logit = op_logit; in.noise = noise; in.N = N; in.noise_scale = noise_scale;
        in.t = t; in.k = k;
        mcmc_perturb_positions_cpu(in);
    });
}


// std::mt19937_64(seed): its first n outputs (pins the oracle's restated engine).
int sxr_mt64_outputs(uint64_t seed, int64_t n, uint64_t* out) {
    return guarded([&] {
        std::mt19937_64 g(seed);
        for (int64_t i = 0; i < n; i++) out[i] = g();
    });
}

// The reference's own Trainer::mcmc_refine (Trainer.cpp:1273-1435) on its CPU backend, run
// n_refines times. params / exp_avg / exp_avg_sq: the six groups (D3 order) as [cap_max, dims]
// arrays, rows [0, count) meaningful on input, all cap_max rows written back. stats[3*r + {0,1,2}]
// = (count after, |relocated_dead|, |added_src|) of refine r; the index lists of every refine are
// appended to dead/src/added (capacity list_cap each).
int sxr_trainer_mcmc_refine(float* const* params, float* const* exp_avg, float* const* exp_avg_sq,
                            int sh_degree, int64_t count, int64_t cap_max, float min_opacity,
                            uint64_t seed, int n_refines, int64_t* stats, int64_t* dead,
                            int64_t* src, int64_t* added, int64_t list_cap) {
    return guarded([&] {
        auto cpu = make_cpu_backend();
        SplatCloud c;
        c.count = count;
        c.sh_degree = sh_degree;
        const int64_t K3 = static_cast<int64_t>(c.sh_rest_coeffs()) * 3;
        const int64_t dims[6] = {3, 4, 3, 1, 3, K3};
        std::vector<float>* vec[6] = {&c.means, &c.quats, &c.scales, &c.opacities, &c.sh0, &c.shN};
        for (int g = 0; g < 6; g++) vec[g]->assign(params[g], params[g] + count * dims[g]);
        TrainConfig cfg;
        cfg.total_iters = 100;
        cfg.mcmc.enabled = true;
        cfg.mcmc.cap_max = cap_max;
        cfg.mcmc.min_opacity = min_opacity;
        cfg.mcmc.seed = seed;
        Trainer tr(*cpu, std::move(c), cfg);
        const Trainer::ParamGroup groups[6] = {
            Trainer::ParamGroup::Means, Trainer::ParamGroup::Quats, Trainer::ParamGroup::Scales,
            Trainer::ParamGroup::Opacities, Trainer::ParamGroup::Sh0, Trainer::ParamGroup::ShN};
        for (int g = 0; g < 6; g++) {
            if (dims[g] == 0) continue;
            Trainer::AdamState& st = tr.adam_state(groups[g]);
            std::copy(exp_avg[g], exp_avg[g] + count * dims[g], st.exp_avg.begin());
            std::copy(exp_avg_sq[g], exp_avg_sq[g] + count * dims[g], st.exp_avg_sq.begin());
        }
        int64_t nd = 0, na = 0;
        for (int r = 0; r < n_refines; r++) {
            const Trainer::McmcRefineResult res = tr.mcmc_refine();
            stats[3 * r] = tr.cloud().count;
            stats[3 * r + 1] = static_cast<int64_t>(res.relocated_dead.size());
            stats[3 * r + 2] = static_cast<int64_t>(res.added_src.size());
            for (size_t j = 0; j < res.relocated_dead.size() && nd < list_cap; j++, nd++) {
                dead[nd] = res.relocated_dead[j];
                src[nd] = res.relocation_src[j];
            }
            for (size_t j = 0; j < res.added_src.size() && na < list_cap; j++) added[na++] = res.added_src[j];
        }
        const SplatCloud& out = tr.cloud();
        const std::vector<float>* ov[6] = {&out.means, &out.quats, &out.scales, &out.opacities,
                                           &out.sh0, &out.shN};
        for (int g = 0; g < 6; g++) {
            if (dims[g] == 0) continue;
            std::copy(ov[g]->begin(), ov[g]->begin() + cap_max * dims[g], params[g]);
            Trainer::AdamState& st = tr.adam_state(groups[g]);
            std::copy(st.exp_avg.begin(), st.exp_avg.begin() + cap_max * dims[g], exp_avg[g]);
            std::copy(st.exp_avg_sq.begin(), st.exp_avg_sq.begin() + cap_max * dims[g], exp_avg_sq[g]);
        }
    });
}


// ---- PLY IO, export filter and eval metrics of the reference (PlyIO.cpp, Trainer.cpp) ----
namespace {
SplatCloud cloud_from(int64_t n, int deg, const float* means, const float* scales,
                      const float* quats, const float* op, const float* sh0, const float* shN) {
    SplatCloud c;
    c.count = n;
    c.sh_degree = deg;
    const int64_t K3 = static_cast<int64_t>(c.sh_rest_coeffs()) * 3;
    c.means.assign(means, means + n * 3);
    c.scales.assign(scales, scales + n * 3);
    c.quats.assign(quats, quats + n * 4);
    c.opacities.assign(op, op + n);
    c.sh0.assign(sh0, sh0 + n * 3);
    c.shN.assign(shN, shN + n * K3);
    return c;
}
void cloud_to(const SplatCloud& c, float* means, float* scales, float* quats, float* op,
              float* sh0, float* shN) {
    put(means, c.means);
    put(scales, c.scales);
    put(quats, c.quats);
    put(op, c.opacities);
    put(sh0, c.sh0);
    put(shN, c.shN);
}
}  // namespace

int sxr_ply_write(int64_t n, int deg, const float* means, const float* scales, const float* quats,
                  const float* op, const float* sh0, const float* shN, const char* path, int pad) {
    return guarded([&] { write_inria_ply(cloud_from(n, deg, means, scales, quats, op, sh0, shN), path, pad != 0); });
}

int sxr_ply_info(const char* path, int64_t* n, int* deg) {
    return guarded([&] {
        const SplatCloud c = read_inria_ply(path);
        *n = c.count;
        *deg = c.sh_degree;
    });
}

int sxr_ply_read(const char* path, float* means, float* scales, float* quats, float* op,
                 float* sh0, float* shN) {
    return guarded([&] { cloud_to(read_inria_ply(path), means, scales, quats, op, sh0, shN); });
}

// filter_cloud_for_export: the kept rows are written back into the input arrays' first rows.
int sxr_filter_for_export(int64_t n, int deg, float* means, float* scales, float* quats, float* op,
                          float* sh0, float* shN, float min_opacity, int64_t* stats) {
    return guarded([&] {
        ExportFilterStats st;
        const SplatCloud out = filter_cloud_for_export(
            cloud_from(n, deg, means, scales, quats, op, sh0, shN), min_opacity, &st);
        cloud_to(out, means, scales, quats, op, sh0, shN);
        stats[0] = st.input;
        stats[1] = st.removed_nonfinite;
        stats[2] = st.removed_low_opacity;
        stats[3] = st.kept;
    });
}

int sxr_psnr(const float* a, const float* b, int64_t n, float* out) {
    return guarded([&] { *out = psnr(a, b, n); });
}

int sxr_color_correct(const float* img, const float* ref, int64_t n, float* out) {
    return guarded([&] { color_correct_affine(img, ref, n, out); });
}


// ---- the reference's SXCK checkpoint files (Checkpoint.cpp) ----
// cfg_i: sh_degree, factor, test_split, total_iters, mcmc_enabled, antialiased;
// cfg_l: cap_max, mcmc_seed; cfg_f: scene_scale, ssim_weight. params / m / v: the six groups
// (D3 order) of n rows each.
namespace {
CheckpointConfig ck_config(const int32_t* ci, const int64_t* cl, const float* cf) {
    CheckpointConfig c;
    c.sh_degree = ci[0];
    c.factor = ci[1];
    c.test_split = ci[2];
    c.total_iters = ci[3];
    c.mcmc_enabled = static_cast<uint8_t>(ci[4]);
    c.antialiased = static_cast<uint8_t>(ci[5]);
    c.cap_max = cl[0];
    c.mcmc_seed = static_cast<uint64_t>(cl[1]);
    c.scene_scale = cf[0];
    c.ssim_weight = cf[1];
    return c;
}
}  // namespace

int sxr_checkpoint_save(const int32_t* ci, const int64_t* cl, const float* cf, int32_t iter,
                        int64_t n, float* const* params, float* const* m, float* const* v,
                        const char* rng, const char* path, int fp16) {
    return guarded([&] {
        TrainerCheckpoint ck;
        ck.config = ck_config(ci, cl, cf);
        ck.iter = iter;
        ck.cloud.count = n;
        ck.cloud.sh_degree = ck.config.sh_degree;
        const int64_t K3 = static_cast<int64_t>(ck.cloud.sh_rest_coeffs()) * 3;
        const int64_t dims[6] = {3, 4, 3, 1, 3, K3};
        std::vector<float>* g[6] = {&ck.cloud.means, &ck.cloud.quats, &ck.cloud.scales,
                                    &ck.cloud.opacities, &ck.cloud.sh0, &ck.cloud.shN};
        for (int k = 0; k < 6; k++) {
            g[k]->assign(params[k], params[k] + n * dims[k]);
            ck.moments[k].exp_avg.assign(m[k], m[k] + n * dims[k]);
            ck.moments[k].exp_avg_sq.assign(v[k], v[k] + n * dims[k]);
        }
        ck.mcmc_rng_state = rng ? rng : "";
        save_checkpoint_file(ck, path, fp16 != 0);
    });
}

int sxr_checkpoint_load(const char* path, int32_t* ci, int64_t* cl, float* cf, int32_t* iter,
                        int64_t* n, float* const* params, float* const* m, float* const* v,
                        char* rng, int64_t rng_cap, int64_t* rng_len) {
    return guarded([&] {
        const TrainerCheckpoint ck = load_checkpoint_file(path);
        ci[0] = ck.config.sh_degree; ci[1] = ck.config.factor; ci[2] = ck.config.test_split;
        ci[3] = ck.config.total_iters; ci[4] = ck.config.mcmc_enabled; ci[5] = ck.config.antialiased;
        cl[0] = ck.config.cap_max; cl[1] = static_cast<int64_t>(ck.config.mcmc_seed);
        cf[0] = ck.config.scene_scale; cf[1] = ck.config.ssim_weight;
        *iter = ck.iter;
        *n = ck.cloud.count;
        *rng_len = static_cast<int64_t>(ck.mcmc_rng_state.size());
        if (rng && rng_cap >= *rng_len) std::memcpy(rng, ck.mcmc_rng_state.data(), ck.mcmc_rng_state.size());
        if (!params) return;  // header-only call
        const std::vector<float>* g[6] = {&ck.cloud.means, &ck.cloud.quats, &ck.cloud.scales,
                                          &ck.cloud.opacities, &ck.cloud.sh0, &ck.cloud.shN};
        for (int k = 0; k < 6; k++) {
            put(params[k], *g[k]);
            put(m[k], ck.moments[k].exp_avg);
            put(v[k], ck.moments[k].exp_avg_sq);
        }
    });
}

int sxr_checkpoint_verify(const int32_t* ci_s, const int64_t* cl_s, const float* cf_s,
                          const int32_t* ci_c, const int64_t* cl_c, const float* cf_c) {
    return guarded([&] { verify_checkpoint_config(ck_config(ci_s, cl_s, cf_s), ck_config(ci_c, cl_c, cf_c)); });
}


// ---- the reference's COLMAP loader + TrainingInput conversion ----
// First call with viewmats NULL: counts only. Then arrays of n_images cameras / n_points seeds;
// names are written NUL-separated into names (capacity names_cap).
int sxr_colmap_load(const char* sparse, const char* images, int64_t* n_images, int64_t* n_points,
                    float* viewmats, float* Ks, int32_t* widths, int32_t* heights, float* points,
                    uint8_t* rgb, char* names, int64_t names_cap) {
    return guarded([&] {
        const TrainingInput ti = training_input_from_colmap(load_colmap_bundle(sparse), images);
        *n_images = static_cast<int64_t>(ti.cameras.size());
        *n_points = static_cast<int64_t>(ti.seed_points.size() / 3);
        if (!viewmats) return;
        int64_t off = 0;
        for (size_t i = 0; i < ti.cameras.size(); i++) {
            const TrainingCamera& c = ti.cameras[i];
            std::memcpy(viewmats + i * 16, c.viewmat, 64);
            std::memcpy(Ks + i * 9, c.K, 36);
            widths[i] = c.width;
            heights[i] = c.height;
            const std::string& p = c.image_path;
            if (off + static_cast<int64_t>(p.size()) + 1 <= names_cap) {
                std::memcpy(names + off, p.c_str(), p.size() + 1);
                off += static_cast<int64_t>(p.size()) + 1;
            }
        }
        put(points, ti.seed_points);
        put(rgb, ti.seed_rgb);
    });
}


// ---- the reference's SPZ files (SpzIO.cpp over the vendored spz v2.1.0) ----
int sxr_spz_write(int64_t n, int deg, const float* means, const float* scales, const float* quats,
                  const float* op, const float* sh0, const float* shN, const char* path,
                  float min_opacity, int antialiased, int64_t* stats) {
    return guarded([&] {
        SpzSaveOptions o;
        o.min_opacity = min_opacity;
        o.antialiased = antialiased != 0;
        ExportFilterStats st;
        o.filter_stats = &st;
        save_spz(cloud_from(n, deg, means, scales, quats, op, sh0, shN), path, o);
        stats[0] = st.input;
        stats[1] = st.removed_nonfinite;
        stats[2] = st.removed_low_opacity;
        stats[3] = st.kept;
    });
}

int sxr_spz_info(const char* path, int64_t* n, int* deg, int* antialiased) {
    return guarded([&] {
        bool aa = false;
        const SplatCloud c = load_spz(path, &aa);
        *n = c.count;
        *deg = c.sh_degree;
        *antialiased = aa ? 1 : 0;
    });
}

int sxr_spz_read(const char* path, float* means, float* scales, float* quats, float* op,
                 float* sh0, float* shN) {
    return guarded([&] { cloud_to(load_spz(path, nullptr), means, scales, quats, op, sh0, shN); });
}


// ---- the reference's trainer schedules and init (Trainer.cpp:270-330, :470-508) ----
float sxr_means_lr_at(int total_iters, float lr_means, float scene_scale, int iter) {
    TrainConfig c;
    c.total_iters = total_iters;
    c.lr_means = lr_means;
    c.scene_scale = scene_scale;
    return means_lr_at(c, iter);
}

uint32_t sxr_sh_degree_at(int total_iters, float interval_ratio, int iter, int sh_degree) {
    TrainConfig c;
    c.total_iters = total_iters;
    c.sh_degree_interval_ratio = interval_ratio;
    return sh_degree_at(c, iter, sh_degree);
}

float sxr_scene_scale(const float* viewmats, int64_t n) {
    std::vector<TrainingCamera> cams(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; i++) std::memcpy(cams[i].viewmat, viewmats + i * 16, 64);
    return scene_scale_from_cameras(cams);
}

// init_splats into caller arrays sized min(M, max_points) rows (sh_degree's shN width).
int sxr_init_splats(const float* pts, const uint8_t* rgb, int64_t M, int64_t max_points,
                    float init_opacity, float init_scale, int sh_degree, float* means,
                    float* scales, float* quats, float* op, float* sh0, float* shN) {
    return guarded([&] {
        TrainingInput ti;
        ti.seed_points.assign(pts, pts + M * 3);
        ti.seed_rgb.assign(rgb, rgb + M * 3);
        InitOptions o;
        o.max_points = max_points;
        o.init_opacity = init_opacity;
        o.init_scale = init_scale;
        o.sh_degree = sh_degree;
        cloud_to(init_splats(ti, o), means, scales, quats, op, sh0, shN);
    });
}

}  // extern "C"
