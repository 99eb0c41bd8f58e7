/*
 * sx_oracle.h — CPU oracle of splatx-metal's 3DGS training step. TEST INFRASTRUCTURE ONLY:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may load it,
 * and only as the checker or the timed CPU reference — never as a product path.
 *
 * A plain-C (C11, no FMA contraction, glibc libm) restatement of the reference's CPU algorithms:
 * forward kernels follow Sources/SplatXCore/CpuKernels.cpp (file:line per function in
 * sx_oracle.c); the backward kernels, which the reference has no CPU code for, are restated from
 * its kernel specs and Metal sources and pinned against the gsplat autograd goldens; the training
 * step follows Trainer::step (Trainer.cpp:974-1131).
 * Output buffers are caller-allocated and (for accumulating outputs) zero-initialised.
 */
#ifndef SX_ORACLE_H
#define SX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Threads used by the OpenMP loops (n <= 0 leaves it unchanged); returns the effective count. */
int32_t sxo_set_threads(int32_t n);
uint32_t sxo_bits_for_count(int64_t count);

void sxo_fused_adam(float* param, const float* grad, float* exp_avg, float* exp_avg_sq,
                    const uint8_t* valid, int64_t n_elems, int64_t n_gauss, float lr, float b1,
                    float b2, float eps);

void sxo_projection_fused_fwd(const float* means, const float* covars6, const float* quats,
                              const float* scales, const float* opacities, const float* viewmats,
                              const float* Ks, int64_t N, int64_t C, int32_t width, int32_t height,
                              float eps2d, float near_plane, float far_plane, float radius_clip,
                              int32_t calc_comp, int32_t* radii, float* means2d, float* depths,
                              float* conics, float* comps);

void sxo_projection_fused_bwd(const float* means, const float* covars6, const float* quats,
                              const float* scales, const float* viewmats, const float* Ks,
                              int64_t N, int64_t C, int32_t width, int32_t height, float eps2d,
                              const int32_t* radii, const float* conics, const float* comps,
                              const float* v_means2d, const float* v_depths, const float* v_conics,
                              const float* v_comps, float* v_means, float* v_covars,
                              float* v_quats, float* v_scales, float* v_viewmats);

void sxo_sh_fwd(const float* dirs, const float* coeffs, const uint8_t* masks, uint32_t degree,
                int64_t B, int64_t N, int64_t K, uint32_t D, float* colors);
void sxo_sh_bwd(const float* dirs, const float* coeffs, const uint8_t* masks, uint32_t degree,
                int64_t B, int64_t N, int64_t K, uint32_t D, const float* v_colors,
                float* v_coeffs, float* v_dirs);

/* Intersection: count (returns n_isects) then emit in the reference's order. conics/opacities
 * both NULL selects AABB, both non-NULL AccuTile. */
int64_t sxo_isect_count(const float* means2d, const int32_t* radii, const float* conics,
                        const float* opacities, int64_t n, uint32_t tile_size, uint32_t tile_width,
                        uint32_t tile_height, int32_t* tiles_per_gauss);
void sxo_isect_emit(const float* means2d, const int32_t* radii, const float* depths,
                    const float* conics, const float* opacities, int64_t I, int64_t N,
                    uint32_t tile_size, uint32_t tile_width, uint32_t tile_height,
                    const int32_t* tiles_per_gauss, uint64_t* isect_ids, int32_t* flatten_ids);
/* Stable ascending sort of u64 keys carrying i32 values. Returns -1 when a key has bits at or
 * above key_n_bits (the reference throws there), else 0. */
int32_t sxo_sort_isect(const uint64_t* keys, const int32_t* values, int64_t n,
                       uint32_t key_n_bits, uint64_t* keys_sorted, int32_t* values_sorted);
void sxo_isect_offset_encode(const uint64_t* isect_ids, int64_t n_isects, int64_t I,
                             uint32_t tile_width, uint32_t tile_height, int32_t* offsets);

void sxo_rasterize_fwd(const float* means2d, const float* conics, const float* colors,
                       const float* opacities, const float* backgrounds, const uint8_t* masks,
                       const int32_t* offsets, const int32_t* flatten_ids, int64_t I, int64_t N,
                       int64_t n_isects, uint32_t width, uint32_t height, uint32_t tile_size,
                       uint32_t tile_width, uint32_t tile_height, float* render_colors,
                       float* render_alphas, int32_t* last_ids);
void sxo_rasterize_bwd(const float* means2d, const float* conics, const float* colors,
                       const float* opacities, const float* backgrounds, const uint8_t* masks,
                       const int32_t* offsets, const int32_t* flatten_ids, int64_t I, int64_t N,
                       int64_t n_isects, uint32_t width, uint32_t height, uint32_t tile_size,
                       uint32_t tile_width, uint32_t tile_height, const float* render_alphas,
                       const int32_t* last_ids, const float* v_render_colors,
                       const float* v_render_alphas, float* v_means2d, float* v_conics,
                       float* v_colors, float* v_opacities, float* v_means2d_abs);

double sxo_ssim_fwd(const float* img1, const float* img2, int64_t I, int64_t H, int64_t W,
                    int64_t C, int32_t need_coeffs, float* map, float* coeff_mu,
                    float* coeff_sigma, float* coeff_cross);
void sxo_ssim_bwd(const float* img1, const float* img2, int64_t I, int64_t H, int64_t W,
                  int64_t C, const float* coeff_mu, const float* coeff_sigma,
                  const float* coeff_cross, float v_loss, float* v_img1);

void sxo_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
void sxo_rng_philox_u32(uint64_t seed, uint64_t offset, int64_t count, uint32_t* out);
void sxo_rng_normal_f32(uint64_t seed, uint64_t offset, int64_t count, float* out);
void sxo_make_binoms_lut(int32_t n_max, float* lut);
/* Returns -1 when a ratio lies outside [1, n_max] (the reference throws there), else 0. */
int32_t sxo_mcmc_relocation(const float* opacities, const float* scales, const int32_t* ratios,
                            const float* binoms, int64_t N, int32_t n_max, float min_opacity,
                            float* new_opacities, float* new_scales);
void sxo_mcmc_perturb_positions(float* positions, const float* quats, const float* scales_log,
                                const float* opacities_logit, const float* noise, int64_t N,
                                float noise_scale, float t, float k);

/* The host round-trip training step (Trainer::step). params/exp_avg/exp_avg_sq: six groups in the
 * D3 order (means, quats, log-scales, logit opacities, sh0, shN), `count` rows each, updated in
 * place. Returns 0, or -1 on a contract violation. */
typedef struct SxoStepConfig {
    int32_t sh_degree;
    uint32_t degrees_to_use;
    float lr[6];
    float b1, b2, eps;
    float eps2d, near_plane, far_plane, radius_clip;
    float ssim_weight;
    int32_t antialiased;
    float opacity_reg, scale_reg;
    int32_t inject_noise;
    uint64_t noise_seed, noise_offset;
    float noise_scale;
    int32_t forward_only;
} SxoStepConfig;

/* The activations of Trainer::step's host path: exp of the log-scales, sigmoid of the logits. */
void sxo_train_activations(const float* log_scales, const float* logits, int64_t N, float* s_lin,
                           float* sig);

/* Training loss of a render against its target and the gradient with respect to the render
 * (the host loss of Trainer::step, L1 + optional SSIM; v holds H*W*3 floats). */
float sxo_train_loss(const float* render, const float* gt, int32_t H, int32_t W, float ssim_weight,
                     float* v_render);

int32_t sxo_train_step(float* const* params, float* const* exp_avg, float* const* exp_avg_sq,
                       int64_t count, const float* viewmat, const float* K, int32_t width,
                       int32_t height, const float* gt_rgb, const SxoStepConfig* cfg,
                       float* loss_out, int64_t* n_isects_out, float* render_out);

/* ---- MCMC refine (Trainer::mcmc_refine, Trainer.cpp:1195-1435) ----
 * mt19937_64: the 64-bit Mersenne Twister of Matsumoto and Nishimura (2000), with the parameters
 * the C++ standard fixes for std::mt19937_64 ([rand.predef]); the reference's multinomial engine. */
typedef struct SxoMt64 {
    uint64_t x[312];
    int32_t i;
} SxoMt64;
void sxo_mt64_seed(SxoMt64* g, uint64_t seed);
uint64_t sxo_mt64_next(SxoMt64* g);

/* multinomial_with_replacement (Trainer.cpp:1199-1217). Returns -1 for a negative/NaN weight or a
 * zero sum (the reference throws there), else 0. */
int32_t sxo_multinomial(const float* weights, int64_t n, int64_t n_samples, SxoMt64* rng,
                        int64_t* out);

/* One refine on host arrays: six groups in the D3 order, [arena rows, dims[g]] each (dims[g] may
 * be 0), rows [0, count) alive. relocate (Trainer.cpp:1284-1340), then add (:1342-1394). The index
 * lists receive up to `count` (dead, sources) and cap_max - count (added) entries. Returns -1 on a
 * contract violation (the reference throws), else 0. */
typedef struct SxoMcmcResult {
    int64_t count, n_relocated, n_added;
} SxoMcmcResult;
int32_t sxo_mcmc_refine(SxoMt64* rng, float* const* params, float* const* exp_avg,
                        float* const* exp_avg_sq, const int64_t* dims, int64_t count,
                        int64_t cap_max, float min_opacity, int64_t* relocated_dead,
                        int64_t* relocation_src, int64_t* added_src, SxoMcmcResult* out);

#ifdef __cplusplus
}
#endif

#endif
