// sx_internal.h — host-side launchers shared between the translation units of libsplatx_cuda.
// Every launcher enqueues on `stream` and throws sx::RuntimeError on a launch failure.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/splatx_cuda.h"
#include "sx_geometry_exact.cuh"

// A loaded COLMAP sparse model (colmap.cu).
struct SxColmap {
    struct Camera {
        int32_t id = 0, model = 0;
        int64_t width = 0, height = 0;
        std::vector<double> params;
        float fx = 0, fy = 0, cx = 0, cy = 0;
    };
    struct Image {
        int32_t id = 0, camera_id = 0;
        double q[4] = {}, t[3] = {};
        std::string name;
    };
    std::vector<Camera> cameras;
    std::vector<Image> images;
    std::vector<double> xyz;     // [M, 3]
    std::vector<uint8_t> rgb;    // [M, 3]
    std::string images_dir;
};

namespace sx {

// ---------------- per-step parameters of the resident step ----------------
// The values that change from step to step (camera, learning rates, regularisers, noise) live in
// device memory and are read by the step's kernels, so one captured CUDA graph replays any step
// of the same shape.
struct FwdGaussConst {
    PinholeCam cam;
    float campos[3];
    ProjParams p;
    TileGrid g;
};
struct BwdGaussConst {
    float R[9], t[3], campos[3];
    float fx, fy, cx, cy;
};
struct StepParams {
    FwdGaussConst fwd;
    BwdGaussConst bwd;
    float lr[6];
    float opacity_reg_w, scale_reg_w;
    float noise_scale;
    int32_t inject_noise;
    uint64_t noise_seed, noise_offset;
};
// Host: the step constants from a row-major world->camera viewmat and K (campos = -R^T t summed
// in the reference's order, Trainer.cpp:754-757).
void fill_step_camera(StepParams& sp, const float* viewmat, const float* K, int width, int height,
                      const ProjParams& p, uint32_t tile_width, uint32_t tile_height);

// ---------------- forward.cu (compiled with -fmad=false) ----------------
void launch_projection_fwd(const SxProjectionFusedInputs& in, const SxProjectionFusedOutputs& out,
                           cudaStream_t s);
void launch_sh_fwd(const SxShInputs& in, float* colors, cudaStream_t s);
void launch_isect_count(const SxIsectTilesInputs& in, int32_t* tiles_per_gauss, cudaStream_t s);
void launch_isect_emit(const SxIsectTilesInputs& in, uint32_t tile_n_bits,
                       const int64_t* cum_tiles_per_gauss, uint64_t* isect_ids,
                       int32_t* flatten_ids, cudaStream_t s);
void launch_offset_encode(const uint64_t* isect_ids, int64_t n_isects, int64_t I,
                          uint32_t tile_n_bits, int64_t n_tiles, int32_t* offsets,
                          cudaStream_t s);

// Executor forward: one thread per Gaussian — activations, projection, SH colour + post-op,
// AccuTile count, depth sort key.
struct FwdGaussArgs {
    const float* means;
    const float* quats;
    const float* log_scales;
    const float* opac_logit;
    const float* sh0;
    const float* shN;
    int32_t K;  // bands stored per Gaussian
    uint32_t degree;
    int32_t count;
    const StepParams* step;  // device: camera and projection constants
    int32_t antialiased;
    // outputs
    uint8_t* valid;        // [N] radii>0
    float* means2d;        // [N,2]
    float* conics;         // [N,3]
    float* opac_raster;    // [N] sigmoid (x compensation when antialiased)
    float* comps;          // [N] compensation (antialiased only)
    float* act;            // tiles of 4: exp(log-scale) x3, sigmoid(opacity logit) (valid only)
    float* colors;         // [N,3] SH + 0.5, clamped at 0
    uint8_t* relu_mask;    // [N] bit c set when channel c was not clamped
    int32_t* tiles;        // [N] AccuTile tile count
    int32_t* entries;      // [N] supertiles holding those tiles (null: not counted)
    uint32_t* depth_keys;  // [N] f32 bits of depth, 0xffffffff when no tile
    int32_t* gauss_ids;    // [N] identity (the sort's values)
    float4* rec;           // [N,3] packed raster records of the visible Gaussians (RasterArgs::rec)
};
void launch_fwd_gauss(const FwdGaussArgs& a, cudaStream_t s);

// Resident-arena layout conversion: [n, d] rows <-> 32-Gaussian tiles, rows r0 .. r0+n-1.
void launch_rows_to_tiles(const float* rows, float* tiles, int d, int64_t n, int64_t r0,
                          cudaStream_t s);
void launch_tiles_to_rows(const float* tiles, float* rows, int d, int64_t n, int64_t r0,
                          cudaStream_t s);

// Executor emit: Gaussians in depth order write (tile id, gaussian id) pairs at their offsets.
struct EmitArgs {
    const int32_t* order;      // [n] gaussian ids sorted by depth
    const int32_t* offsets;    // [n] exclusive scan of tiles[order[j]]
    const int32_t* tiles;      // [N]
    const float* means2d;
    const float* conics;
    const float* opac_raster;
    int32_t n;                 // visible+culled count (== count)
    uint32_t tile_width, tile_height;
    const int64_t* n_isects;   // device total
    int64_t capacity;
    uint32_t* tile_keys;       // [capacity]
    int32_t* gauss_vals;       // [capacity]
    int32_t* overflow;         // device flag
};
void launch_emit_depth_ordered(const EmitArgs& a, cudaStream_t s);

// ---------------- supertile binning (forward.cu: emit; tile_bins.cu: the rest) ----------------
// The executor's tile lists without a sort over every intersection. A supertile is a block of
// kStTiles x kStTiles tiles; each visible Gaussian holds one ENTRY per supertile its AccuTile tiles
// fall in, carrying the 64-bit mask of those tiles (bit (ty % 8) * 8 + tx % 8). Entries are
// written in depth order and sorted stably by supertile (one 7..14-bit pass over ~1/10 as many
// items as intersections); each supertile's run is cut into chunks of kStChunk entries, and
// per-chunk tile counts, their prefixes and the tile offsets give every (entry, tile) pair its
// slot — the same list a stable sort of depth-ordered (tile, Gaussian) pairs produces.
constexpr int kStTiles = 8;
constexpr int kStChunk = 64;
constexpr int64_t kStMaxSupertiles = 16384;  // the entry sort's whole-key histogram bound

struct EmitStArgs {
    const int32_t* order;      // [n] gaussian ids sorted by depth
    const int32_t* offsets;    // [n] exclusive scan of entries[order[j]]
    const int32_t* entries;    // [N] entries per Gaussian
    const float* means2d;
    const float* conics;
    const float* opac_raster;
    int32_t n;
    uint32_t tile_width, tile_height, st_width;
    const int32_t* overflow;   // device flag: set -> nothing is written
    uint32_t* st_keys;         // [capacity] supertile of the entry
    int32_t* entry_ids;        // [capacity] the entry's own index (the sort's values)
    uint4* entry;              // [capacity] (tile mask lo, tile mask hi, Gaussian id, 0)
};
void launch_emit_supertiles(const EmitStArgs& a, cudaStream_t s);

struct StBinArgs {
    const int32_t* sorted;     // [entries] entry indices, stably sorted by supertile
    const int32_t* st_offsets; // [n_st] first sorted position of each supertile
    const int64_t* n_entries;  // device: entries to bin (0 after an overflow)
    const uint4* entry;        // (tile mask lo, tile mask hi, Gaussian id, 0) by entry index
    const int32_t* overflow;   // device flag: set -> every tile empty, nothing written
    int32_t n_st, st_width;
    uint32_t tile_width, tile_height;
    int64_t max_chunks;        // chunk capacity (st_chunk_capacity)
    int32_t* st_chunk0;        // [n_st + 1] first chunk of each supertile
    int32_t* n_chunks;         // device scalar
    uint32_t* chunk_counts;    // [max_chunks][64]: counts, then exclusive prefixes per supertile
    int32_t* tile_counts;      // [n_tiles] scratch
    uint32_t* done;            // device counter, 0 between steps (st_prefix's last CTA resets it)
    int32_t* tile_offsets;     // [n_tiles] output: first slot of each tile
    int32_t* flatten_ids;      // [capacity] output: Gaussian ids, tile-major, depth order
};
int64_t st_chunk_capacity(int64_t capacity, int64_t n_st);
void launch_bin_supertiles(const StBinArgs& a, cudaStream_t s);

// ---------------- sort.cu ----------------
// Scan: inclusive int32 -> int64 (API) with `n` known on the host.
size_t scan_i64_workspace(int64_t n);
void launch_scan_i64(const int32_t* in, int64_t* out, int64_t n, void* ws, cudaStream_t s);
// Allocation-free variant: block totals live in a fixed file-scope device array (sort.cu).
void launch_scan_i64_noalloc(const int32_t* in, int64_t* out, int64_t n, cudaStream_t s);
int64_t noalloc_scan_max_n();
// Exclusive scan of in[gather[j]] (gather may be null) -> int32 out, total -> *total (device).
// With gather and `side`, the same pass also sums side[0..n) (in plain order) into *side_total.
size_t scan_gather_workspace(int64_t n);
void launch_scan_gather_excl(const int32_t* in, const int32_t* gather, int32_t* out,
                             int64_t* total, int64_t n, void* ws, cudaStream_t s,
                             const int32_t* side = nullptr, int64_t* side_total = nullptr);

// Stable LSD radix sort (8-bit digits) of (key, value) pairs. `n_dev` (optional) overrides n with
// a device-resident count no larger than n (grids are sized by n).
size_t radix_sort_u64_workspace(int64_t n);
void radix_sort_u64(const uint64_t* keys_in, const int32_t* vals_in, uint64_t* keys_out,
                    int32_t* vals_out, int64_t n, uint32_t key_bits, void* ws, cudaStream_t s);
// The executor's single-sweep u32 sort (histogram + one kernel per pass with decoupled
// look-back). keys_out may be null: the sorted keys are then not written. With full_offsets, the
// exclusive scan of the whole-key histogram (full_bins bins) is written there as int32 offsets.
// A look-back wait that runs out sets kStatusSortLookbackTimeout in *status.
size_t onesweep_u32_workspace(int64_t n, uint32_t key_bits, int64_t full_bins);
void onesweep_sort_u32(const uint32_t* keys_in, const int32_t* vals_in, uint32_t* keys_out,
                       int32_t* vals_out, int64_t n, const int64_t* n_dev, uint32_t key_bits,
                       int32_t* full_offsets, int64_t full_bins, void* ws, uint32_t* status,
                       cudaStream_t s);
size_t radix_sort_u32_workspace(int64_t n);
void radix_sort_u32(const uint32_t* keys_in, const int32_t* vals_in, uint32_t* keys_out,
                    int32_t* vals_out, int64_t n, const int64_t* n_dev, uint32_t key_bits,
                    void* ws, cudaStream_t s);
// Tile offsets from tile-sorted u32 keys (executor): offsets[t] = first index with key >= t.
void launch_tile_offsets_u32(const uint32_t* sorted_tiles, const int64_t* n_dev, int64_t cap,
                             int64_t n_tiles, int32_t* offsets, cudaStream_t s);

// ---------------- raster.cu ----------------
struct RasterArgs {
    const float* means2d;
    const float* conics;
    const float* colors;
    const float* opacities;
    const float* backgrounds;
    const uint8_t* masks;
    const int32_t* offsets;
    const int32_t* flatten_ids;
    int64_t I, n_isects;
    const int64_t* n_isects_dev;  // overrides n_isects when non-null
    uint32_t width, height, tile_width, tile_height;
    // Diagnostic: when non-null, the forward adds the (pixel, Gaussian) pairs it evaluates to
    // pair_count[0] and the backward to pair_count[1] (one atomic per warp). Only without
    // backgrounds, masks and absgrad.
    unsigned long long* pair_count;
    // When non-null, the kernels stage Gaussian g from rec[3g .. 3g+2] = {x, y, opacity, 0},
    // {conic a, b, c, 0}, {r, g, b, 0} (16-byte aligned; written by the executor's forward) and
    // ignore means2d / conics / colors / opacities. Only without backgrounds, masks and absgrad.
    const float4* rec;
};
void launch_raster_fwd(const RasterArgs& a, float* render_colors, float* render_alphas,
                       int32_t* last_ids, cudaStream_t s);
void launch_raster_bwd(const RasterArgs& a, const float* render_alphas, const int32_t* last_ids,
                       const float* v_render_colors, const float* v_render_alphas,
                       float* v_means2d, float* v_conics, float* v_colors, float* v_opacities,
                       float* v_means2d_abs, cudaStream_t s);

// ---------------- ssim.cu ----------------
size_t ssim_fwd_workspace(int64_t I, int64_t H, int64_t W, int64_t C);
void launch_ssim_fwd(const float* img1, const float* img2, int64_t I, int64_t H, int64_t W,
                     int64_t C, bool need_coeffs, float* map, float* cmu, float* csg, float* ccr,
                     double* mean_out, void* ws, cudaStream_t s);
void launch_ssim_bwd(const float* img1, const float* img2, int64_t I, int64_t H, int64_t W,
                     int64_t C, const float* cmu, const float* csg, const float* ccr, float G,
                     float* v_img1, cudaStream_t s);
// Executor loss: fused L1 (+ SSIM) gradient into v_render and device loss scalar.
size_t loss_workspace(int64_t H, int64_t W);
void launch_train_loss(const float* render, const float* gt, int64_t H, int64_t W,
                       float ssim_weight, float* map, float* cmu, float* csg, float* ccr,
                       float* v_render, float* loss_out, void* ws, const int32_t* skip_flag,
                       cudaStream_t s);

// ---------------- backward.cu ----------------
void launch_adam(const SxAdamInputs& in, cudaStream_t s);
void launch_projection_bwd(const SxProjectionFusedInputs& in, const SxProjectionFusedGradsIn& g,
                           const SxProjectionFusedGrads& out, cudaStream_t s);
void launch_sh_bwd(const SxShInputs& in, const float* v_colors, float* v_coeffs, float* v_dirs,
                   cudaStream_t s);
void launch_rng_normal(uint64_t seed, uint64_t offset, int64_t count, float* out, cudaStream_t s);
void launch_rng_u32(uint64_t seed, uint64_t offset, int64_t count, uint32_t* out, cudaStream_t s);
void launch_relocation(const SxRelocationInputs& in, float* new_op, float* new_sc, cudaStream_t s);
void launch_perturb(const SxPerturbInputs& in, cudaStream_t s);

// Executor backward: one thread per Gaussian — relu mask, SH bwd, projection bwd (C=1),
// activation chains + regularisers, Adam on the six groups, optional MCMC noise.
struct BwdGaussArgs {
    float* means;
    float* quats;
    float* log_scales;
    float* opac_logit;
    float* sh0;
    float* shN;
    float* m[6];
    float* v[6];
    int32_t K;
    uint32_t degree;
    int32_t count;
    const StepParams* step;  // device: camera constants, learning rates, regularisers, noise
    int32_t width, height;
    float eps2d;
    int32_t antialiased;
    const uint8_t* valid;
    const float* conics;
    const float* comps;
    const uint8_t* relu_mask;
    float* v_means2d;  // consumed and re-zeroed
    float* v_conics;
    float* v_colors;
    float* v_opac;
    float b1, b2, eps;
    const int32_t* skip_flag;  // device: non-zero -> the step overflowed, leave params untouched
    const float* act;          // tiles of 4: the forward's exp(log-scale) x3, sigmoid(logit)
    float* v_dir;              // tiles of 3: SH direction gradient, bwd_sh -> bwd_geom
    // Gradient-accumulation mode (view-parallel training): 0 = Adam in place; 1 = the six groups'
    // gradients (data terms only) are ADDED to gacc (same tiled layout as the parameters) and
    // gvis (tiles of 1) counts the views a Gaussian was visible in; 2 = as 1 but the view is the
    // first of its step, so gacc / gvis are WRITTEN (rows the view does not see get zeros) and
    // need no clearing beforehand. Modes 1 and 2 run no Adam and no noise.
    int32_t accumulate;
    float* gacc[6];
    float* gvis;
    // Row subset (view-parallel exchange overlap): with map_world > 0 the launch covers rows
    // r * map_shard + [map_c0, map_c1) for every rank r < map_world instead of [0, count).
    int32_t map_world;
    int64_t map_shard, map_c0, map_c1;
};

// ---------------- io.cu (host) ----------------
void ply_write(const SxCloud& c, const char* path, bool pad_sh_full);
void ply_info(const char* path, int64_t* count, int32_t* degree);
void ply_read(const char* path, const SxCloud& out);
void filter_for_export(const SxCloud& c, float min_opacity, uint8_t* keep, SxExportFilterStats& st);
// spz.cu (host)
void spz_write(const SxCloud& c, const char* path, float min_opacity, bool antialiased,
               SxExportFilterStats& st);
void spz_info(const char* path, int64_t* count, int32_t* degree, int32_t* antialiased);
void spz_read(const char* path, const SxCloud& out);

// ---------------- checkpoint.cu ----------------
struct ArenaView;
void checkpoint_verify(const SxCheckpointConfig& saved, const SxCheckpointConfig& current);
void checkpoint_header(const char* path, SxCheckpointHeader& out);
void checkpoint_save(const ArenaView& a, float* stage, int64_t stage_rows,
                     const SxCheckpointConfig& cfg, int32_t iter, int64_t count,
                     const std::string& rng_state, const char* path, bool fp16);
void checkpoint_load(const ArenaView& a, float* stage, int64_t stage_rows, const char* path,
                     const SxCheckpointConfig* current, SxCheckpointHeader& out,
                     std::string& rng_state);

// ---------------- colmap.cu (host) ----------------
SxColmap* colmap_open(const char* sparse_dir, const char* images_dir);
void colmap_cameras(const SxColmap& b, float* viewmats, float* Ks, int32_t* widths, int32_t* heights);

// ---------------- eval.cu ----------------
size_t eval_workspace();  // bytes of the per-block double partials
void launch_clamp01(float* x, int64_t n, cudaStream_t s);
// *out = sum of (a - b)^2 in double (fixed-order reduction)
void launch_sum_sqdiff(const float* a, const float* b, int64_t n, double* parts, double* out,
                       cudaStream_t s);
// out = color_correct_affine(img, ref); moments: 12 doubles of device scratch
void launch_color_correct(const float* img, const float* ref, int64_t n_px, double* parts,
                          double* moments, float* out, cudaStream_t s);
void launch_rgba8(const float* rgb, int64_t n_px, uint8_t* out, cudaStream_t s);

// ---------------- MCMC refine on the resident arena (backward.cu) ----------------
// Position noise of rows [0, count) of the tiled arena (the in-step noise, run on its own).
void launch_noise_rows(float* means, const float* quats, const float* log_scales,
                       const float* opac_logit, int64_t count, uint64_t seed, uint64_t offset,
                       float noise_scale, cudaStream_t s);
// Gathers the three log-scales of rows idx[j] (tiled layout) into out[j*3 + k].
void launch_gather_log_scales(const float* log_scales, const int64_t* idx, int64_t n, float* out,
                              cudaStream_t s);
// Writes the relocated source rows: opacity logit and three log-scales of row idx[j]. Rows may
// repeat in idx; repeats carry identical values.
void launch_write_sources(float* opac_logit, float* log_scales, const int64_t* idx,
                          const float* logits, const float* log_scales_new, int64_t n, cudaStream_t s);
// Copies every parameter group's row src[j] to row dst[j] (tiled layout, dims[g] floats per row).
struct RowCopyArgs {
    float* p[6];
    int32_t dims[6];
};
void launch_copy_rows(const RowCopyArgs& a, const int64_t* dst, const int64_t* src, int64_t n,
                      cudaStream_t s);
// Zeroes both Adam moments of rows idx[j] in every group.
struct MomentRowsArgs {
    float* m[6];
    float* v[6];
    int32_t dims[6];
};
void launch_zero_moment_rows(const MomentRowsArgs& a, const int64_t* idx, int64_t n, cudaStream_t s);

// MCMC refine orchestration (mcmc.cu). The arena is the executor's tiled parameters and moments.
struct ArenaView {
    float* p[6];
    float* m[6];
    float* v[6];
    int32_t dims[6];
    int64_t rows;
    int device;
    cudaStream_t stream;
};
struct McmcRefineOut {
    int64_t count = 0;
    std::vector<int64_t> relocated_dead, relocation_src, added_src;
};
struct McmcRefine;
McmcRefine* mcmc_new();
void mcmc_delete(McmcRefine* m);
void mcmc_seed(McmcRefine* m, uint64_t seed);
std::string mcmc_rng_state(const McmcRefine* m);
void mcmc_set_rng_state(McmcRefine* m, const std::string& text);
// Relocate then add on rows [0, count) (synchronous); out.count = the alive rows afterwards.
void mcmc_refine(McmcRefine* m, const ArenaView& a, int64_t count, int64_t cap_max,
                 float min_opacity, McmcRefineOut& out);

// Adam over the resident rows [row_begin, row_end) (multiples of 32) from accumulated gradients:
// gradient = gacc / n_views (+ regularisers), rows with gvis == 0 untouched, then MCMC noise on
// rows < count, and the rows' gacc / gvis re-zeroed.
struct ApplyGradsArgs {
    float* p[6];
    float* m[6];
    float* v[6];
    float* gacc[6];
    float* gvis;
    int32_t K;
    int64_t row_begin, row_end, count;
    float inv_views;
    float lr[6];
    float b1, b2, eps;
    float opacity_reg_w, scale_reg_w;
    int32_t inject_noise;
    uint64_t noise_seed, noise_offset;
    float noise_scale;
};
void launch_apply_grads(const ApplyGradsArgs& a, cudaStream_t s);

// View-parallel exchange fused into one kernel over peer memory (CUDA IPC mappings over NVLink):
// for the owner shard [row_begin, row_end) of this rank, the gradients and visibility of every
// rank are read and summed in rank order (the reduce-scatter), Adam (+ regularisers, + noise) runs
// on the local moments, and every changed row is stored into every rank's parameter replica (the
// all-gather). Rows visible in no view are neither read beyond the visibility nor sent. The
// accumulators are not cleared: the caller zeroes them once every rank has finished reading.
constexpr int kMaxPeers = 8;
constexpr int kPeerBufs = 14;  // IPC buffers per rank: grads 0..5, visibility, params 0..5, flags
struct PeerApplyArgs {
    ApplyGradsArgs a;  // the local buffers, rows and Adam settings (a.gacc / a.gvis unused)
    int32_t world, rank;
    const float* gacc[kMaxPeers][6];  // every rank's accumulated gradients (self included)
    const float* gvis[kMaxPeers];
    float* params[kMaxPeers][6];      // every rank's parameter replica (self included)
    // The executor's status word (may be null): when a bounded wait of this step ran out (a
    // barrier whose peers did not all arrive, a sort look-back), the gradients may be incomplete
    // and the peers may still be reading, so the kernel returns without reading or writing.
    const uint32_t* status;
};
void launch_exchange_apply(const PeerApplyArgs& a, cudaStream_t s);

// Cross-GPU barrier over peer memory: every rank stores `epoch` into slot `rank` of every rank's
// flag array (released at system scope), then waits until all slots of its own array reached
// `epoch`. Each wait is bounded; a wait that runs out sets kStatusPeerBarrierTimeout in *status
// and the kernel returns. One block, world threads.
struct PeerBarrierArgs {
    uint32_t* flags[kMaxPeers];  // every rank's flag array (kMaxPeers slots each), self included
    int32_t world, rank;
    uint32_t epoch;
    uint32_t* status;
};
void launch_peer_barrier(const PeerBarrierArgs& b, cudaStream_t s);
// Rank 0 of `world` ranks whose other flag arrays (on the current device) nobody signals: the
// barrier's bounded wait runs out for world > 1. Returns the status bits the kernel set. Then,
// on a 32-row arena of this device (gradients and visibility 1), the exchange that follows a
// barrier in step_exchange: *applied = it changed the parameters (must be 0 after a timeout).
uint32_t peer_barrier_selftest(int world, int* applied);
void launch_bwd_gauss(const BwdGaussArgs& a, cudaStream_t s);

}  // namespace sx
