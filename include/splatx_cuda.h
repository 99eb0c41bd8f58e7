/*
 * splatx_cuda.h — C-ABI of the B200 (sm_100a) 3DGS training-step library.
 *
 * This is the drop-in boundary that replaces the Metal backend of splatx-metal. Every entry point
 * below stands in for one method of the reference's C++ kernel contract
 * (Sources/SplatXCore/include/splatx/KernelBackend.h) or of its resident step executor, and each
 * declaration cites the reference interface it replaces. Plain pointers and sizes only: no C++,
 * no torch types. A Swift, C or C++ host binds this header directly.
 *
 * Pointer conventions
 *   - Per-kernel entry points (sxcuda_* below the executor section) take DEVICE pointers and a
 *     CUDA stream (sxcuda_stream_t == cudaStream_t; NULL = the legacy default stream). They are
 *     asynchronous unless stated otherwise; inputs must stay alive until the stream reaches them.
 *   - The executor entry points (sxcuda_executor_*) mirror TrainStepExecutor and take HOST
 *     pointers (the reference's std::vector semantics); they synchronise before returning.
 *   - Entry points that need scratch follow the query protocol: pass workspace == NULL to receive
 *     the byte count in *workspace_bytes, then call again with a device buffer of that size.
 *     The library never allocates device memory on those calls.
 *
 * Errors (mirrors the reference: std::invalid_argument / std::runtime_error at KernelBackend,
 * 0/1 + err_buf at splatx_train_c.h:141-144)
 *   SXCUDA_OK       0  success
 *   SXCUDA_EINVAL   1  contract violation (the reference throws std::invalid_argument)
 *   SXCUDA_ERUNTIME 2  device or runtime failure (std::runtime_error), including an unsupported
 *                      camera model (Validate.h:50-53 raises runtime_error for it)
 *   The NUL-terminated message of the last failing call on this thread: sxcuda_last_error().
 *
 * Layouts follow the reference's D3/D6 contract (docs/kernel-specs/00-index.md §2): SoA flattened
 * fp32 arrays, quats [w,x,y,z], conics upper-triangular (a,b,c) with a 12-byte stride, bool masks
 * as uint8 0/1, isect keys u64 = image<<(32+tile_bits) | tile<<32 | f32bits(depth).
 */
#ifndef SPLATX_CUDA_H
#define SPLATX_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SXCUDA_OK 0
#define SXCUDA_EINVAL 1
#define SXCUDA_ERUNTIME 2

typedef void* sxcuda_stream_t;

/* ---------------------------------------------------------------------------------------------
 * Library helpers
 * ------------------------------------------------------------------------------------------- */

/* Message of the last failing call on the calling thread ("" when none). */
const char* sxcuda_last_error(void);
/* ABI version of this header (bumped on any struct or signature change). */
int32_t sxcuda_abi_version(void);
/* bits_for_count (CpuKernels.h:92-97): bits needed to index 0..count-1; count<=1 gives 0. */
uint32_t sxcuda_bits_for_count(int64_t count);
/* Host-side binoms LUT for MCMC relocation (make_binoms_lut, CpuKernels.h:178 /
 * CpuKernels.cpp:906): lut[n*n_max+k] = C(n,k) as float, 0 for k>n. lut_host holds n_max*n_max. */
int32_t sxcuda_make_binoms_lut(int32_t n_max, float* lut_host);

/* ---------------------------------------------------------------------------------------------
 * Resident training-step executor — replaces MetalTrainStepExecutor
 * (TrainStepExecutor, KernelBackend.h:386-392; desc/sync/io structs KernelBackend.h:338-384;
 *  factory KernelBackend::make_train_step_executor, KernelBackend.h:505-508).
 * Host pointers. One executor per device; it owns every device buffer it uses.
 * ------------------------------------------------------------------------------------------- */

/* TrainStepExecutorDesc (KernelBackend.h:338-346). */
typedef struct SxTrainStepExecutorDesc {
    int64_t arena_rows; /* parameter rows (MCMC cap_max); never reallocated between steps */
    int32_t sh_degree;  /* 0..3, K = (sh_degree+1)^2 */
    float eps2d, near_plane, far_plane, radius_clip;
    float b1, b2, eps;  /* Adam */
    float ssim_weight;  /* lambda in [0,1]; 0 bypasses SSIM entirely */
    int32_t antialiased;
} SxTrainStepExecutorDesc;

/* ResidentParamSync (KernelBackend.h:354-359). Group order: 0 means[3], 1 quats[4],
 * 2 scales[3] (log), 3 opacities[1] (logit), 4 sh0[3], 5 shN[(K-1)*3] (NULL when K==1). */
typedef struct SxResidentParamSync {
    float* params[6];
    float* exp_avg[6];
    float* exp_avg_sq[6];
    int64_t rows;
} SxResidentParamSync;

/* ResidentStepInputs (KernelBackend.h:361-378), plus gt_on_device (not in the reference): when
 * non-zero, gt_rgb is a DEVICE pointer and no host->device copy of it is made. */
typedef struct SxResidentStepInputs {
    const float* viewmat; /* [16] world->cam row-major (host) */
    const float* K;       /* [9] (host) */
    int32_t width, height;
    const float* gt_rgb;  /* [H,W,3]; may be NULL when forward_only */
    int64_t count;        /* alive rows, 1..arena_rows */
    uint32_t degrees_to_use;
    float lr[6];
    float opacity_reg_w, scale_reg_w;
    int32_t forward_only;
    int32_t want_render;
    int32_t inject_noise;
    uint64_t noise_seed, noise_offset;
    float noise_scale;
    int32_t gt_on_device;
} SxResidentStepInputs;

/* ResidentStepOutputs (KernelBackend.h:380-384). render_colors: caller-owned HOST buffer of
 * H*W*3 floats, filled when want_render (may be NULL otherwise). */
typedef struct SxResidentStepOutputs {
    float loss;
    int64_t n_isects;
    float* render_colors;
} SxResidentStepOutputs;

typedef struct SxExecutor SxExecutor;

/* make_train_step_executor (KernelBackend.h:505-508) on CUDA device `device`. */
int32_t sxcuda_executor_create(const SxTrainStepExecutorDesc* desc, int32_t device,
                               SxExecutor** out);
void sxcuda_executor_destroy(SxExecutor* ex);
/* TrainStepExecutor::upload_params / download_params (KernelBackend.h:389-390). */
int32_t sxcuda_executor_upload_params(SxExecutor* ex, const SxResidentParamSync* sync);
int32_t sxcuda_executor_download_params(SxExecutor* ex, const SxResidentParamSync* sync);
/* TrainStepExecutor::step (KernelBackend.h:391): one synchronous step, loss and n_isects read
 * back. Grows the intersection capacity and replays the step when a step overflows it. */
int32_t sxcuda_executor_step(SxExecutor* ex, const SxResidentStepInputs* in,
                             SxResidentStepOutputs* out);
/* Asynchronous step (no reference counterpart; it is the same step with the loss and n_isects
 * left on the device). Enqueued on the executor's stream; read them later with
 * sxcuda_executor_last_result. Overflowed steps leave parameters untouched and are counted. */
int32_t sxcuda_executor_step_async(SxExecutor* ex, const SxResidentStepInputs* in);
/* Waits for the executor's stream and reports the last step's loss / n_isects and the number of
 * async steps skipped because they overflowed the intersection capacity since the last call. */
int32_t sxcuda_executor_last_result(SxExecutor* ex, float* loss, int64_t* n_isects,
                                    int64_t* overflowed_steps);
/* Grows the intersection capacity ahead of time (so async steps do not overflow). */
int32_t sxcuda_executor_reserve_isects(SxExecutor* ex, int64_t n_isects);
/* The executor's CUDA stream (cudaStream_t), for callers that time or order around it. */
sxcuda_stream_t sxcuda_executor_stream(SxExecutor* ex);
/* Kernel launches issued by the last step (counted by the executor itself). */
int64_t sxcuda_executor_last_launch_count(SxExecutor* ex);
/* Per-segment GPU timing of each step (the counterpart of the reference's SPLATX_KERNEL_TIMING
 * "[ktime]" segments, MetalBackend.cpp:57-72,1909-1937). When on, CUDA events are recorded between
 * the step's segments on the executor's stream. */
int32_t sxcuda_executor_set_profiling(SxExecutor* ex, int32_t on);
/* Segment names (static strings) and milliseconds of the last profiled step; *count receives the
 * number of segments written (at most `capacity`). Synchronises the executor's stream. */
int32_t sxcuda_executor_segment_times(SxExecutor* ex, const char** names, float* ms,
                                      int32_t capacity, int32_t* count);
/* Raster work counting (pairs evaluated): while on, steps run their kernels
 * directly (no graphs) with counting variants of the raster kernels. sxcuda_executor_raster_pairs
 * returns the last such step's (pixel, Gaussian) pairs: forward = pairs a pixel still blending
 * evaluated (up to its early stop), backward = pairs the replay evaluated (at or before the
 * pixel's last contributor). Synchronises the executor's stream. */
int32_t sxcuda_executor_set_pair_counting(SxExecutor* ex, int32_t on);
int32_t sxcuda_executor_raster_pairs(SxExecutor* ex, int64_t* fwd_pairs, int64_t* bwd_pairs);
/* How the step builds its tile-sorted intersection list (the reference's isect_tiles + sort_isect
 * + isect_offset_encode, KernelBackend.h:150-190; the list is the same either way).
 * mode 0 (default): supertile binning wherever the tile grid has at most 16,384 blocks of 8x8
 * tiles, the pair sort beyond; mode 1: always the pair sort (emit every (tile, Gaussian) pair in
 * depth order, sort stably by tile). Any other mode: EINVAL. */
int32_t sxcuda_executor_set_tile_lists(SxExecutor* ex, int32_t mode);
/* The last step's supertile binning: *n_entries (Gaussian, supertile) entries over *n_supertiles
 * supertiles; both 0 when the step used the pair sort. Synchronises the executor's stream. */
int32_t sxcuda_executor_bin_stats(SxExecutor* ex, int64_t* n_entries, int64_t* n_supertiles);
/* The last profiled sxcuda_executor_step_exchange as a timeline: event names (static strings:
 * "start", "raster_bwd_end", "bwd_chunk<c>_end" on the executor's stream, "barrier<c>_end" and
 * "exchange<c>_end" on the exchange stream, "closing_barrier_end", "clear_end") and their
 * milliseconds from "start", in recording order. Synchronises both streams. */
int32_t sxcuda_executor_exchange_timeline(SxExecutor* ex, const char** names, float* ms,
                                          int32_t capacity, int32_t* count);

/* Read-back of the last step's intermediate tensors, for parity checks of the resident step
 * against a host implementation. The reference's host path holds the same tensors between its
 * kernel calls (Trainer.cpp:974-1131: projection outputs, colours, tiles_per_gauss, sorted
 * flatten_ids, isect offsets, render / alpha / last_ids, and the loss gradient fed to
 * rasterize_bwd); the resident executor keeps them in device buffers until the next step. HOST
 * pointers, each may be NULL (skipped); every call synchronises the executor's stream. Fails
 * before any step has run. */
typedef struct SxExecutorGaussianTrace {
    uint8_t* valid;           /* [count] radii > 0 (projection_fused_fwd's cull) */
    float* means2d;           /* [count,2] (rows with valid 0: unspecified) */
    float* conics;            /* [count,3] (rows with valid 0: unspecified) */
    float* opacities;         /* [count] raster opacity: sigmoid, x compensation when antialiased */
    float* colors;            /* [count,3] SH colour + 0.5 clamped at 0 (valid rows) */
    int32_t* tiles_per_gauss; /* [count] AccuTile tile count (isect_tiles' tiles_per_gauss) */
    uint32_t* depth_keys;     /* [count] f32 bits of the camera depth; 0xffffffff without tiles */
    int32_t* depth_order;     /* [count] Gaussian ids in ascending depth key, ties by id */
} SxExecutorGaussianTrace;
/* Per-Gaussian forward outputs of the last step; *count receives its alive row count. */
int32_t sxcuda_executor_read_gaussians(SxExecutor* ex, const SxExecutorGaussianTrace* out,
                                       int64_t* count);
/* The last step's tile-sorted intersection list: flatten_ids in the reference's sorted order
 * (tile, depth, Gaussian id — sort_isect's values_sorted, KernelBackend.h:164-176) and the
 * start offset of every tile (isect_offset_encode, KernelBackend.h:178-190). *n_isects and
 * *n_tiles receive the sizes; flatten_ids needs capacity >= n_isects and tile_offsets
 * tiles_capacity >= n_tiles, else EINVAL (the sizes are still written). */
int32_t sxcuda_executor_read_isects(SxExecutor* ex, int32_t* flatten_ids, int64_t capacity,
                                    int32_t* tile_offsets, int64_t tiles_capacity,
                                    int64_t* n_isects, int64_t* n_tiles);
/* The last step's images, H*W pixels of its camera: render [H,W,3], alpha [H,W], last_ids [H,W]
 * (rasterize_fwd's outputs) and v_render [H,W,3], the loss gradient with respect to the render
 * (0.8-weighted L1 sign term + the SSIM term, the input of rasterize_bwd; not written by a
 * forward-only step). */
int32_t sxcuda_executor_read_images(SxExecutor* ex, float* render_colors, float* render_alphas,
                                    int32_t* last_ids, float* v_render_colors);

/* ---------------------------------------------------------------------------------------------
 * View-parallel training (no counterpart in the reference, which trains on one GPU; the
 * multi-GPU plan of this port). Each GPU's executor accumulates the gradients of several views
 * (no Adam), the caller reduce-scatters them over the GPUs, each GPU applies Adam to its owner
 * shard of rows, and the caller all-gathers the parameters. The resident layout stores Gaussians
 * in tiles of 32 (a group's d components as d runs of 32 floats per tile), so rows [r0, r1) with
 * r0, r1 multiples of 32 are the contiguous floats [r0*d, r1*d) of every group's buffer.
 * ------------------------------------------------------------------------------------------- */

/* Forward + backward of one view; the six groups' data-term gradients are ADDED to the
 * executor's gradient buffers and the visibility count of each visible Gaussian is incremented.
 * Parameters, moments, lr, regularisers and noise fields of `in` are not used. Asynchronous (as
 * sxcuda_executor_step_async); a view whose intersections overflow the capacity is skipped and
 * counted by sxcuda_executor_last_result. */
int32_t sxcuda_executor_step_accumulate(SxExecutor* ex, const SxResidentStepInputs* in);

typedef struct SxApplyGradsInputs {
    int64_t row_begin, row_end; /* multiples of 32 within the executor's padded rows */
    int64_t count;              /* alive rows (rows >= count are never updated) */
    int32_t n_views;            /* views summed into the gradients: gradient = sum / n_views */
    float lr[6];
    float opacity_reg_w, scale_reg_w; /* per-element weights, added once per step */
    int32_t inject_noise;
    uint64_t noise_seed, noise_offset;
    float noise_scale;
} SxApplyGradsInputs;

/* Adam (no bias correction, as fused_adam) on rows [row_begin, row_end) from the accumulated
 * gradients; rows with visibility 0 are untouched; then MCMC noise on those rows (< count); the
 * rows' gradient buffers and visibility are re-zeroed. Rows outside the range keep their
 * gradients: zero them with another call or sxcuda_executor_clear_grads. Asynchronous. */
int32_t sxcuda_executor_apply_grads(SxExecutor* ex, const SxApplyGradsInputs* in);

/* Zeroes every gradient buffer and the visibility count (after a reduce-scatter has consumed
 * them). Asynchronous. */
int32_t sxcuda_executor_clear_grads(SxExecutor* ex);

/* Device buffers of the resident arena, for collectives on the executor's stream. grads and
 * visibility are allocated by the first call (zeroed). dims[5] is 0 for SH degree 0. */
typedef struct SxResidentBuffers {
    float* params[6];
    float* grads[6];
    float* visibility;
    int64_t dims[6];
    int64_t padded_rows;
} SxResidentBuffers;
int32_t sxcuda_executor_resident_buffers(SxExecutor* ex, SxResidentBuffers* out);

/* The exchange fused into one kernel over peer memory (an alternative to the reduce-scatter /
 * apply_grads / all-gather sequence above, with the same result up to the order of the gradient
 * sum). Each rank exports CUDA IPC handles of its gradient, visibility and parameter buffers, the
 * caller shares them (e.g. all_gather_object) and every rank opens the others'. Per step, after a
 * cross-rank barrier that follows every rank's last step_accumulate:
 *   sxcuda_executor_exchange_apply  for the owner rows [row_begin, row_end): every rank's
 *       gradients and visibility summed in rank order, Adam (+ regularisers, + noise) on the local
 *       moments, and each changed row stored into every rank's parameter replica;
 * then, after a second barrier (all reads and stores done), sxcuda_executor_clear_grads. The
 * barriers are the caller's (a stream-ordered collective); the kernel itself never waits.
 * sxcuda_executor_step_exchange below instead overlaps the exchange with the last view's
 * backward and takes its barriers on the device over the mapped flag arrays. */
#define SXCUDA_IPC_HANDLE_BYTES 64
#define SXCUDA_PEER_BUFS 14
typedef struct SxPeerHandles {
    /* grads 0..5, visibility, params 0..5, barrier flags */
    unsigned char handle[SXCUDA_PEER_BUFS][SXCUDA_IPC_HANDLE_BYTES];
    int64_t padded_rows;     /* arena layout, checked on open */
    int32_t sh_degree;
    uint32_t barrier_epoch;  /* device barriers taken so far; every rank's must agree on open */
} SxPeerHandles;
int32_t sxcuda_executor_peer_handles(SxExecutor* ex, SxPeerHandles* out);
/* all: world entries indexed by rank (this rank's entry is not opened). At most 8 ranks; the
 * executor's padded rows must split into whole 32-row tiles per rank. */
int32_t sxcuda_executor_open_peers(SxExecutor* ex, int32_t rank, int32_t world,
                                   const SxPeerHandles* all);
int32_t sxcuda_executor_exchange_apply(SxExecutor* ex, const SxApplyGradsInputs* in);
/* The last view of a view-parallel step with the exchange overlapped (after open_peers). `in`
 * accumulates like sxcuda_executor_step_accumulate; its per-Gaussian backward runs in `chunks`
 * (1..8) row chunks, chunk c holding rows r*S + [c0, c1) of every rank r (S = padded_rows /
 * world, 32-row aligned bounds). After chunk c, a second stream waits on a device barrier (every
 * rank finished chunk c: each rank stores the epoch into every rank's flag array at system scope
 * and polls its own) and runs exchange_apply on this rank's owner rows of chunk c while the next
 * chunk's backward runs. A closing barrier (every rank's reads and stores done) ends the step.
 * The accumulators are not cleared in memory: they keep the step's sums, and the executor's next
 * accumulating view (step_accumulate or step_exchange) writes them instead of adding (rows it
 * does not see get zeros), so no clearing pass runs between steps. `ap` carries the apply inputs; row_begin / row_end must
 * be this rank's owner rows [rank*S, (rank+1)*S). Every rank calls it in the same order.
 * Barrier waits are bounded (about a second); one that runs out makes the next result read
 * (sxcuda_executor_last_result) fail with "peer barrier". Asynchronous. */
int32_t sxcuda_executor_step_exchange(SxExecutor* ex, const SxResidentStepInputs* in,
                                      const SxApplyGradsInputs* ap, int32_t chunks);
/* Check of the device barrier's bounded wait on one GPU: the barrier kernel runs as rank 0 of
 * `world` (1..8) ranks whose other flag arrays, allocated on `device`, nobody signals. With
 * world > 1 the wait runs out after about a second and *status receives 2 (the "peer barrier"
 * bit); with world 1 it passes at once and *status is 0. Synchronous; the context stays usable
 * (the device's current setting is restored). */
int32_t sxcuda_peer_barrier_selftest(int32_t device, int32_t world, uint32_t* status);
/* The same barrier, followed by what sxcuda_executor_step_exchange enqueues after one: this
 * rank's exchange, on a 32-row arena of `device` whose gradients and visibility are 1. The
 * exchange reads the step's status word and changes nothing when a wait of the step ran out, so
 * after a timed-out barrier (world > 1) *applied (the parameters changed) is 0; with world 1 it
 * is 1. Synchronous. */
int32_t sxcuda_peer_exchange_selftest(int32_t device, int32_t world, uint32_t* status,
                                      int32_t* applied);

/* ---------------------------------------------------------------------------------------------
 * MCMC refine on the resident arena: Trainer::mcmc_refine (Trainer.cpp:1273-1281: relocate
 * :1284-1340, add :1342-1394, Adam row zeroing :1422-1435) and Trainer::mcmc_inject_noise
 * (Trainer.cpp:1396-1420), run against the executor's device-resident parameters instead of the
 * reference's download / host mutation / re-upload (sync_host_for_mutation, Trainer.cpp:1275).
 * The executor owns the refine's std::mt19937_64 (Trainer::mcmc_rng_, Trainer.h:495; seeded 42
 * like McmcOptions::seed until sxcuda_executor_mcmc_seed). The dead/alive split, the multinomial
 * draws and the float exp/log around the relocation kernel run on the host with the reference's
 * arithmetic; the relocation kernel and the row surgery run on the device.
 * ------------------------------------------------------------------------------------------- */

/* mcmc_rng_.seed(seed) (Trainer.cpp:713). */
int32_t sxcuda_executor_mcmc_seed(SxExecutor* ex, uint64_t seed);

/* The engine state as the text `os << std::mt19937_64` writes in the classic locale (the
 * checkpoint's mcmc_rng_state, Trainer.cpp:1506-1509). With buf NULL or cap too small, only *len
 * (the text length, no terminator) is written and SXCUDA_EINVAL is returned for a short buffer. */
int32_t sxcuda_executor_mcmc_rng_state(SxExecutor* ex, char* buf, int64_t cap, int64_t* len);
/* Restores a state written by sxcuda_executor_mcmc_rng_state (Trainer.cpp:1556-1563). */
int32_t sxcuda_executor_mcmc_set_rng_state(SxExecutor* ex, const char* text, int64_t len);

typedef struct SxMcmcRefineInputs {
    int64_t count;     /* alive rows before the refine, 1..arena_rows */
    int64_t cap_max;   /* McmcOptions::cap_max (Trainer.h:190): count <= cap_max <= arena_rows */
    float min_opacity; /* McmcOptions::min_opacity (Trainer.h:191), in (0,1) */
} SxMcmcRefineInputs;

/* McmcRefineResult (Trainer.h:414-420). The three lists are optional caller HOST buffers of
 * list_capacity entries each (NULL to skip); n_* are the full lengths, lists are truncated to
 * list_capacity. */
typedef struct SxMcmcRefineResult {
    int64_t count;          /* alive rows after the refine (count + n_added) */
    int64_t n_relocated;    /* |relocated_dead| == |relocation_src| */
    int64_t n_added;        /* |added_src| */
    int64_t* relocated_dead;
    int64_t* relocation_src;
    int64_t* added_src;
    int64_t list_capacity;
} SxMcmcRefineResult;

/* One refine (relocate, then add) on rows [0, count). Synchronous: returns after the surgery has
 * run on the executor's stream. Rows count..count+n_added-1 become alive; the caller passes the
 * new count to later steps. */
int32_t sxcuda_executor_mcmc_refine(SxExecutor* ex, const SxMcmcRefineInputs* in,
                                    SxMcmcRefineResult* out);

/* MCMC position noise on rows [0, count) outside a step (the refine step's noise, after the
 * refine: Trainer.cpp:966): means += Sigma (n * sigmoid(-100 (sigmoid(op) - 0.005)) *
 * noise_scale) with n = Philox normals (seed, offset; counter 3*row + k) — the same noise the
 * step applies with inject_noise. Asynchronous. */
int32_t sxcuda_executor_inject_noise(SxExecutor* ex, int64_t count, uint64_t seed, uint64_t offset,
                                     float noise_scale);

/* ---------------------------------------------------------------------------------------------
 * Evaluation and rendering around the resident arena.
 * ------------------------------------------------------------------------------------------- */

/* The training eval of one view (TrainC.cpp:653-696): the render of `in`'s camera (forward only,
 * degrees_to_use as given) clamped to [0,1]; psnr = 10 log10(1/mse) against in->gt_rgb (a host
 * image, or a device image with gt_on_device), cc_psnr after the affine per-channel colour
 * correction (color_correct_affine, Trainer.cpp:364-392), ssim / cc_ssim = mean SSIM of the
 * clamped / corrected render against the target (eval_ssim, Trainer.cpp:405-418; NaN when H or
 * W < 11). psnr values are the reference's float results widened to double. Synchronous. */
typedef struct SxEvalResult {
    double psnr, cc_psnr, ssim, cc_ssim;
} SxEvalResult;
int32_t sxcuda_executor_eval_view(SxExecutor* ex, const SxResidentStepInputs* in,
                                  SxEvalResult* out);

/* Forward-only render of `in`'s camera quantised on the device to RGBA8 into a HOST buffer of
 * width*height*4 bytes (NaN -> 0, clamp to [0,1], round(v*255) half to even, alpha 255 — the
 * quantisation of sx_render_session_frame, TrainC.cpp:1549-1565). Synchronous. */
int32_t sxcuda_executor_render_rgba8(SxExecutor* ex, const SxResidentStepInputs* in,
                                     uint8_t* out_rgba);

/* A Gaussian cloud in the reference's host layout (SplatCloud, SplatCloud.h:8-18): count rows of
 * means [3], log-scales [3], quats [4] (w first), opacity logits [1], sh0 [3] and shN
 * [K][3] coefficient-major, K = (sh_degree+1)^2 - 1. */
typedef struct SxCloud {
    int64_t count;
    int32_t sh_degree;
    float* means;
    float* scales;
    float* quats;
    float* opacities;
    float* sh0;
    float* shN;
} SxCloud;

/* INRIA PLY (write_inria_ply / read_inria_ply, PlyIO.h:20-21, PlyIO.cpp:18-123): binary little
 * endian, f_rest channel-major, zero-padded to 45 with pad_sh_full when 0 < K < 15.
 * sxcuda_ply_info reads the header (count, SH degree); sxcuda_ply_read fills caller buffers sized
 * from it (degree 0..3). */
int32_t sxcuda_ply_write(const SxCloud* cloud, const char* path, int32_t pad_sh_full);
int32_t sxcuda_ply_info(const char* path, int64_t* count, int32_t* sh_degree);
int32_t sxcuda_ply_read(const char* path, const SxCloud* out);

/* filter_cloud_for_export (PlyIO.h:48-49, PlyIO.cpp:131-188): keep[i] = 0 for rows with a
 * non-finite value, then for rows with sigmoid(opacity) <= min_opacity, else 1. */
typedef struct SxExportFilterStats {
    int64_t input, removed_nonfinite, removed_low_opacity, kept;
} SxExportFilterStats;
int32_t sxcuda_filter_for_export(const SxCloud* cloud, float min_opacity, uint8_t* keep,
                                 SxExportFilterStats* stats);

/* The end-of-training export: rows [0, count) of the resident arena downloaded, filtered
 * (min_opacity 0.005 in the reference) and written as a PLY. stats may be NULL. */
int32_t sxcuda_executor_export_ply(SxExecutor* ex, int64_t count, const char* path,
                                   float min_opacity, int32_t pad_sh_full,
                                   SxExportFilterStats* stats);

/* Niantic SPZ files (save_spz / load_spz, SpzIO.h, SpzIO.cpp over the spz library v2.1.0):
 * version 3 written (24-bit positions, smallest-three quaternions), versions 1..3 read; the cloud
 * passes the export filter first; the file frame is right-up-back (the training world is the
 * PLY's right-down-front); loaded opacity logits are clamped to +-ln(509). SH degree 0..3. */
int32_t sxcuda_spz_write(const SxCloud* cloud, const char* path, float min_opacity,
                         int32_t antialiased, SxExportFilterStats* stats);
int32_t sxcuda_spz_info(const char* path, int64_t* count, int32_t* sh_degree, int32_t* antialiased);
int32_t sxcuda_spz_read(const char* path, const SxCloud* out);
int32_t sxcuda_executor_export_spz(SxExecutor* ex, int64_t count, const char* path,
                                   float min_opacity, int32_t antialiased,
                                   SxExportFilterStats* stats);

/* The session-style render API (sx_render_session_*, splatx_train_c.h:578-682, TrainC.cpp:
 * 1440-1584): open loads a PLY once (sh_degree 0 = the file's; 1..3 = a cap, above the file's is
 * an error) onto CUDA device `device` and keeps it resident; frame renders an arbitrary pinhole
 * camera at any size into a caller RGBA8 buffer; close releases it. Errors: open returns NULL,
 * frame returns -1 (argument violation) or -2 (render failure); both write a NUL-terminated
 * message into err_buf. The reference's metallib fields have no CUDA meaning and are absent. */
typedef struct SxRenderSession SxRenderSession;
typedef struct SxRenderSessionArgs {
    const char* ply_path;
    int32_t antialiased;
    int32_t sh_degree;
    int32_t device;
} SxRenderSessionArgs;
SxRenderSession* sxcuda_render_session_open(const SxRenderSessionArgs* args, char* err_buf,
                                            int32_t err_buf_len);
int32_t sxcuda_render_session_frame(SxRenderSession* session, const float* viewmat, float fx,
                                    float fy, float cx, float cy, int32_t width, int32_t height,
                                    uint8_t* out_rgba, char* err_buf, int32_t err_buf_len);
void sxcuda_render_session_close(SxRenderSession* session);

/* COLMAP sparse model -> training cameras and seed points (load_colmap_bundle,
 * ColmapLoader.h:17-21 / ColmapLoader.cpp; training_input_from_colmap, TrainingInput.h:27,
 * TrainingInput.cpp:10-47). Binary model when cameras.bin exists, else text; PINHOLE and
 * SIMPLE_PINHOLE only (distortion models are rejected by name). Cameras are the images in file
 * order: viewmat [16] row-major world->camera, K [9], width, height, image path images_dir/name.
 * Seed points in float, colours u8. Host only. */
typedef struct SxColmap SxColmap;
int32_t sxcuda_colmap_open(const char* sparse_dir, const char* images_dir, SxColmap** out);
void sxcuda_colmap_close(SxColmap* b);
int32_t sxcuda_colmap_counts(const SxColmap* b, int64_t* n_images, int64_t* n_points);
int32_t sxcuda_colmap_cameras(const SxColmap* b, float* viewmats, float* Ks, int32_t* widths,
                              int32_t* heights);
/* The NUL-free path of image i; with buf NULL or cap too short only *len is written (EINVAL for
 * a short buffer). */
int32_t sxcuda_colmap_image_path(const SxColmap* b, int64_t i, char* buf, int64_t cap, int64_t* len);
int32_t sxcuda_colmap_seed(const SxColmap* b, float* points, uint8_t* rgb);

/* ---------------------------------------------------------------------------------------------
 * SXCK checkpoints of the resident arena (Checkpoint.h:1-145, Checkpoint.cpp): the reference's
 * byte format, written atomically (temp + fsync + rename), fp32 lossless or fp16 (half, exp_avg_sq
 * stored as half(sqrt(v)), paired zeroing on load). The fp16 conversion runs on the device.
 * ------------------------------------------------------------------------------------------- */

/* CheckpointConfig (Checkpoint.h:84-95): the resume fingerprint. */
typedef struct SxCheckpointConfig {
    int32_t sh_degree, factor, test_split, total_iters;
    uint8_t mcmc_enabled, antialiased;
    int64_t cap_max;
    uint64_t mcmc_seed;
    float scene_scale, ssim_weight;
} SxCheckpointConfig;

/* CheckpointHeader (Checkpoint.h:138-144). */
typedef struct SxCheckpointHeader {
    SxCheckpointConfig config;
    int32_t iter;
    int64_t alive_count;
    int32_t fp16;
    uint32_t version;
} SxCheckpointHeader;

/* verify_checkpoint_config (Checkpoint.cpp:146-178): SXCUDA_ERUNTIME naming the first mismatched
 * field and both values. */
int32_t sxcuda_checkpoint_verify_config(const SxCheckpointConfig* saved,
                                        const SxCheckpointConfig* current);
/* load_checkpoint_header (Checkpoint.cpp:320-323). */
int32_t sxcuda_checkpoint_info(const char* path, SxCheckpointHeader* out);
/* save_checkpoint_file of rows [0, count) of the arena (parameters and both moments) at step
 * `iter`; with config->mcmc_enabled the executor's MCMC engine state is stored. */
int32_t sxcuda_executor_save_checkpoint(SxExecutor* ex, const SxCheckpointConfig* config,
                                        int32_t iter, int64_t count, const char* path,
                                        int32_t fp16);
/* load_checkpoint_file into the arena (rows beyond the saved count zeroed), after verifying the
 * fingerprint against `current` (NULL skips the check); restores the MCMC engine state when the
 * file has one. out receives the header (alive count and iter to resume at). */
int32_t sxcuda_executor_load_checkpoint(SxExecutor* ex, const char* path,
                                        const SxCheckpointConfig* current,
                                        SxCheckpointHeader* out);

/* ---------------------------------------------------------------------------------------------
 * Per-kernel entry points (device pointers) — the 37-kernel verification surface.
 * ------------------------------------------------------------------------------------------- */

/* fused_adam — KernelBackend::fused_adam (KernelBackend.h:404-406), AdamInputs
 * (KernelBackend.h:18-27); kernel AdamMCMC.metal:20-46. No bias correction; rows with
 * valid[g]==0 are skipped entirely. n_elems==0 is a no-op. */
typedef struct SxAdamInputs {
    float* param;
    const float* grad;
    float* exp_avg;
    float* exp_avg_sq;
    const uint8_t* valid; /* [n_gauss] or NULL */
    int64_t n_elems, n_gauss;
    float lr, b1, b2, eps;
} SxAdamInputs;
int32_t sxcuda_fused_adam(const SxAdamInputs* in, sxcuda_stream_t stream);

/* ProjectionFusedInputs (KernelBackend.h:31-45). covars != NULL selects the 6-triu path. */
typedef struct SxProjectionFusedInputs {
    const float* means;     /* [N,3] */
    const float* covars;    /* [N,6] or NULL */
    const float* quats;     /* [N,4] wxyz */
    const float* scales;    /* [N,3] linear */
    const float* opacities; /* [N] post-sigmoid or NULL */
    const float* viewmats;  /* [C,16] row-major */
    const float* Ks;        /* [C,9] */
    int64_t N, C;
    int32_t width, height;
    float eps2d, near_plane, far_plane, radius_clip;
    uint32_t camera_model; /* 0 = PINHOLE (the only supported model) */
    int32_t calc_compensations;
} SxProjectionFusedInputs;

/* ProjectionFusedOutputs (KernelBackend.h:47-54). Culled slots get radii 0 and leave the other
 * outputs unwritten, except compensations which the entry point zero-fills first. */
typedef struct SxProjectionFusedOutputs {
    int32_t* radii;       /* [C,N,2] */
    float* means2d;       /* [C,N,2] */
    float* depths;        /* [C,N] */
    float* conics;        /* [C,N,3] */
    float* compensations; /* [C,N] when calc_compensations, else NULL */
} SxProjectionFusedOutputs;

/* projection_ewa_3dgs_fused_fwd — KernelBackend::projection_fused_fwd (KernelBackend.h:407-409);
 * kernel ProjectionEWA.metal:62-180; CPU reference CpuKernels.cpp:168-273. */
int32_t sxcuda_projection_fused_fwd(const SxProjectionFusedInputs* in,
                                    const SxProjectionFusedOutputs* out, sxcuda_stream_t stream);

/* ProjectionFusedGradsIn (KernelBackend.h:57-66). */
typedef struct SxProjectionFusedGradsIn {
    const int32_t* radii;
    const float* conics;
    const float* compensations;   /* required when v_compensations != NULL */
    const float* v_means2d;
    const float* v_depths;
    const float* v_conics;
    const float* v_compensations; /* optional */
    int32_t viewmats_grad;
} SxProjectionFusedGradsIn;

/* ProjectionFusedGrads (KernelBackend.h:68-74); buffers are zero-filled by the entry point. */
typedef struct SxProjectionFusedGrads {
    float* v_means;    /* [N,3] */
    float* v_covars;   /* [N,6] on the covars path, else NULL */
    float* v_quats;    /* [N,4] on the quat/scale path */
    float* v_scales;   /* [N,3] on the quat/scale path */
    float* v_viewmats; /* [C,16] when viewmats_grad */
} SxProjectionFusedGrads;

/* projection_ewa_3dgs_fused_bwd — KernelBackend::projection_fused_bwd (KernelBackend.h:410-413);
 * kernel ProjectionEWA.metal:358-560. */
int32_t sxcuda_projection_fused_bwd(const SxProjectionFusedInputs* in,
                                    const SxProjectionFusedGradsIn* gin,
                                    const SxProjectionFusedGrads* out, sxcuda_stream_t stream);

/* ShInputs (KernelBackend.h:77-86). */
typedef struct SxShInputs {
    const float* dirs;     /* [B*N,3] unnormalised */
    const float* coeffs;   /* [N,K,D] */
    const uint8_t* masks;  /* [B*N] or NULL */
    uint32_t degrees_to_use;
    int64_t B, N, K;
    uint32_t D;
    int32_t compute_v_dirs;
} SxShInputs;

/* sh_fwd — KernelBackend::sh_fwd (KernelBackend.h:414-416); kernel SphericalHarmonics.metal:
 * 399-414. colors [B*N,D]; masked-out rows are left unwritten. */
int32_t sxcuda_sh_fwd(const SxShInputs* in, float* colors, sxcuda_stream_t stream);
/* sh_bwd — KernelBackend::sh_bwd (KernelBackend.h:417-419); kernel SphericalHarmonics.metal:
 * 422-446. v_coeffs [N,K,D] and v_dirs [B*N,3] (when compute_v_dirs) are zero-filled first. */
int32_t sxcuda_sh_bwd(const SxShInputs* in, const float* v_colors, float* v_coeffs,
                      float* v_dirs, sxcuda_stream_t stream);

/* IsectTilesInputs (KernelBackend.h:106-115). conics+opacities select AccuTile, neither AABB. */
typedef struct SxIsectTilesInputs {
    const float* means2d;
    const int32_t* radii;
    const float* depths;
    const float* conics;
    const float* opacities;
    int64_t I, N;
    uint32_t tile_size, tile_width, tile_height;
} SxIsectTilesInputs;

/* Pass 1 of KernelBackend::isect_tiles (KernelBackend.h:420-422): isect_tile_count
 * (IntersectTile.metal:225-254) + the int64 inclusive prefix scan (PrefixScan.metal) + the
 * n_isects readback (MetalBackend.cpp:1849-1858). Writes tiles_per_gauss [I*N] and
 * cum_tiles_per_gauss [I*N]; stores n_isects to *n_isects_host (synchronises the stream). */
int32_t sxcuda_isect_tile_count(const SxIsectTilesInputs* in, int32_t* tiles_per_gauss,
                                int64_t* cum_tiles_per_gauss, int64_t* n_isects_host,
                                void* workspace, size_t* workspace_bytes,
                                sxcuda_stream_t stream);
/* Pass 2 of isect_tiles: isect_tile_emit (IntersectTile.metal:259-298). Keys and flatten ids in
 * the reference's emit order (element idx, then sweep u, then v / AABB y then x). */
int32_t sxcuda_isect_tile_emit(const SxIsectTilesInputs* in, const int64_t* cum_tiles_per_gauss,
                               uint64_t* isect_ids, int32_t* flatten_ids,
                               sxcuda_stream_t stream);
/* prefix_scan_i64 — KernelBackend::prefix_scan_i64 (KernelBackend.h:428-430): inclusive int32 ->
 * int64 cumsum, bit-exact. */
int32_t sxcuda_prefix_scan_i64(const int32_t* in, int64_t* out, int64_t n, void* workspace,
                               size_t* workspace_bytes, sxcuda_stream_t stream);
/* Allocation-free variant of sxcuda_prefix_scan_i64 (no counterpart in the reference). For callers
 * that cannot allocate device memory at call time and so cannot hand over the workspace the
 * regular entry point needs — e.g. a host that hands out its whole device-memory budget at
 * start-up, or a latency-critical loop that must never hit cudaMalloc's implicit device-wide
 * synchronisation. The scratch (one int64 per 4096 inputs) is a fixed 512 KiB device array inside
 * the library, held on every GPU that uses it until the process exits, so n is limited to
 * 268,435,456; larger n returns SXCUDA_EINVAL. The call allocates nothing: it issues no
 * cudaMalloc/cudaFree and no allocating library routine. The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress, with that device current) and caches it; make
 * that first call before any stream capture. Under CUDA's lazy module loading that first call
 * (or any earlier call into this library on the device) is also what loads the library's device
 * code and backs the array, which takes device memory: a host that hands out its whole device
 * budget should make it before doing so. Every call on a device shares the one array and
 * leaves its last contents there (nothing in it needs to start at zero): calls that overlap on
 * the GPU — two streams, or two host threads at once — race on it, so order them on one stream.
 * Output is bit-identical to sxcuda_prefix_scan_i64. */
int32_t sxcuda_prefix_scan_i64_noalloc(const int32_t* in, int64_t* out, int64_t n,
                                       sxcuda_stream_t stream);
/* sort_isect — KernelBackend::sort_isect (KernelBackend.h:435-437), SortIsectInputs
 * (KernelBackend.h:143-153): stable ascending sort of u64 keys (only the low key_n_bits are
 * significant) carrying i32 values. Inputs are not modified. */
int32_t sxcuda_sort_isect(const uint64_t* keys, const int32_t* values, uint64_t* keys_sorted,
                          int32_t* values_sorted, int64_t n, uint32_t key_n_bits,
                          void* workspace, size_t* workspace_bytes, sxcuda_stream_t stream);
/* isect_offset_encode — KernelBackend::isect_offset_encode (KernelBackend.h:441-443);
 * kernel IntersectTile.metal:310-335. offsets [I*tile_height*tile_width]; n_isects==0 fills 0. */
int32_t sxcuda_isect_offset_encode(const uint64_t* isect_ids_sorted, int64_t n_isects,
                                   int64_t I, uint32_t tile_width, uint32_t tile_height,
                                   int32_t* offsets, sxcuda_stream_t stream);

/* RasterizeFwdInputs (KernelBackend.h:175-188). tile_size must be 16. */
typedef struct SxRasterizeFwdInputs {
    const float* means2d;       /* [I,N,2] */
    const float* conics;        /* [I,N,3] */
    const float* colors;        /* [I,N,3] */
    const float* opacities;     /* [I,N] */
    const float* backgrounds;   /* [I,3] or NULL */
    const uint8_t* masks;       /* [I,TH,TW] or NULL */
    const int32_t* isect_offsets; /* [I,TH,TW] */
    const int32_t* flatten_ids; /* [n_isects] sorted */
    int64_t I, N, n_isects;
    uint32_t image_width, image_height;
    uint32_t tile_size, tile_width, tile_height;
} SxRasterizeFwdInputs;

/* rasterize_to_pixels_3dgs_fwd — KernelBackend::rasterize_fwd (KernelBackend.h:450-452);
 * kernel Rasterize3DGSFwd.metal:57-204. Outputs [I,H,W,3], [I,H,W], [I,H,W]. */
int32_t sxcuda_rasterize_fwd(const SxRasterizeFwdInputs* in, float* render_colors,
                             float* render_alphas, int32_t* last_ids, sxcuda_stream_t stream);

/* RasterizeBwdGradsIn (KernelBackend.h:207-213). */
typedef struct SxRasterizeBwdGradsIn {
    const float* render_alphas;
    const int32_t* last_ids;
    const float* v_render_colors;
    const float* v_render_alphas;
    int32_t absgrad;
} SxRasterizeBwdGradsIn;

/* RasterizeBwdGrads (KernelBackend.h:220-226); zero-filled by the entry point. */
typedef struct SxRasterizeBwdGrads {
    float* v_means2d;     /* [I,N,2] */
    float* v_conics;      /* [I,N,3] */
    float* v_colors;      /* [I,N,3] */
    float* v_opacities;   /* [I,N] */
    float* v_means2d_abs; /* [I,N,2] when absgrad, else NULL */
} SxRasterizeBwdGrads;

/* rasterize_to_pixels_3dgs_bwd — KernelBackend::rasterize_bwd (KernelBackend.h:458-461);
 * kernel Rasterize3DGSBwd.metal:70-298. Atomic accumulation (not bit-deterministic). */
int32_t sxcuda_rasterize_bwd(const SxRasterizeFwdInputs* in, const SxRasterizeBwdGradsIn* gin,
                             const SxRasterizeBwdGrads* out, sxcuda_stream_t stream);

/* rng_normal_f32 / rng_philox_u32 — KernelBackend.h:466-474 (RngNormalInputs :234-238);
 * Philox4x32-10, counter (t, offset_lo, offset_hi, 0), key seed; kernels Rng.metal. */
int32_t sxcuda_rng_normal_f32(uint64_t seed, uint64_t offset, int64_t count, float* out,
                              sxcuda_stream_t stream);
int32_t sxcuda_rng_philox_u32(uint64_t seed, uint64_t offset, int64_t count, uint32_t* out,
                              sxcuda_stream_t stream);

/* RelocationInputs (KernelBackend.h:246-254); mcmc_relocation — KernelBackend.h:478-480;
 * kernel AdamMCMC.metal:63-97. binoms is a DEVICE [n_max*n_max] LUT. */
typedef struct SxRelocationInputs {
    const float* opacities;
    const float* scales;
    const int32_t* ratios;
    const float* binoms;
    int64_t N;
    int32_t n_max;
    float min_opacity;
} SxRelocationInputs;
int32_t sxcuda_mcmc_relocation(const SxRelocationInputs* in, float* new_opacities,
                               float* new_scales, sxcuda_stream_t stream);

/* PerturbInputs (KernelBackend.h:265-275); mcmc_perturb_positions — KernelBackend.h:483-485;
 * kernel AdamMCMC.metal:112-140. positions updated in place. */
typedef struct SxPerturbInputs {
    float* positions;
    const float* quats;
    const float* scales_log;
    const float* opacities_logit;
    const float* noise;
    int64_t N;
    float noise_scale, t, k;
} SxPerturbInputs;
int32_t sxcuda_mcmc_perturb_positions(const SxPerturbInputs* in, sxcuda_stream_t stream);

/* SsimInputs (KernelBackend.h:283-291), layout [I,H,W,C]. */
typedef struct SxSsimInputs {
    const float* img1;
    const float* img2;
    int64_t I, H, W, C;
    int32_t need_coeffs;
} SxSsimInputs;

/* ssim_fwd — KernelBackend::ssim_fwd (KernelBackend.h:491-493); kernel Ssim.metal:66-173.
 * ssim_map and the three coefficient maps (when need_coeffs) are [I,H-10,W-10,C]. The mean of the
 * map is reduced on the device in f64 in a fixed order and stored to *ssim_mean_device (a DEVICE
 * double). Workspace query protocol. */
int32_t sxcuda_ssim_fwd(const SxSsimInputs* in, float* ssim_map, float* coeff_mu,
                        float* coeff_sigma, float* coeff_cross, double* ssim_mean_device,
                        void* workspace, size_t* workspace_bytes, sxcuda_stream_t stream);

/* SsimGradsIn (KernelBackend.h:313-318); ssim_bwd — KernelBackend.h:499-501; kernel
 * Ssim.metal:190-268. v_img1 [I,H,W,C], every pixel written. */
typedef struct SxSsimGradsIn {
    const float* coeff_mu;
    const float* coeff_sigma;
    const float* coeff_cross;
    float v_loss;
} SxSsimGradsIn;
int32_t sxcuda_ssim_bwd(const SxSsimInputs* in, const SxSsimGradsIn* gin, float* v_img1,
                        sxcuda_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SPLATX_CUDA_H */
