// capi.cu — the extern "C" boundary (include/splatx_cuda.h): entry validation with the
// reference's semantics (Sources/SplatXCore/include/splatx/Validate.h), error translation
// (invalid_argument -> SXCUDA_EINVAL, everything else -> SXCUDA_ERUNTIME, message kept per thread)
// and the workspace-query protocol.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <memory>
#include <stdexcept>
#include <vector>
#include <mutex>
#include <set>
#include <utility>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/splatx_cuda.h"
#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

static std::atomic<int64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void smem_limit_once(const void* kernel, int bytes, const char* what) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), what);
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({kernel, dev})) return;
    cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
    done.insert({kernel, dev});
}
int64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }

SxExecutor* executor_new(const SxTrainStepExecutorDesc& d, int device);
void executor_delete(SxExecutor* ex);
void executor_upload(SxExecutor* ex, const SxResidentParamSync& s);
void executor_download(SxExecutor* ex, const SxResidentParamSync& s);
void executor_step(SxExecutor* ex, const SxResidentStepInputs& in, SxResidentStepOutputs& out);
void executor_step_async(SxExecutor* ex, const SxResidentStepInputs& in);
void executor_step_accumulate(SxExecutor* ex, const SxResidentStepInputs& in);
void executor_apply_grads(SxExecutor* ex, const SxApplyGradsInputs& in);
void executor_clear_grads(SxExecutor* ex);
void executor_buffers(SxExecutor* ex, SxResidentBuffers& out);
void executor_last_result(SxExecutor* ex, float* loss, int64_t* n_isects, int64_t* overflowed);
void executor_read_gaussians(SxExecutor* ex, const SxExecutorGaussianTrace& o, int64_t* count);
void executor_read_isects(SxExecutor* ex, int32_t* ids, int64_t cap, int32_t* offs,
                          int64_t tiles_cap, int64_t* n, int64_t* n_tiles);
void executor_read_images(SxExecutor* ex, float* rc, float* ra, int32_t* li, float* vr);
void executor_reserve(SxExecutor* ex, int64_t n);
void executor_peer_handles(SxExecutor* ex, SxPeerHandles& out);
void executor_save_checkpoint(SxExecutor* ex, const SxCheckpointConfig& cfg, int32_t iter,
                              int64_t count, const char* path, bool fp16);
void executor_load_checkpoint(SxExecutor* ex, const char* path, const SxCheckpointConfig* current,
                              SxCheckpointHeader& out);
void executor_eval_view(SxExecutor* ex, const SxResidentStepInputs& in, SxEvalResult& out);
void executor_render_rgba8(SxExecutor* ex, const SxResidentStepInputs& in, uint8_t* rgba);
void executor_export_ply(SxExecutor* ex, int64_t n, const char* path, float min_opacity, bool pad,
                         SxExportFilterStats& st);
void executor_export_spz(SxExecutor* ex, int64_t n, const char* path, float min_opacity,
                         bool antialiased, SxExportFilterStats& st);
void executor_open_peers(SxExecutor* ex, int rank, int world, const SxPeerHandles* all);
void executor_exchange_apply(SxExecutor* ex, const SxApplyGradsInputs& in);
void executor_step_exchange(SxExecutor* ex, const SxResidentStepInputs& in,
                            const SxApplyGradsInputs& ap, int chunks);
void executor_mcmc_seed(SxExecutor* ex, uint64_t seed);
std::string executor_mcmc_rng_state(SxExecutor* ex);
void executor_mcmc_set_rng_state(SxExecutor* ex, const std::string& t);
void executor_mcmc_refine(SxExecutor* ex, int64_t count, int64_t cap_max, float min_opacity,
                          McmcRefineOut& out);
void executor_inject_noise(SxExecutor* ex, int64_t count, uint64_t seed, uint64_t offset,
                           float noise_scale);
cudaStream_t executor_stream(SxExecutor* ex);
int64_t executor_launches(SxExecutor* ex);
void executor_set_profiling(SxExecutor* ex, bool on);
int executor_segments(SxExecutor* ex, const char** names, float* ms, int cap);
int executor_exchange_timeline(SxExecutor* ex, const char** names, float* ms, int cap);
void executor_set_pair_counting(SxExecutor* ex, bool on);
void executor_set_tile_lists(SxExecutor* ex, int mode);
void executor_bin_stats(SxExecutor* ex, int64_t* n_entries, int64_t* n_st);
void executor_raster_pairs(SxExecutor* ex, int64_t* out);

namespace {

thread_local std::string t_last_error;

// Every entry point leaves the calling thread's current CUDA device as it found it (the
// executor and the kernels select their own device internally).
struct DeviceRestore {
    int dev = -1;
    DeviceRestore() {
        if (cudaGetDevice(&dev) != cudaSuccess) {
            cudaGetLastError();
            dev = -1;
        }
    }
    ~DeviceRestore() {
        if (dev >= 0) cudaSetDevice(dev);
    }
};

template <typename F>
int32_t guarded(F&& f) {
    DeviceRestore restore;
    try {
        f();
        t_last_error.clear();
        return SXCUDA_OK;
    } catch (const std::invalid_argument& e) {
        t_last_error = e.what();
        return SXCUDA_EINVAL;
    } catch (const std::exception& e) {
        t_last_error = e.what();
        return SXCUDA_ERUNTIME;
    } catch (...) {
        t_last_error = "unknown error";
        return SXCUDA_ERUNTIME;
    }
}

cudaStream_t as_stream(sxcuda_stream_t s) { return static_cast<cudaStream_t>(s); }

// Workspace protocol: NULL workspace -> report size; otherwise require enough bytes.
bool workspace_query(void* ws, size_t* bytes, size_t need, const char* what) {
    if (!bytes) throw_invalid(what, "null workspace_bytes");
    if (!ws) {
        *bytes = need;
        return true;
    }
    if (*bytes < need) throw_invalid(what, "workspace too small");
    return false;
}

void validate_projection(const SxProjectionFusedInputs* in, const char* w) {
    if (!in) throw_invalid(w, "null inputs");
    if (in->camera_model != 0)
        throw RuntimeError(std::string(w) + ": only PINHOLE (camera_model=0) supported");
    if (!in->means || !in->viewmats || !in->Ks) throw_invalid(w, "null means/viewmats/Ks");
    if (!in->covars && (!in->quats || !in->scales))
        throw_invalid(w, "need covars (6-triu) or quats+scales");
    if (in->N < 0 || in->C < 0) throw_invalid(w, "negative N or C");
    if (in->N * in->C > INT32_MAX) throw_invalid(w, "C*N must fit in int32");
}

void validate_sh(const SxShInputs* in, const char* w) {
    if (!in) throw_invalid(w, "null inputs");
    if (!in->dirs || !in->coeffs) throw_invalid(w, "null dirs/coeffs");
    if (in->B < 0 || in->N < 0) throw_invalid(w, "negative B or N");
    if (in->K < 1 || in->D == 0) throw_invalid(w, "K and D must be positive");
    if (in->degrees_to_use > 4) throw_invalid(w, "degrees_to_use must be 0..4");
    const int64_t bands = static_cast<int64_t>(in->degrees_to_use) + 1;
    if (bands * bands > in->K) throw_invalid(w, "(degrees_to_use+1)^2 must be <= K");
}

void validate_isect(const SxIsectTilesInputs* in, const char* w) {
    if (!in) throw_invalid(w, "null inputs");
    if (!in->means2d || !in->radii || !in->depths) throw_invalid(w, "null means2d/radii/depths");
    if ((in->conics != nullptr) != (in->opacities != nullptr))
        throw_invalid(w, "conics and opacities must be given together (AccuTile) or both null (AABB)");
    if (in->I < 0 || in->N < 0) throw_invalid(w, "negative I or N");
    if (in->tile_size == 0 || in->tile_width == 0 || in->tile_height == 0)
        throw_invalid(w, "tile_size/tile_width/tile_height must be positive");
    const uint32_t tb = bits_for_count(static_cast<int64_t>(in->tile_width) * in->tile_height);
    if (bits_for_count(in->I) + tb > 32) throw_invalid(w, "image_n_bits + tile_n_bits must be <= 32");
    if (in->N > 0 && in->I > INT32_MAX / in->N) throw_invalid(w, "I*N must fit in int32 (flatten_ids)");
}

void validate_raster(const SxRasterizeFwdInputs* in, const char* w) {
    if (!in) throw_invalid(w, "null inputs");
    if (!in->means2d || !in->conics || !in->colors || !in->opacities || !in->isect_offsets)
        throw_invalid(w, "null means2d/conics/colors/opacities/isect_offsets");
    if (in->n_isects > 0 && !in->flatten_ids) throw_invalid(w, "null flatten_ids");
    if (in->I < 0 || in->N < 0 || in->n_isects < 0) throw_invalid(w, "negative I/N/n_isects");
    if (in->n_isects > 0 && in->N == 0)
        throw_invalid(w, "n_isects > 0 requires N > 0 (flatten_ids reference gaussians)");
    if (in->tile_size != static_cast<uint32_t>(kTile))
        throw_invalid(w, "tile_size must be 16 (the rasterizer instantiation)");
    if (in->image_width == 0 || in->image_height == 0)
        throw_invalid(w, "image_width/image_height must be positive");
    if (in->tile_width == 0 || in->tile_height == 0)
        throw_invalid(w, "tile_width/tile_height must be positive");
    if (static_cast<uint64_t>(in->tile_width) * in->tile_size < in->image_width ||
        static_cast<uint64_t>(in->tile_height) * in->tile_size < in->image_height)
        throw_invalid(w, "tile grid must cover the image");
    if (in->n_isects > INT32_MAX) throw_invalid(w, "n_isects must fit in int32 (last_ids)");
    const int64_t n_tiles = static_cast<int64_t>(in->tile_width) * in->tile_height;
    if (in->I > 0 && n_tiles > INT32_MAX / in->I)
        throw_invalid(w, "I*n_tiles must fit in int32 (offsets table)");
}

RasterArgs raster_args(const SxRasterizeFwdInputs& in) {
    RasterArgs a{};
    a.means2d = in.means2d;
    a.conics = in.conics;
    a.colors = in.colors;
    a.opacities = in.opacities;
    a.backgrounds = in.backgrounds;
    a.masks = in.masks;
    a.offsets = in.isect_offsets;
    a.flatten_ids = in.flatten_ids;
    a.I = in.I;
    a.n_isects = in.n_isects;
    a.n_isects_dev = nullptr;
    a.width = in.image_width;
    a.height = in.image_height;
    a.tile_width = in.tile_width;
    a.tile_height = in.tile_height;
    return a;
}

void validate_ssim(const SxSsimInputs* in, const char* w) {
    if (!in) throw_invalid(w, "null inputs");
    if (!in->img1 || !in->img2) throw_invalid(w, "null img1/img2");
    if (in->I <= 0 || in->C <= 0)
        throw_invalid(w, "I and C must be positive (ssim mean undefined on empty batch)");
    if (in->H < 11 || in->W < 11) throw_invalid(w, "H and W must be >= 11 (valid map would be empty)");
    if (in->H > UINT32_MAX || in->W > UINT32_MAX) throw_invalid(w, "H/W exceed uint32");
    if (in->I > static_cast<int64_t>(65535) / in->C) throw_invalid(w, "I*C exceeds the grid z limit");
}

}  // namespace
}  // namespace sx

using namespace sx;

extern "C" {

const char* sxcuda_last_error(void) { return t_last_error.c_str(); }

int32_t sxcuda_abi_version(void) { return 1; }

uint32_t sxcuda_bits_for_count(int64_t count) { return bits_for_count(count); }

int32_t sxcuda_make_binoms_lut(int32_t n_max, float* lut) {
    return guarded([&] {
        if (n_max < 1) throw_invalid("make_binoms_lut", "n_max must be >= 1");
        if (!lut) throw_invalid("make_binoms_lut", "null lut");
        // Pascal's triangle in exact 64-bit integers (C(50,25) < 2^63), cast to float once.
        std::string row_store(sizeof(uint64_t) * n_max, '\0');
        uint64_t* row = reinterpret_cast<uint64_t*>(&row_store[0]);
        for (int n = 0; n < n_max; ++n) {
            for (int k = n; k >= 1; --k) row[k] += row[k - 1];
            row[0] = 1;
            for (int k = 0; k < n_max; ++k)
                lut[static_cast<size_t>(n) * n_max + k] = k <= n ? static_cast<float>(row[k]) : 0.0f;
        }
    });
}

// ---------------------------------------------------------------- executor ----------------------
int32_t sxcuda_executor_create(const SxTrainStepExecutorDesc* desc, int32_t device,
                               SxExecutor** out) {
    return guarded([&] {
        if (!desc || !out) throw_invalid("executor_create", "null desc/out");
        *out = executor_new(*desc, device);
    });
}

void sxcuda_executor_destroy(SxExecutor* ex) {
    try {
        executor_delete(ex);
    } catch (...) {
    }
}

int32_t sxcuda_executor_upload_params(SxExecutor* ex, const SxResidentParamSync* s) {
    return guarded([&] {
        if (!ex || !s) throw_invalid("executor_upload_params", "null executor/sync");
        executor_upload(ex, *s);
    });
}

int32_t sxcuda_executor_download_params(SxExecutor* ex, const SxResidentParamSync* s) {
    return guarded([&] {
        if (!ex || !s) throw_invalid("executor_download_params", "null executor/sync");
        executor_download(ex, *s);
    });
}

int32_t sxcuda_executor_step(SxExecutor* ex, const SxResidentStepInputs* in,
                             SxResidentStepOutputs* out) {
    return guarded([&] {
        if (!ex || !in || !out) throw_invalid("executor_step", "null executor/inputs/outputs");
        executor_step(ex, *in, *out);
    });
}

int32_t sxcuda_executor_step_async(SxExecutor* ex, const SxResidentStepInputs* in) {
    return guarded([&] {
        if (!ex || !in) throw_invalid("executor_step_async", "null executor/inputs");
        executor_step_async(ex, *in);
    });
}

int32_t sxcuda_executor_step_accumulate(SxExecutor* ex, const SxResidentStepInputs* in) {
    return guarded([&] {
        if (!ex || !in) throw_invalid("executor_step_accumulate", "null executor/inputs");
        executor_step_accumulate(ex, *in);
    });
}

int32_t sxcuda_executor_apply_grads(SxExecutor* ex, const SxApplyGradsInputs* in) {
    return guarded([&] {
        if (!ex || !in) throw_invalid("executor_apply_grads", "null executor/inputs");
        executor_apply_grads(ex, *in);
    });
}

int32_t sxcuda_executor_clear_grads(SxExecutor* ex) {
    return guarded([&] {
        if (!ex) throw_invalid("executor_clear_grads", "null executor");
        executor_clear_grads(ex);
    });
}

int32_t sxcuda_executor_resident_buffers(SxExecutor* ex, SxResidentBuffers* out) {
    return guarded([&] {
        if (!ex || !out) throw_invalid("executor_resident_buffers", "null executor/output");
        executor_buffers(ex, *out);
    });
}

int32_t sxcuda_executor_read_gaussians(SxExecutor* ex, const SxExecutorGaussianTrace* out,
                                       int64_t* count) {
    return guarded([&] {
        if (!ex || !out) throw_invalid("executor_read_gaussians", "null executor/output");
        executor_read_gaussians(ex, *out, count);
    });
}

int32_t sxcuda_executor_read_isects(SxExecutor* ex, int32_t* flatten_ids, int64_t capacity,
                                    int32_t* tile_offsets, int64_t tiles_capacity,
                                    int64_t* n_isects, int64_t* n_tiles) {
    return guarded([&] {
        if (!ex) throw_invalid("executor_read_isects", "null executor");
        executor_read_isects(ex, flatten_ids, capacity, tile_offsets, tiles_capacity, n_isects,
                             n_tiles);
    });
}

int32_t sxcuda_executor_read_images(SxExecutor* ex, float* render_colors, float* render_alphas,
                                    int32_t* last_ids, float* v_render_colors) {
    return guarded([&] {
        if (!ex) throw_invalid("executor_read_images", "null executor");
        executor_read_images(ex, render_colors, render_alphas, last_ids, v_render_colors);
    });
}

int32_t sxcuda_executor_eval_view(SxExecutor* ex, const SxResidentStepInputs* in,
                                  SxEvalResult* out) {
    return guarded([&] {
        if (!ex || !in || !out) throw_invalid("executor_eval_view", "null executor/inputs/result");
        executor_eval_view(ex, *in, *out);
    });
}

int32_t sxcuda_executor_render_rgba8(SxExecutor* ex, const SxResidentStepInputs* in,
                                     uint8_t* out_rgba) {
    return guarded([&] {
        if (!ex || !in) throw_invalid("executor_render_rgba8", "null executor/inputs");
        executor_render_rgba8(ex, *in, out_rgba);
    });
}

int32_t sxcuda_ply_write(const SxCloud* cloud, const char* path, int32_t pad_sh_full) {
    return guarded([&] {
        if (!cloud) throw_invalid("ply_write", "null cloud");
        ply_write(*cloud, path, pad_sh_full != 0);
    });
}

int32_t sxcuda_ply_info(const char* path, int64_t* count, int32_t* sh_degree) {
    return guarded([&] { ply_info(path, count, sh_degree); });
}

int32_t sxcuda_ply_read(const char* path, const SxCloud* out) {
    return guarded([&] {
        if (!out) throw_invalid("ply_read", "null cloud");
        ply_read(path, *out);
    });
}

int32_t sxcuda_filter_for_export(const SxCloud* cloud, float min_opacity, uint8_t* keep,
                                 SxExportFilterStats* stats) {
    return guarded([&] {
        if (!cloud) throw_invalid("filter_for_export", "null cloud");
        SxExportFilterStats st;
        filter_for_export(*cloud, min_opacity, keep, st);
        if (stats) *stats = st;
    });
}

int32_t sxcuda_spz_write(const SxCloud* cloud, const char* path, float min_opacity,
                         int32_t antialiased, SxExportFilterStats* stats) {
    return guarded([&] {
        if (!cloud) throw_invalid("spz_write", "null cloud");
        SxExportFilterStats st;
        spz_write(*cloud, path, min_opacity, antialiased != 0, st);
        if (stats) *stats = st;
    });
}

int32_t sxcuda_spz_info(const char* path, int64_t* count, int32_t* sh_degree, int32_t* antialiased) {
    return guarded([&] { spz_info(path, count, sh_degree, antialiased); });
}

int32_t sxcuda_spz_read(const char* path, const SxCloud* out) {
    return guarded([&] {
        if (!out) throw_invalid("spz_read", "null cloud");
        spz_read(path, *out);
    });
}

int32_t sxcuda_executor_export_spz(SxExecutor* ex, int64_t count, const char* path,
                                   float min_opacity, int32_t antialiased,
                                   SxExportFilterStats* stats) {
    return guarded([&] {
        if (!ex || !path) throw_invalid("executor_export_spz", "null executor/path");
        SxExportFilterStats st;
        executor_export_spz(ex, count, path, min_opacity, antialiased != 0, st);
        if (stats) *stats = st;
    });
}

int32_t sxcuda_executor_export_ply(SxExecutor* ex, int64_t count, const char* path,
                                   float min_opacity, int32_t pad_sh_full,
                                   SxExportFilterStats* stats) {
    return guarded([&] {
        if (!ex || !path) throw_invalid("executor_export_ply", "null executor/path");
        SxExportFilterStats st;
        executor_export_ply(ex, count, path, min_opacity, pad_sh_full != 0, st);
        if (stats) *stats = st;
    });
}

int32_t sxcuda_colmap_open(const char* sparse_dir, const char* images_dir, SxColmap** out) {
    return guarded([&] {
        if (!out) throw_invalid("colmap_open", "null output");
        *out = nullptr;
        *out = colmap_open(sparse_dir, images_dir);
    });
}

void sxcuda_colmap_close(SxColmap* b) { delete b; }

int32_t sxcuda_colmap_counts(const SxColmap* b, int64_t* n_images, int64_t* n_points) {
    return guarded([&] {
        if (!b) throw_invalid("colmap_counts", "null bundle");
        if (n_images) *n_images = static_cast<int64_t>(b->images.size());
        if (n_points) *n_points = static_cast<int64_t>(b->xyz.size() / 3);
    });
}

int32_t sxcuda_colmap_cameras(const SxColmap* b, float* viewmats, float* Ks, int32_t* widths,
                              int32_t* heights) {
    return guarded([&] {
        if (!b || !viewmats || !Ks || !widths || !heights)
            throw_invalid("colmap_cameras", "null bundle/output");
        colmap_cameras(*b, viewmats, Ks, widths, heights);
    });
}

int32_t sxcuda_colmap_image_path(const SxColmap* b, int64_t i, char* buf, int64_t cap,
                                 int64_t* len) {
    return guarded([&] {
        if (!b || !len) throw_invalid("colmap_image_path", "null bundle/len");
        if (i < 0 || i >= static_cast<int64_t>(b->images.size()))
            throw_invalid("colmap_image_path", "image index out of range");
        const std::string p = b->images_dir + "/" + b->images[static_cast<size_t>(i)].name;
        *len = static_cast<int64_t>(p.size());
        if (!buf) return;
        if (cap < *len) throw_invalid("colmap_image_path", "buffer too small");
        std::memcpy(buf, p.data(), p.size());
    });
}

int32_t sxcuda_colmap_seed(const SxColmap* b, float* points, uint8_t* rgb) {
    return guarded([&] {
        if (!b || (!b->xyz.empty() && (!points || !rgb))) throw_invalid("colmap_seed", "null output");
        for (size_t k = 0; k < b->xyz.size(); ++k) points[k] = static_cast<float>(b->xyz[k]);
        if (!b->rgb.empty()) std::memcpy(rgb, b->rgb.data(), b->rgb.size());
    });
}

int32_t sxcuda_checkpoint_verify_config(const SxCheckpointConfig* saved,
                                        const SxCheckpointConfig* current) {
    return guarded([&] {
        if (!saved || !current) throw_invalid("checkpoint_verify_config", "null config");
        checkpoint_verify(*saved, *current);
    });
}

int32_t sxcuda_checkpoint_info(const char* path, SxCheckpointHeader* out) {
    return guarded([&] {
        if (!out) throw_invalid("checkpoint_info", "null output");
        checkpoint_header(path, *out);
    });
}

int32_t sxcuda_executor_save_checkpoint(SxExecutor* ex, const SxCheckpointConfig* config,
                                        int32_t iter, int64_t count, const char* path,
                                        int32_t fp16) {
    return guarded([&] {
        if (!ex || !config) throw_invalid("save_checkpoint", "null executor/config");
        executor_save_checkpoint(ex, *config, iter, count, path, fp16 != 0);
    });
}

int32_t sxcuda_executor_load_checkpoint(SxExecutor* ex, const char* path,
                                        const SxCheckpointConfig* current,
                                        SxCheckpointHeader* out) {
    return guarded([&] {
        if (!ex || !out) throw_invalid("load_checkpoint", "null executor/output");
        executor_load_checkpoint(ex, path, current, *out);
    });
}

int32_t sxcuda_executor_peer_handles(SxExecutor* ex, SxPeerHandles* out) {
    return guarded([&] {
        if (!ex || !out) throw_invalid("executor_peer_handles", "null executor/output");
        executor_peer_handles(ex, *out);
    });
}

int32_t sxcuda_executor_open_peers(SxExecutor* ex, int32_t rank, int32_t world,
                                   const SxPeerHandles* all) {
    return guarded([&] {
        if (!ex || !all) throw_invalid("executor_open_peers", "null executor/handles");
        executor_open_peers(ex, rank, world, all);
    });
}

int32_t sxcuda_executor_exchange_apply(SxExecutor* ex, const SxApplyGradsInputs* in) {
    return guarded([&] {
        if (!ex || !in) throw_invalid("executor_exchange_apply", "null executor/inputs");
        executor_exchange_apply(ex, *in);
    });
}

int32_t sxcuda_executor_step_exchange(SxExecutor* ex, const SxResidentStepInputs* in,
                                      const SxApplyGradsInputs* ap, int32_t chunks) {
    return guarded([&] {
        if (!ex || !in || !ap) throw_invalid("executor_step_exchange", "null executor/inputs");
        executor_step_exchange(ex, *in, *ap, chunks);
    });
}

int32_t sxcuda_executor_mcmc_seed(SxExecutor* ex, uint64_t seed) {
    return guarded([&] {
        if (!ex) throw_invalid("executor_mcmc_seed", "null executor");
        executor_mcmc_seed(ex, seed);
    });
}

int32_t sxcuda_executor_mcmc_rng_state(SxExecutor* ex, char* buf, int64_t cap, int64_t* len) {
    return guarded([&] {
        if (!ex || !len) throw_invalid("executor_mcmc_rng_state", "null executor/len");
        const std::string t = executor_mcmc_rng_state(ex);
        *len = static_cast<int64_t>(t.size());
        if (!buf) return;
        if (cap < *len) throw_invalid("executor_mcmc_rng_state", "buffer too small");
        std::memcpy(buf, t.data(), t.size());
    });
}

int32_t sxcuda_executor_mcmc_set_rng_state(SxExecutor* ex, const char* text, int64_t len) {
    return guarded([&] {
        if (!ex || !text || len <= 0) throw_invalid("executor_mcmc_set_rng_state", "empty state");
        executor_mcmc_set_rng_state(ex, std::string(text, static_cast<size_t>(len)));
    });
}

int32_t sxcuda_executor_mcmc_refine(SxExecutor* ex, const SxMcmcRefineInputs* in,
                                    SxMcmcRefineResult* out) {
    return guarded([&] {
        if (!ex || !in || !out) throw_invalid("executor_mcmc_refine", "null executor/inputs/result");
        if (out->list_capacity < 0) throw_invalid("executor_mcmc_refine", "negative list_capacity");
        McmcRefineOut r;
        executor_mcmc_refine(ex, in->count, in->cap_max, in->min_opacity, r);
        out->count = r.count;
        out->n_relocated = static_cast<int64_t>(r.relocated_dead.size());
        out->n_added = static_cast<int64_t>(r.added_src.size());
        auto put = [&](int64_t* dst, const std::vector<int64_t>& v) {
            if (!dst) return;
            const size_t n = std::min(v.size(), static_cast<size_t>(out->list_capacity));
            if (n) std::memcpy(dst, v.data(), n * sizeof(int64_t));
        };
        put(out->relocated_dead, r.relocated_dead);
        put(out->relocation_src, r.relocation_src);
        put(out->added_src, r.added_src);
    });
}

int32_t sxcuda_executor_inject_noise(SxExecutor* ex, int64_t count, uint64_t seed, uint64_t offset,
                                     float noise_scale) {
    return guarded([&] {
        if (!ex) throw_invalid("executor_inject_noise", "null executor");
        executor_inject_noise(ex, count, seed, offset, noise_scale);
    });
}

int32_t sxcuda_executor_last_result(SxExecutor* ex, float* loss, int64_t* n_isects,
                                    int64_t* overflowed) {
    return guarded([&] {
        if (!ex) throw_invalid("executor_last_result", "null executor");
        executor_last_result(ex, loss, n_isects, overflowed);
    });
}

int32_t sxcuda_executor_reserve_isects(SxExecutor* ex, int64_t n) {
    return guarded([&] {
        if (!ex) throw_invalid("executor_reserve_isects", "null executor");
        if (n < 0) throw_invalid("executor_reserve_isects", "negative n");
        executor_reserve(ex, n);
    });
}

sxcuda_stream_t sxcuda_executor_stream(SxExecutor* ex) {
    return ex ? static_cast<sxcuda_stream_t>(executor_stream(ex)) : nullptr;
}

int64_t sxcuda_executor_last_launch_count(SxExecutor* ex) { return ex ? executor_launches(ex) : 0; }

int32_t sxcuda_executor_set_profiling(SxExecutor* ex, int32_t on) {
    return guarded([&] {
        if (!ex) throw_invalid("executor_set_profiling", "null executor");
        executor_set_profiling(ex, on != 0);
    });
}

int32_t sxcuda_executor_segment_times(SxExecutor* ex, const char** names, float* ms,
                                      int32_t capacity, int32_t* count) {
    return guarded([&] {
        if (!ex || !names || !ms || !count) throw_invalid("executor_segment_times", "null argument");
        *count = executor_segments(ex, names, ms, capacity);
    });
}

int32_t sxcuda_peer_barrier_selftest(int32_t device, int32_t world, uint32_t* status) {
    return guarded([&] {
        if (!status) throw_invalid("peer_barrier_selftest", "null status");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        *status = peer_barrier_selftest(world, nullptr);
    });
}

int32_t sxcuda_peer_exchange_selftest(int32_t device, int32_t world, uint32_t* status,
                                      int32_t* applied) {
    return guarded([&] {
        if (!status || !applied) throw_invalid("peer_exchange_selftest", "null output");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        int a = 0;
        *status = peer_barrier_selftest(world, &a);
        *applied = a;
    });
}

int32_t sxcuda_executor_set_pair_counting(SxExecutor* ex, int32_t on) {
    return guarded([&] {
        if (!ex) throw_invalid("executor_set_pair_counting", "null executor");
        executor_set_pair_counting(ex, on != 0);
    });
}

int32_t sxcuda_executor_bin_stats(SxExecutor* ex, int64_t* n_entries, int64_t* n_supertiles) {
    return guarded([&] {
        if (!ex) throw_invalid("executor_bin_stats", "null executor");
        executor_bin_stats(ex, n_entries, n_supertiles);
    });
}

int32_t sxcuda_executor_set_tile_lists(SxExecutor* ex, int32_t mode) {
    return guarded([&] {
        if (!ex) throw_invalid("executor_set_tile_lists", "null executor");
        if (mode != 0 && mode != 1) throw_invalid("executor_set_tile_lists", "mode must be 0 or 1");
        executor_set_tile_lists(ex, mode);
    });
}

int32_t sxcuda_executor_raster_pairs(SxExecutor* ex, int64_t* fwd_pairs, int64_t* bwd_pairs) {
    return guarded([&] {
        if (!ex || !fwd_pairs || !bwd_pairs) throw_invalid("executor_raster_pairs", "null argument");
        int64_t o[2];
        executor_raster_pairs(ex, o);
        *fwd_pairs = o[0];
        *bwd_pairs = o[1];
    });
}

int32_t sxcuda_executor_exchange_timeline(SxExecutor* ex, const char** names, float* ms,
                                          int32_t capacity, int32_t* count) {
    return guarded([&] {
        if (!ex || !names || !ms || !count)
            throw_invalid("executor_exchange_timeline", "null argument");
        *count = executor_exchange_timeline(ex, names, ms, capacity);
    });
}

// ---------------------------------------------------------------- per-kernel ----------------------
int32_t sxcuda_fused_adam(const SxAdamInputs* in, sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "fused_adam";
        if (!in) throw_invalid(w, "null inputs");
        if (in->n_elems == 0) return;
        if (!in->param || !in->grad || !in->exp_avg || !in->exp_avg_sq) throw_invalid(w, "null tensor");
        if (in->n_elems < 0 || in->n_gauss <= 0 || in->n_elems % in->n_gauss != 0)
            throw_invalid(w, "n_elems must be a positive multiple of n_gauss");
        launch_adam(*in, as_stream(stream));
    });
}

int32_t sxcuda_projection_fused_fwd(const SxProjectionFusedInputs* in,
                                    const SxProjectionFusedOutputs* out, sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "projection_fused_fwd";
        validate_projection(in, w);
        if (!out || (in->N * in->C > 0 && (!out->radii || !out->means2d || !out->depths || !out->conics)))
            throw_invalid(w, "null outputs");
        if (in->calc_compensations && in->N * in->C > 0 && !out->compensations)
            throw_invalid(w, "null compensations output");
        launch_projection_fwd(*in, *out, as_stream(stream));
    });
}

int32_t sxcuda_projection_fused_bwd(const SxProjectionFusedInputs* in,
                                    const SxProjectionFusedGradsIn* g,
                                    const SxProjectionFusedGrads* out, sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "projection_fused_bwd";
        validate_projection(in, w);
        if (!g || !out) throw_invalid(w, "null grads");
        if (!g->radii || !g->conics || !g->v_means2d || !g->v_depths || !g->v_conics)
            throw_invalid(w, "null radii/conics/v_means2d/v_depths/v_conics");
        if (g->v_compensations && !g->compensations)
            throw_invalid(w, "v_compensations requires compensations (fwd output)");
        if (!out->v_means) throw_invalid(w, "null v_means");
        if (in->covars ? !out->v_covars : (!out->v_quats || !out->v_scales))
            throw_invalid(w, "null v_covars or v_quats/v_scales");
        if (g->viewmats_grad && !out->v_viewmats) throw_invalid(w, "null v_viewmats");
        launch_projection_bwd(*in, *g, *out, as_stream(stream));
    });
}

int32_t sxcuda_sh_fwd(const SxShInputs* in, float* colors, sxcuda_stream_t stream) {
    return guarded([&] {
        validate_sh(in, "sh_fwd");
        if (!colors && in->B * in->N > 0) throw_invalid("sh_fwd", "null colors");
        launch_sh_fwd(*in, colors, as_stream(stream));
    });
}

int32_t sxcuda_sh_bwd(const SxShInputs* in, const float* v_colors, float* v_coeffs, float* v_dirs,
                      sxcuda_stream_t stream) {
    return guarded([&] {
        validate_sh(in, "sh_bwd");
        if (!v_colors || !v_coeffs) throw_invalid("sh_bwd", "null v_colors/v_coeffs");
        if (in->compute_v_dirs && !v_dirs) throw_invalid("sh_bwd", "null v_dirs");
        launch_sh_bwd(*in, v_colors, v_coeffs, v_dirs, as_stream(stream));
    });
}

int32_t sxcuda_isect_tile_count(const SxIsectTilesInputs* in, int32_t* tiles_per_gauss,
                                int64_t* cum, int64_t* n_isects_host, void* ws, size_t* ws_bytes,
                                sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "isect_tiles";
        validate_isect(in, w);
        const int64_t n = in->I * in->N;
        if (workspace_query(ws, ws_bytes, scan_i64_workspace(n), w)) return;
        if (n > 0 && (!tiles_per_gauss || !cum)) throw_invalid(w, "null tiles_per_gauss/cum");
        if (!n_isects_host) throw_invalid(w, "null n_isects_host");
        cudaStream_t s = as_stream(stream);
        *n_isects_host = 0;
        if (n == 0) return;
        launch_isect_count(*in, tiles_per_gauss, s);
        launch_scan_i64(tiles_per_gauss, cum, n, ws, s);
        int64_t total = 0;
        cuda_check(cudaMemcpyAsync(&total, cum + n - 1, sizeof(int64_t), cudaMemcpyDeviceToHost, s),
                   "n_isects readback");
        cuda_check(cudaStreamSynchronize(s), "n_isects readback");
        if (total < 0 || total > INT32_MAX)
            throw_invalid(w, "n_isects must fit in int32 (offsets/last_ids)");
        *n_isects_host = total;
    });
}

int32_t sxcuda_isect_tile_emit(const SxIsectTilesInputs* in, const int64_t* cum,
                               uint64_t* isect_ids, int32_t* flatten_ids, sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "isect_tiles";
        validate_isect(in, w);
        if (in->I * in->N > 0 && (!cum || !isect_ids || !flatten_ids))
            throw_invalid(w, "null cum/isect_ids/flatten_ids");
        const uint32_t tb = bits_for_count(static_cast<int64_t>(in->tile_width) * in->tile_height);
        launch_isect_emit(*in, tb, cum, isect_ids, flatten_ids, as_stream(stream));
    });
}

int32_t sxcuda_prefix_scan_i64(const int32_t* in, int64_t* out, int64_t n, void* ws,
                               size_t* ws_bytes, sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "prefix_scan_i64";
        if (n < 0) throw_invalid(w, "negative n");
        if (workspace_query(ws, ws_bytes, scan_i64_workspace(n), w)) return;
        if (n > 0 && (!in || !out)) throw_invalid(w, "null in/out");
        launch_scan_i64(in, out, n, ws, as_stream(stream));
    });
}

int32_t sxcuda_prefix_scan_i64_noalloc(const int32_t* in, int64_t* out, int64_t n,
                                       sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "prefix_scan_i64_noalloc";
        if (n < 0) throw_invalid(w, "negative n");
        if (n > noalloc_scan_max_n())
            throw_invalid(w, "n exceeds the fixed scratch capacity of 268435456 elements");
        if (n > 0 && (!in || !out)) throw_invalid(w, "null in/out");
        launch_scan_i64_noalloc(in, out, n, as_stream(stream));
    });
}

int32_t sxcuda_sort_isect(const uint64_t* keys, const int32_t* values, uint64_t* keys_sorted,
                          int32_t* values_sorted, int64_t n, uint32_t key_n_bits, void* ws,
                          size_t* ws_bytes, sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "sort_isect";
        if (n < 0) throw_invalid(w, "negative n");
        if (n > INT32_MAX) throw_invalid(w, "n must fit in int32 (flatten_ids)");
        if (key_n_bits < 1 || key_n_bits > 64) throw_invalid(w, "key_n_bits must be 1..64");
        if (workspace_query(ws, ws_bytes, radix_sort_u64_workspace(n), w)) return;
        if (n > 0 && (!keys || !values || !keys_sorted || !values_sorted))
            throw_invalid(w, "null keys/values");
        radix_sort_u64(keys, values, keys_sorted, values_sorted, n, key_n_bits, ws, as_stream(stream));
    });
}

int32_t sxcuda_isect_offset_encode(const uint64_t* ids, int64_t n_isects, int64_t I,
                                   uint32_t tile_width, uint32_t tile_height, int32_t* offsets,
                                   sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "isect_offset_encode";
        if (n_isects < 0) throw_invalid(w, "negative n_isects");
        if (n_isects > 0 && !ids) throw_invalid(w, "null isect_ids");
        if (I < 0) throw_invalid(w, "negative I");
        if (n_isects > 0 && I == 0) throw_invalid(w, "n_isects > 0 requires I > 0 (keys encode image ids)");
        if (tile_width == 0 || tile_height == 0) throw_invalid(w, "tile_width/tile_height must be positive");
        const int64_t n_tiles = static_cast<int64_t>(tile_width) * tile_height;
        if (bits_for_count(I) + bits_for_count(n_tiles) > 32)
            throw_invalid(w, "image_n_bits + tile_n_bits must be <= 32");
        if (n_isects > INT32_MAX) throw_invalid(w, "n_isects must fit in int32 (offsets values)");
        if (I > 0 && n_tiles > INT32_MAX / I) throw_invalid(w, "I*n_tiles must fit in int32 (offsets table)");
        if (I * n_tiles > 0 && !offsets) throw_invalid(w, "null offsets");
        launch_offset_encode(ids, n_isects, I, bits_for_count(n_tiles), n_tiles, offsets,
                             as_stream(stream));
    });
}

int32_t sxcuda_rasterize_fwd(const SxRasterizeFwdInputs* in, float* rc, float* ra, int32_t* li,
                             sxcuda_stream_t stream) {
    return guarded([&] {
        validate_raster(in, "rasterize_fwd");
        if (!rc || !ra || !li) throw_invalid("rasterize_fwd", "null outputs");
        launch_raster_fwd(raster_args(*in), rc, ra, li, as_stream(stream));
    });
}

int32_t sxcuda_rasterize_bwd(const SxRasterizeFwdInputs* in, const SxRasterizeBwdGradsIn* g,
                             const SxRasterizeBwdGrads* out, sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "rasterize_bwd";
        validate_raster(in, w);
        if (!g || !out) throw_invalid(w, "null grads");
        if (!g->render_alphas || !g->last_ids) throw_invalid(w, "null render_alphas/last_ids (fwd outputs)");
        if (!g->v_render_colors || !g->v_render_alphas)
            throw_invalid(w, "null v_render_colors/v_render_alphas");
        if (!out->v_means2d || !out->v_conics || !out->v_colors || !out->v_opacities)
            throw_invalid(w, "null gradient outputs");
        if (g->absgrad && !out->v_means2d_abs) throw_invalid(w, "null v_means2d_abs");
        cudaStream_t s = as_stream(stream);
        const int64_t IN = in->I * in->N;
        auto zero = [&](float* p, int64_t n) {
            if (p && n > 0) cuda_check(cudaMemsetAsync(p, 0, sizeof(float) * n, s), "memset grads");
        };
        zero(out->v_means2d, IN * 2);
        zero(out->v_conics, IN * 3);
        zero(out->v_colors, IN * 3);
        zero(out->v_opacities, IN);
        if (g->absgrad) zero(out->v_means2d_abs, IN * 2);
        if (in->n_isects == 0) return;  // all-zero gradients
        launch_raster_bwd(raster_args(*in), g->render_alphas, g->last_ids, g->v_render_colors,
                          g->v_render_alphas, out->v_means2d, out->v_conics, out->v_colors,
                          out->v_opacities, g->absgrad ? out->v_means2d_abs : nullptr, s);
    });
}

int32_t sxcuda_rng_normal_f32(uint64_t seed, uint64_t offset, int64_t count, float* out,
                              sxcuda_stream_t stream) {
    return guarded([&] {
        if (count < 0) throw_invalid("rng_normal_f32", "negative count");
        if (count > static_cast<int64_t>(UINT32_MAX)) throw_invalid("rng_normal_f32", "count must fit in uint32");
        if (count > 0 && !out) throw_invalid("rng_normal_f32", "null out");
        launch_rng_normal(seed, offset, count, out, as_stream(stream));
    });
}

int32_t sxcuda_rng_philox_u32(uint64_t seed, uint64_t offset, int64_t count, uint32_t* out,
                              sxcuda_stream_t stream) {
    return guarded([&] {
        if (count < 0) throw_invalid("rng_philox_u32", "negative count");
        if (count > static_cast<int64_t>(UINT32_MAX)) throw_invalid("rng_philox_u32", "count must fit in uint32");
        if (count > 0 && !out) throw_invalid("rng_philox_u32", "null out");
        launch_rng_u32(seed, offset, count, out, as_stream(stream));
    });
}

int32_t sxcuda_mcmc_relocation(const SxRelocationInputs* in, float* new_op, float* new_sc,
                               sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "mcmc_relocation";
        if (!in) throw_invalid(w, "null inputs");
        if (!in->opacities || !in->scales || !in->ratios || !in->binoms)
            throw_invalid(w, "null opacities/scales/ratios/binoms");
        if (in->N < 0) throw_invalid(w, "negative N");
        if (in->n_max < 1) throw_invalid(w, "n_max must be >= 1");
        if (in->N > static_cast<int64_t>(UINT32_MAX)) throw_invalid(w, "N exceeds uint32");
        if (in->N > 0 && (!new_op || !new_sc)) throw_invalid(w, "null outputs");
        launch_relocation(*in, new_op, new_sc, as_stream(stream));
    });
}

int32_t sxcuda_mcmc_perturb_positions(const SxPerturbInputs* in, sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "mcmc_perturb_positions";
        if (!in) throw_invalid(w, "null inputs");
        if (in->N == 0) return;
        if (!in->positions || !in->quats || !in->scales_log || !in->opacities_logit || !in->noise)
            throw_invalid(w, "null positions/quats/scales_log/opacities_logit/noise");
        if (in->N < 0) throw_invalid(w, "negative N");
        if (in->N > static_cast<int64_t>(UINT32_MAX)) throw_invalid(w, "N exceeds uint32");
        launch_perturb(*in, as_stream(stream));
    });
}

int32_t sxcuda_ssim_fwd(const SxSsimInputs* in, float* map, float* cmu, float* csg, float* ccr,
                        double* mean_dev, void* ws, size_t* ws_bytes, sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "ssim_fwd";
        validate_ssim(in, w);
        if (workspace_query(ws, ws_bytes, ssim_fwd_workspace(in->I, in->H, in->W, in->C), w)) return;
        if (!map || !mean_dev) throw_invalid(w, "null ssim_map/mean");
        if (in->need_coeffs && (!cmu || !csg || !ccr)) throw_invalid(w, "null coefficient maps");
        launch_ssim_fwd(in->img1, in->img2, in->I, in->H, in->W, in->C, in->need_coeffs != 0, map,
                        cmu, csg, ccr, mean_dev, ws, as_stream(stream));
    });
}

int32_t sxcuda_ssim_bwd(const SxSsimInputs* in, const SxSsimGradsIn* g, float* v_img1,
                        sxcuda_stream_t stream) {
    return guarded([&] {
        const char* w = "ssim_bwd";
        validate_ssim(in, w);
        if (!g || !g->coeff_mu || !g->coeff_sigma || !g->coeff_cross)
            throw_invalid(w, "null coeff maps (run ssim_fwd with need_coeffs=true)");
        if (!v_img1) throw_invalid(w, "null v_img1");
        const double M = static_cast<double>(in->I) * in->C * (in->H - 10) * (in->W - 10);
        const float G = static_cast<float>(-static_cast<double>(g->v_loss) / M);
        launch_ssim_bwd(in->img1, in->img2, in->I, in->H, in->W, in->C, g->coeff_mu, g->coeff_sigma,
                        g->coeff_cross, G, v_img1, as_stream(stream));
    });
}


// ---- render session (sx_render_session_*, TrainC.cpp:1440-1584) ----------------------------
struct SxRenderSession {
    SxExecutor* ex = nullptr;
    int64_t count = 0;
    int32_t sh_degree = 0;
    ~SxRenderSession() {
        if (ex) sx::executor_delete(ex);
    }
};

namespace {
void fill_err(char* buf, int32_t len, const std::string& msg) {
    if (!buf || len <= 0) return;
    const size_t n = std::min(static_cast<size_t>(len - 1), msg.size());
    std::memcpy(buf, msg.data(), n);
    buf[n] = '\0';
}
}  // namespace

SxRenderSession* sxcuda_render_session_open(const SxRenderSessionArgs* args, char* err_buf,
                                            int32_t err_buf_len) {
    DeviceRestore restore;
    try {
        if (!args) throw std::invalid_argument("args must be given (zero-initialise, then fill)");
        if (!args->ply_path) throw std::invalid_argument("ply_path must be given");
        if (args->sh_degree < 0 || args->sh_degree > 3)
            throw std::invalid_argument("sh_degree must be 0..3 (0 = derived from the PLY)");
        int64_t n = 0;
        int32_t deg = 0;
        sx::ply_info(args->ply_path, &n, &deg);
        if (n < 1) throw std::invalid_argument("the PLY holds no Gaussians (count must be >= 1)");
        if (deg > 3) throw std::invalid_argument("PLY SH degree 4 is outside the render path (0..3)");
        if (args->sh_degree > 0 && args->sh_degree > deg)
            throw std::invalid_argument("sh_degree " + std::to_string(args->sh_degree) +
                                        " exceeds PLY sh_degree " + std::to_string(deg) +
                                        " (higher-band coefficients absent)");
        const int K = (deg + 1) * (deg + 1) - 1;
        std::vector<float> means(n * 3), scales(n * 3), quats(n * 4), op(n), sh0(n * 3),
            shN(static_cast<size_t>(n) * K * 3 + 1);
        SxCloud c{n, deg, means.data(), scales.data(), quats.data(), op.data(), sh0.data(), shN.data()};
        sx::ply_read(args->ply_path, c);
        int rdeg = deg;
        if (args->sh_degree > 0 && args->sh_degree < deg) {  // truncate the higher bands
            rdeg = args->sh_degree;
            const int Kn = (rdeg + 1) * (rdeg + 1) - 1;
            for (int64_t i = 0; i < n; ++i)
                std::memmove(shN.data() + i * Kn * 3, shN.data() + i * K * 3, sizeof(float) * Kn * 3);
        }
        const int Kr = (rdeg + 1) * (rdeg + 1) - 1;
        SxTrainStepExecutorDesc d{};
        d.arena_rows = n;
        d.sh_degree = rdeg;
        d.eps2d = 0.3f;
        d.near_plane = 0.01f;
        d.far_plane = 1e10f;
        d.radius_clip = 0.0f;
        d.b1 = 0.9f;
        d.b2 = 0.999f;
        d.eps = 1e-15f;
        d.ssim_weight = 0.2f;
        d.antialiased = args->antialiased != 0;
        auto session = std::make_unique<SxRenderSession>();
        session->ex = sx::executor_new(d, args->device);
        session->count = n;
        session->sh_degree = rdeg;
        std::vector<float> zeros(static_cast<size_t>(n) * std::max(Kr * 3, 4) + 1, 0.0f);
        SxResidentParamSync sync{};
        float* params[6] = {means.data(), quats.data(), scales.data(), op.data(), sh0.data(), shN.data()};
        for (int g = 0; g < 6; ++g) {
            sync.params[g] = params[g];
            sync.exp_avg[g] = zeros.data();
            sync.exp_avg_sq[g] = zeros.data();
        }
        sync.rows = n;
        sx::executor_upload(session->ex, sync);
        return session.release();
    } catch (const std::exception& e) {
        fill_err(err_buf, err_buf_len, e.what());
        return nullptr;
    } catch (...) {
        fill_err(err_buf, err_buf_len, "unknown error");
        return nullptr;
    }
}

int32_t sxcuda_render_session_frame(SxRenderSession* session, const float* viewmat, float fx,
                                    float fy, float cx, float cy, int32_t width, int32_t height,
                                    uint8_t* out_rgba, char* err_buf, int32_t err_buf_len) {
    if (!session || !viewmat || !out_rgba) {
        fill_err(err_buf, err_buf_len, "session/viewmat/out_rgba must be given");
        return -1;
    }
    if (width < 1 || height < 1) {
        fill_err(err_buf, err_buf_len, "width/height must be positive");
        return -1;
    }
    if (!(fx > 0.0f) || !(fy > 0.0f) || !std::isfinite(cx) || !std::isfinite(cy)) {
        fill_err(err_buf, err_buf_len, "fx/fy must be positive and cx/cy finite");
        return -1;
    }
    DeviceRestore restore;
    try {
        const float K[9] = {fx, 0.0f, cx, 0.0f, fy, cy, 0.0f, 0.0f, 1.0f};
        SxResidentStepInputs in{};
        in.viewmat = viewmat;
        in.K = K;
        in.width = width;
        in.height = height;
        in.count = session->count;
        in.degrees_to_use = static_cast<uint32_t>(session->sh_degree);
        in.forward_only = 1;
        executor_render_rgba8(session->ex, in, out_rgba);
        return 0;
    } catch (const std::exception& e) {
        fill_err(err_buf, err_buf_len, e.what());
        return -2;
    } catch (...) {
        fill_err(err_buf, err_buf_len, "unknown error");
        return -2;
    }
}

void sxcuda_render_session_close(SxRenderSession* session) {
    DeviceRestore restore;
    delete session;
}

}  // extern "C"
