// executor.cu — the device-resident training step (replaces MetalTrainStepExecutor,
// Sources/SplatXCore/MetalBackend.cpp:1628-2460).
//
// One step, all on the executor's stream, no host synchronisation until the final read-back:
//   fwd_gauss            activations + projection + SH colour + AccuTile count (per Gaussian)
//   depth sort           stable radix sort of the Gaussians by depth bits (ties: index order)
//   gather scan          exclusive scan of tile counts in depth order -> n_isects (device)
//   capacity check       n_isects > capacity -> the step degrades to a no-op and is replayed
//   emit                 Gaussians in depth order write (tile, id) pairs
//   tile sort            stable radix sort by tile id  => order (tile, depth, index) — exactly
//                        the reference's stable sort of (tile<<32 | depth) keys in emit order
//   tile offsets, raster forward, fused L1+SSIM loss/gradient, raster backward
//   bwd_gauss            SH + projection backward, chains, Adam x6, MCMC noise (per Gaussian)
// The only host synchronisation is the read-back of (loss, n_isects, overflow) at the end.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <memory>
#include <vector>

#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

__global__ void capacity_check_kernel(const int64_t* __restrict__ n_isects, int64_t cap,
                                      int64_t* __restrict__ n_eff, int32_t* __restrict__ overflow,
                                      int64_t* __restrict__ overflow_count) {
    const int64_t n = *n_isects;
    const bool over = n > cap || *overflow != 0;
    *n_eff = over ? 0 : n;
    *overflow = over ? 1 : 0;
    if (over) *overflow_count += 1;
}

// The supertile path's check: the tile total and the entry total (both summed by the depth-order
// scan) against the capacity; the effective counts are 0 after an overflow.
__global__ void bin_capacity_check_kernel(const int64_t* __restrict__ n_isects,
                                          const int64_t* __restrict__ n_entries, int64_t cap,
                                          int64_t* __restrict__ n_eff, int64_t* __restrict__ n_eff_entries,
                                          int32_t* __restrict__ overflow,
                                          int64_t* __restrict__ overflow_count) {
    const int64_t n = *n_isects, ne = *n_entries;
    const bool over = n > cap || ne > cap || *overflow != 0;
    *n_eff = over ? 0 : n;
    *n_eff_entries = over ? 0 : ne;
    *overflow = over ? 1 : 0;
    if (over) *overflow_count += 1;
}

// Tile ids wider than this are rejected. Up to kStMaxSupertiles supertiles the tile lists come
// from the supertile binning; wider grids emit (tile, Gaussian) pairs and sort them. The sort
// workspace covers both: kMaxTileBits-bit keys and a whole-key histogram of kHistTileBins bins.
constexpr uint32_t kMaxTileBits = 24;
constexpr int64_t kHistTileBins = 16384;
// The single-sweep sort keeps counts in 30 bits.
constexpr int64_t kMaxIsects = (int64_t{1} << 30) - 1;

template <typename T>
T* dalloc(size_t count, std::vector<void*>& owned) {
    void* p = nullptr;
    if (count == 0) count = 1;
    cuda_check(cudaMalloc(&p, sizeof(T) * count),
               "executor allocation (device memory exhausted?)");
    owned.push_back(p);
    return static_cast<T*>(p);
}

}  // namespace

}  // namespace sx

struct SxExecutor {
    SxTrainStepExecutorDesc d{};
    int device = 0;
    cudaStream_t stream = nullptr;
    int32_t K = 1;
    int64_t rows = 0;
    // Resident parameters and moments are tiled: Gaussians in tiles of 32, a group's dims[g]
    // components as runs of 32 floats inside each tile (tile_index). `padded` = rows rounded up
    // to 32. Host sync converts to and from the reference's [rows, dims] layout through a fixed
    // staging buffer of kStageRows rows.
    int64_t padded = 0;
    static constexpr int64_t kStageRows = 1 << 16;
    float* stage = nullptr;
    int64_t dims[6] = {3, 4, 3, 1, 3, 0};
    std::vector<void*> owned;

    float* p[6] = {};
    float* m1[6] = {};
    float* m2[6] = {};

    uint8_t* valid = nullptr;
    float* means2d = nullptr;
    float* conics = nullptr;
    float* opac_raster = nullptr;
    float* comps = nullptr;
    float* act = nullptr;    // tiles of 4: forward activations reused by the backward
    float* v_dir = nullptr;  // tiles of 3: SH direction gradient between the backward kernels
    // view-parallel training: accumulated gradients (tiled like the parameters) and visibility
    float* gacc[6] = {};
    float* gvis = nullptr;
    float* colors = nullptr;
    float4* raster_rec = nullptr;  // [N,3] packed raster records (RasterArgs::rec)
    uint8_t* relu_mask = nullptr;
    int32_t* tiles = nullptr;
    uint32_t* depth_keys = nullptr;
    int32_t* gauss_ids = nullptr;
    int32_t* order = nullptr;
    int32_t* excl_offsets = nullptr;
    int32_t* entries = nullptr;  // supertile entries per Gaussian
    void* ws_scan = nullptr;
    void* ws_depth = nullptr;
    float* v_means2d = nullptr;
    float* v_conics = nullptr;
    float* v_colors = nullptr;
    float* v_opac = nullptr;

    int64_t cap = 0;
    uint32_t* tile_keys = nullptr;
    int32_t* gauss_vals = nullptr;
    uint32_t* tile_keys_sorted = nullptr;
    int32_t* flatten_ids = nullptr;
    void* ws_tile = nullptr;
    // supertile binning (the entries' sort keys and ids live in tile_keys / gauss_vals)
    uint4* entry = nullptr;          // [cap] (tile mask lo, hi, Gaussian id, 0)
    int32_t* st_sorted = nullptr;
    int64_t max_chunks = 0;
    uint32_t* chunk_counts = nullptr;
    std::vector<void*> isect_bufs;

    int64_t img_cap = 0;
    int64_t tiles_cap = 0;
    size_t loss_ws_cap = 0;
    float* gt = nullptr;
    float* render = nullptr;
    float* alphas = nullptr;
    int32_t* last_ids = nullptr;
    float* v_render = nullptr;
    float* v_ralpha_zero = nullptr;
    float* cmu = nullptr;
    float* csg = nullptr;
    float* ccr = nullptr;
    void* ws_loss = nullptr;
    int32_t* tile_offsets = nullptr;
    int32_t* tile_counts = nullptr;
    std::vector<void*> image_bufs;

    // device scalars
    int64_t* n_isects = nullptr;
    int64_t* n_eff = nullptr;
    int64_t* n_entries = nullptr;      // supertile entries of the step (scan total)
    int64_t* n_eff_entries = nullptr;  // 0 after an overflow
    int32_t* n_chunks = nullptr;
    uint32_t* bin_done = nullptr;      // st_prefix's finishing counter (0 between steps)
    int32_t* st_offsets = nullptr;     // [kStMaxSupertiles]
    int32_t* st_chunk0 = nullptr;      // [kStMaxSupertiles + 1]
    int32_t* overflow = nullptr;
    int64_t* overflow_count = nullptr;
    float* loss = nullptr;
    uint32_t* status = nullptr;  // error bits set by kernels whose bounded waits ran out
    // pinned host mirror: loss, n_isects, overflow, overflow_count, status
    struct HostOut {
        float loss;
        int32_t overflow;
        int64_t n_isects;
        int64_t overflow_count;
        uint32_t status;
    }* h = nullptr;
    HostOut* dev_out = nullptr;
    // the ground-truth upload runs on its own stream, overlapping the forward segments:
    // gt_free (main stream, after the loss) -> copy -> gt_ready (waited on before the loss)
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t gt_ready = nullptr, gt_free = nullptr;

    sx::McmcRefine* mcmc = nullptr;  // created by the first refine / seed call

    int64_t last_launches = 0;
    int64_t last_count = 0;
    uint32_t last_w = 0, last_h = 0;

    // per-segment timing (the reference's [ktime] segments): CUDA events recorded between
    // segments of every step while profiling is on; read back (and averaged) in one go.
    bool profiling = false;
    std::vector<cudaEvent_t> event_pool;
    std::vector<std::vector<cudaEvent_t>> step_events;
    std::vector<const char*> seg_names;
    void seg_begin() {
        if (!profiling) return;
        step_events.emplace_back();
        seg_names.clear();
        mark(nullptr);
    }
    void mark(const char* name_of_finished_segment) {
        if (!profiling) return;
        cudaEvent_t e;
        if (event_pool.empty()) {
            sx::cuda_check(cudaEventCreate(&e), "event");
        } else {
            e = event_pool.back();
            event_pool.pop_back();
        }
        sx::cuda_check(cudaEventRecord(e, stream), "event record");
        step_events.back().push_back(e);
        if (name_of_finished_segment) seg_names.push_back(name_of_finished_segment);
    }
    // Raster pair counting (diagnostic): while on, steps run their kernels directly and the
    // raster kernels add the (pixel, Gaussian) pairs they evaluate to d_pairs [fwd, bwd], zeroed
    // at the start of each such step.
    bool count_pairs = false;
    bool pair_sort = false;  // tile lists from the (tile, Gaussian) pair sort even where binning applies
    bool last_binned = false;
    unsigned long long* d_pairs = nullptr;
    int64_t raster_pairs(int64_t* out) {
        sx::cuda_check(cudaStreamSynchronize(stream), "pairs sync");
        unsigned long long hp[2] = {0, 0};
        if (d_pairs)
            sx::cuda_check(cudaMemcpy(hp, d_pairs, sizeof(hp), cudaMemcpyDeviceToHost), "pairs d2h");
        out[0] = static_cast<int64_t>(hp[0]);
        out[1] = static_cast<int64_t>(hp[1]);
        return 0;
    }
    // The overlapped exchange's timeline while profiling: events on the main and the exchange
    // stream, read back as milliseconds from the step's start (the last profiled step_exchange).
    std::vector<std::pair<const char*, cudaEvent_t>> xline;
    void xmark(const char* name, cudaStream_t s) {
        if (!profiling) return;
        cudaEvent_t e;
        if (event_pool.empty()) {
            sx::cuda_check(cudaEventCreate(&e), "event");
        } else {
            e = event_pool.back();
            event_pool.pop_back();
        }
        sx::cuda_check(cudaEventRecord(e, s), "event record");
        xline.emplace_back(name, e);
    }
    int exchange_timeline(const char** names, float* ms, int cap) {
        sx::cuda_check(cudaStreamSynchronize(stream), "timeline sync");
        if (xstream) sx::cuda_check(cudaStreamSynchronize(xstream), "timeline sync");
        const int n = static_cast<int>(xline.size());
        int k = 0;
        for (; k < n && k < cap; ++k) {
            names[k] = xline[k].first;
            sx::cuda_check(cudaEventElapsedTime(&ms[k], xline[0].second, xline[k].second), "elapsed");
        }
        return k;
    }
    // Average ms per segment over the profiled steps since the last call; clears them.
    int segments(const char** names, float* ms, int cap) {
        sx::cuda_check(cudaStreamSynchronize(stream), "segment sync");
        const int n = static_cast<int>(seg_names.size());
        int k = 0;
        for (; k < n && k < cap; ++k) {
            double tot = 0.0;
            int cnt = 0;
            for (auto& ev : step_events) {
                if (static_cast<int>(ev.size()) <= k + 1) continue;
                float t = 0.f;
                sx::cuda_check(cudaEventElapsedTime(&t, ev[k], ev[k + 1]), "elapsed");
                tot += t;
                ++cnt;
            }
            names[k] = seg_names[k];
            ms[k] = cnt ? static_cast<float>(tot / cnt) : 0.f;
        }
        for (auto& ev : step_events)
            for (cudaEvent_t e : ev) event_pool.push_back(e);
        step_events.clear();
        return k;
    }

    ~SxExecutor() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        if (copy_stream) cudaStreamSynchronize(copy_stream);
        invalidate_graphs();
        close_peers();
        if (mcmc) sx::mcmc_delete(mcmc);
        for (void* q : owned) cudaFree(q);
        for (void* q : isect_bufs) cudaFree(q);
        for (void* q : image_bufs) cudaFree(q);
        if (h) cudaFreeHost(h);
        if (h_eval) cudaFreeHost(h_eval);
        if (step_ring) cudaFreeHost(step_ring);
        for (cudaEvent_t e : ring_ev)
            if (e) cudaEventDestroy(e);
        for (void* q : eval_bufs) cudaFree(q);
        for (auto& xe : xline) cudaEventDestroy(xe.second);
        for (cudaEvent_t e : event_pool) cudaEventDestroy(e);
        for (auto& ev : step_events)
            for (cudaEvent_t e : ev) cudaEventDestroy(e);
        if (gt_ready) cudaEventDestroy(gt_ready);
        if (gt_free) cudaEventDestroy(gt_free);
        for (cudaEvent_t e : xev)
            if (e) cudaEventDestroy(e);
        if (xdone) cudaEventDestroy(xdone);
        if (xstream) cudaStreamSynchronize(xstream);
        if (xstream) cudaStreamDestroy(xstream);
        if (copy_stream) cudaStreamDestroy(copy_stream);
        if (stream) cudaStreamDestroy(stream);
    }

    void init(const SxTrainStepExecutorDesc& desc, int dev) {
        using namespace sx;
        d = desc;
        device = dev;
        if (d.arena_rows < 1) throw_invalid("TrainStepExecutor", "arena_rows must be >= 1");
        if (d.sh_degree < 0 || d.sh_degree > 3)
            throw_invalid("TrainStepExecutor", "sh_degree must be in [0,3]");
        if (!(d.ssim_weight >= 0.0f && d.ssim_weight <= 1.0f))
            throw_invalid("TrainStepExecutor", "ssim_weight must be in [0,1]");
        K = (d.sh_degree + 1) * (d.sh_degree + 1);
        rows = d.arena_rows;
        if (rows * K * 3 > INT32_MAX)
            throw_invalid("TrainStepExecutor", "arena_rows*K*3 exceeds int32");
        dims[5] = (K - 1) * 3;
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        cuda_check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
        padded = (rows + 31) / 32 * 32;
        stage = dalloc<float>(static_cast<size_t>(std::min<int64_t>(rows, kStageRows) * 45), owned);
        for (int g = 0; g < 6; ++g) {
            if (dims[g] == 0) continue;
            const size_t n = static_cast<size_t>(padded * dims[g]);
            p[g] = dalloc<float>(n, owned);
            m1[g] = dalloc<float>(n, owned);
            m2[g] = dalloc<float>(n, owned);
            cuda_check(cudaMemsetAsync(p[g], 0, n * 4, stream), "zero arena");
            cuda_check(cudaMemsetAsync(m1[g], 0, n * 4, stream), "zero arena");
            cuda_check(cudaMemsetAsync(m2[g], 0, n * 4, stream), "zero arena");
        }
        const size_t R = static_cast<size_t>(rows);
        valid = dalloc<uint8_t>(R, owned);
        means2d = dalloc<float>(R * 2, owned);
        conics = dalloc<float>(R * 3, owned);
        opac_raster = dalloc<float>(R, owned);
        comps = dalloc<float>(R, owned);
        act = dalloc<float>(static_cast<size_t>(padded) * 4, owned);
        v_dir = dalloc<float>(static_cast<size_t>(padded) * 3, owned);
        colors = dalloc<float>(R * 3, owned);
        raster_rec = dalloc<float4>(R * 3, owned);
        relu_mask = dalloc<uint8_t>(R, owned);
        tiles = dalloc<int32_t>(R, owned);
        depth_keys = dalloc<uint32_t>(R, owned);
        gauss_ids = dalloc<int32_t>(R, owned);
        order = dalloc<int32_t>(R, owned);
        excl_offsets = dalloc<int32_t>(R, owned);
        entries = dalloc<int32_t>(R, owned);
        ws_scan = dalloc<unsigned char>(scan_gather_workspace(rows), owned);
        ws_depth = dalloc<unsigned char>(onesweep_u32_workspace(rows, 32, 0), owned);
        v_means2d = dalloc<float>(R * 2, owned);
        v_conics = dalloc<float>(R * 3, owned);
        v_colors = dalloc<float>(R * 3, owned);
        v_opac = dalloc<float>(R, owned);
        cuda_check(cudaMemsetAsync(v_means2d, 0, R * 2 * 4, stream), "zero grads");
        cuda_check(cudaMemsetAsync(v_conics, 0, R * 3 * 4, stream), "zero grads");
        cuda_check(cudaMemsetAsync(v_colors, 0, R * 3 * 4, stream), "zero grads");
        cuda_check(cudaMemsetAsync(v_opac, 0, R * 4, stream), "zero grads");
        // the step's scalar results share one struct so the read-back is a single copy
        dev_out = reinterpret_cast<HostOut*>(dalloc<unsigned char>(sizeof(HostOut), owned));
        cuda_check(cudaMemsetAsync(dev_out, 0, sizeof(HostOut), stream), "zero");
        loss = &dev_out->loss;
        overflow = &dev_out->overflow;
        n_isects = &dev_out->n_isects;
        overflow_count = &dev_out->overflow_count;
        status = &dev_out->status;
        n_eff = dalloc<int64_t>(1, owned);
        n_entries = dalloc<int64_t>(2, owned);
        n_eff_entries = n_entries + 1;
        n_chunks = dalloc<int32_t>(1, owned);
        bin_done = dalloc<uint32_t>(1, owned);
        cuda_check(cudaMemsetAsync(bin_done, 0, sizeof(uint32_t), stream), "zero counter");
        st_offsets = dalloc<int32_t>(static_cast<size_t>(kStMaxSupertiles), owned);
        st_chunk0 = dalloc<int32_t>(static_cast<size_t>(kStMaxSupertiles) + 1, owned);
        dev_step = reinterpret_cast<StepParams*>(dalloc<unsigned char>(sizeof(StepParams), owned));
        cuda_check(cudaMallocHost(&step_ring, sizeof(StepParams) * kStepRing), "pinned step ring");
        for (int k = 0; k < kStepRing; ++k)
            cuda_check(cudaEventCreateWithFlags(&ring_ev[k], cudaEventDisableTiming), "event");
        cuda_check(cudaStreamCreateWithFlags(&copy_stream, cudaStreamNonBlocking), "copy stream");
        cuda_check(cudaEventCreateWithFlags(&gt_ready, cudaEventDisableTiming), "event");
        cuda_check(cudaEventCreateWithFlags(&gt_free, cudaEventDisableTiming), "event");
        cuda_check(cudaMallocHost(&h, sizeof(HostOut)), "pinned host");
        std::memset(h, 0, sizeof(HostOut));
        reserve(1 << 16);
        cuda_check(cudaStreamSynchronize(stream), "executor init");
    }

    void reserve(int64_t n) {
        using namespace sx;
        if (n <= cap && tile_keys) return;
        int64_t c = std::max<int64_t>(cap, 1024);
        while (c < n) c += c / 2;
        if (c > kMaxIsects) c = kMaxIsects;
        if (n > c) throw_invalid("TrainStepExecutor", "n_isects must be below 2^30");
        cuda_check(cudaStreamSynchronize(stream), "reserve sync");
        invalidate_graphs();  // the graphs hold the old buffers' addresses
        for (void* q : isect_bufs) cudaFree(q);
        isect_bufs.clear();
        tile_keys = dalloc<uint32_t>(c, isect_bufs);
        gauss_vals = dalloc<int32_t>(c, isect_bufs);
        tile_keys_sorted = dalloc<uint32_t>(c, isect_bufs);
        flatten_ids = dalloc<int32_t>(c, isect_bufs);
        entry = dalloc<uint4>(c, isect_bufs);
        st_sorted = dalloc<int32_t>(c, isect_bufs);
        max_chunks = st_chunk_capacity(c, kStMaxSupertiles);
        chunk_counts = dalloc<uint32_t>(static_cast<size_t>(max_chunks) * 64, isect_bufs);
        // sized for the largest tile-id width the executor accepts (kMaxTileBits) and the
        // whole-key histogram that yields the tile ranges
        ws_tile = dalloc<unsigned char>(onesweep_u32_workspace(c, kMaxTileBits, kHistTileBins),
                                        isect_bufs);
        cap = c;
    }

    void ensure_image(int64_t W, int64_t H, int64_t n_tiles) {
        using namespace sx;
        const int64_t hw = W * H;
        const size_t loss_ws = loss_workspace(H, W);
        if (hw <= img_cap && n_tiles <= tiles_cap && loss_ws <= loss_ws_cap && ws_loss) return;
        cuda_check(cudaStreamSynchronize(stream), "image realloc sync");
        cuda_check(cudaStreamSynchronize(copy_stream), "image realloc sync");
        invalidate_graphs();  // the graphs hold the old buffers' addresses
        for (void* q : image_bufs) cudaFree(q);
        image_bufs.clear();
        img_cap = std::max(hw, img_cap);
        tiles_cap = std::max(n_tiles, tiles_cap);
        loss_ws_cap = std::max(loss_ws, loss_ws_cap);
        const size_t n = static_cast<size_t>(img_cap);
        gt = dalloc<float>(n * 3, image_bufs);
        render = dalloc<float>(n * 3, image_bufs);
        alphas = dalloc<float>(n, image_bufs);
        last_ids = dalloc<int32_t>(n, image_bufs);
        v_render = dalloc<float>(n * 3, image_bufs);
        v_ralpha_zero = dalloc<float>(n, image_bufs);
        cuda_check(cudaMemsetAsync(v_ralpha_zero, 0, n * 4, stream), "zero");
        cmu = dalloc<float>(n * 3, image_bufs);
        csg = dalloc<float>(n * 3, image_bufs);
        ccr = dalloc<float>(n * 3, image_bufs);
        ws_loss = dalloc<unsigned char>(loss_ws_cap, image_bufs);
        tile_offsets = dalloc<int32_t>(static_cast<size_t>(tiles_cap) + 1, image_bufs);
        tile_counts = dalloc<int32_t>(static_cast<size_t>(tiles_cap) + 1, image_bufs);
    }

    void sync(const SxResidentParamSync& s, bool to_device) {
        using namespace sx;
        if (s.rows < 1 || s.rows > rows)
            throw_invalid("TrainStepExecutor", "sync rows out of [1, arena_rows]");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        for (int g = 0; g < 6; ++g) {
            if (dims[g] == 0) continue;
            if (!s.params[g] || !s.exp_avg[g] || !s.exp_avg_sq[g])
                throw_invalid("TrainStepExecutor", "null sync pointer");
            const int d = static_cast<int>(dims[g]);
            float* dev[3] = {p[g], m1[g], m2[g]};
            float* host[3] = {s.params[g], s.exp_avg[g], s.exp_avg_sq[g]};
            for (int a = 0; a < 3; ++a) {
                for (int64_t r0 = 0; r0 < s.rows; r0 += kStageRows) {
                    const int64_t n = std::min<int64_t>(kStageRows, s.rows - r0);
                    const size_t bytes = static_cast<size_t>(n * d) * sizeof(float);
                    float* h_rows = host[a] + r0 * d;
                    if (to_device) {
                        cuda_check(cudaMemcpyAsync(stage, h_rows, bytes, cudaMemcpyHostToDevice,
                                                   stream),
                                   "upload");
                        launch_rows_to_tiles(stage, dev[a], d, n, r0, stream);
                    } else {
                        launch_tiles_to_rows(dev[a], stage, d, n, r0, stream);
                        cuda_check(cudaMemcpyAsync(h_rows, stage, bytes, cudaMemcpyDeviceToHost,
                                                   stream),
                                   "download");
                    }
                }
            }
        }
        cuda_check(cudaStreamSynchronize(stream), "param sync");
    }

    void validate(const SxResidentStepInputs& in) const {
        using namespace sx;
        const char* w = "TrainStepExecutor::step";
        if (in.count < 1 || in.count > rows) throw_invalid(w, "count out of [1, arena_rows]");
        if (in.width < 1 || in.height < 1) throw_invalid(w, "width/height must be positive");
        if (!in.viewmat || !in.K) throw_invalid(w, "null viewmat/K");
        if (!in.forward_only && !in.gt_rgb) throw_invalid(w, "null gt_rgb");
        const bool use_ssim = d.ssim_weight > 0.0f && !in.forward_only;
        if (use_ssim && (in.height < kSsimWin || in.width < kSsimWin))
            throw_invalid(w, "ssim requires H, W >= 11");
        if (in.degrees_to_use > static_cast<uint32_t>(d.sh_degree))
            throw_invalid(w, "degrees_to_use exceeds the executor's sh_degree");
    }

    // Enqueue one step; returns nothing, results stay on the device.
    void ensure_grads() {
        using namespace sx;
        if (gvis) return;
        for (int g = 0; g < 6; ++g) {
            if (dims[g] == 0) continue;
            const size_t n = static_cast<size_t>(padded * dims[g]);
            gacc[g] = dalloc<float>(n, owned);
            cuda_check(cudaMemsetAsync(gacc[g], 0, n * 4, stream), "zero grads");
        }
        gvis = dalloc<float>(static_cast<size_t>(padded), owned);
        cuda_check(cudaMemsetAsync(gvis, 0, static_cast<size_t>(padded) * 4, stream), "zero grads");
    }

    // The accumulators hold the last overlapped exchange's sums; the next accumulating view
    // writes them rather than adding.
    bool grads_stale = false;

    void clear_grads() {
        using namespace sx;
        ensure_grads();
        grads_stale = false;
        for (int g = 0; g < 6; ++g)
            if (gacc[g])
                cuda_check(cudaMemsetAsync(gacc[g], 0, static_cast<size_t>(padded * dims[g]) * 4, stream),
                           "zero grads");
        cuda_check(cudaMemsetAsync(gvis, 0, static_cast<size_t>(padded) * 4, stream), "zero grads");
    }

    sx::ApplyGradsArgs grads_args(const SxApplyGradsInputs& in) {
        using namespace sx;
        const char* w = "TrainStepExecutor::apply_grads";
        if (in.row_begin < 0 || in.row_end < in.row_begin || in.row_end > padded ||
            in.row_begin % 32 || in.row_end % 32)
            throw_invalid(w, "rows must be multiples of 32 within the padded arena");
        if (in.n_views < 1) throw_invalid(w, "n_views must be >= 1");
        if (in.count < 0 || in.count > rows) throw_invalid(w, "count out of [0, arena_rows]");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        ensure_grads();
        ApplyGradsArgs a{};
        for (int g = 0; g < 6; ++g) {
            a.p[g] = p[g];
            a.m[g] = m1[g];
            a.v[g] = m2[g];
            a.gacc[g] = gacc[g];
            a.lr[g] = in.lr[g];
        }
        a.gvis = gvis;
        a.K = K;
        a.row_begin = in.row_begin;
        a.row_end = in.row_end;
        a.count = in.count;
        a.inv_views = 1.0f / static_cast<float>(in.n_views);
        a.b1 = d.b1;
        a.b2 = d.b2;
        a.eps = d.eps;
        a.opacity_reg_w = in.opacity_reg_w;
        a.scale_reg_w = in.scale_reg_w;
        a.inject_noise = in.inject_noise;
        a.noise_seed = in.noise_seed;
        a.noise_offset = in.noise_offset;
        a.noise_scale = in.noise_scale;
        return a;
    }

    void apply_grads(const SxApplyGradsInputs& in) { sx::launch_apply_grads(grads_args(in), stream); }

    // ---- view-parallel exchange over peer memory (CUDA IPC) ---------------------------------
    int peer_world = 0, peer_rank = 0;
    std::vector<void*> peer_opened;
    sx::PeerApplyArgs peer{};
    // cross-GPU barrier flags: slot r of this rank's array holds the last epoch rank r signalled.
    // Zeroed once at allocation; epochs only grow, so a reopened exchange continues from the
    // epoch every rank agrees on (checked in open_peers).
    uint32_t* peer_flags = nullptr;
    uint32_t peer_epoch = 0;
    sx::PeerBarrierArgs barrier{};
    // the overlapped exchange's stream: chunk c's exchange waits on xev[c] (the backward of
    // chunk c on the main stream); the main stream waits on xdone before the closing barrier
    static constexpr int kMaxChunks = 8;
    cudaStream_t xstream = nullptr;
    cudaEvent_t xev[kMaxChunks] = {};
    cudaEvent_t xdone = nullptr;

    void ensure_peer_flags() {
        using namespace sx;
        if (peer_flags) return;
        peer_flags = dalloc<uint32_t>(kMaxPeers, owned);
        cuda_check(cudaMemsetAsync(peer_flags, 0, sizeof(uint32_t) * kMaxPeers, stream), "zero flags");
        cuda_check(cudaStreamSynchronize(stream), "zero flags");
    }

    // IPC handles of [grads 0..5, visibility, params 0..5, barrier flags] (zero bytes for an
    // empty group)
    void peer_handles(SxPeerHandles& out) {
        using namespace sx;
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        ensure_grads();
        ensure_peer_flags();
        std::memset(&out, 0, sizeof(out));
        void* bufs[kPeerBufs] = {};
        for (int g = 0; g < 6; ++g) {
            bufs[g] = gacc[g];
            bufs[7 + g] = p[g];
        }
        bufs[6] = gvis;
        bufs[13] = peer_flags;
        for (int k = 0; k < kPeerBufs; ++k) {
            if (!bufs[k]) continue;
            cudaIpcMemHandle_t h;
            cuda_check(cudaIpcGetMemHandle(&h, bufs[k]), "cudaIpcGetMemHandle");
            static_assert(sizeof(h) == sizeof(out.handle[0]), "IPC handle size");
            std::memcpy(out.handle[k], &h, sizeof(h));
        }
        out.padded_rows = padded;
        out.sh_degree = d.sh_degree;
        out.barrier_epoch = peer_epoch;
    }

    void close_peers() {
        for (void* q : peer_opened) cudaIpcCloseMemHandle(q);
        peer_opened.clear();
        peer_world = 0;
    }

    void open_peers(int rank, int world, const SxPeerHandles* all) {
        using namespace sx;
        if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
            throw_invalid("open_peers", "world must be in [1, 8] and rank in [0, world)");
        if (padded % (32 * world)) throw_invalid("open_peers", "arena rows must split into whole 32-row tiles per rank");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        ensure_grads();
        ensure_peer_flags();
        for (int r = 0; r < world; ++r)
            if (all[r].padded_rows != padded || all[r].sh_degree != d.sh_degree)
                throw_invalid("open_peers", "every rank's executor needs the same arena rows and SH degree");
        for (int r = 0; r < world; ++r)
            if (all[r].barrier_epoch != peer_epoch)
                throw_invalid("open_peers", "every rank's executor must have taken the same number "
                                            "of peer barriers (handles from peer_handles of this session)");
        close_peers();
        peer = PeerApplyArgs{};
        peer.world = world;
        peer.rank = rank;
        barrier = PeerBarrierArgs{};
        barrier.world = world;
        barrier.rank = rank;
        barrier.status = status;
        peer.status = status;
        for (int r = 0; r < world; ++r) {
            for (int k = 0; k < kPeerBufs; ++k) {
                void* ptr = nullptr;
                const bool empty = k < 6 ? dims[k] == 0 : (k > 6 && k < 13 && dims[k - 7] == 0);
                if (empty) continue;
                if (r == rank) {
                    ptr = k < 6     ? static_cast<void*>(gacc[k])
                          : k == 6  ? static_cast<void*>(gvis)
                          : k == 13 ? static_cast<void*>(peer_flags)
                                    : static_cast<void*>(p[k - 7]);
                } else {
                    cudaIpcMemHandle_t h;
                    std::memcpy(&h, all[r].handle[k], sizeof(h));
                    cuda_check(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess),
                               "cudaIpcOpenMemHandle");
                    peer_opened.push_back(ptr);
                }
                if (k < 6) peer.gacc[r][k] = static_cast<const float*>(ptr);
                else if (k == 6) peer.gvis[r] = static_cast<const float*>(ptr);
                else if (k == 13) barrier.flags[r] = static_cast<uint32_t*>(ptr);
                else peer.params[r][k - 7] = static_cast<float*>(ptr);
            }
        }
        peer_world = world;
        peer_rank = rank;
    }

    void exchange_apply(const SxApplyGradsInputs& in) {
        using namespace sx;
        if (peer_world < 1) throw_invalid("exchange_apply", "open_peers first");
        PeerApplyArgs x = peer;
        x.a = grads_args(in);
        launch_exchange_apply(x, stream);
    }

    void peer_barrier(cudaStream_t s) {
        sx::PeerBarrierArgs b = barrier;
        b.epoch = ++peer_epoch;
        sx::launch_peer_barrier(b, s);
    }

    // The last view of a step with the exchange overlapped: forward and backward of `in`
    // accumulate like step_accumulate, but the per-Gaussian backward runs in `chunks` row chunks
    // (chunk c = rows r * S + [c0, c1) of every rank r, S = padded / world). As soon as chunk c
    // is done here, the exchange stream waits for every rank to finish it (device barrier over
    // peer memory) and runs the exchange of this rank's owner rows of chunk c, while the next
    // chunk's backward runs. A closing barrier (every rank's exchange done) precedes zeroing the
    // accumulators. Asynchronous; barrier timeouts surface in the next result read.
    void step_exchange(const SxResidentStepInputs& in, const SxApplyGradsInputs& ap, int chunks) {
        using namespace sx;
        const char* w = "TrainStepExecutor::step_exchange";
        if (peer_world < 1) throw_invalid(w, "open_peers first");
        if (chunks < 1 || chunks > kMaxChunks) throw_invalid(w, "chunks must be in [1, 8]");
        const int64_t S = padded / peer_world;
        if (ap.row_begin != peer_rank * S || ap.row_end != (peer_rank + 1) * S)
            throw_invalid(w, "row_begin / row_end must be this rank's owner rows");
        if (S / 32 < chunks) chunks = static_cast<int>(std::max<int64_t>(1, S / 32));
        const ApplyGradsArgs base = grads_args(ap);  // validates; before anything is enqueued
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        if (!xstream) {
            // the highest priority: the block scheduler dispatches an exchange's blocks ahead of
            // the queued blocks of the next backward chunk, so the two run side by side instead of
            // one after the other
            int lo = 0, hi = 0;
            cuda_check(cudaDeviceGetStreamPriorityRange(&lo, &hi), "stream priorities");
            cuda_check(cudaStreamCreateWithPriority(&xstream, cudaStreamNonBlocking, hi),
                       "exchange stream");
            for (cudaEvent_t& e : xev)
                cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "exchange event");
            cuda_check(cudaEventCreateWithFlags(&xdone, cudaEventDisableTiming), "exchange event");
        }
        split_chunks = chunks;
        split_shard = S;
        if (profiling) {
            for (auto& xe : xline) event_pool.push_back(xe.second);
            xline.clear();
            xmark("start", stream);
        }
        enqueue(in, true, chunks);
        static const char* kBarrierEnd[kMaxChunks] = {
            "barrier0_end", "barrier1_end", "barrier2_end", "barrier3_end",
            "barrier4_end", "barrier5_end", "barrier6_end", "barrier7_end"};
        static const char* kExchangeEnd[kMaxChunks] = {
            "exchange0_end", "exchange1_end", "exchange2_end", "exchange3_end",
            "exchange4_end", "exchange5_end", "exchange6_end", "exchange7_end"};
        for (int c = 0; c < chunks; ++c) {
            const int64_t c0 = chunk_begin(c), c1 = chunk_begin(c + 1);
            cuda_check(cudaStreamWaitEvent(xstream, xev[c], 0), "exchange wait");
            peer_barrier(xstream);
            xmark(kBarrierEnd[c], xstream);
            PeerApplyArgs x = peer;
            x.a = base;
            x.a.row_begin = peer_rank * S + c0;
            x.a.row_end = peer_rank * S + c1;
            launch_exchange_apply(x, xstream);
            xmark(kExchangeEnd[c], xstream);
        }
        cuda_check(cudaEventRecord(xdone, xstream), "exchange done");
        cuda_check(cudaStreamWaitEvent(stream, xdone, 0), "exchange join");
        peer_barrier(stream);
        xmark("closing_barrier_end", stream);
        // No clearing pass: the accumulators keep this step's sums until the next accumulating
        // view, which writes them instead of adding (BwdGaussArgs::accumulate 2). After a barrier
        // that ran out the next result read fails, so nothing continues on the stale sums.
        grads_stale = true;
        xmark("clear_end", stream);
    }
    int split_chunks = 0;
    int64_t split_shard = 0;
    int64_t chunk_begin(int c) const {  // 32-row aligned chunk boundaries of a shard
        return (split_shard / 32) * c / split_chunks * 32;
    }

    sx::ArenaView arena() const {
        sx::ArenaView a{};
        for (int g = 0; g < 6; ++g) {
            a.p[g] = p[g];
            a.m[g] = m1[g];
            a.v[g] = m2[g];
            a.dims[g] = static_cast<int32_t>(dims[g]);
        }
        a.rows = rows;
        a.device = device;
        a.stream = stream;
        return a;
    }
    sx::McmcRefine* refiner() {
        if (!mcmc) mcmc = sx::mcmc_new();
        return mcmc;
    }

    void inject_noise(int64_t count, uint64_t seed, uint64_t offset, float noise_scale) {
        using namespace sx;
        if (count < 0 || count > rows) throw_invalid("inject_noise", "count out of [0, arena_rows]");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        launch_noise_rows(p[0], p[1], p[2], p[3], count, seed, offset, noise_scale, stream);
    }

    void buffers(SxResidentBuffers& o) {
        ensure_grads();
        for (int g = 0; g < 6; ++g) {
            o.params[g] = p[g];
            o.grads[g] = gacc[g];
            o.dims[g] = dims[g];
        }
        o.visibility = gvis;
        o.padded_rows = padded;
    }

    // ---- CUDA graphs of the step -----------------------------------------------------------
    // A step is two graphs, split where the loss waits for the ground truth (copied on the copy
    // stream while the forward runs): `pre` (fwd_gauss .. raster_fwd) and `post` (loss .. bwd).
    // Everything that changes between steps of one shape lives in dev_step, so a graph captured
    // once replays every later step of that shape. A new shape runs directly once and is
    // captured the next time it is seen; profiling always runs directly.
    struct GraphKey {
        uint32_t W = 0, H = 0;
        int32_t N = 0;
        int64_t cap = 0;
        uint32_t degree = 0;
        bool forward_only = false;
        int32_t accumulate = 0;  // BwdGaussArgs::accumulate
        int32_t chunks = 0;  // > 0: the backward split for the overlapped exchange (never a graph)
        bool pair_sort = false;
        bool operator==(const GraphKey& o) const {
            return W == o.W && H == o.H && N == o.N && cap == o.cap && degree == o.degree &&
                   forward_only == o.forward_only && accumulate == o.accumulate &&
                   pair_sort == o.pair_sort;
        }
    };
    bool use_graphs = true;
    bool graphs_ready = false, pending_valid = false;
    GraphKey gkey, pending_key;
    cudaGraphExec_t pre_exec = nullptr, post_exec = nullptr;
    int64_t graph_launches = 0;
    sx::StepParams host_step{};
    sx::StepParams* dev_step = nullptr;
    static constexpr int kStepRing = 16;
    sx::StepParams* step_ring = nullptr;  // pinned
    cudaEvent_t ring_ev[kStepRing] = {};
    int ring_pos = 0;

    void invalidate_graphs() {
        if (pre_exec) cudaGraphExecDestroy(pre_exec);
        if (post_exec) cudaGraphExecDestroy(post_exec);
        pre_exec = post_exec = nullptr;
        graphs_ready = false;
        pending_valid = false;
    }

    cudaGraphExec_t capture(void (SxExecutor::*part)(const GraphKey&), const GraphKey& key) {
        using namespace sx;
        cuda_check(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "begin capture");
        try {
            (this->*part)(key);
        } catch (...) {
            cudaGraph_t g = nullptr;
            cudaStreamEndCapture(stream, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        cudaGraph_t g = nullptr;
        cuda_check(cudaStreamEndCapture(stream, &g), "end capture");
        cudaGraphExec_t e = nullptr;
        const cudaError_t err = cudaGraphInstantiate(&e, g, 0);
        cudaGraphDestroy(g);
        cuda_check(err, "graph instantiate");
        return e;
    }

    void enqueue(const SxResidentStepInputs& in, bool accumulate = false, int chunks = 0) {
        using namespace sx;
        validate(in);
        if (accumulate) {
            if (in.forward_only) throw_invalid("TrainStepExecutor", "accumulate needs a backward");
            ensure_grads();
        }
        // the first accumulating view after an overlapped exchange writes the accumulators
        // (rows it does not see get zeros) instead of adding to the exchanged step's sums
        const int32_t mode = !accumulate ? 0 : (grads_stale ? 2 : 1);
        if (accumulate) grads_stale = false;
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        GraphKey key;
        key.N = static_cast<int32_t>(in.count);
        key.W = static_cast<uint32_t>(in.width);
        key.H = static_cast<uint32_t>(in.height);
        key.degree = in.degrees_to_use;
        key.forward_only = in.forward_only != 0;
        key.accumulate = mode;
        key.chunks = chunks;
        const uint32_t tw = (key.W + kTile - 1) / kTile, th = (key.H + kTile - 1) / kTile;
        const int64_t n_tiles = static_cast<int64_t>(tw) * th;
        const int64_t HW = static_cast<int64_t>(key.W) * key.H;
        if (bits_for_count(n_tiles) > kMaxTileBits)
            throw_invalid("TrainStepExecutor::step", "image has too many tiles");
        ensure_image(key.W, key.H, n_tiles);
        key.cap = cap;
        key.pair_sort = pair_sort;

        // per-step parameters (pageable source: staged before the call returns)
        fill_step_camera(host_step, in.viewmat, in.K, in.width, in.height,
                         ProjParams{d.eps2d, d.near_plane, d.far_plane, d.radius_clip, d.antialiased},
                         tw, th);
        for (int g = 0; g < 6; ++g) host_step.lr[g] = in.lr[g];
        host_step.opacity_reg_w = in.opacity_reg_w;
        host_step.scale_reg_w = in.scale_reg_w;
        host_step.inject_noise = in.inject_noise;
        host_step.noise_seed = in.noise_seed;
        host_step.noise_offset = in.noise_offset;
        host_step.noise_scale = in.noise_scale;
        // staged through a ring of pinned slots: a pageable source could make the copy wait for
        // the stream, and a slot is reused only after its copy has run
        const int slot = ring_pos;
        ring_pos = (ring_pos + 1) % kStepRing;
        cuda_check(cudaEventSynchronize(ring_ev[slot]), "step parameter slot");
        step_ring[slot] = host_step;
        cuda_check(cudaMemcpyAsync(dev_step, &step_ring[slot], sizeof(StepParams),
                                   cudaMemcpyHostToDevice, stream),
                   "step parameters");
        cuda_check(cudaEventRecord(ring_ev[slot], stream), "step parameter slot");
        // the ground truth into the executor's buffer on the copy stream, overlapping the forward
        if (!in.forward_only) {
            cuda_check(cudaStreamWaitEvent(copy_stream, gt_free, 0), "gt wait");
            cuda_check(cudaMemcpyAsync(gt, in.gt_rgb, sizeof(float) * HW * 3,
                                       in.gt_on_device ? cudaMemcpyDeviceToDevice
                                                       : cudaMemcpyHostToDevice,
                                       copy_stream),
                       "gt upload");
            cuda_check(cudaEventRecord(gt_ready, copy_stream), "gt event");
        }

        const int64_t before = launch_count();
        auto wait_gt = [&] {
            if (!in.forward_only) cuda_check(cudaStreamWaitEvent(stream, gt_ready, 0), "gt ready");
        };
        if (count_pairs) {
            if (!d_pairs) d_pairs = dalloc<unsigned long long>(2, owned);
            cuda_check(cudaMemsetAsync(d_pairs, 0, 2 * sizeof(unsigned long long), stream), "zero pairs");
        }
        if (profiling || count_pairs || !use_graphs) {
            seg_begin();
            enqueue_pre(key);
            wait_gt();
            enqueue_post(key);
            last_launches = launch_count() - before;
        } else {
            if (!(graphs_ready && key == gkey)) {
                if (pending_valid && key == pending_key) {
                    GraphKey whole = key;  // the graphs are of the unsplit step
                    whole.chunks = 0;
                    invalidate_graphs();
                    pre_exec = capture(&SxExecutor::enqueue_pre, whole);
                    post_exec = capture(&SxExecutor::enqueue_post, whole);
                    graph_launches = launch_count() - before;
                    gkey = whole;
                    graphs_ready = true;
                } else {  // first step of this shape: direct, captured next time
                    enqueue_pre(key);
                    wait_gt();
                    enqueue_post(key);
                    last_launches = launch_count() - before;
                    pending_key = key;
                    pending_valid = true;
                    finish_step(in);
                    return;
                }
            }
            cuda_check(cudaGraphLaunch(pre_exec, stream), "graph launch");
            wait_gt();
            if (key.chunks > 0) {  // the split backward records events between its chunks
                const int64_t b = launch_count();
                enqueue_post(key);
                last_launches = graph_launches + (launch_count() - b);
            } else {
                cuda_check(cudaGraphLaunch(post_exec, stream), "graph launch");
                last_launches = graph_launches;
            }
        }
        finish_step(in);
    }

    // Whether a step of this image builds its tile lists by supertile binning.
    static bool binned_grid(uint32_t W, uint32_t H, bool pair_sort) {
        using namespace sx;
        const int64_t tw = (W + kTile - 1) / kTile, th = (H + kTile - 1) / kTile;
        const int64_t n_st = ((tw + kStTiles - 1) / kStTiles) * ((th + kStTiles - 1) / kStTiles);
        return !pair_sort && n_st <= kStMaxSupertiles;
    }

    void finish_step(const SxResidentStepInputs& in) {
        using namespace sx;
        last_binned = binned_grid(static_cast<uint32_t>(in.width), static_cast<uint32_t>(in.height),
                                  pair_sort);
        if (!in.forward_only) cuda_check(cudaEventRecord(gt_free, stream), "gt free");
        last_count = in.count;
        last_w = static_cast<uint32_t>(in.width);
        last_h = static_cast<uint32_t>(in.height);
    }

    // fwd_gauss .. raster_fwd
    void enqueue_pre(const GraphKey& key) {
        using namespace sx;
        const int32_t N = key.N;
        const uint32_t W = key.W, H = key.H;
        const uint32_t tw = (W + kTile - 1) / kTile, th = (H + kTile - 1) / kTile;
        const int64_t n_tiles = static_cast<int64_t>(tw) * th;
        cudaStream_t s = stream;
        cuda_check(cudaMemsetAsync(overflow, 0, sizeof(int32_t), s), "reset overflow");

        FwdGaussArgs fa{};
        fa.means = p[0];
        fa.quats = p[1];
        fa.log_scales = p[2];
        fa.opac_logit = p[3];
        fa.sh0 = p[4];
        fa.shN = p[5];
        fa.K = K;
        fa.degree = key.degree;
        fa.count = N;
        fa.step = dev_step;
        fa.antialiased = d.antialiased;
        fa.valid = valid;
        fa.means2d = means2d;
        fa.conics = conics;
        fa.opac_raster = opac_raster;
        fa.comps = comps;
        fa.act = act;
        fa.colors = colors;
        fa.relu_mask = relu_mask;
        fa.tiles = tiles;
        fa.depth_keys = depth_keys;
        fa.gauss_ids = gauss_ids;
        fa.rec = raster_rec;
        const uint32_t stw = (tw + kStTiles - 1) / kStTiles, sth = (th + kStTiles - 1) / kStTiles;
        const int64_t n_st = static_cast<int64_t>(stw) * sth;
        const bool binned = binned_grid(W, H, key.pair_sort);  // else: pairs + tile sort
        fa.entries = binned ? entries : nullptr;
        launch_fwd_gauss(fa, s);
        mark("fwd_gauss");

        onesweep_sort_u32(depth_keys, gauss_ids, nullptr, order, N, nullptr, 32, nullptr, 0, ws_depth,
                          status, s);
        mark("depth_sort");
        if (binned) {
            launch_scan_gather_excl(entries, order, excl_offsets, n_entries, N, ws_scan, s, tiles,
                                    n_isects);
            SX_LAUNCH(bin_capacity_check_kernel, 1, 1, 0, s, n_isects, n_entries, cap, n_eff,
                      n_eff_entries, overflow, overflow_count);
            mark("scan");
            EmitStArgs ea{};
            ea.order = order;
            ea.offsets = excl_offsets;
            ea.entries = entries;
            ea.means2d = means2d;
            ea.conics = conics;
            ea.opac_raster = opac_raster;
            ea.n = N;
            ea.tile_width = tw;
            ea.tile_height = th;
            ea.st_width = stw;
            ea.overflow = overflow;
            ea.st_keys = tile_keys;
            ea.entry_ids = gauss_vals;
            ea.entry = entry;
            launch_emit_supertiles(ea, s);
            mark("emit");

            onesweep_sort_u32(tile_keys, gauss_vals, nullptr, st_sorted, cap, n_eff_entries,
                              std::max<uint32_t>(1, bits_for_count(n_st)), st_offsets, n_st,
                              ws_tile, status, s);
            StBinArgs ba{};
            ba.sorted = st_sorted;
            ba.entry = entry;
            ba.st_offsets = st_offsets;
            ba.n_entries = n_eff_entries;
            ba.overflow = overflow;
            ba.n_st = static_cast<int32_t>(n_st);
            ba.st_width = static_cast<int32_t>(stw);
            ba.tile_width = tw;
            ba.tile_height = th;
            ba.max_chunks = max_chunks;
            ba.st_chunk0 = st_chunk0;
            ba.n_chunks = n_chunks;
            ba.chunk_counts = chunk_counts;
            ba.tile_counts = tile_counts;
            ba.done = bin_done;
            ba.tile_offsets = tile_offsets;
            ba.flatten_ids = flatten_ids;
            launch_bin_supertiles(ba, s);
        } else {
            launch_scan_gather_excl(tiles, order, excl_offsets, n_isects, N, ws_scan, s);
            SX_LAUNCH(capacity_check_kernel, 1, 1, 0, s, n_isects, cap, n_eff, overflow,
                      overflow_count);
            mark("scan");

            EmitArgs ea{};
            ea.order = order;
            ea.offsets = excl_offsets;
            ea.tiles = tiles;
            ea.means2d = means2d;
            ea.conics = conics;
            ea.opac_raster = opac_raster;
            ea.n = N;
            ea.tile_width = tw;
            ea.tile_height = th;
            ea.n_isects = n_isects;
            ea.capacity = cap;
            ea.tile_keys = tile_keys;
            ea.gauss_vals = gauss_vals;
            ea.overflow = overflow;
            launch_emit_depth_ordered(ea, s);
            mark("emit");

            const uint32_t tile_bits = bits_for_count(n_tiles);
            if (n_tiles <= kHistTileBins) {
                // the whole-key histogram's scan is the tile ranges: no sorted keys needed
                onesweep_sort_u32(tile_keys, gauss_vals, nullptr, flatten_ids, cap, n_eff,
                                  tile_bits > 0 ? tile_bits : 1, tile_offsets, n_tiles, ws_tile,
                                  status, s);
            } else {
                onesweep_sort_u32(tile_keys, gauss_vals, tile_keys_sorted, flatten_ids, cap, n_eff,
                                  tile_bits > 0 ? tile_bits : 1, nullptr, 0, ws_tile, status, s);
                launch_tile_offsets_u32(tile_keys_sorted, n_eff, cap, n_tiles, tile_offsets, s);
            }
        }
        mark("tile_sort");

        launch_raster_fwd(raster_args(key), render, alphas, last_ids, s);
        mark("raster_fwd");
    }

    sx::RasterArgs raster_args(const GraphKey& key) const {
        sx::RasterArgs ra{};
        ra.means2d = means2d;
        ra.conics = conics;
        ra.colors = colors;
        ra.opacities = opac_raster;
        ra.offsets = tile_offsets;
        ra.flatten_ids = flatten_ids;
        ra.rec = raster_rec;
        ra.I = 1;
        ra.n_isects = cap;
        ra.n_isects_dev = n_eff;
        ra.width = key.W;
        ra.height = key.H;
        ra.tile_width = (key.W + sx::kTile - 1) / sx::kTile;
        ra.tile_height = (key.H + sx::kTile - 1) / sx::kTile;
        ra.pair_count = count_pairs ? d_pairs : nullptr;
        return ra;
    }

    // loss .. bwd (or the zeroed loss of a forward-only step)
    void enqueue_post(const GraphKey& key) {
        using namespace sx;
        cudaStream_t s = stream;
        if (key.forward_only) {
            cuda_check(cudaMemsetAsync(loss, 0, sizeof(float), s), "zero loss");
            return;
        }
        launch_train_loss(render, gt, key.H, key.W, d.ssim_weight, nullptr, cmu, csg, ccr,
                          v_render, loss, ws_loss, overflow, s);
        mark("loss");
        const RasterArgs ra = raster_args(key);
        launch_raster_bwd(ra, alphas, last_ids, v_render, v_ralpha_zero, v_means2d, v_conics,
                          v_colors, v_opac, nullptr, s);
        mark("raster_bwd");
        if (key.chunks > 0) xmark("raster_bwd_end", s);
        BwdGaussArgs ba{};
        ba.means = p[0];
        ba.quats = p[1];
        ba.log_scales = p[2];
        ba.opac_logit = p[3];
        ba.sh0 = p[4];
        ba.shN = p[5];
        for (int g = 0; g < 6; ++g) {
            ba.m[g] = m1[g];
            ba.v[g] = m2[g];
        }
        ba.K = K;
        ba.degree = key.degree;
        ba.count = key.N;
        ba.step = dev_step;
        ba.width = static_cast<int32_t>(key.W);
        ba.height = static_cast<int32_t>(key.H);
        ba.eps2d = d.eps2d;
        ba.antialiased = d.antialiased;
        ba.valid = valid;
        ba.conics = conics;
        ba.comps = comps;
        ba.relu_mask = relu_mask;
        ba.v_means2d = v_means2d;
        ba.v_conics = v_conics;
        ba.v_colors = v_colors;
        ba.v_opac = v_opac;
        ba.b1 = d.b1;
        ba.b2 = d.b2;
        ba.eps = d.eps;
        ba.skip_flag = overflow;
        ba.act = act;
        ba.v_dir = v_dir;
        ba.accumulate = key.accumulate;
        for (int g = 0; g < 6; ++g) ba.gacc[g] = gacc[g];
        ba.gvis = gvis;
        if (key.chunks == 0) {
            launch_bwd_gauss(ba, s);
        } else {
            ba.map_world = peer_world;
            ba.map_shard = split_shard;
            for (int c = 0; c < key.chunks; ++c) {
                ba.map_c0 = chunk_begin(c);
                ba.map_c1 = chunk_begin(c + 1);
                launch_bwd_gauss(ba, s);
                cuda_check(cudaEventRecord(xev[c], s), "chunk event");
                static const char* kBwdEnd[kMaxChunks] = {
                    "bwd_chunk0_end", "bwd_chunk1_end", "bwd_chunk2_end", "bwd_chunk3_end",
                    "bwd_chunk4_end", "bwd_chunk5_end", "bwd_chunk6_end", "bwd_chunk7_end"};
                xmark(kBwdEnd[c], s);
            }
        }
        mark("bwd_gauss");
    }

    void read_back() {
        using namespace sx;
        cudaStream_t s = stream;
        cuda_check(cudaMemcpyAsync(h, dev_out, sizeof(HostOut), cudaMemcpyDeviceToHost, s), "d2h");
        cuda_check(cudaStreamSynchronize(s), "step");
        if (h->status != 0) {
            cuda_check(cudaMemsetAsync(status, 0, 4, s), "reset status");
            cuda_check(cudaStreamSynchronize(s), "reset status");
            std::string what;
            if (h->status & kStatusSortLookbackTimeout) what += "sort look-back";
            if (h->status & kStatusPeerBarrierTimeout) what += what.empty() ? "peer barrier" : ", peer barrier";
            if (what.empty()) what = "unknown";
            throw RuntimeError("TrainStepExecutor::step: a device-side bounded wait ran out (" + what +
                               "); the step's results are invalid");
        }
    }

    // ---- evaluation, RGBA frames and export ----------------------------------------------------
    std::vector<void*> eval_bufs;
    double* d_eval = nullptr;      // [0] psnr sum, [1] cc sum, [2] ssim, [3] cc ssim, [4..15] moments
    double* d_parts = nullptr;     // per-block partials
    void* ssim_ws = nullptr;
    size_t ssim_ws_cap = 0;
    uint8_t* rgba = nullptr;
    int64_t rgba_cap = 0;
    double* h_eval = nullptr;      // pinned mirror of d_eval[0..3]

    void ensure_eval(int64_t W, int64_t H) {
        using namespace sx;
        const size_t ws = ssim_fwd_workspace(1, std::max<int64_t>(H, 11), std::max<int64_t>(W, 11), 3);
        if (d_eval && ws <= ssim_ws_cap && W * H <= rgba_cap) return;
        cuda_check(cudaStreamSynchronize(stream), "eval realloc sync");
        for (void* q : eval_bufs) cudaFree(q);
        eval_bufs.clear();
        ssim_ws_cap = std::max(ws, ssim_ws_cap);
        rgba_cap = std::max(W * H, rgba_cap);
        d_eval = dalloc<double>(16, eval_bufs);
        d_parts = dalloc<double>(eval_workspace() / sizeof(double), eval_bufs);
        ssim_ws = dalloc<unsigned char>(ssim_ws_cap, eval_bufs);
        rgba = dalloc<uint8_t>(static_cast<size_t>(rgba_cap) * 4, eval_bufs);
        if (!h_eval) cuda_check(cudaMallocHost(&h_eval, sizeof(double) * 4), "pinned eval");
    }

    void render_only(const SxResidentStepInputs& in) {
        SxResidentStepInputs f = in;
        f.forward_only = 1;
        f.want_render = 0;
        SxResidentStepOutputs o{0.f, 0, nullptr};
        step(f, o);
    }

    void eval_view(const SxResidentStepInputs& in, SxEvalResult& out) {
        using namespace sx;
        if (!in.gt_rgb) throw_invalid("eval_view", "null gt_rgb");
        render_only(in);
        const int64_t W = in.width, H = in.height, n = W * H * 3;
        ensure_eval(W, H);
        cuda_check(cudaMemcpyAsync(gt, in.gt_rgb, sizeof(float) * n,
                                   in.gt_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                                   stream),
                   "eval target");
        launch_clamp01(render, n, stream);
        launch_sum_sqdiff(render, gt, n, d_parts, d_eval + 0, stream);
        launch_color_correct(render, gt, W * H, d_parts, d_eval + 4, v_render, stream);
        launch_sum_sqdiff(v_render, gt, n, d_parts, d_eval + 1, stream);
        const bool ssim_ok = H >= kSsimWin && W >= kSsimWin;
        if (ssim_ok) {
            launch_ssim_fwd(render, gt, 1, H, W, 3, false, cmu, nullptr, nullptr, nullptr, d_eval + 2,
                            ssim_ws, stream);
            launch_ssim_fwd(v_render, gt, 1, H, W, 3, false, cmu, nullptr, nullptr, nullptr,
                            d_eval + 3, ssim_ws, stream);
        }
        cuda_check(cudaMemcpyAsync(h_eval, d_eval, sizeof(double) * 4, cudaMemcpyDeviceToHost, stream),
                   "eval d2h");
        cuda_check(cudaStreamSynchronize(stream), "eval");
        // psnr (Trainer.cpp:349-360): float(10 log10(1 / mse)), +inf for identical images
        auto psnr = [&](double sum) {
            const double mse = sum / static_cast<double>(n);
            if (mse <= 0.0) return static_cast<double>(std::numeric_limits<float>::infinity());
            return static_cast<double>(static_cast<float>(10.0 * std::log10(1.0 / mse)));
        };
        out.psnr = psnr(h_eval[0]);
        out.cc_psnr = psnr(h_eval[1]);
        const double nan = std::numeric_limits<double>::quiet_NaN();
        out.ssim = ssim_ok ? h_eval[2] : nan;
        out.cc_ssim = ssim_ok ? h_eval[3] : nan;
    }

    void render_rgba8(const SxResidentStepInputs& in, uint8_t* host_rgba) {
        using namespace sx;
        if (!host_rgba) throw_invalid("render_rgba8", "null out_rgba");
        render_only(in);
        const int64_t npx = static_cast<int64_t>(in.width) * in.height;
        ensure_eval(in.width, in.height);
        launch_rgba8(render, npx, rgba, stream);
        cuda_check(cudaMemcpyAsync(host_rgba, rgba, static_cast<size_t>(npx) * 4,
                                   cudaMemcpyDeviceToHost, stream),
                   "rgba d2h");
        cuda_check(cudaStreamSynchronize(stream), "rgba");
    }

    // Parameters of rows [0, n) in the reference's [rows, d] layout (moments untouched).
    void download_rows(int64_t n, float* const host[6]) {
        using namespace sx;
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        for (int g = 0; g < 6; ++g) {
            if (dims[g] == 0) continue;
            const int d = static_cast<int>(dims[g]);
            for (int64_t r0 = 0; r0 < n; r0 += kStageRows) {
                const int64_t m = std::min<int64_t>(kStageRows, n - r0);
                launch_tiles_to_rows(p[g], stage, d, m, r0, stream);
                cuda_check(cudaMemcpyAsync(host[g] + r0 * d, stage, sizeof(float) * m * d,
                                           cudaMemcpyDeviceToHost, stream),
                           "download");
            }
        }
        cuda_check(cudaStreamSynchronize(stream), "download");
    }

    void export_spz(int64_t n, const char* path, float min_opacity, bool antialiased,
                    SxExportFilterStats& st) {
        using namespace sx;
        if (n < 0 || n > rows) throw_invalid("export_spz", "count out of [0, arena_rows]");
        std::vector<std::vector<float>> h(6);
        float* hp[6] = {};
        for (int g = 0; g < 6; ++g) {
            h[g].resize(static_cast<size_t>(n * dims[g]) + 1);
            hp[g] = h[g].data();
        }
        download_rows(n, hp);
        const SxCloud c{n, d.sh_degree, hp[0], hp[2], hp[1], hp[3], hp[4], hp[5]};
        spz_write(c, path, min_opacity, antialiased, st);
    }

    void export_ply(int64_t n, const char* path, float min_opacity, bool pad, SxExportFilterStats& st) {
        using namespace sx;
        if (n < 0 || n > rows) throw_invalid("export_ply", "count out of [0, arena_rows]");
        std::vector<std::vector<float>> h(6);
        float* hp[6] = {};
        for (int g = 0; g < 6; ++g) {
            h[g].resize(static_cast<size_t>(n * dims[g]) + 1);
            hp[g] = h[g].data();
        }
        download_rows(n, hp);
        SxCloud c{n, d.sh_degree, hp[0], hp[2], hp[1], hp[3], hp[4], hp[5]};
        std::vector<uint8_t> keep(static_cast<size_t>(n) + 1);
        filter_for_export(c, min_opacity, keep.data(), st);
        int64_t j = 0;  // compact the kept rows in place (j <= i)
        for (int64_t i = 0; i < n; ++i) {
            if (!keep[i]) continue;
            if (j != i)
                for (int g = 0; g < 6; ++g)
                    std::memmove(hp[g] + j * dims[g], hp[g] + i * dims[g], sizeof(float) * dims[g]);
            ++j;
        }
        c.count = j;
        ply_write(c, path, pad);
    }

    void step(const SxResidentStepInputs& in, SxResidentStepOutputs& out) {
        using namespace sx;
        for (int attempt = 0; attempt < 8; ++attempt) {
            enqueue(in);
            read_back();
            if (!h->overflow) break;
            // the step was a no-op on the parameters: grow and replay it
            cuda_check(cudaMemsetAsync(overflow_count, 0, 8, stream), "reset overflow count");
            reserve(h->n_isects + h->n_isects / 4);
            if (attempt == 7) throw RuntimeError("TrainStepExecutor::step: capacity growth failed");
        }
        out.loss = in.forward_only ? 0.f : h->loss;
        out.n_isects = h->n_isects;
        if (in.want_render && out.render_colors) {
            const size_t bytes = sizeof(float) * static_cast<size_t>(in.width) * in.height * 3;
            cuda_check(cudaMemcpyAsync(out.render_colors, render, bytes, cudaMemcpyDeviceToHost,
                                       stream),
                       "render d2h");
            cuda_check(cudaStreamSynchronize(stream), "render d2h");
        }
    }

    // ---- read-back of the last step's intermediate buffers (parity checks) ------------------
    void require_step(const char* who) const {
        if (last_count <= 0 || last_w == 0 || last_h == 0)
            sx::throw_invalid(who, "no step has run on this executor");
    }
    void d2h(void* dst, const void* src, size_t bytes) {
        if (!dst || bytes == 0) return;
        sx::cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, stream), "trace d2h");
    }
    void read_gaussians(const SxExecutorGaussianTrace& o, int64_t* count_out) {
        using namespace sx;
        require_step("executor_read_gaussians");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        const size_t n = static_cast<size_t>(last_count);
        d2h(o.valid, valid, n);
        d2h(o.means2d, means2d, n * 2 * sizeof(float));
        d2h(o.conics, conics, n * 3 * sizeof(float));
        d2h(o.opacities, opac_raster, n * sizeof(float));
        d2h(o.colors, colors, n * 3 * sizeof(float));
        d2h(o.tiles_per_gauss, tiles, n * sizeof(int32_t));
        d2h(o.depth_keys, depth_keys, n * sizeof(uint32_t));
        d2h(o.depth_order, order, n * sizeof(int32_t));
        cuda_check(cudaStreamSynchronize(stream), "trace d2h");
        if (count_out) *count_out = last_count;
    }
    void read_isects(int32_t* ids, int64_t capacity, int32_t* offs, int64_t tiles_capacity,
                     int64_t* n_out, int64_t* tiles_out) {
        using namespace sx;
        require_step("executor_read_isects");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        read_back();
        const int64_t n = h->n_isects;
        const int64_t n_tiles = static_cast<int64_t>((last_w + kTile - 1) / kTile) *
                                ((last_h + kTile - 1) / kTile);
        if (n_out) *n_out = n;
        if (tiles_out) *tiles_out = n_tiles;
        if (h->overflow) throw_invalid("executor_read_isects", "the last step overflowed its capacity");
        if ((ids && capacity < n) || (offs && tiles_capacity < n_tiles))
            throw_invalid("executor_read_isects", "output capacity below n_isects / n_tiles");
        d2h(ids, flatten_ids, static_cast<size_t>(n) * sizeof(int32_t));
        d2h(offs, tile_offsets, static_cast<size_t>(n_tiles) * sizeof(int32_t));
        cuda_check(cudaStreamSynchronize(stream), "trace d2h");
    }
    void bin_stats(int64_t* n_entries_out, int64_t* n_st_out) {
        using namespace sx;
        require_step("executor_bin_stats");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        int64_t ne = 0, n_st = 0;
        if (last_binned) {
            cuda_check(cudaMemcpyAsync(&ne, n_entries, sizeof(int64_t), cudaMemcpyDeviceToHost, stream),
                       "bin stats d2h");
            cuda_check(cudaStreamSynchronize(stream), "bin stats sync");
            const int64_t tw = (last_w + kTile - 1) / kTile, th = (last_h + kTile - 1) / kTile;
            n_st = ((tw + kStTiles - 1) / kStTiles) * ((th + kStTiles - 1) / kStTiles);
        }
        if (n_entries_out) *n_entries_out = ne;
        if (n_st_out) *n_st_out = n_st;
    }
    void read_images(float* rc, float* ra, int32_t* li, float* vr) {
        using namespace sx;
        require_step("executor_read_images");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        const size_t hw = static_cast<size_t>(last_w) * last_h;
        d2h(rc, render, hw * 3 * sizeof(float));
        d2h(ra, alphas, hw * sizeof(float));
        d2h(li, last_ids, hw * sizeof(int32_t));
        d2h(vr, v_render, hw * 3 * sizeof(float));
        cuda_check(cudaStreamSynchronize(stream), "trace d2h");
    }

};

namespace sx {
void fill_step_camera(StepParams& sp, const float* vm, const float* Kmat, int width, int height,
                      const ProjParams& p, uint32_t tile_width, uint32_t tile_height) {
    sp.fwd.cam = make_cam(vm, Kmat, width, height);
    // campos = -R^T t, summed in the reference's order (Trainer.cpp:754-757)
    for (int i = 0; i < 3; ++i)
        sp.fwd.campos[i] = -(vm[0 * 4 + i] * vm[0 * 4 + 3] + vm[1 * 4 + i] * vm[1 * 4 + 3] +
                             vm[2 * 4 + i] * vm[2 * 4 + 3]);
    sp.fwd.p = p;
    sp.fwd.g = TileGrid{static_cast<float>(kTile), static_cast<int>(tile_width),
                        static_cast<int>(tile_height)};
    const int rows[9] = {0, 1, 2, 4, 5, 6, 8, 9, 10};
    for (int i = 0; i < 9; ++i) sp.bwd.R[i] = vm[rows[i]];
    sp.bwd.t[0] = vm[3];
    sp.bwd.t[1] = vm[7];
    sp.bwd.t[2] = vm[11];
    for (int i = 0; i < 3; ++i) sp.bwd.campos[i] = sp.fwd.campos[i];
    sp.bwd.fx = Kmat[0];
    sp.bwd.fy = Kmat[4];
    sp.bwd.cx = Kmat[2];
    sp.bwd.cy = Kmat[5];
}

// C-ABI glue lives in capi.cu; these helpers expose the executor to it.
SxExecutor* executor_new(const SxTrainStepExecutorDesc& d, int device) {
    std::unique_ptr<SxExecutor> ex(new SxExecutor());
    ex->init(d, device);
    return ex.release();
}
void executor_delete(SxExecutor* ex) { delete ex; }
void executor_upload(SxExecutor* ex, const SxResidentParamSync& s) { ex->sync(s, true); }
void executor_download(SxExecutor* ex, const SxResidentParamSync& s) { ex->sync(s, false); }
void executor_step(SxExecutor* ex, const SxResidentStepInputs& in, SxResidentStepOutputs& out) {
    ex->step(in, out);
}
void executor_step_async(SxExecutor* ex, const SxResidentStepInputs& in) { ex->enqueue(in); }
void executor_step_accumulate(SxExecutor* ex, const SxResidentStepInputs& in) {
    ex->enqueue(in, true);
}
void executor_step_exchange(SxExecutor* ex, const SxResidentStepInputs& in,
                            const SxApplyGradsInputs& ap, int chunks) {
    ex->step_exchange(in, ap, chunks);
}
void executor_apply_grads(SxExecutor* ex, const SxApplyGradsInputs& in) { ex->apply_grads(in); }
void executor_clear_grads(SxExecutor* ex) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    ex->clear_grads();
}
void executor_buffers(SxExecutor* ex, SxResidentBuffers& out) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    ex->buffers(out);
}
void executor_last_result(SxExecutor* ex, float* loss, int64_t* n_isects, int64_t* overflowed) {
    ex->read_back();
    if (loss) *loss = ex->h->loss;
    if (n_isects) *n_isects = ex->h->n_isects;
    if (overflowed) *overflowed = ex->h->overflow_count;
    cuda_check(cudaMemsetAsync(ex->overflow_count, 0, 8, ex->stream), "reset overflow count");
}
void executor_reserve(SxExecutor* ex, int64_t n) { ex->reserve(n); }
void executor_read_gaussians(SxExecutor* ex, const SxExecutorGaussianTrace& o, int64_t* count) {
    ex->read_gaussians(o, count);
}
void executor_read_isects(SxExecutor* ex, int32_t* ids, int64_t cap, int32_t* offs,
                          int64_t tiles_cap, int64_t* n, int64_t* n_tiles) {
    ex->read_isects(ids, cap, offs, tiles_cap, n, n_tiles);
}
void executor_read_images(SxExecutor* ex, float* rc, float* ra, int32_t* li, float* vr) {
    ex->read_images(rc, ra, li, vr);
}
void executor_peer_handles(SxExecutor* ex, SxPeerHandles& out) { ex->peer_handles(out); }
void executor_save_checkpoint(SxExecutor* ex, const SxCheckpointConfig& cfg, int32_t iter,
                              int64_t count, const char* path, bool fp16) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    if (cfg.sh_degree != ex->d.sh_degree)
        throw_invalid("save_checkpoint", "config sh_degree differs from the executor's");
    const std::string rng = cfg.mcmc_enabled ? mcmc_rng_state(ex->refiner()) : std::string();
    checkpoint_save(ex->arena(), ex->stage, std::min<int64_t>(ex->rows, SxExecutor::kStageRows), cfg,
                    iter, count, rng, path, fp16);
}
void executor_load_checkpoint(SxExecutor* ex, const char* path, const SxCheckpointConfig* current,
                              SxCheckpointHeader& out) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    std::string rng;
    checkpoint_load(ex->arena(), ex->stage, std::min<int64_t>(ex->rows, SxExecutor::kStageRows), path,
                    current, out, rng);
    if (!rng.empty()) mcmc_set_rng_state(ex->refiner(), rng);
}
void executor_eval_view(SxExecutor* ex, const SxResidentStepInputs& in, SxEvalResult& out) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    ex->eval_view(in, out);
}
void executor_render_rgba8(SxExecutor* ex, const SxResidentStepInputs& in, uint8_t* rgba) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    ex->render_rgba8(in, rgba);
}
void executor_export_ply(SxExecutor* ex, int64_t n, const char* path, float min_opacity, bool pad,
                         SxExportFilterStats& st) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    ex->export_ply(n, path, min_opacity, pad, st);
}
void executor_export_spz(SxExecutor* ex, int64_t n, const char* path, float min_opacity,
                         bool antialiased, SxExportFilterStats& st) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    ex->export_spz(n, path, min_opacity, antialiased, st);
}
void executor_open_peers(SxExecutor* ex, int rank, int world, const SxPeerHandles* all) {
    ex->open_peers(rank, world, all);
}
void executor_exchange_apply(SxExecutor* ex, const SxApplyGradsInputs& in) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    ex->exchange_apply(in);
}
void executor_mcmc_seed(SxExecutor* ex, uint64_t seed) { mcmc_seed(ex->refiner(), seed); }
std::string executor_mcmc_rng_state(SxExecutor* ex) { return mcmc_rng_state(ex->refiner()); }
void executor_mcmc_set_rng_state(SxExecutor* ex, const std::string& t) {
    mcmc_set_rng_state(ex->refiner(), t);
}
void executor_mcmc_refine(SxExecutor* ex, int64_t count, int64_t cap_max, float min_opacity,
                          McmcRefineOut& out) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    mcmc_refine(ex->refiner(), ex->arena(), count, cap_max, min_opacity, out);
}
void executor_inject_noise(SxExecutor* ex, int64_t count, uint64_t seed, uint64_t offset,
                           float noise_scale) {
    ex->inject_noise(count, seed, offset, noise_scale);
}
cudaStream_t executor_stream(SxExecutor* ex) { return ex->stream; }
int64_t executor_launches(SxExecutor* ex) { return ex->last_launches; }
void executor_set_profiling(SxExecutor* ex, bool on) { ex->profiling = on; }
void executor_set_pair_counting(SxExecutor* ex, bool on) { ex->count_pairs = on; }
void executor_set_tile_lists(SxExecutor* ex, int mode) { ex->pair_sort = mode == 1; }
void executor_bin_stats(SxExecutor* ex, int64_t* n_entries, int64_t* n_st) {
    ex->bin_stats(n_entries, n_st);
}
void executor_raster_pairs(SxExecutor* ex, int64_t* out) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    ex->raster_pairs(out);
}
int executor_exchange_timeline(SxExecutor* ex, const char** names, float* ms, int cap) {
    cuda_check(cudaSetDevice(ex->device), "cudaSetDevice");
    return ex->exchange_timeline(names, ms, cap);
}
// Segment times (ms) of the last step; returns the number of segments written.
int executor_segments(SxExecutor* ex, const char** names, float* ms, int cap) {
    return ex->segments(names, ms, cap);
}
}  // namespace sx
