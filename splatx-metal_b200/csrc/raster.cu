// raster.cu — tile rasterisation forward and backward (16x16 pixel tiles, one CTA per tile, a
// vertical run of kPix pixels per thread), the contract of Rasterize3DGSFwd.metal / Rasterize3DGSBwd.metal:
//   sigma = 0.5 (a dx^2 + c dy^2) + b dx dy, dx = mean - (pixel + 0.5)
//   alpha = min(0.99, opacity exp(-sigma)); skipped when sigma < 0 or alpha < 1/255
//   front-to-back blending with EXCLUSIVE early stop at next_T <= 1e-4
//   last_ids = absolute index (in the sorted list) of the last contributor, 0 if none
// Gaussian batches are staged in shared memory as 16-byte records (xy+opacity, conic, rgb) so
// each pair evaluation is three broadcast LDS.128. The resident executor hands the kernels packed
// 48-byte records (written by its forward), staged with cp.async while the previous batch is
// evaluated; the per-kernel API gathers the same records from its separate arrays.
#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

// A thread owns a vertical run of kPix pixels of one column, so a tile has 256/kPix threads. Every
// Gaussian record read from shared memory, every warp vote and (backward) every
// warp reduction and atomic serves the thread's kPix pixels; dx is common to the run.
constexpr int kPix = 2;
constexpr int kRasterThreads = kTileThreads / kPix;
constexpr int kBatch = 128;  // Gaussians staged in shared memory per batch

struct TileRun {
    uint32_t image_id, tile_id;
    uint32_t px, py0;  // pixels (px, py0 + p), p < kPix
    bool col_in;
    uint32_t height;
    __device__ __forceinline__ bool in(int p) const { return col_in && py0 + p < height; }
};

__device__ __forceinline__ TileRun tile_run(const RasterArgs& a) {
    TileRun c;
    const uint32_t tpi = a.tile_width * a.tile_height;
    c.image_id = blockIdx.x / tpi;
    c.tile_id = blockIdx.x % tpi;
    const uint32_t tx = c.tile_id % a.tile_width, ty = c.tile_id / a.tile_width;
    // warps cover 8x8 pixel blocks (lane -> column lane & 7, run lane >> 3; warp -> one of the
    // tile's 2x2 blocks): compact blocks keep the warp's last-contributor indices close together,
    // so the backward replays fewer Gaussians that only some of its pixels need
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    c.px = tx * kTile + (w & 1) * 8 + (lane & 7);
    c.py0 = ty * kTile + (w >> 1) * 8 + kPix * (lane >> 3);
    c.col_in = c.px < a.width;
    c.height = a.height;
    return c;
}

__device__ __forceinline__ void tile_range(const RasterArgs& a, uint32_t image_id,
                                           uint32_t tile_id, int& start, int& end) {
    const uint32_t tpi = a.tile_width * a.tile_height;
    const int32_t* off = a.offsets + static_cast<int64_t>(image_id) * tpi;
    const int64_t n = a.n_isects_dev ? *a.n_isects_dev : a.n_isects;
    start = off[tile_id];
    end = (image_id == a.I - 1 && tile_id == tpi - 1) ? static_cast<int>(n) : off[tile_id + 1];
}

// sigma = 0.5 (a dx dx + c dy dy) + b dx dy with a fixed rounding sequence (two explicit fused
// multiply-adds), shared by forward and backward so the backward replays the forward's alphas bit
// for bit. adx = (a dx) dx and bdx = b dx are shared by the thread's two pixels (same dx).
__device__ __forceinline__ float conic_sigma(float adx, float bdx, float c, float dy) {
    const float q = __fmaf_rn(__fmul_rn(c, dy), dy, adx);
    return __fmaf_rn(0.5f, q, __fmul_rn(bdx, dy));
}

// A staged batch: the Gaussians' ids and their three 16-byte records (xy + opacity, conic, rgb).
// Batches are double-buffered: batch i+1 is copied in while batch i is evaluated.
static_assert(kBatch == kRasterThreads, "one staged Gaussian per thread and batch");
struct RasterStage {
    int id[kBatch];
    float4 xyo[kBatch];
    float4 con[kBatch];
    float4 rgb[kBatch];
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Stage Gaussian g into slot k: from its packed record (a.rec, three 16-byte cp.async copies that
// land while the thread goes on), or gathered from the separate arrays (the per-kernel API).
template <bool REC>
__device__ __forceinline__ void stage_one(const RasterArgs& a, RasterStage& st, int k, int g) {
    st.id[k] = g;
    if constexpr (REC) {
        const float4* r = a.rec + 3 * static_cast<int64_t>(g);
        cp_async16(&st.xyo[k], r);
        cp_async16(&st.con[k], r + 1);
        cp_async16(&st.rgb[k], r + 2);
    } else {
        st.xyo[k] = make_float4(a.means2d[2 * g], a.means2d[2 * g + 1], a.opacities[g], 0.f);
        st.con[k] = make_float4(a.conics[3 * g], a.conics[3 * g + 1], a.conics[3 * g + 2], 0.f);
        st.rgb[k] = make_float4(a.colors[3 * g], a.colors[3 * g + 1], a.colors[3 * g + 2], 0.f);
    }
}

// One front-to-back blend step of one pixel (exclusive early stop at next_T <= 1e-4).
__device__ __forceinline__ void blend_step(const float4& xyo, const float4& cn, const float4* s_rgb,
                                           int t, int gidx, float adx, float bdx, float fy,
                                           float& T, float (&o)[3], int& cur, bool& done) {
    const float dy = xyo.y - fy;
    const float sigma = conic_sigma(adx, bdx, cn.z, dy);
    if (sigma < 0.f) return;
    const float alpha = smin(kMaxAlpha, xyo.z * expf(-sigma));
    if (alpha < kAlphaThreshold) return;
    const float next_T = T * (1.0f - alpha);
    if (next_T <= kTransmittanceThreshold) {
        done = true;
        return;
    }
    const float w = alpha * T;
    const float4 rgb = s_rgb[t];
    o[0] = fmaf(rgb.x, w, o[0]);
    o[1] = fmaf(rgb.y, w, o[1]);
    o[2] = fmaf(rgb.z, w, o[2]);
    cur = gidx;
    T = next_T;
}

// COUNT (diagnostic, no background / mask): add the pairs evaluated — a pixel not yet stopped
// meeting a staged Gaussian — to a.pair_count[0], one atomic per warp. REC: stage from the packed
// records (a.rec) instead of the separate arrays.
template <bool HAS_BG, bool HAS_MASK, bool COUNT = false, bool REC = false>
__global__ void __launch_bounds__(kRasterThreads)
raster_fwd_kernel(RasterArgs a, float* __restrict__ rc, float* __restrict__ ra,
                  int32_t* __restrict__ li) {
    const TileRun c = tile_run(a);
    const uint32_t tpi = a.tile_width * a.tile_height;
    const int64_t img_px = static_cast<int64_t>(a.width) * a.height;
    const int64_t pix0 = static_cast<int64_t>(c.image_id) * img_px +
                         static_cast<int64_t>(c.py0) * a.width + c.px;
    const float* bg = HAS_BG ? a.backgrounds + c.image_id * 3 : nullptr;
    if (HAS_MASK && a.masks[static_cast<int64_t>(c.image_id) * tpi + c.tile_id] == 0) {
#pragma unroll
        for (int p = 0; p < kPix; ++p) {
            if (!c.in(p)) continue;
            const int64_t pix = pix0 + static_cast<int64_t>(p) * a.width;
            for (int k = 0; k < 3; ++k) rc[pix * 3 + k] = HAS_BG ? bg[k] : 0.f;
            ra[pix] = 0.f;
            li[pix] = 0;
        }
        return;
    }
    int start, end;
    tile_range(a, c.image_id, c.tile_id, start, end);

    __shared__ RasterStage st[2];

    const float fx = static_cast<float>(c.px) + 0.5f;
    float fy[kPix], T[kPix], o[kPix][3];
    int cur[kPix];
    bool done[kPix];
    bool all_done = true;
    uint32_t evals = 0;
#pragma unroll
    for (int p = 0; p < kPix; ++p) {
        fy[p] = static_cast<float>(c.py0 + p) + 0.5f;
        T[p] = 1.0f;
        o[p][0] = o[p][1] = o[p][2] = 0.f;
        cur[p] = 0;
        done[p] = !c.in(p);
        all_done = all_done && done[p];
    }
    // front to back in batches of kBatch; batch i+1 is staged while batch i is evaluated, and the
    // ids of batch i+2 are loaded a batch ahead of their use
    const int k = threadIdx.x;
    const int nb = (end - start + kBatch - 1) / kBatch;
    int next_id = start + k < end ? a.flatten_ids[start + k] : -1;
    if (next_id >= 0) stage_one<REC>(a, st[0], k, next_id);
    cp_async_commit();
    next_id = nb > 1 && start + kBatch + k < end ? a.flatten_ids[start + kBatch + k] : -1;
    for (int i = 0; i < nb; ++i) {
        const int b0 = start + i * kBatch;
        if (i + 1 < nb) {
            if (next_id >= 0) stage_one<REC>(a, st[(i + 1) & 1], k, next_id);
            cp_async_commit();
            const int idx2 = b0 + 2 * kBatch + k;
            next_id = i + 2 < nb && idx2 < end ? a.flatten_ids[idx2] : -1;
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const RasterStage& cur_st = st[i & 1];
        const float4* s_rgb = cur_st.rgb;
        const int cnt = min(kBatch, end - b0);
        for (int t = 0; t < cnt && !all_done; ++t) {
            const float4 cn = cur_st.con[t];
            const float4 xyo = cur_st.xyo[t];
            const float dx = xyo.x - fx;
            const float adx = __fmul_rn(__fmul_rn(cn.x, dx), dx), bdx = __fmul_rn(cn.y, dx);
            all_done = true;
#pragma unroll
            for (int p = 0; p < kPix; ++p) {
                if (COUNT && !done[p]) ++evals;
                if (!done[p]) blend_step(xyo, cn, s_rgb, t, b0 + t, adx, bdx, fy[p], T[p], o[p], cur[p], done[p]);
                all_done = all_done && done[p];
            }
        }
        // the barrier also frees this buffer for the copies the next iteration issues
        if (__syncthreads_and(all_done)) break;
    }
    cp_async_wait<0>();  // no copy may land in shared memory after the block has left
#pragma unroll
    for (int p = 0; p < kPix; ++p) {
        if (!c.in(p)) continue;
        const int64_t pix = pix0 + static_cast<int64_t>(p) * a.width;
        ra[pix] = 1.0f - T[p];
        if (HAS_BG) {
            rc[pix * 3 + 0] = fmaf(T[p], bg[0], o[p][0]);
            rc[pix * 3 + 1] = fmaf(T[p], bg[1], o[p][1]);
            rc[pix * 3 + 2] = fmaf(T[p], bg[2], o[p][2]);
        } else {
            rc[pix * 3 + 0] = o[p][0];
            rc[pix * 3 + 1] = o[p][1];
            rc[pix * 3 + 2] = o[p][2];
        }
        li[pix] = cur[p];
    }
    if constexpr (COUNT) {
        const uint32_t w = __reduce_add_sync(kFullMask, evals);
        if ((threadIdx.x & 31) == 0) atomicAdd(a.pair_count, static_cast<unsigned long long>(w));
    }
}

// Per-pixel backward state of the back-to-front replay.
struct BwdPixel {
    float T, T_final, acc[3], vc[3], va, bg_dot, fy;
    int bin_final;
    bool in;
};

__device__ __forceinline__ void bwd_pixel_init(BwdPixel& q, bool in, int64_t pix, float fy,
                                               const float* render_alphas, const int32_t* last_ids,
                                               const float* v_rc, const float* v_ra,
                                               const float* bg) {
    q.in = in;
    q.fy = fy;
    q.T_final = 1.0f - render_alphas[pix];
    q.T = q.T_final;
    q.acc[0] = q.acc[1] = q.acc[2] = 0.f;
    q.bin_final = in ? last_ids[pix] : 0;
    q.vc[0] = v_rc[pix * 3];
    q.vc[1] = v_rc[pix * 3 + 1];
    q.vc[2] = v_rc[pix * 3 + 2];
    q.va = v_ra[pix];
    q.bg_dot = bg ? bg[0] * q.vc[0] + bg[1] * q.vc[1] + bg[2] * q.vc[2] : 0.f;
}

// Does the Gaussian contribute to this pixel (the forward's alpha test)?
__device__ __forceinline__ bool bwd_hit(const BwdPixel& q, int gidx, const float4& xyo,
                                        const float4& cn, float adx, float bdx, float& dy,
                                        float& vis, float& alpha) {
    if (!q.in || gidx > q.bin_final) return false;
    dy = xyo.y - q.fy;
    const float sigma = conic_sigma(adx, bdx, cn.z, dy);
    vis = expf(-sigma);
    alpha = smin(kMaxAlpha, xyo.z * vis);
    return !(sigma < 0.f || alpha < kAlphaThreshold);
}

// One contributing pixel of the back-to-front replay: colour and opacity gradients into v, and
// the pixel's v_sigma folded into the per-thread sums the conic / mean gradients need
// (ws = v_sigma; S += ws, Sy += ws dy, Syy += ws dy^2 — dx is shared by the thread's pixels).
// absgrad needs per-pixel |v_means2d|, so it takes the per-pixel form instead.
template <bool HAS_BG, int NV>
__device__ __forceinline__ void bwd_accumulate(BwdPixel& q, const float4& xyo, const float4& cn,
                                               const float4& rgb, float dx, float dy, float vis,
                                               float alpha, float (&v)[NV], float& S, float& Sy,
                                               float& Syy) {
    const float rcp = __frcp_rn(fmaxf(kMinOneMinusAlpha, 1.0f - alpha));  // == 1 / x, rounded
    q.T *= rcp;
    const float fac = alpha * q.T;
    v[0] += fac * q.vc[0];
    v[1] += fac * q.vc[1];
    v[2] += fac * q.vc[2];
    float v_alpha = (rgb.x * q.T - q.acc[0] * rcp) * q.vc[0] +
                    (rgb.y * q.T - q.acc[1] * rcp) * q.vc[1] +
                    (rgb.z * q.T - q.acc[2] * rcp) * q.vc[2];
    v_alpha += q.T_final * rcp * q.va;
    if (HAS_BG) v_alpha += -q.T_final * rcp * q.bg_dot;
    const float opac = xyo.z;
    if (opac * vis <= kMaxAlpha) {
        const float ws = -opac * vis * v_alpha;
        if constexpr (NV == 11) {
            v[3] += 0.5f * ws * dx * dx;
            v[4] += ws * dx * dy;
            v[5] += 0.5f * ws * dy * dy;
            const float gx = ws * (cn.x * dx + cn.y * dy);
            const float gy = ws * (cn.y * dx + cn.z * dy);
            v[6] += gx;
            v[7] += gy;
            v[9] += fabsf(gx);
            v[10] += fabsf(gy);
        } else {
            S += ws;
            Sy += ws * dy;
            Syy += ws * dy * dy;
        }
        v[8] += vis * v_alpha;
    }
    q.acc[0] = fmaf(rgb.x, fac, q.acc[0]);
    q.acc[1] = fmaf(rgb.y, fac, q.acc[1]);
    q.acc[2] = fmaf(rgb.z, fac, q.acc[2]);
}

// Backward: back-to-front replay from T_final, per-pixel gradients summed over the thread's
// pixels, a warp transpose-reduction of the per-Gaussian gradient vector and one atomic per value
// per warp (spread over lanes).
// COUNT (diagnostic, no background / mask / absgrad): add the pairs whose alpha the replay
// evaluates — a pixel meeting a Gaussian at or before its last contributor — to
// a.pair_count[1], one atomic per warp.
template <bool HAS_BG, bool HAS_MASK, bool ABSGRAD, bool COUNT = false, bool REC = false>
__global__ void __launch_bounds__(kRasterThreads)
raster_bwd_kernel(RasterArgs a, const float* __restrict__ render_alphas,
                  const int32_t* __restrict__ last_ids, const float* __restrict__ v_rc,
                  const float* __restrict__ v_ra, float* __restrict__ v_m2,
                  float* __restrict__ v_con, float* __restrict__ v_col,
                  float* __restrict__ v_op, float* __restrict__ v_m2abs) {
    constexpr int NV = ABSGRAD ? 11 : 9;
    const TileRun c = tile_run(a);
    const uint32_t tpi = a.tile_width * a.tile_height;
    if (HAS_MASK && a.masks[static_cast<int64_t>(c.image_id) * tpi + c.tile_id] == 0) return;
    const int64_t img_px = static_cast<int64_t>(a.width) * a.height;
    const int64_t ibase = static_cast<int64_t>(c.image_id) * img_px;
    int start, end;
    tile_range(a, c.image_id, c.tile_id, start, end);

    __shared__ RasterStage st[2];

    const int lane = threadIdx.x & 31;
    const int slot = transpose_reduce_slot<NV>(lane);
    float* dst_base = nullptr;
    int dst_stride = 0, dst_comp = 0;
    if (slot >= 0) {
        if (slot < 3) { dst_base = v_col; dst_stride = 3; dst_comp = slot; }
        else if (slot < 6) { dst_base = v_con; dst_stride = 3; dst_comp = slot - 3; }
        else if (slot < 8) { dst_base = v_m2; dst_stride = 2; dst_comp = slot - 6; }
        else if (slot == 8) { dst_base = v_op; dst_stride = 1; dst_comp = 0; }
        else { dst_base = v_m2abs; dst_stride = 2; dst_comp = slot - 9; }
    }

    const float* bg = HAS_BG ? a.backgrounds + c.image_id * 3 : nullptr;
    const float fx = static_cast<float>(c.px) + 0.5f;
    BwdPixel q[kPix];
    int run_bin_final = 0;
#pragma unroll
    for (int p = 0; p < kPix; ++p) {
        // pixels outside the image read a valid (unused) address
        const bool in = c.in(p);
        const int64_t pix = ibase + (in ? static_cast<int64_t>(c.py0 + p) * a.width + c.px : img_px - 1);
        bwd_pixel_init(q[p], in, pix, static_cast<float>(c.py0 + p) + 0.5f, render_alphas, last_ids,
                       v_rc, v_ra, bg);
        run_bin_final = max(run_bin_final, q[p].bin_final);
    }
    const int warp_bin_final = __reduce_max_sync(kFullMask, run_bin_final);
    // The replay starts at the tile's last contributor: the Gaussians behind it (most of a
    // saturated tile's list) are neither staged nor visited.
    __shared__ int s_tile_bin_final;
    if (threadIdx.x == 0) s_tile_bin_final = 0;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) atomicMax(&s_tile_bin_final, warp_bin_final);
    __syncthreads();
    const int first = min(end - 1, s_tile_bin_final);
    uint32_t evals = 0;

    // back to front from `first` in batches of kBatch, double-buffered as in the forward
    const int k = threadIdx.x;
    const int nb = first >= start ? (first - start + kBatch) / kBatch : 0;
    int next_id = nb > 0 && first - k >= start ? a.flatten_ids[first - k] : -1;
    if (next_id >= 0) stage_one<REC>(a, st[0], k, next_id);
    cp_async_commit();
    next_id = nb > 1 && first - kBatch - k >= start ? a.flatten_ids[first - kBatch - k] : -1;
    for (int i = 0; i < nb; ++i) {
        const int batch_end = first - i * kBatch;
        if (i + 1 < nb) {
            if (next_id >= 0) stage_one<REC>(a, st[(i + 1) & 1], k, next_id);
            cp_async_commit();
            const int idx2 = batch_end - 2 * kBatch - k;
            next_id = i + 2 < nb && idx2 >= start ? a.flatten_ids[idx2] : -1;
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const RasterStage& cur_st = st[i & 1];
        const int batch_size = min(kBatch, batch_end + 1 - start);
        for (int t = max(0, batch_end - warp_bin_final); t < batch_size; ++t) {
            const float4 cn = cur_st.con[t];
            const int gidx = batch_end - t;
            const float4 xyo = cur_st.xyo[t];
            const float dx = xyo.x - fx;
            const float adx = __fmul_rn(__fmul_rn(cn.x, dx), dx), bdx = __fmul_rn(cn.y, dx);
            float dy[kPix], vis[kPix], al[kPix];
            bool h[kPix];
            bool any = false;
#pragma unroll
            for (int p = 0; p < kPix; ++p) {
                dy[p] = vis[p] = al[p] = 0.f;
                h[p] = bwd_hit(q[p], gidx, xyo, cn, adx, bdx, dy[p], vis[p], al[p]);
                if (COUNT && q[p].in && gidx <= q[p].bin_final) ++evals;
                any = any || h[p];
            }
            if (!__any_sync(kFullMask, any)) continue;
            float v[NV];
#pragma unroll
            for (int k = 0; k < NV; ++k) v[k] = 0.f;
            const float4 rgb = cur_st.rgb[t];
            float S = 0.f, Sy = 0.f, Syy = 0.f;
#pragma unroll
            for (int p = 0; p < kPix; ++p)
                if (h[p]) bwd_accumulate<HAS_BG, NV>(q[p], xyo, cn, rgb, dx, dy[p], vis[p], al[p], v, S, Sy, Syy);
            if constexpr (NV == 9) {  // conic and mean gradients from the thread's pixel sums
                const float dxS = dx * S;
                v[3] = 0.5f * dx * dxS;
                v[4] = dx * Sy;
                v[5] = 0.5f * Syy;
                v[6] = cn.x * dxS + cn.y * Sy;
                v[7] = cn.y * dxS + cn.z * Sy;
            }
            const float r = warp_transpose_reduce<NV>(v, lane);
            if (slot >= 0) {
                const int g = cur_st.id[t];
                atomicAdd(dst_base + static_cast<int64_t>(g) * dst_stride + dst_comp, r);
            }
        }
        __syncthreads();  // every warp is done with this buffer before the next copies into it
    }
    if constexpr (COUNT) {
        const uint32_t w = __reduce_add_sync(kFullMask, evals);
        if (lane == 0) atomicAdd(a.pair_count + 1, static_cast<unsigned long long>(w));
    }
}

}  // namespace

void launch_raster_fwd(const RasterArgs& a, float* rc, float* ra, int32_t* li, cudaStream_t s) {
    const int64_t blocks = a.I * static_cast<int64_t>(a.tile_width) * a.tile_height;
    if (blocks == 0) return;
    const bool bg = a.backgrounds != nullptr, mk = a.masks != nullptr;
    if (a.rec) {
        if (bg || mk) throw_invalid("raster_fwd", "packed records need no background and no mask");
        if (a.pair_count)
            SX_LAUNCH((raster_fwd_kernel<false, false, true, true>), static_cast<unsigned>(blocks),
                      kRasterThreads, 0, s, a, rc, ra, li);
        else
            SX_LAUNCH((raster_fwd_kernel<false, false, false, true>), static_cast<unsigned>(blocks),
                      kRasterThreads, 0, s, a, rc, ra, li);
        return;
    }
    if (a.pair_count) {
        if (bg || mk) throw_invalid("raster_fwd", "pair counting needs no background and no mask");
        SX_LAUNCH((raster_fwd_kernel<false, false, true>), static_cast<unsigned>(blocks),
                  kRasterThreads, 0, s, a, rc, ra, li);
        return;
    }
    if (bg && mk)
        SX_LAUNCH((raster_fwd_kernel<true, true>), static_cast<unsigned>(blocks), kRasterThreads, 0, s, a, rc, ra, li);
    else if (bg)
        SX_LAUNCH((raster_fwd_kernel<true, false>), static_cast<unsigned>(blocks), kRasterThreads, 0, s, a, rc, ra, li);
    else if (mk)
        SX_LAUNCH((raster_fwd_kernel<false, true>), static_cast<unsigned>(blocks), kRasterThreads, 0, s, a, rc, ra, li);
    else
        SX_LAUNCH((raster_fwd_kernel<false, false>), static_cast<unsigned>(blocks), kRasterThreads, 0, s, a, rc, ra, li);
}

void launch_raster_bwd(const RasterArgs& a, const float* render_alphas, const int32_t* last_ids,
                       const float* v_rc, const float* v_ra, float* v_m2, float* v_con,
                       float* v_col, float* v_op, float* v_m2abs, cudaStream_t s) {
    const int64_t blocks = a.I * static_cast<int64_t>(a.tile_width) * a.tile_height;
    if (blocks == 0) return;
    const bool bg = a.backgrounds != nullptr, mk = a.masks != nullptr, ab = v_m2abs != nullptr;
    if (a.rec) {
        if (bg || mk || ab)
            throw_invalid("raster_bwd", "packed records need no background, mask or absgrad");
        if (a.pair_count)
            SX_LAUNCH((raster_bwd_kernel<false, false, false, true, true>), static_cast<unsigned>(blocks),
                      kRasterThreads, 0, s, a, render_alphas, last_ids, v_rc, v_ra, v_m2, v_con, v_col,
                      v_op, v_m2abs);
        else
            SX_LAUNCH((raster_bwd_kernel<false, false, false, false, true>), static_cast<unsigned>(blocks),
                      kRasterThreads, 0, s, a, render_alphas, last_ids, v_rc, v_ra, v_m2, v_con, v_col,
                      v_op, v_m2abs);
        return;
    }
    if (a.pair_count) {
        if (bg || mk || ab)
            throw_invalid("raster_bwd", "pair counting needs no background, mask or absgrad");
        SX_LAUNCH((raster_bwd_kernel<false, false, false, true>), static_cast<unsigned>(blocks),
                  kRasterThreads, 0, s, a, render_alphas, last_ids, v_rc, v_ra, v_m2, v_con, v_col,
                  v_op, v_m2abs);
        return;
    }
#define SX_RB(BG, MK, AB)                                                                        \
    SX_LAUNCH((raster_bwd_kernel<BG, MK, AB>), static_cast<unsigned>(blocks), kRasterThreads, 0, s, \
              a, render_alphas, last_ids, v_rc, v_ra, v_m2, v_con, v_col, v_op, v_m2abs)
    if (bg) {
        if (mk) { if (ab) SX_RB(true, true, true); else SX_RB(true, true, false); }
        else { if (ab) SX_RB(true, false, true); else SX_RB(true, false, false); }
    } else {
        if (mk) { if (ab) SX_RB(false, true, true); else SX_RB(false, true, false); }
        else { if (ab) SX_RB(false, false, true); else SX_RB(false, false, false); }
    }
#undef SX_RB
}

}  // namespace sx
