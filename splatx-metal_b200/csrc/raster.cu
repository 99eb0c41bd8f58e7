// raster.cu — tile rasterisation forward and backward (16x16 pixel tiles, one CTA of 256 threads
// per tile, one thread per pixel), the contract of Rasterize3DGSFwd.metal / Rasterize3DGSBwd.metal:
//   sigma = 0.5 (a dx^2 + c dy^2) + b dx dy, dx = mean - (pixel + 0.5)
//   alpha = min(0.99, opacity exp(-sigma)); skipped when sigma < 0 or alpha < 1/255
//   front-to-back blending with EXCLUSIVE early stop at next_T <= 1e-4
//   last_ids = absolute index (in the sorted list) of the last contributor, 0 if none
// Gaussian batches are staged in shared memory as 16-byte records (xy+opacity, conic, rgb) so
// each pair evaluation is three broadcast LDS.128.
#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

struct TileCoord {
    uint32_t image_id, tile_id;
    uint32_t px, py;
    bool inside;
};

__device__ __forceinline__ TileCoord tile_coord(const RasterArgs& a) {
    TileCoord c;
    const uint32_t tpi = a.tile_width * a.tile_height;
    c.image_id = blockIdx.x / tpi;
    c.tile_id = blockIdx.x % tpi;
    const uint32_t tx = c.tile_id % a.tile_width, ty = c.tile_id / a.tile_width;
    c.px = tx * kTile + (threadIdx.x & (kTile - 1));
    c.py = ty * kTile + (threadIdx.x >> 4);
    c.inside = c.px < a.width && c.py < a.height;
    return c;
}

__device__ __forceinline__ void tile_range(const RasterArgs& a, const TileCoord& c, int& start,
                                           int& end) {
    const uint32_t tpi = a.tile_width * a.tile_height;
    const int32_t* off = a.offsets + static_cast<int64_t>(c.image_id) * tpi;
    const int64_t n = a.n_isects_dev ? *a.n_isects_dev : a.n_isects;
    start = off[c.tile_id];
    end = (c.image_id == a.I - 1 && c.tile_id == tpi - 1) ? static_cast<int>(n) : off[c.tile_id + 1];
}

template <bool HAS_BG, bool HAS_MASK>
__global__ void __launch_bounds__(kTileThreads)
raster_fwd_kernel(RasterArgs a, float* __restrict__ rc, float* __restrict__ ra,
                  int32_t* __restrict__ li) {
    const TileCoord c = tile_coord(a);
    const uint32_t tpi = a.tile_width * a.tile_height;
    const int64_t img_px = static_cast<int64_t>(a.width) * a.height;
    const int64_t pix = static_cast<int64_t>(c.image_id) * img_px +
                        static_cast<int64_t>(c.py) * a.width + c.px;
    const float* bg = HAS_BG ? a.backgrounds + c.image_id * 3 : nullptr;
    if (HAS_MASK && a.masks[static_cast<int64_t>(c.image_id) * tpi + c.tile_id] == 0) {
        if (c.inside) {
            for (int k = 0; k < 3; ++k) rc[pix * 3 + k] = HAS_BG ? bg[k] : 0.f;
            ra[pix] = 0.f;
            li[pix] = 0;
        }
        return;
    }
    int start, end;
    tile_range(a, c, start, end);

    __shared__ float4 s_xyo[kTileThreads];
    __shared__ float4 s_con[kTileThreads];
    __shared__ float4 s_rgb[kTileThreads];

    const float px = static_cast<float>(c.px) + 0.5f, py = static_cast<float>(c.py) + 0.5f;
    float T = 1.0f;
    int cur = 0;
    float o0 = 0.f, o1 = 0.f, o2 = 0.f;
    bool done = !c.inside;
    for (int b0 = start; b0 < end; b0 += kTileThreads) {
        const int idx = b0 + static_cast<int>(threadIdx.x);
        if (idx < end) {
            const int g = a.flatten_ids[idx];
            s_xyo[threadIdx.x] = make_float4(a.means2d[2 * g], a.means2d[2 * g + 1], a.opacities[g], 0.f);
            s_con[threadIdx.x] = make_float4(a.conics[3 * g], a.conics[3 * g + 1], a.conics[3 * g + 2], 0.f);
            s_rgb[threadIdx.x] = make_float4(a.colors[3 * g], a.colors[3 * g + 1], a.colors[3 * g + 2], 0.f);
        }
        __syncthreads();
        const int cnt = min(kTileThreads, end - b0);
        if (!done) {
            for (int t = 0; t < cnt; ++t) {
                const float4 xyo = s_xyo[t];
                const float4 cn = s_con[t];
                const float dx = xyo.x - px, dy = xyo.y - py;
                const float sigma = 0.5f * (cn.x * dx * dx + cn.z * dy * dy) + cn.y * dx * dy;
                if (sigma < 0.f) continue;
                const float alpha = smin(kMaxAlpha, xyo.z * expf(-sigma));
                if (alpha < kAlphaThreshold) continue;
                const float next_T = T * (1.0f - alpha);
                if (next_T <= kTransmittanceThreshold) {
                    done = true;
                    break;
                }
                const float w = alpha * T;
                const float4 rgb = s_rgb[t];
                o0 = fmaf(rgb.x, w, o0);
                o1 = fmaf(rgb.y, w, o1);
                o2 = fmaf(rgb.z, w, o2);
                cur = b0 + t;
                T = next_T;
            }
        }
        if (__syncthreads_and(done)) break;
    }
    if (c.inside) {
        ra[pix] = 1.0f - T;
        if (HAS_BG) {
            rc[pix * 3 + 0] = fmaf(T, bg[0], o0);
            rc[pix * 3 + 1] = fmaf(T, bg[1], o1);
            rc[pix * 3 + 2] = fmaf(T, bg[2], o2);
        } else {
            rc[pix * 3 + 0] = o0;
            rc[pix * 3 + 1] = o1;
            rc[pix * 3 + 2] = o2;
        }
        li[pix] = cur;
    }
}

// Backward: back-to-front replay from T_final, per-pixel gradients, a warp transpose-reduction
// of the per-Gaussian gradient vector and one atomic per value per warp (spread over lanes).
template <bool HAS_BG, bool HAS_MASK, bool ABSGRAD>
__global__ void __launch_bounds__(kTileThreads)
raster_bwd_kernel(RasterArgs a, const float* __restrict__ render_alphas,
                  const int32_t* __restrict__ last_ids, const float* __restrict__ v_rc,
                  const float* __restrict__ v_ra, float* __restrict__ v_m2,
                  float* __restrict__ v_con, float* __restrict__ v_col,
                  float* __restrict__ v_op, float* __restrict__ v_m2abs) {
    constexpr int NV = ABSGRAD ? 11 : 9;
    const TileCoord c = tile_coord(a);
    const uint32_t tpi = a.tile_width * a.tile_height;
    if (HAS_MASK && a.masks[static_cast<int64_t>(c.image_id) * tpi + c.tile_id] == 0) return;
    const int64_t img_px = static_cast<int64_t>(a.width) * a.height;
    const int64_t local = c.inside ? static_cast<int64_t>(c.py) * a.width + c.px : img_px - 1;
    const int64_t pix = static_cast<int64_t>(c.image_id) * img_px + local;
    int start, end;
    tile_range(a, c, start, end);

    __shared__ int s_id[kTileThreads];
    __shared__ float4 s_xyo[kTileThreads];
    __shared__ float4 s_con[kTileThreads];
    __shared__ float4 s_rgb[kTileThreads];

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

    const float px = static_cast<float>(c.px) + 0.5f, py = static_cast<float>(c.py) + 0.5f;
    const float T_final = 1.0f - render_alphas[pix];
    float T = T_final;
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f;
    const int bin_final = c.inside ? last_ids[pix] : 0;
    const float vc0 = v_rc[pix * 3], vc1 = v_rc[pix * 3 + 1], vc2 = v_rc[pix * 3 + 2];
    const float va = v_ra[pix];
    float bg_dot = 0.f;
    if (HAS_BG) {
        const float* bg = a.backgrounds + c.image_id * 3;
        bg_dot = bg[0] * vc0 + bg[1] * vc1 + bg[2] * vc2;
    }
    const int warp_bin_final = __reduce_max_sync(kFullMask, bin_final);

    for (int batch_end = end - 1; batch_end >= start; batch_end -= kTileThreads) {
        __syncthreads();
        const int idx = batch_end - static_cast<int>(threadIdx.x);
        if (idx >= start) {
            const int g = a.flatten_ids[idx];
            s_id[threadIdx.x] = g;
            s_xyo[threadIdx.x] = make_float4(a.means2d[2 * g], a.means2d[2 * g + 1], a.opacities[g], 0.f);
            s_con[threadIdx.x] = make_float4(a.conics[3 * g], a.conics[3 * g + 1], a.conics[3 * g + 2], 0.f);
            s_rgb[threadIdx.x] = make_float4(a.colors[3 * g], a.colors[3 * g + 1], a.colors[3 * g + 2], 0.f);
        }
        __syncthreads();
        const int batch_size = min(kTileThreads, batch_end + 1 - start);
        for (int t = max(0, batch_end - warp_bin_final); t < batch_size; ++t) {
            bool valid = c.inside && (batch_end - t <= bin_final);
            float4 xyo = make_float4(0.f, 0.f, 0.f, 0.f), cn = xyo;
            float dx = 0.f, dy = 0.f, vis = 0.f, alpha = 0.f;
            if (valid) {
                xyo = s_xyo[t];
                cn = s_con[t];
                dx = xyo.x - px;
                dy = xyo.y - py;
                const float sigma = 0.5f * (cn.x * dx * dx + cn.z * dy * dy) + cn.y * dx * dy;
                vis = expf(-sigma);
                alpha = smin(kMaxAlpha, xyo.z * vis);
                if (sigma < 0.f || alpha < kAlphaThreshold) valid = false;
            }
            if (!__any_sync(kFullMask, valid)) continue;
            float v[NV];
#pragma unroll
            for (int q = 0; q < NV; ++q) v[q] = 0.f;
            if (valid) {
                const float4 rgb = s_rgb[t];
                const float rcp = 1.0f / fmaxf(kMinOneMinusAlpha, 1.0f - alpha);
                T *= rcp;
                const float fac = alpha * T;
                v[0] = fac * vc0;
                v[1] = fac * vc1;
                v[2] = fac * vc2;
                float v_alpha = (rgb.x * T - acc0 * rcp) * vc0 + (rgb.y * T - acc1 * rcp) * vc1 +
                                (rgb.z * T - acc2 * rcp) * vc2;
                v_alpha += T_final * rcp * va;
                if (HAS_BG) v_alpha += -T_final * rcp * bg_dot;
                const float opac = xyo.z;
                if (opac * vis <= kMaxAlpha) {
                    const float v_sigma = -opac * vis * v_alpha;
                    v[3] = 0.5f * v_sigma * dx * dx;
                    v[4] = v_sigma * dx * dy;
                    v[5] = 0.5f * v_sigma * dy * dy;
                    v[6] = v_sigma * (cn.x * dx + cn.y * dy);
                    v[7] = v_sigma * (cn.y * dx + cn.z * dy);
                    v[8] = vis * v_alpha;
                    if (ABSGRAD) {
                        v[NV - 2] = fabsf(v[6]);
                        v[NV - 1] = fabsf(v[7]);
                    }
                }
                acc0 = fmaf(rgb.x, fac, acc0);
                acc1 = fmaf(rgb.y, fac, acc1);
                acc2 = fmaf(rgb.z, fac, acc2);
            }
            const float r = warp_transpose_reduce<NV>(v, lane);
            if (slot >= 0) {
                const int g = s_id[t];
                atomicAdd(dst_base + static_cast<int64_t>(g) * dst_stride + dst_comp, r);
            }
        }
    }
}

}  // namespace

void launch_raster_fwd(const RasterArgs& a, float* rc, float* ra, int32_t* li, cudaStream_t s) {
    const int64_t blocks = a.I * static_cast<int64_t>(a.tile_width) * a.tile_height;
    if (blocks == 0) return;
    const bool bg = a.backgrounds != nullptr, mk = a.masks != nullptr;
    if (bg && mk)
        SX_LAUNCH((raster_fwd_kernel<true, true>), static_cast<unsigned>(blocks), kTileThreads, 0, s, a, rc, ra, li);
    else if (bg)
        SX_LAUNCH((raster_fwd_kernel<true, false>), static_cast<unsigned>(blocks), kTileThreads, 0, s, a, rc, ra, li);
    else if (mk)
        SX_LAUNCH((raster_fwd_kernel<false, true>), static_cast<unsigned>(blocks), kTileThreads, 0, s, a, rc, ra, li);
    else
        SX_LAUNCH((raster_fwd_kernel<false, false>), static_cast<unsigned>(blocks), kTileThreads, 0, s, a, rc, ra, li);
}

void launch_raster_bwd(const RasterArgs& a, const float* render_alphas, const int32_t* last_ids,
                       const float* v_rc, const float* v_ra, float* v_m2, float* v_con,
                       float* v_col, float* v_op, float* v_m2abs, cudaStream_t s) {
    const int64_t blocks = a.I * static_cast<int64_t>(a.tile_width) * a.tile_height;
    if (blocks == 0) return;
    const bool bg = a.backgrounds != nullptr, mk = a.masks != nullptr, ab = v_m2abs != nullptr;
#define SX_RB(BG, MK, AB)                                                                        \
    SX_LAUNCH((raster_bwd_kernel<BG, MK, AB>), static_cast<unsigned>(blocks), kTileThreads, 0, s, \
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
