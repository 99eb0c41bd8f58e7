// sx_geometry_exact.cuh — projection forward and tile-intersection geometry whose integer outputs
// (radii, culling, tile sets, keys) must match the CPU contract bit for bit.
//
// Include ONLY from translation units compiled with `-fmad=false`: every expression below is
// evaluated in the CPU reference's order with separately rounded multiplies and adds, IEEE
// division and sqrt, and correctly rounded log. The formulas follow
//   projection: Sources/SplatXCore/CpuKernels.cpp:168-273 + Math.cpp:9-44 (quat/scale covariance)
//   AABB tiles: CpuKernels.cpp:371-393 (IntersectTile.metal:46-60)
//   AccuTile:   CpuKernels.cpp:395-560 (IntersectTile.metal:62-220; SpeedySplat arXiv:2412.00578)
#pragma once

#include "sx_common.cuh"

namespace sx {

// Camera of one view, prepared once per launch by the host (all values are plain copies of the
// viewmat / K entries; the derived FOV limits are recomputed on the device per thread so they are
// rounded exactly like the reference).
struct PinholeCam {
    float R[9];  // row-major rotation of the world->camera transform
    float t[3];
    float fx, fy, cx, cy;
    int width, height;
};

__host__ inline PinholeCam make_cam(const float* viewmat16, const float* K9, int width, int height) {
    PinholeCam c;
    const int rows[9] = {0, 1, 2, 4, 5, 6, 8, 9, 10};
    for (int i = 0; i < 9; ++i) c.R[i] = viewmat16[rows[i]];
    c.t[0] = viewmat16[3];
    c.t[1] = viewmat16[7];
    c.t[2] = viewmat16[11];
    c.fx = K9[0];
    c.fy = K9[4];
    c.cx = K9[2];
    c.cy = K9[5];
    c.width = width;
    c.height = height;
    return c;
}

struct ProjParams {
    float eps2d, near_plane, far_plane, radius_clip;
    int calc_comp;
};

struct ProjResult {
    int rx, ry;  // 0,0 when culled
    float m2x, m2y, depth;
    float conic[3];
    float comp;  // compensation (computed before the det<=0 cull, as the contract does)
};

// 3x3 product with the reference's accumulation order: s = 0; s += a_ik * b_kj for k = 0..2.
__device__ __forceinline__ void mat3_mul_ref(const float* a, const float* b, float* c) {
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < 3; ++k) s = s + a[i * 3 + k] * b[k * 3 + j];
            c[i * 3 + j] = s;
        }
}

// World covariance from an unnormalised quaternion [w,x,y,z] and linear scales:
// R(q/|q|) diag(s) (R diag(s))^T, normalised by division as Math.cpp:9-17 does.
__device__ __forceinline__ void covar_from_quat_scale(const float* q, const float* s, float* C) {
    float w = q[0], x = q[1], y = q[2], z = q[3];
    const float n = sqrtf(w * w + x * x + y * y + z * z);
    if (n > 0.0f) {
        w = w / n;
        x = x / n;
        y = y / n;
        z = z / n;
    }
    float M[9];
    M[0] = 1.f - 2.f * (y * y + z * z);
    M[1] = 2.f * (x * y - w * z);
    M[2] = 2.f * (x * z + w * y);
    M[3] = 2.f * (x * y + w * z);
    M[4] = 1.f - 2.f * (x * x + z * z);
    M[5] = 2.f * (y * z - w * x);
    M[6] = 2.f * (x * z - w * y);
    M[7] = 2.f * (y * z + w * x);
    M[8] = 1.f - 2.f * (x * x + y * y);
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) M[i * 3 + j] = M[i * 3 + j] * s[j];
    float Mt[9];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) Mt[i * 3 + j] = M[j * 3 + i];
    mat3_mul_ref(M, Mt, C);
}

// EWA projection of one Gaussian with the culling cascade near/far -> det<=0 -> opacity ->
// radius_clip -> off-image. `opacity` < 0 means "no opacities given" (fixed 3.33 extend).
// `Cw` is the full 3x3 world covariance.
__device__ __forceinline__ ProjResult project_exact(const float* mw, const float* Cw,
                                                    float opacity, bool has_opacity,
                                                    const PinholeCam& cam, const ProjParams& p) {
    ProjResult r;
    r.rx = 0;
    r.ry = 0;
    r.comp = 0.f;
    const float* R = cam.R;
    const float mx = R[0] * mw[0] + R[1] * mw[1] + R[2] * mw[2] + cam.t[0];
    const float my = R[3] * mw[0] + R[4] * mw[1] + R[5] * mw[2] + cam.t[1];
    const float mz = R[6] * mw[0] + R[7] * mw[1] + R[8] * mw[2] + cam.t[2];
    if (mz < p.near_plane || mz > p.far_plane) return r;

    float RC[9], Rt[9], Cc[9];
    mat3_mul_ref(R, Cw, RC);
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) Rt[i * 3 + j] = R[j * 3 + i];
    mat3_mul_ref(RC, Rt, Cc);

    const float fx = cam.fx, fy = cam.fy, cx = cam.cx, cy = cam.cy;
    const float Wf = static_cast<float>(cam.width), Hf = static_cast<float>(cam.height);
    const float tan_fovx = 0.5f * Wf / fx;
    const float tan_fovy = 0.5f * Hf / fy;
    const float lim_x_pos = (Wf - cx) / fx + 0.3f * tan_fovx;
    const float lim_x_neg = cx / fx + 0.3f * tan_fovx;
    const float lim_y_pos = (Hf - cy) / fy + 0.3f * tan_fovy;
    const float lim_y_neg = cy / fy + 0.3f * tan_fovy;

    const float rz = 1.0f / mz, rz2 = rz * rz;
    const float txc = mz * smin(lim_x_pos, smax(-lim_x_neg, mx * rz));
    const float tyc = mz * smin(lim_y_pos, smax(-lim_y_neg, my * rz));
    const float J00 = fx * rz, J02 = -fx * txc * rz2;
    const float J11 = fy * rz, J12 = -fy * tyc * rz2;
    const float JC0[3] = {J00 * Cc[0] + J02 * Cc[6], J00 * Cc[1] + J02 * Cc[7],
                          J00 * Cc[2] + J02 * Cc[8]};
    const float JC1[3] = {J11 * Cc[3] + J12 * Cc[6], J11 * Cc[4] + J12 * Cc[7],
                          J11 * Cc[5] + J12 * Cc[8]};
    float c00 = JC0[0] * J00 + JC0[2] * J02;
    const float c01 = JC0[1] * J11 + JC0[2] * J12;
    const float c10 = JC1[0] * J00 + JC1[2] * J02;
    float c11 = JC1[1] * J11 + JC1[2] * J12;
    const float m2x = fx * mx * rz + cx;
    const float m2y = fy * my * rz + cy;

    const float det_orig = c00 * c11 - c01 * c10;
    c00 = c00 + p.eps2d;
    c11 = c11 + p.eps2d;
    const float det = c00 * c11 - c01 * c10;
    const float comp = sqrtf(smax(kMinCompensation * kMinCompensation, det_orig / det));
    r.comp = comp;
    if (det <= 0.0f) return r;

    const float rdet = 1.0f / det;
    r.conic[0] = c11 * rdet;
    r.conic[1] = -c10 * rdet;
    r.conic[2] = c00 * rdet;

    float extend = kGaussianExtend;
    if (has_opacity) {
        float op = opacity;
        if (p.calc_comp) op = op * comp;
        if (op < kAlphaThreshold) return r;
        extend = smin(kGaussianExtend, sqrtf(2.0f * log_cr(op / kAlphaThreshold)));
    }
    const float radius_x = ceilf(extend * sqrtf(c00));
    const float radius_y = ceilf(extend * sqrtf(c11));
    if (radius_x <= p.radius_clip && radius_y <= p.radius_clip) return r;
    if (m2x + radius_x <= 0.0f || m2x - radius_x >= Wf || m2y + radius_y <= 0.0f ||
        m2y - radius_y >= Hf)
        return r;
    r.rx = static_cast<int>(radius_x);
    r.ry = static_cast<int>(radius_y);
    r.m2x = m2x;
    r.m2y = m2y;
    r.depth = mz;
    return r;
}

// ---------------------------------------------------------------------------------------------
// Tile intersection. `emit(tile_id)` is called for every intersected tile in the reference's
// emit order; the return value is the tile count. Both paths are shared by the count and emit
// passes so that emit can never write more than count.
// ---------------------------------------------------------------------------------------------

struct TileGrid {
    float tile_size_f;
    int tile_width, tile_height;
};

template <typename Emit>
__device__ __forceinline__ uint32_t aabb_tiles(float mean_x, float mean_y, float radius_x,
                                               float radius_y, const TileGrid& g, Emit&& emit) {
    const float tile_radius_x = radius_x / g.tile_size_f;
    const float tile_radius_y = radius_y / g.tile_size_f;
    const float tile_x = mean_x / g.tile_size_f;
    const float tile_y = mean_y / g.tile_size_f;
    const int min_x = min(max(0, static_cast<int>(floorf(tile_x - tile_radius_x))), g.tile_width);
    const int min_y = min(max(0, static_cast<int>(floorf(tile_y - tile_radius_y))), g.tile_height);
    const int max_x = min(max(0, static_cast<int>(ceilf(tile_x + tile_radius_x))), g.tile_width);
    const int max_y = min(max(0, static_cast<int>(ceilf(tile_y + tile_radius_y))), g.tile_height);
    for (int i = min_y; i < max_y; ++i)
        for (int j = min_x; j < max_x; ++j) emit(static_cast<uint32_t>(i * g.tile_width + j));
    return static_cast<uint32_t>((max_y - min_y) * (max_x - min_x));
}

// Closed-form AABB count (no iteration) for the count pass.
__device__ __forceinline__ uint32_t aabb_count(float mean_x, float mean_y, float radius_x,
                                               float radius_y, const TileGrid& g) {
    return aabb_tiles(mean_x, mean_y, radius_x, radius_y, g, [](uint32_t) {});
}

struct F2 {
    float x, y;
};

// v-range where the line u = coord crosses the level set q = t, in the sweep frame.
__device__ __forceinline__ F2 accutile_line(float A, float B, float C, float disc, float t, F2 p,
                                            bool isY, float coord) {
    const float p_u = isY ? p.y : p.x;
    const float p_v = isY ? p.x : p.y;
    const float coeff = isY ? A : C;
    const float h = coord - p_u;
    const float sq = sqrtf(disc * h * h + t * coeff);
    F2 r;
    r.x = (-B * h - sq) / coeff + p_v;
    r.y = (-B * h + sq) / coeff + p_v;
    return r;
}

// AccuTile: opacity-aware level set + SNUGBOX + strip sweep along the shorter axis.
// The sweep's per-Gaussian constants, in the sweep frame: x is the swept axis (strips u), y the
// other (tile ranges v); `isY` says the frame is the image's transposed one.
struct AccuSweep {
    float A, B, C, disc, t;
    F2 p;            // the mean (image frame)
    F2 bmin, bmax;   // the level set's bounding box (sweep frame)
    float argmin_y, argmax_y;
    int rmin_x, rmax_x, rmin_y, rmax_y;
    float block;     // the tile size
    bool isY;
};

// The sweep's constants of one Gaussian; false when it covers no tile. TS > 0 fixes the tile size
// at compile time (it must equal g.tile_size_f): the divisions by the tile size then fold into
// multiplications by its reciprocal, which for a power of two round identically.
template <int TS = 0>
__device__ __forceinline__ bool accutile_setup(const float* conic, float opacity, float mean_x,
                                               float mean_y, const TileGrid& g, AccuSweep& S) {
    static_assert(TS == 0 || (TS & (TS - 1)) == 0, "a compile-time tile size is a power of two");
    const float A = conic[0], B = conic[1], C = conic[2];
    const float disc = B * B - A * C;
    const float t = fminf(kGaussianExtend * kGaussianExtend,
                          2.0f * log_cr(opacity / kAlphaThreshold));
    if (t <= 0.f) return false;  // approved guard: no tiles when opacity <= alpha threshold

    const float neg_t_over_disc = -t / disc;
    const float x_extent = sqrtf(neg_t_over_disc * C);
    const float y_extent = sqrtf(neg_t_over_disc * A);
    F2 bmin = {mean_x - x_extent, mean_y - y_extent};
    F2 bmax = {mean_x + x_extent, mean_y + y_extent};
    const float Bx_over_C = B * x_extent / C;
    const float By_over_A = B * y_extent / A;
    F2 argmin = {mean_y + Bx_over_C, mean_x + By_over_A};
    F2 argmax = {mean_y - Bx_over_C, mean_x - By_over_A};

    const float BLOCK = TS > 0 ? static_cast<float>(TS) : g.tile_size_f;
    int rmin_x = max(0, min(g.tile_width, static_cast<int>(bmin.x / BLOCK)));
    int rmin_y = max(0, min(g.tile_height, static_cast<int>(bmin.y / BLOCK)));
    int rmax_x = max(0, min(g.tile_width, static_cast<int>(bmax.x / BLOCK + 1.f)));
    int rmax_y = max(0, min(g.tile_height, static_cast<int>(bmax.y / BLOCK + 1.f)));
    const int y_span = rmax_y - rmin_y;
    const int x_span = rmax_x - rmin_x;
    if (y_span * x_span == 0) return false;

    const bool isY = y_span < x_span;  // sweep the shorter axis
    if (isY) {
        int tmp;
        tmp = rmin_x; rmin_x = rmin_y; rmin_y = tmp;
        tmp = rmax_x; rmax_x = rmax_y; rmax_y = tmp;
        float f;
        f = bmin.x; bmin.x = bmin.y; bmin.y = f;
        f = bmax.x; bmax.x = bmax.y; bmax.y = f;
        f = argmin.x; argmin.x = argmin.y; argmin.y = f;
        f = argmax.x; argmax.x = argmax.y; argmax.y = f;
    }
    S.A = A; S.B = B; S.C = C; S.disc = disc; S.t = t;
    S.p = F2{mean_x, mean_y};
    S.bmin = bmin; S.bmax = bmax;
    S.argmin_y = argmin.y; S.argmax_y = argmax.y;
    S.rmin_x = rmin_x; S.rmax_x = rmax_x; S.rmin_y = rmin_y; S.rmax_y = rmax_y;
    S.block = BLOCK;
    S.isY = isY;
    return true;
}

__device__ __forceinline__ F2 accutile_line_at(const AccuSweep& S, float coord) {
    return accutile_line(S.A, S.B, S.C, S.disc, S.t, S.p, S.isY, coord);
}

// Tile range [v0, v1) of the strip between the lines min_line and max_line = min_line + tile,
// whose level-set crossings are line_min and line_max (empty when v1 <= v0).
template <int TS = 0>
__device__ __forceinline__ void accutile_strip(const AccuSweep& S, float min_line, float max_line,
                                               F2 line_min, F2 line_max, int& v0, int& v1) {
    const float BLOCK = TS > 0 ? static_cast<float>(TS) : S.block;
    const float ell_min = (min_line <= S.argmin_y && S.argmin_y < max_line)
                              ? S.bmin.y
                              : fminf(line_min.x, line_max.x);
    const float ell_max = (min_line <= S.argmax_y && S.argmax_y < max_line)
                              ? S.bmax.y
                              : fmaxf(line_min.y, line_max.y);
    v0 = max(S.rmin_y, min(S.rmax_y, static_cast<int>(ell_min / BLOCK)));
    v1 = min(S.rmax_y, max(S.rmin_y, static_cast<int>(ell_max / BLOCK + 1.f)));
}

// accutile_strips reports the sweep strip by strip: strip(u, v0, v1) for every strip u whose
// tile range [v0, v1) is non-empty, in sweep order; the tile of (u, v) is u*tile_width + v when
// the sweep runs along y (isY) and v*tile_width + u otherwise. Returns false when the Gaussian
// covers no tile. Each strip reuses the crossing of its lower line from the strip before; a line
// beyond the level set's extent (max_line > bmax.x) keeps the previous crossing.
// accutile_tiles enumerates the same tiles one by one.
template <int TS = 0, typename Strip>
__device__ __forceinline__ bool accutile_strips(const float* conic, float opacity, float mean_x,
                                                float mean_y, const TileGrid& g, bool& isY_out,
                                                Strip&& strip) {
    AccuSweep S;
    if (!accutile_setup<TS>(conic, opacity, mean_x, mean_y, g, S)) return false;
    isY_out = S.isY;
    const float BLOCK = TS > 0 ? static_cast<float>(TS) : S.block;
    F2 line_max = {S.bmax.y, S.bmin.y};  // neutral pair
    float min_line = S.rmin_x * BLOCK;
    F2 line_min = (S.bmin.x <= min_line) ? accutile_line_at(S, min_line) : line_max;
    for (int u = S.rmin_x; u < S.rmax_x; ++u) {
        const float max_line = min_line + BLOCK;
        if (max_line <= S.bmax.x) line_max = accutile_line_at(S, max_line);
        int v0, v1;
        accutile_strip<TS>(S, min_line, max_line, line_min, line_max, v0, v1);
        if (v1 > v0) strip(u, v0, v1);
        line_min = line_max;
        min_line = max_line;
    }
    return true;
}

// The crossing accutile_strips holds as line_max once it has swept the strips before line b
// (b > rmin_x): the crossing of line b when that line lies within the level set's extent, else
// that of the last line that did (lines advance by whole tiles, so it is line
// floor(bmax.x / tile)), else the neutral pair.
template <int TS>
__device__ __forceinline__ F2 accutile_line_max_before(const AccuSweep& S, int b) {
    static_assert(TS > 0, "exact only for a compile-time power-of-two tile size");
    const float BLOCK = static_cast<float>(TS);
    const float x = b * BLOCK;
    if (x <= S.bmax.x) return accutile_line_at(S, x);
    const int bp = static_cast<int>(floorf(S.bmax.x / BLOCK));
    if (bp >= S.rmin_x + 1) return accutile_line_at(S, bp * BLOCK);
    return F2{S.bmax.y, S.bmin.y};
}

template <int TS = 0, typename Emit>
__device__ __forceinline__ uint32_t accutile_tiles(const float* conic, float opacity,
                                                   float mean_x, float mean_y, const TileGrid& g,
                                                   Emit&& emit) {
    uint32_t count = 0;
    bool isY = false;
    accutile_strips<TS>(conic, opacity, mean_x, mean_y, g, isY, [&](int u, int v0, int v1) {
        for (int v = v0; v < v1; ++v) {
            ++count;
            emit(static_cast<uint32_t>(isY ? u * g.tile_width + v : v * g.tile_width + u));
        }
    });
    return count;
}

// Tile count only (the same sweep, summed per strip).
template <int TS = 0>
__device__ __forceinline__ uint32_t accutile_count(const float* conic, float opacity, float mean_x,
                                                   float mean_y, const TileGrid& g) {
    uint32_t count = 0;
    bool isY = false;
    accutile_strips<TS>(conic, opacity, mean_x, mean_y, g, isY,
                    [&](int, int v0, int v1) { count += static_cast<uint32_t>(v1 - v0); });
    return count;
}

}  // namespace sx
