// forward.cu — projection, SH forward, tile intersection and offset encoding (per-kernel API) and
// the executor's fused per-Gaussian forward + depth-ordered emit.
//
// Built with -fmad=false: the projection and tile geometry must round exactly like the CPU
// contract (integer radii / tile sets / keys are compared bit for bit). Where a multiply-add is
// wanted (SH colour) it is written as an explicit fmaf.
#include "sx_common.cuh"
#include "sx_geometry_exact.cuh"
#include "sx_internal.h"
#include "sx_sh.cuh"

namespace sx {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ PinholeCam cam_from_device(const float* vm, const float* K, int w, int h) {
    PinholeCam c;
    c.R[0] = vm[0]; c.R[1] = vm[1]; c.R[2] = vm[2];
    c.R[3] = vm[4]; c.R[4] = vm[5]; c.R[5] = vm[6];
    c.R[6] = vm[8]; c.R[7] = vm[9]; c.R[8] = vm[10];
    c.t[0] = vm[3]; c.t[1] = vm[7]; c.t[2] = vm[11];
    c.fx = K[0]; c.fy = K[4]; c.cx = K[2]; c.cy = K[5];
    c.width = w; c.height = h;
    return c;
}

// ---------------------------------------------------------------- projection (API) ----------
__global__ void __launch_bounds__(kThreads)
projection_fwd_kernel(const float* __restrict__ means, const float* __restrict__ covars,
                      const float* __restrict__ quats, const float* __restrict__ scales,
                      const float* __restrict__ opacities, const float* __restrict__ viewmats,
                      const float* __restrict__ Ks, int64_t N, int64_t C, int width, int height,
                      ProjParams p, int32_t* __restrict__ radii, float* __restrict__ means2d,
                      float* __restrict__ depths, float* __restrict__ conics,
                      float* __restrict__ comps) {
    const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (idx >= N * C) return;
    const int64_t cid = idx / N, gid = idx % N;
    const PinholeCam cam = cam_from_device(viewmats + cid * 16, Ks + cid * 9, width, height);
    float Cw[9];
    if (covars) {
        const float* cv = covars + gid * 6;
        Cw[0] = cv[0]; Cw[1] = cv[1]; Cw[2] = cv[2];
        Cw[3] = cv[1]; Cw[4] = cv[3]; Cw[5] = cv[4];
        Cw[6] = cv[2]; Cw[7] = cv[4]; Cw[8] = cv[5];
    } else {
        covar_from_quat_scale(quats + gid * 4, scales + gid * 3, Cw);
    }
    const float op = opacities ? opacities[gid] : 0.f;
    const ProjResult r = project_exact(means + gid * 3, Cw, op, opacities != nullptr, cam, p);
    radii[idx * 2] = r.rx;
    radii[idx * 2 + 1] = r.ry;
    if (r.rx == 0 && r.ry == 0) return;  // culled: other outputs stay unwritten
    means2d[idx * 2] = r.m2x;
    means2d[idx * 2 + 1] = r.m2y;
    depths[idx] = r.depth;
    conics[idx * 3] = r.conic[0];
    conics[idx * 3 + 1] = r.conic[1];
    conics[idx * 3 + 2] = r.conic[2];
    if (p.calc_comp) comps[idx] = r.comp;
}

// ---------------------------------------------------------------- SH forward (API) -----------
__global__ void __launch_bounds__(kThreads)
sh_fwd_kernel(const float* __restrict__ dirs, const float* __restrict__ coeffs,
              const uint8_t* __restrict__ masks, int degree, int64_t BN, int64_t N, int64_t K,
              int D, float* __restrict__ colors) {
    const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (idx >= BN * D) return;
    const int64_t elem = idx / D;
    const int c = static_cast<int>(idx % D);
    if (masks && masks[elem] == 0) return;
    const float* co = coeffs + (elem % N) * K * D;
    float Y[25];
    float x = 0.f, y = 0.f, z = 0.f;
    if (degree >= 1) {
        const float* d = dirs + elem * 3;
        const float inorm = 1.0f / sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
        x = d[0] * inorm;
        y = d[1] * inorm;
        z = d[2] * inorm;
    }
    sh_basis(degree, x, y, z, Y);
    float acc = Y[0] * co[c];
    const int nb = sh_bands(degree);
    for (int k = 1; k < nb; ++k) acc = fmaf(Y[k], co[k * D + c], acc);
    colors[elem * D + c] = acc;
}

// ---------------------------------------------------------------- isect count / emit (API) ---
__global__ void __launch_bounds__(kThreads)
isect_count_kernel(const float* __restrict__ means2d, const int32_t* __restrict__ radii,
                   const float* __restrict__ conics, const float* __restrict__ opacities,
                   int64_t n, TileGrid g, int32_t* __restrict__ tiles) {
    const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (idx >= n) return;
    const float rx = static_cast<float>(radii[idx * 2]);
    const float ry = static_cast<float>(radii[idx * 2 + 1]);
    if (rx <= 0.f || ry <= 0.f) {
        tiles[idx] = 0;
        return;
    }
    const float mx = means2d[idx * 2], my = means2d[idx * 2 + 1];
    uint32_t c;
    if (conics)
        c = accutile_count(conics + idx * 3, opacities[idx], mx, my, g);
    else
        c = aabb_count(mx, my, rx, ry, g);
    tiles[idx] = static_cast<int32_t>(c);
}

__global__ void __launch_bounds__(kThreads)
isect_emit_kernel(const float* __restrict__ means2d, const int32_t* __restrict__ radii,
                  const float* __restrict__ depths, const float* __restrict__ conics,
                  const float* __restrict__ opacities, const int64_t* __restrict__ cum,
                  int64_t n, int64_t N, uint32_t tile_n_bits, TileGrid g,
                  uint64_t* __restrict__ isect_ids, int32_t* __restrict__ flatten_ids) {
    const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (idx >= n) return;
    const float rx = static_cast<float>(radii[idx * 2]);
    const float ry = static_cast<float>(radii[idx * 2 + 1]);
    if (rx <= 0.f || ry <= 0.f) return;
    const uint64_t iid_enc = static_cast<uint64_t>(idx / N) << (32 + tile_n_bits);
    const uint64_t depth_enc = static_cast<uint64_t>(__float_as_uint(depths[idx]));
    int64_t cur = (idx == 0) ? 0 : cum[idx - 1];
    const int32_t fid = static_cast<int32_t>(idx);
    auto emit = [&](uint32_t tile) {
        isect_ids[cur] = iid_enc | (static_cast<uint64_t>(tile) << 32) | depth_enc;
        flatten_ids[cur] = fid;
        ++cur;
    };
    const float mx = means2d[idx * 2], my = means2d[idx * 2 + 1];
    if (conics)
        accutile_tiles(conics + idx * 3, opacities[idx], mx, my, g, emit);
    else
        aabb_tiles(mx, my, rx, ry, g, emit);
}

// ---------------------------------------------------------------- offset encode (API) --------
__global__ void __launch_bounds__(kThreads)
offset_encode_kernel(const uint64_t* __restrict__ ids, int64_t n, int64_t total,
                     uint32_t tile_n_bits, int64_t n_tiles, int32_t* __restrict__ offsets) {
    const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (idx >= n) return;
    const uint64_t mask = (static_cast<uint64_t>(1) << tile_n_bits) - 1;
    auto flat = [&](uint64_t key) {
        const uint64_t hi = key >> 32;
        return static_cast<int64_t>(hi >> tile_n_bits) * n_tiles + static_cast<int64_t>(hi & mask);
    };
    const int64_t cur = flat(ids[idx]);
    if (idx == 0)
        for (int64_t i = 0; i <= cur; ++i) offsets[i] = 0;
    if (idx == n - 1)
        for (int64_t i = cur + 1; i < total; ++i) offsets[i] = static_cast<int32_t>(n);
    if (idx > 0) {
        if ((ids[idx - 1] >> 32) == (ids[idx] >> 32)) return;
        const int64_t prev = flat(ids[idx - 1]);
        for (int64_t i = prev + 1; i <= cur; ++i) offsets[i] = static_cast<int32_t>(idx);
    }
}

// ---------------------------------------------------------------- executor forward -----------

// 4-byte global -> shared copy that holds no register while it is in flight.
__device__ __forceinline__ void cp_async4(float* smem, const float* gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Mask bits of tiles [lo, hi) (0 <= lo < hi <= kStTiles) of strip r inside its supertile:
// one row of the mask when the sweep runs along y (u = tile row), one column otherwise.
__device__ __forceinline__ uint64_t st_strip_bits(int r, int lo, int hi, bool isY) {
    if (isY) {
        const uint32_t run = ((1u << (hi - lo)) - 1u) << lo;
        return static_cast<uint64_t>(run) << (kStTiles * r);
    }
    const uint64_t top = hi == kStTiles ? ~0ull : ((1ull << (kStTiles * hi)) - 1ull);
    const uint64_t rows = top & ~((1ull << (kStTiles * lo)) - 1ull);
    return (rows & 0x0101010101010101ull) << r;
}

// Tiles and supertile entries of one Gaussian from one AccuTile sweep (the count of what
// supertile_entries emits: per block of kStTiles strips, the kStTiles-blocks of v between the
// block's smallest and largest v).
struct StCount {
    uint32_t tiles, entries;
};
__device__ __forceinline__ StCount accutile_supertile_count(const float* conic, float opacity,
                                                            float mean_x, float mean_y,
                                                            const TileGrid& g) {
    StCount c{0u, 0u};
    bool isY = false;
    int ub = -1, vlo = 0, vhi = 0;
    accutile_strips<kTile>(conic, opacity, mean_x, mean_y, g, isY, [&](int u, int v0, int v1) {
        c.tiles += static_cast<uint32_t>(v1 - v0);
        const int b = u / kStTiles;
        if (b != ub) {
            if (ub >= 0) c.entries += static_cast<uint32_t>(vhi / kStTiles - vlo / kStTiles + 1);
            ub = b;
            vlo = v0;
            vhi = v1 - 1;
        } else {
            vlo = min(vlo, v0);
            vhi = max(vhi, v1 - 1);
        }
    });
    if (ub >= 0) c.entries += static_cast<uint32_t>(vhi / kStTiles - vlo / kStTiles + 1);
    return c;
}

constexpr int kFwdThreads = 128;

__global__ void __launch_bounds__(kFwdThreads)
fwd_gauss_kernel(FwdGaussArgs a) {
    // this thread's SH coefficients (sh0 x3, then the rest), copied in while the projection runs
    __shared__ float sh_st[48][kFwdThreads];
    const FwdGaussConst& k = a.step->fwd;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.count) return;
    const int t = threadIdx.x;
    const int nb = sh_bands(static_cast<int>(a.degree));  // bands the colour uses
    {
        const float* c0 = a.sh0 + tile_index(i, 3);
        const float* cn = a.shN + tile_index(i, 3 * (a.K - 1));
#pragma unroll
        for (int c = 0; c < 3; ++c) cp_async4(&sh_st[c][t], c0 + 32 * c);
        for (int j = 0; j < 3 * (nb - 1); ++j) cp_async4(&sh_st[3 + j][t], cn + 32 * j);
    }
    // resident 32-Gaussian tiles: every load below is 128 contiguous bytes per warp
    const float* pm = a.means + tile_index(i, 3);
    const float* pq = a.quats + tile_index(i, 4);
    const float* ps = a.log_scales + tile_index(i, 3);
    const float m[3] = {pm[0], pm[32], pm[64]};
    const float q[4] = {pq[0], pq[32], pq[64], pq[96]};
    const float s[3] = {exp_cr(ps[0]), exp_cr(ps[32]), exp_cr(ps[64])};
    const float opac = sigmoid_cr(a.opac_logit[tile_index(i, 1)]);

    float Cw[9];
    covar_from_quat_scale(q, s, Cw);
    const ProjResult r = project_exact(m, Cw, opac, true, k.cam, k.p);
    const bool valid = (r.rx > 0 && r.ry > 0);
    a.valid[i] = valid ? 1 : 0;
    if (a.antialiased) a.comps[i] = valid ? r.comp : 0.f;
    // AA: culled slots carry comp 0 (zero-initialised in the contract) -> opacity 0.
    const float op_r = a.antialiased ? (valid ? opac * r.comp : 0.f) : opac;
    a.opac_raster[i] = op_r;
    a.gauss_ids[i] = i;
    if (!valid) {
        a.tiles[i] = 0;
        if (a.entries) a.entries[i] = 0;
        a.depth_keys[i] = 0xffffffffu;
        cp_async_wait_all();  // no copy may land after the thread is gone
        return;
    }
    {
        float* pa = a.act + tile_index(i, 4);
        pa[0] = s[0];
        pa[32] = s[1];
        pa[64] = s[2];
        pa[96] = opac;
    }
    a.means2d[i * 2] = r.m2x;
    a.means2d[i * 2 + 1] = r.m2y;
    a.conics[i * 3] = r.conic[0];
    a.conics[i * 3 + 1] = r.conic[1];
    a.conics[i * 3 + 2] = r.conic[2];

    // SH colour (dirs = mean - campos), +0.5 and clamp at 0 with the relu mask
    {
        const float dx = m[0] - k.campos[0], dy = m[1] - k.campos[1], dz = m[2] - k.campos[2];
        float Y[16];
        const int deg = static_cast<int>(a.degree);
        float x = 0.f, y = 0.f, z = 0.f;
        if (deg >= 1) {
            const float inorm = 1.0f / sqrtf(dx * dx + dy * dy + dz * dz);
            x = dx * inorm;
            y = dy * inorm;
            z = dz * inorm;
        }
        sh_basis(deg, x, y, z, Y);
        cp_async_wait_all();  // this thread's coefficients have landed
        float col[3] = {Y[0] * sh_st[0][t], Y[0] * sh_st[1][t], Y[0] * sh_st[2][t]};
#pragma unroll
        for (int b = 1; b < 16; ++b) {  // constant indices keep Y in registers
            if (b >= nb) break;
            col[0] = fmaf(Y[b], sh_st[3 + (b - 1) * 3 + 0][t], col[0]);
            col[1] = fmaf(Y[b], sh_st[3 + (b - 1) * 3 + 1][t], col[1]);
            col[2] = fmaf(Y[b], sh_st[3 + (b - 1) * 3 + 2][t], col[2]);
        }
        uint8_t mask = 0;
        float out[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const float pre = col[c] + 0.5f;
            if (pre > 0.0f) mask |= static_cast<uint8_t>(1u << c);
            out[c] = smax(pre, 0.0f);
            a.colors[i * 3 + c] = out[c];
        }
        a.relu_mask[i] = mask;
        if (a.rec) {  // the raster kernels' packed record of this Gaussian
            float4* rp = a.rec + 3 * static_cast<int64_t>(i);
            rp[0] = make_float4(r.m2x, r.m2y, op_r, 0.f);
            rp[1] = make_float4(r.conic[0], r.conic[1], r.conic[2], 0.f);
            rp[2] = make_float4(out[0], out[1], out[2], 0.f);
        }
    }

    uint32_t nt = 0;
    if (a.entries) {
        const StCount sc = accutile_supertile_count(r.conic, op_r, r.m2x, r.m2y, k.g);
        nt = sc.tiles;
        a.entries[i] = static_cast<int32_t>(sc.entries);
    } else {
        nt = accutile_count<kTile>(r.conic, op_r, r.m2x, r.m2y, k.g);
    }
    a.tiles[i] = static_cast<int32_t>(nt);
    a.depth_keys[i] = nt > 0 ? __float_as_uint(r.depth) : 0xffffffffu;
}

// Emit, warp-cooperative. A warp takes 32 consecutive Gaussians in depth order; their output
// ranges [offsets[j], offsets[j] + tiles) are adjacent, so the warp owns one contiguous run of
// (tile, id) pairs. Each lane records its Gaussian's AccuTile strips (the same sweep that counted
// them) in shared memory; then the warp enumerates all of the run's pairs together, lane t
// writing pair t, t+32, ... — every store instruction covers 128 consecutive bytes. A lane finds
// the owner of pair t by a binary search over the warp's inclusive tile prefix (shuffles) and the
// strip by a binary search over that Gaussian's strip starts. Gaussians with more than
// kEmitMaxStrips strips (very large footprints) emit on their own afterwards.
constexpr int kEmitWarps = 8;
constexpr int kEmitMaxStrips = 16;

struct EmitSmem {
    uint16_t u[32][kEmitMaxStrips];
    uint16_t v0[32][kEmitMaxStrips];
    uint16_t start[32][kEmitMaxStrips];
};

__global__ void __launch_bounds__(kEmitWarps * 32)
emit_depth_ordered_kernel(EmitArgs a, TileGrid g) {
    __shared__ EmitSmem sm_all[kEmitWarps];
    const unsigned full = 0xffffffffu;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j0 = (blockIdx.x * kEmitWarps + warp) * 32;
    if (j0 >= a.n) return;  // warp-uniform
    EmitSmem& sm = sm_all[warp];
    const int j = j0 + lane;
    int32_t gid = 0, nt = 0;
    int64_t base = 0;
    if (j < a.n) {
        gid = a.order[j];
        nt = a.tiles[gid];
        base = a.offsets[j];
        if (nt > 0 && base + nt > a.capacity) {  // the step overflowed: write nothing
            atomicExch(a.overflow, 1);
            nt = 0;
        }
    }
    // strips of this lane's Gaussian
    bool isY = false, spill = false;
    int ns = 0;
    if (nt > 0) {
        int run = 0;
        accutile_strips<kTile>(a.conics + static_cast<int64_t>(gid) * 3, a.opac_raster[gid],
                        a.means2d[gid * 2], a.means2d[gid * 2 + 1], g, isY,
                        [&](int u, int v0, int v1) {
                            if (ns < kEmitMaxStrips && run <= 0xffff) {
                                sm.u[lane][ns] = static_cast<uint16_t>(u);
                                sm.v0[lane][ns] = static_cast<uint16_t>(v0);
                                sm.start[lane][ns] = static_cast<uint16_t>(run);
                            } else {
                                spill = true;
                            }
                            ++ns;
                            run += v1 - v0;
                        });
    }
    // cooperative emission of every non-spilled lane's tiles
    const int coop = spill ? 0 : nt;
    int incl = coop;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(full, incl, o);
        if (lane >= o) incl += y;
    }
    const int excl = incl - coop;
    const int total = __shfl_sync(full, incl, 31);
    __syncwarp();
    uint32_t* tk = a.tile_keys;
    int32_t* gv = a.gauss_vals;
    for (int t0 = 0; t0 < total; t0 += 32) {
        const int t = t0 + lane;
        // owner lane k: the number of lanes whose inclusive prefix is <= t
        int k = 0;
#pragma unroll
        for (int step = 16; step > 0; step >>= 1) {
            const int c = k + step;
            const int ic = __shfl_sync(full, incl, c - 1);
            if (ic <= t) k = c;
        }
        k = min(k, 31);
        const int ek = __shfl_sync(full, excl, k);
        const int nsk = __shfl_sync(full, ns, k);
        const bool isYk = __shfl_sync(full, static_cast<int>(isY), k) != 0;
        const int gk = __shfl_sync(full, gid, k);
        const int64_t bk = __shfl_sync(full, base, k);
        if (t < total) {
            const int q = t - ek;
            int s = 0;  // last strip whose start <= q
            int hi = min(nsk, kEmitMaxStrips) - 1;
            while (s < hi) {
                const int mid = (s + hi + 1) >> 1;
                if (sm.start[k][mid] <= q) s = mid; else hi = mid - 1;
            }
            const int u = sm.u[k][s];
            const int v = sm.v0[k][s] + (q - sm.start[k][s]);
            tk[bk + q] = static_cast<uint32_t>(isYk ? u * g.tile_width + v : v * g.tile_width + u);
            gv[bk + q] = gk;
        }
    }
    // very large footprints: the lane emits its own tiles
    if (spill) {
        int64_t cur = base;
        accutile_tiles<kTile>(a.conics + static_cast<int64_t>(gid) * 3, a.opac_raster[gid],
                       a.means2d[gid * 2], a.means2d[gid * 2 + 1], g, [&](uint32_t tile) {
                           tk[cur] = tile;
                           gv[cur] = gid;
                           ++cur;
                       });
    }
}

// Emit of the supertile entries (EmitStArgs), warp-cooperative. A warp takes 32 Gaussians in
// depth order (lane = Gaussian) and their AccuTile sweep constants; the work is then spread over
// the lanes as ITEMS, one per (Gaussian, block of kStTiles strips), 32 at a time, so a Gaussian
// with many strips no longer holds its warp while the others idle. An item sweeps its block's
// strips (its first line's crossing taken as the sequential sweep would hold it:
// accutile_line_max_before), ORs each strip's bits into the masks of the supertiles it touches
// (four registers, v-block mod 4; blocks over more than four supertiles rebuild their masks from
// the strips kept in shared memory), and writes one entry per supertile of the block: the
// supertile id as the sort key, (mask, Gaussian id) as the payload. Its slots within the
// Gaussian's range come from a shared counter per Gaussian; their order inside the range does not
// matter, since a Gaussian has at most one entry per supertile and the stable sort by supertile
// keeps the ranges' depth order. Nothing is written after an overflow.
constexpr int kEmitStThreads = 256;

__device__ __forceinline__ AccuSweep shfl_sweep(const AccuSweep& S, int k) {
    AccuSweep o;
    o.A = __shfl_sync(kFullMask, S.A, k);
    o.B = __shfl_sync(kFullMask, S.B, k);
    o.C = __shfl_sync(kFullMask, S.C, k);
    o.disc = __shfl_sync(kFullMask, S.disc, k);
    o.t = __shfl_sync(kFullMask, S.t, k);
    o.p.x = __shfl_sync(kFullMask, S.p.x, k);
    o.p.y = __shfl_sync(kFullMask, S.p.y, k);
    o.bmin.x = __shfl_sync(kFullMask, S.bmin.x, k);
    o.bmin.y = __shfl_sync(kFullMask, S.bmin.y, k);
    o.bmax.x = __shfl_sync(kFullMask, S.bmax.x, k);
    o.bmax.y = __shfl_sync(kFullMask, S.bmax.y, k);
    o.argmin_y = __shfl_sync(kFullMask, S.argmin_y, k);
    o.argmax_y = __shfl_sync(kFullMask, S.argmax_y, k);
    o.rmin_x = __shfl_sync(kFullMask, S.rmin_x, k);
    o.rmax_x = __shfl_sync(kFullMask, S.rmax_x, k);
    o.rmin_y = __shfl_sync(kFullMask, S.rmin_y, k);
    o.rmax_y = __shfl_sync(kFullMask, S.rmax_y, k);
    o.block = S.block;
    o.isY = __shfl_sync(kFullMask, static_cast<int>(S.isY), k) != 0;
    return o;
}

__global__ void __launch_bounds__(kEmitStThreads)
emit_supertiles_kernel(EmitStArgs a, TileGrid g) {
    __shared__ int32_t s_v0[kStTiles][kEmitStThreads];  // an item's strips, for wide blocks
    __shared__ int32_t s_v1[kStTiles][kEmitStThreads];
    __shared__ uint32_t s_next[kEmitStThreads];          // per Gaussian: entries claimed so far
    const int t = threadIdx.x, lane = t & 31;
    const int64_t j = static_cast<int64_t>(blockIdx.x) * kEmitStThreads + t;
    if (*a.overflow) return;  // uniform
    const int stw = static_cast<int>(a.st_width);
    int32_t gid = 0, ne = 0, nblk = 0;
    int64_t base = 0;
    AccuSweep S{};
    if (j < a.n) {
        gid = a.order[j];
        ne = a.entries[gid];
        if (ne > 0) {
            base = a.offsets[j];
            if (accutile_setup<kTile>(a.conics + static_cast<int64_t>(gid) * 3, a.opac_raster[gid],
                                      a.means2d[static_cast<int64_t>(gid) * 2],
                                      a.means2d[static_cast<int64_t>(gid) * 2 + 1], g, S))
                nblk = (S.rmax_x - 1) / kStTiles - S.rmin_x / kStTiles + 1;
        }
    }
    s_next[t] = 0u;
    int incl = nblk;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFullMask, incl, o);
        if (lane >= o) incl += y;
    }
    const int total = __shfl_sync(kFullMask, incl, 31);
    __syncwarp();
    for (int r0 = 0; r0 < total; r0 += 32) {  // uniform over the warp
        const int it = r0 + lane;
        int k = 0;  // owner: the number of lanes whose inclusive prefix is <= it
#pragma unroll
        for (int step = 16; step > 0; step >>= 1) {
            const int c = k + step;
            if (__shfl_sync(kFullMask, incl, c - 1) <= it) k = c;
        }
        k = min(k, 31);
        const int q = it - (__shfl_sync(kFullMask, incl, k) - __shfl_sync(kFullMask, nblk, k));
        const AccuSweep O = shfl_sweep(S, k);
        const int32_t ogid = __shfl_sync(kFullMask, gid, k);
        const int32_t one = __shfl_sync(kFullMask, ne, k);
        const int64_t obase = __shfl_sync(kFullMask, base, k);
        if (it >= total) continue;
        const int ub = O.rmin_x / kStTiles + q;
        const int u_lo = max(O.rmin_x, ub * kStTiles), u_hi = min(O.rmax_x, ub * kStTiles + kStTiles);
        constexpr float BLOCK = static_cast<float>(kTile);
        // the sequential sweep's state entering strip u_lo
        F2 line_max = u_lo == O.rmin_x ? F2{O.bmax.y, O.bmin.y}
                                       : accutile_line_max_before<kTile>(O, u_lo);
        float min_line = u_lo * BLOCK;
        F2 line_min = u_lo != O.rmin_x ? line_max
                    : (O.bmin.x <= min_line ? accutile_line_at(O, min_line) : line_max);
        int vlo = 0, vhi = -1;
        uint32_t present = 0;
        uint64_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;
        for (int u = u_lo; u < u_hi; ++u) {
            const float max_line = min_line + BLOCK;
            if (max_line <= O.bmax.x) line_max = accutile_line_at(O, max_line);
            int v0, v1;
            accutile_strip<kTile>(O, min_line, max_line, line_min, line_max, v0, v1);
            line_min = line_max;
            min_line = max_line;
            if (v1 <= v0) continue;
            const int r = u - ub * kStTiles;
            if (!present) {
                vlo = v0;
                vhi = v1 - 1;
            } else {
                vlo = min(vlo, v0);
                vhi = max(vhi, v1 - 1);
            }
            present |= 1u << r;
            s_v0[r][t] = v0;
            s_v1[r][t] = v1;
            for (int vb = v0 / kStTiles; vb <= (v1 - 1) / kStTiles; ++vb) {
                const int v_first = vb * kStTiles;
                const uint64_t bits = st_strip_bits(r, max(v0, v_first) - v_first,
                                                    min(v1, v_first + kStTiles) - v_first, O.isY);
                const int qq = vb & 3;
                m0 |= qq == 0 ? bits : 0ull;
                m1 |= qq == 1 ? bits : 0ull;
                m2 |= qq == 2 ? bits : 0ull;
                m3 |= qq == 3 ? bits : 0ull;
            }
        }
        if (!present) continue;
        const int vb0 = vlo / kStTiles, vb1 = vhi / kStTiles;
        const uint32_t e0 = atomicAdd(&s_next[(t & ~31) + k], static_cast<uint32_t>(vb1 - vb0 + 1));
        const bool wide = vb1 - vb0 >= 4;
        for (int vb = vb0; vb <= vb1; ++vb) {
            uint64_t m;
            if (!wide) {
                const int qq = vb & 3;
                m = qq == 0 ? m0 : qq == 1 ? m1 : qq == 2 ? m2 : m3;
            } else {
                const int v_first = vb * kStTiles;
                m = 0;
#pragma unroll
                for (int r = 0; r < kStTiles; ++r) {
                    if (!((present >> r) & 1u)) continue;
                    const int lo = max(s_v0[r][t], v_first) - v_first;
                    const int hi = min(s_v1[r][t], v_first + kStTiles) - v_first;
                    if (lo < hi) m |= st_strip_bits(r, lo, hi, O.isY);
                }
            }
            const uint32_t e = e0 + static_cast<uint32_t>(vb - vb0);
            if (e >= static_cast<uint32_t>(one)) continue;  // never beyond the Gaussian's range
            const int sx = O.isY ? vb : ub, sy = O.isY ? ub : vb;
            const int64_t o = obase + e;
            a.st_keys[o] = static_cast<uint32_t>(sy * stw + sx);
            a.entry_ids[o] = static_cast<int32_t>(o);
            a.entry[o] = make_uint4(static_cast<uint32_t>(m), static_cast<uint32_t>(m >> 32),
                                    static_cast<uint32_t>(ogid), 0u);
        }
    }
}

}  // namespace

void launch_projection_fwd(const SxProjectionFusedInputs& in, const SxProjectionFusedOutputs& out,
                           cudaStream_t s) {
    const int64_t CN = in.N * in.C;
    if (in.calc_compensations && out.compensations)
        cuda_check(cudaMemsetAsync(out.compensations, 0, sizeof(float) * CN, s), "memset comps");
    if (CN == 0) return;
    ProjParams p{in.eps2d, in.near_plane, in.far_plane, in.radius_clip, in.calc_compensations};
    SX_LAUNCH(projection_fwd_kernel, blocks_for(CN, kThreads), kThreads, 0, s, in.means,
              in.covars, in.quats, in.scales, in.opacities, in.viewmats, in.Ks, in.N, in.C,
              in.width, in.height, p, out.radii, out.means2d, out.depths, out.conics,
              out.compensations);
}

void launch_sh_fwd(const SxShInputs& in, float* colors, cudaStream_t s) {
    const int64_t BN = in.B * in.N;
    if (BN == 0) return;
    SX_LAUNCH(sh_fwd_kernel, blocks_for(BN * in.D, kThreads), kThreads, 0, s, in.dirs, in.coeffs,
              in.masks, static_cast<int>(in.degrees_to_use), BN, in.N, in.K,
              static_cast<int>(in.D), colors);
}

void launch_isect_count(const SxIsectTilesInputs& in, int32_t* tiles, cudaStream_t s) {
    const int64_t n = in.I * in.N;
    if (n == 0) return;
    TileGrid g{static_cast<float>(in.tile_size), static_cast<int>(in.tile_width),
               static_cast<int>(in.tile_height)};
    SX_LAUNCH(isect_count_kernel, blocks_for(n, kThreads), kThreads, 0, s, in.means2d, in.radii,
              in.conics, in.opacities, n, g, tiles);
}

void launch_isect_emit(const SxIsectTilesInputs& in, uint32_t tile_n_bits, const int64_t* cum,
                       uint64_t* isect_ids, int32_t* flatten_ids, cudaStream_t s) {
    const int64_t n = in.I * in.N;
    if (n == 0) return;
    TileGrid g{static_cast<float>(in.tile_size), static_cast<int>(in.tile_width),
               static_cast<int>(in.tile_height)};
    SX_LAUNCH(isect_emit_kernel, blocks_for(n, kThreads), kThreads, 0, s, in.means2d, in.radii,
              in.depths, in.conics, in.opacities, cum, n, in.N, tile_n_bits, g, isect_ids,
              flatten_ids);
}

void launch_offset_encode(const uint64_t* ids, int64_t n_isects, int64_t I, uint32_t tile_n_bits,
                          int64_t n_tiles, int32_t* offsets, cudaStream_t s) {
    const int64_t total = I * n_tiles;
    if (n_isects == 0) {
        if (total > 0)
            cuda_check(cudaMemsetAsync(offsets, 0, sizeof(int32_t) * total, s), "memset offsets");
        return;
    }
    SX_LAUNCH(offset_encode_kernel, blocks_for(n_isects, kThreads), kThreads, 0, s, ids, n_isects,
              total, tile_n_bits, n_tiles, offsets);
}

void launch_fwd_gauss(const FwdGaussArgs& a, cudaStream_t s) {
    if (a.count <= 0) return;
    if (a.K < 1 || a.K > 16) throw_invalid("fwd_gauss", "K must be in [1, 16]");
    SX_LAUNCH(fwd_gauss_kernel, blocks_for(a.count, kFwdThreads), kFwdThreads, 0, s, a);
}

void launch_emit_supertiles(const EmitStArgs& a, cudaStream_t s) {
    if (a.n <= 0) return;
    TileGrid g{static_cast<float>(kTile), static_cast<int>(a.tile_width),
               static_cast<int>(a.tile_height)};
    SX_LAUNCH(emit_supertiles_kernel, blocks_for(a.n, kEmitStThreads), kEmitStThreads, 0, s, a, g);
}

void launch_emit_depth_ordered(const EmitArgs& a, cudaStream_t s) {
    if (a.n <= 0) return;
    TileGrid g{static_cast<float>(kTile), static_cast<int>(a.tile_width),
               static_cast<int>(a.tile_height)};
    SX_LAUNCH(emit_depth_ordered_kernel, blocks_for(a.n, kEmitWarps * 32), kEmitWarps * 32, 0, s,
              a, g);
}

}  // namespace sx
