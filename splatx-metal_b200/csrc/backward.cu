// backward.cu — projection and SH backward (per-kernel API), fused Adam, Philox RNG, MCMC
// relocation / perturbation, and the executor's fused per-Gaussian backward + optimiser step.
#include <cfloat>

#include "sx_bulk.cuh"
#include "sx_common.cuh"
#include "sx_internal.h"
#include "sx_sh.cuh"
#include "sx_vjp.cuh"

namespace sx {

namespace {

constexpr int kThreads = 256;

// ------------------------------------------------------------------ fused Adam (API) ----------
// m = b1 m + (1-b1) g, v = b2 v + (1-b2) g^2, p -= lr m / (sqrt(v) + eps); no bias correction;
// a row whose valid flag is 0 is left untouched (AdamMCMC.metal:20-46).
__global__ void __launch_bounds__(kThreads)
adam_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
            float* __restrict__ v, const uint8_t* __restrict__ valid, int64_t n, int64_t D,
            float lr, float b1, float b2, float eps) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= n) return;
    if (valid && valid[i / D] == 0) return;
    const float gi = g[i];
    const float mi = fmaf(1.0f - b1, gi, b1 * m[i]);
    const float vi = fmaf(1.0f - b2, gi * gi, b2 * v[i]);
    p[i] += -lr * mi / (sqrtf(vi) + eps);
    m[i] = mi;
    v[i] = vi;
}

__device__ __forceinline__ void adam_update(float& p, float& m, float& v, float g, float lr,
                                            float b1, float b2, float eps) {
    m = fmaf(1.0f - b1, g, b1 * m);
    v = fmaf(1.0f - b2, g * g, b2 * v);
    p += -lr * m / (sqrtf(v) + eps);
}

// ------------------------------------------------------------------ projection bwd (API) ------
__global__ void __launch_bounds__(kThreads)
projection_bwd_kernel(SxProjectionFusedInputs in, SxProjectionFusedGradsIn gin,
                      SxProjectionFusedGrads out) {
    const int64_t CN = in.N * in.C;
    const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    const bool in_grid = idx < CN;
    const int64_t gi = in_grid ? idx : 0;
    const int64_t cid = gi / in.N, gid = gi % in.N;
    const bool alive = in_grid && gin.radii[gi * 2] > 0 && gin.radii[gi * 2 + 1] > 0;
    ProjVjpOut o;
    const bool want_pose = gin.viewmats_grad != 0;
    if (alive) {
        const float* vm = in.viewmats + cid * 16;
        const float R[9] = {vm[0], vm[1], vm[2], vm[4], vm[5], vm[6], vm[8], vm[9], vm[10]};
        const float t[3] = {vm[3], vm[7], vm[11]};
        const float* K = in.Ks + cid * 9;
        ProjVjpIn pi;
        pi.mean_w = in.means + gid * 3;
        pi.quat = in.covars ? nullptr : in.quats + gid * 4;
        pi.scale = in.covars ? nullptr : in.scales + gid * 3;
        pi.covar6 = in.covars ? in.covars + gid * 6 : nullptr;
        pi.R = R;
        pi.t = t;
        pi.fx = K[0]; pi.fy = K[4]; pi.cx = K[2]; pi.cy = K[5];
        pi.width = in.width;
        pi.height = in.height;
        pi.eps2d = in.eps2d;
        pi.conic = gin.conics + gi * 3;
        pi.v_m2x = gin.v_means2d[gi * 2];
        pi.v_m2y = gin.v_means2d[gi * 2 + 1];
        pi.v_depth = gin.v_depths[gi];
        pi.v_conic = gin.v_conics + gi * 3;
        pi.has_comp = gin.v_compensations != nullptr;
        pi.comp = pi.has_comp ? gin.compensations[gi] : 0.f;
        pi.v_comp = pi.has_comp ? gin.v_compensations[gi] : 0.f;
        projection_vjp(pi, o, want_pose);
        const bool single = in.C == 1;
        auto put = [&](float* dst, float val) {
            if (single)
                *dst = val;
            else
                atomicAdd(dst, val);
        };
        for (int k = 0; k < 3; ++k) put(out.v_means + gid * 3 + k, o.v_mean[k]);
        if (in.covars) {
            const float* c = o.v_covar;
            put(out.v_covars + gid * 6 + 0, c[0]);
            put(out.v_covars + gid * 6 + 1, c[1] + c[3]);
            put(out.v_covars + gid * 6 + 2, c[2] + c[6]);
            put(out.v_covars + gid * 6 + 3, c[4]);
            put(out.v_covars + gid * 6 + 4, c[5] + c[7]);
            put(out.v_covars + gid * 6 + 5, c[8]);
        } else {
            for (int k = 0; k < 4; ++k) put(out.v_quats + gid * 4 + k, o.v_quat[k]);
            for (int k = 0; k < 3; ++k) put(out.v_scales + gid * 3 + k, o.v_scale[k]);
        }
    }
    if (want_pose) {
        // 12 pose values per lane; reduce across the warp when every lane has the same camera.
        float vals[12];
#pragma unroll
        for (int i = 0; i < 3; ++i) {
#pragma unroll
            for (int j = 0; j < 3; ++j) vals[i * 4 + j] = alive ? o.v_R[i * 3 + j] : 0.f;
            vals[i * 4 + 3] = alive ? o.v_t[i] : 0.f;
        }
        const int lane = threadIdx.x & 31;
        const int64_t cid0 = __shfl_sync(kFullMask, cid, 0);
        const bool uniform = __all_sync(kFullMask, cid == cid0);
        if (uniform) {
            const float r = warp_transpose_reduce<12>(vals, lane);
            const int slot = transpose_reduce_slot<12>(lane);
            if (slot >= 0) atomicAdd(out.v_viewmats + cid * 16 + slot, r);
        } else if (alive) {
            for (int k = 0; k < 12; ++k) atomicAdd(out.v_viewmats + cid * 16 + k, vals[k]);
        }
    }
}

// ------------------------------------------------------------------ SH bwd (API) --------------
// One thread per (batch, gaussian) element, all D channels: v_coeffs[k][c] += Y_k v_color[c],
// v_dir = normalisation VJP of sum_k (sum_c v_color[c] coeff[k][c]) dY_k.
__global__ void __launch_bounds__(kThreads)
sh_bwd_kernel(const float* __restrict__ dirs, const float* __restrict__ coeffs,
              const uint8_t* __restrict__ masks, const float* __restrict__ v_colors, int degree,
              int64_t BN, int64_t N, int64_t K, int D, bool atomic_coeffs,
              float* __restrict__ v_coeffs, float* __restrict__ v_dirs) {
    const int64_t elem = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (elem >= BN) return;
    if (masks && masks[elem] == 0) return;
    const int64_t gid = elem % N;
    const float* co = coeffs + gid * K * D;
    const float* vc = v_colors + elem * D;
    float x = 0.f, y = 0.f, z = 0.f, inorm = 0.f;
    const float* d = dirs + elem * 3;
    if (degree >= 1) {
        inorm = 1.0f / sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
        x = d[0] * inorm;
        y = d[1] * inorm;
        z = d[2] * inorm;
    }
    float Y[25], g[25];
    sh_basis(degree, x, y, z, Y);
    const int nb = sh_bands(degree);
    float* vco = v_coeffs + gid * K * D;
    for (int k = 0; k < nb; ++k) {
        float gk = 0.f;
        for (int c = 0; c < D; ++c) {
            const float val = Y[k] * vc[c];
            if (atomic_coeffs)
                atomicAdd(vco + k * D + c, val);
            else
                vco[k * D + c] = val;
            gk = fmaf(vc[c], co[k * D + c], gk);
        }
        g[k] = gk;
    }
    if (v_dirs && degree >= 1) {
        float gx, gy, gz;
        sh_basis_vjp(degree, x, y, z, g, gx, gy, gz);
        const float dot = gx * x + gy * y + gz * z;
        v_dirs[elem * 3 + 0] = (gx - dot * x) * inorm;
        v_dirs[elem * 3 + 1] = (gy - dot * y) * inorm;
        v_dirs[elem * 3 + 2] = (gz - dot * z) * inorm;
    }
}

// ------------------------------------------------------------------ RNG -----------------------
__global__ void __launch_bounds__(kThreads)
rng_u32_kernel(uint32_t* __restrict__ out, int64_t count, uint64_t seed, uint64_t offset) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t base = static_cast<int64_t>(t) * 4;
    if (base >= count) return;
    const Philox4 r = philox4x32_10(t, static_cast<uint32_t>(offset),
                                    static_cast<uint32_t>(offset >> 32), 0u,
                                    static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
    for (int j = 0; j < 4 && base + j < count; ++j) out[base + j] = r.v[j];
}

__global__ void __launch_bounds__(kThreads)
rng_normal_kernel(float* __restrict__ out, int64_t count, uint64_t seed, uint64_t offset) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t base = static_cast<int64_t>(t) * 4;
    if (base >= count) return;
    const Philox4 r = philox4x32_10(t, static_cast<uint32_t>(offset),
                                    static_cast<uint32_t>(offset >> 32), 0u,
                                    static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
    float z[4];
    box_muller(r.v[0], r.v[1], z[0], z[1]);
    box_muller(r.v[2], r.v[3], z[2], z[3]);
    for (int j = 0; j < 4 && base + j < count; ++j) out[base + j] = z[j];
}

// ------------------------------------------------------------------ MCMC ----------------------
// Relocation (MCMC paper Eq. 9): opacity 1-(1-o)^(1/n) clamped to [min_op, 1-eps], then the
// scale factor o / sum_{i=1..n} sum_{k<i} C(i-1,k) (-1)^k / sqrt(k+1) * o_new^(k+1), summed in
// ascending (i,k) (AdamMCMC.metal:63-97).
__global__ void __launch_bounds__(kThreads)
relocation_kernel(const float* __restrict__ op, const float* __restrict__ sc,
                  const int32_t* __restrict__ ratios, const float* __restrict__ binoms, int64_t N,
                  int n_max, float min_op, float* __restrict__ new_op, float* __restrict__ new_sc) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= N) return;
    const int n = ratios[i];
    const float o = op[i];
    float no = 1.0f - powf(1.0f - o, 1.0f / static_cast<float>(n));
    no = fminf(fmaxf(no, min_op), 1.0f - FLT_EPSILON);
    new_op[i] = no;
    float denom = 0.0f;
    for (int a = 1; a <= n; ++a)
        for (int k = 0; k <= a - 1; ++k) {
            const float bc = binoms[(a - 1) * n_max + k];
            const float sign = (k & 1) ? -1.0f : 1.0f;
            const float term = (sign / sqrtf(static_cast<float>(k + 1))) *
                               powf(no, static_cast<float>(k + 1));
            denom += bc * term;
        }
    const float coeff = o / denom;
    for (int k = 0; k < 3; ++k) new_sc[i * 3 + k] = coeff * sc[i * 3 + k];
}

// Position noise: means += Sigma (n * sigmoid(-k (sigmoid(op) - t)) * noise_scale), Sigma the
// covariance itself (MCMCPerturbCUDA semantics, AdamMCMC.metal:112-140).
__device__ __forceinline__ void perturb_one(float* pos, const float* q, const float* log_s,
                                            float op_logit, const float* n3, float noise_scale,
                                            float t, float k) {
    float Rm[9], qn[4], inv_norm;
    quat_rotmat(q, Rm, qn, inv_norm);
    const float s[3] = {expf(log_s[0]), expf(log_s[1]), expf(log_s[2])};
    float M[9], C[9];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) M[i * 3 + j] = Rm[i * 3 + j] * s[j];
    m3_mul_bt(M, M, C);
    const float density = 1.0f / (1.0f + expf(-op_logit));
    const float w = (1.0f / (1.0f + expf(k * (density - t)))) * noise_scale;
    const float a = n3[0] * w, b = n3[1] * w, c = n3[2] * w;
#pragma unroll
    for (int i = 0; i < 3; ++i) pos[i] += C[i * 3] * a + C[i * 3 + 1] * b + C[i * 3 + 2] * c;
}

__global__ void __launch_bounds__(kThreads)
perturb_kernel(SxPerturbInputs in) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= in.N) return;
    float p[3] = {in.positions[i * 3], in.positions[i * 3 + 1], in.positions[i * 3 + 2]};
    perturb_one(p, in.quats + i * 4, in.scales_log + i * 3, in.opacities_logit[i],
                in.noise + i * 3, in.noise_scale, in.t, in.k);
    in.positions[i * 3] = p[0];
    in.positions[i * 3 + 1] = p[1];
    in.positions[i * 3 + 2] = p[2];
}

// ------------------------------------------------------------------ executor backward ---------
struct BwdGaussConst {
    float R[9], t[3], campos[3];
    float fx, fy, cx, cy;
};

// One warp owns 32 consecutive Gaussians.
//  * The 14 geometric floats per Gaussian (means, quats, log-scales, logit opacity, sh0) of the
//    parameters and both Adam moments are contiguous 16-byte-aligned slabs for the warp (5,376 B);
//    one lane moves them into shared memory with bulk copies (TMA, untiled) on an mbarrier and,
//    after the update, back with bulk stores — every byte moves in full 16-byte units.
//  * The SH rest coefficients (3*(K-1) floats per Gaussian, 1,440 per warp at degree 3) stream
//    as float4 through registers: lane-consecutive, two float4 of params + both moments in flight
//    per lane, whole float4s of invalid Gaussians skipped. Each coefficient's product with the
//    masked colour gradient (taken before the update) goes to shared memory; the owning lane sums
//    them into the colour-weighted coefficient sums g_k of the SH direction VJP.
//  * Per-Gaussian work (SH basis and its VJP, projection VJP, chains, Adam on the geometric groups,
//    noise) runs one lane per Gaussian out of shared memory.
constexpr int kBwdWarps = 4;
// per array (floats): means [0,96) | quats [96,224) | log-scales [224,320) | opac [320,352) |
// sh0 [352,448)
constexpr int kGeoFloats = 448;
constexpr int kYStride = 17;     // padded SH-basis rows: conflict-free lane-strided writes

__device__ __forceinline__ int geo_off(int g) {
    return g == 0 ? 0 : g == 1 ? 96 : g == 2 ? 224 : g == 3 ? 320 : 352;
}
__device__ __forceinline__ int geo_dim(int g) { return g == 1 ? 4 : g == 3 ? 1 : 3; }

template <int R>
struct BwdSmem {
    static constexpr int kPerWarp = 3 * kGeoFloats + 32 * kYStride + 32 * 4 + 32 * R;  // floats
    static constexpr size_t kBytes = sizeof(float) * kPerWarp * kBwdWarps;
};

// One SH-rest coefficient: product for g_k, then Adam when its Gaussian is valid.
template <int R>
__device__ __forceinline__ void shn_coeff(int f, float& p, float& m, float& v, const float* sC,
                                          const float* sY, float* sP, float lr, float b1, float b2,
                                          float eps) {
    const int gl = f / R;
    const int rem = f - gl * R;
    const int band = rem / 3;
    const int c = rem - band * 3;
    const float vc = sC[gl * 4 + c];
    sP[f] = __fmul_rn(vc, p);
    if (sC[gl * 4 + 3] != 0.f) adam_update(p, m, v, sY[gl * kYStride + band + 1] * vc, lr, b1, b2, eps);
}

template <int R>
__global__ void __launch_bounds__(kBwdWarps * 32, 4)
bwd_gauss_kernel(BwdGaussArgs a, BwdGaussConst k) {
    extern __shared__ __align__(16) float smem[];
    __shared__ uint64_t bars[kBwdWarps];
    if (*a.skip_flag) return;  // uniform: the step overflowed
    const unsigned full = 0xffffffffu;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int base = (blockIdx.x * kBwdWarps + warp) * 32;
    if (base >= a.count) return;  // warp-uniform; only warp-level syncs below
    const int ng = min(32, a.count - base);
    const int i = base + lane;
    const bool in_range = lane < ng;
    const bool valid = in_range && a.valid[i] != 0;
    if (!__any_sync(full, valid) && !a.inject_noise) return;  // nothing to update

    float* geo = smem + warp * BwdSmem<R>::kPerWarp;  // [param | m | v][kGeoFloats]
    float* sY = geo + 3 * kGeoFloats;
    float* sC = sY + 32 * kYStride;  // masked colour gradient (3) + valid flag, per lane
    float* sP = sC + 32 * 4;         // SH-rest coefficient x colour-gradient products
    float* gparam[5] = {a.means, a.quats, a.log_scales, a.opac_logit, a.sh0};
    const bool bulk = ng == 32;
    if (bulk) {
        if (lane == 0) {
            mbar_init(&bars[warp], 1);
            mbar_arrive_expect_tx(&bars[warp], 3 * kGeoFloats * sizeof(float));
#pragma unroll
            for (int g = 0; g < 5; ++g) {
                const int64_t o = static_cast<int64_t>(base) * geo_dim(g);
                const uint32_t bytes = 32u * geo_dim(g) * sizeof(float);
                bulk_load(geo + geo_off(g), gparam[g] + o, bytes, &bars[warp]);
                bulk_load(geo + kGeoFloats + geo_off(g), a.m[g] + o, bytes, &bars[warp]);
                bulk_load(geo + 2 * kGeoFloats + geo_off(g), a.v[g] + o, bytes, &bars[warp]);
            }
        }
    } else {  // the ragged last warp: plain loads into the same layout
#pragma unroll
        for (int g = 0; g < 5; ++g) {
            const int64_t o = static_cast<int64_t>(base) * geo_dim(g);
            for (int e = lane; e < ng * geo_dim(g); e += 32) {
                geo[geo_off(g) + e] = gparam[g][o + e];
                geo[kGeoFloats + geo_off(g) + e] = a.m[g][o + e];
                geo[2 * kGeoFloats + geo_off(g) + e] = a.v[g][o + e];
            }
        }
    }
    __syncwarp();  // the barrier is initialised before any lane waits on it

    // the accumulated screen-space gradients: read, then re-zeroed for the next step
    const int64_t i3 = static_cast<int64_t>(i) * 3;
    float vm2[2] = {0.f, 0.f}, vcon[3] = {0.f, 0.f, 0.f}, vcol[3] = {0.f, 0.f, 0.f}, vop = 0.f;
    float con[3] = {0.f, 0.f, 0.f}, comp = 0.f;
    if (valid) {
        vm2[0] = a.v_means2d[i * 2];
        vm2[1] = a.v_means2d[i * 2 + 1];
        vcon[0] = a.v_conics[i3]; vcon[1] = a.v_conics[i3 + 1]; vcon[2] = a.v_conics[i3 + 2];
        vcol[0] = a.v_colors[i3]; vcol[1] = a.v_colors[i3 + 1]; vcol[2] = a.v_colors[i3 + 2];
        vop = a.v_opac[i];
        con[0] = a.conics[i3]; con[1] = a.conics[i3 + 1]; con[2] = a.conics[i3 + 2];
        if (a.antialiased) comp = a.comps[i];
        const uint8_t rm = a.relu_mask[i];
#pragma unroll
        for (int c = 0; c < 3; ++c)
            if (!(rm & (1u << c))) vcol[c] = 0.f;
        a.v_means2d[i * 2] = 0.f;
        a.v_means2d[i * 2 + 1] = 0.f;
        a.v_conics[i3] = 0.f; a.v_conics[i3 + 1] = 0.f; a.v_conics[i3 + 2] = 0.f;
        a.v_colors[i3] = 0.f; a.v_colors[i3 + 1] = 0.f; a.v_colors[i3 + 2] = 0.f;
        a.v_opac[i] = 0.f;
    }
    sC[lane * 4 + 0] = vcol[0];
    sC[lane * 4 + 1] = vcol[1];
    sC[lane * 4 + 2] = vcol[2];
    sC[lane * 4 + 3] = valid ? 1.f : 0.f;
    if (bulk) {
        const bool ok = __all_sync(full, mbar_wait(&bars[warp], 0));
        if (!ok) {
            if (lane == 0) atomicOr(a.status, kStatusBulkWaitTimeout);
            __syncwarp();
            mbar_wait(&bars[warp], 0);  // once more for the copies still in flight, then give up
            return;
        }
    }
    __syncwarp();

    const int deg = static_cast<int>(a.degree);
    float x = 0.f, y = 0.f, z = 0.f, inorm = 0.f;
    float Y[16];
#pragma unroll
    for (int b = 0; b < 16; ++b) Y[b] = 0.f;
    if (valid) {
        const float* mw = geo + lane * 3;
        const float dx = mw[0] - k.campos[0], dy = mw[1] - k.campos[1], dz = mw[2] - k.campos[2];
        if (deg >= 1) {
            inorm = 1.0f / sqrtf(dx * dx + dy * dy + dz * dz);
            x = dx * inorm;
            y = dy * inorm;
            z = dz * inorm;
        }
        sh_basis(deg, x, y, z, Y);
    }
#pragma unroll
    for (int b = 0; b < 16; ++b) sY[lane * kYStride + b] = Y[b];
    __syncwarp();

    // ---- SH rest coefficients, streamed as float4
    if constexpr (R > 0) {
        const int nf = ng * R;
        const int nq = nf >> 2;
        const int64_t o = static_cast<int64_t>(base) * R;
        float4* __restrict__ P4 = reinterpret_cast<float4*>(a.shN + o);
        float4* __restrict__ M4 = reinterpret_cast<float4*>(a.m[5] + o);
        float4* __restrict__ V4 = reinterpret_cast<float4*>(a.v[5] + o);
        const float lr = a.lr[5], b1 = a.b1, b2 = a.b2, eps = a.eps;
#pragma unroll 2
        for (int q = lane; q < nq; q += 32) {
            const int f0 = q * 4;
            if (sC[(f0 / R) * 4 + 3] == 0.f && sC[((f0 + 3) / R) * 4 + 3] == 0.f) continue;
            float4 p = P4[q], m = M4[q], v = V4[q];
            shn_coeff<R>(f0 + 0, p.x, m.x, v.x, sC, sY, sP, lr, b1, b2, eps);
            shn_coeff<R>(f0 + 1, p.y, m.y, v.y, sC, sY, sP, lr, b1, b2, eps);
            shn_coeff<R>(f0 + 2, p.z, m.z, v.z, sC, sY, sP, lr, b1, b2, eps);
            shn_coeff<R>(f0 + 3, p.w, m.w, v.w, sC, sY, sP, lr, b1, b2, eps);
            P4[q] = p;
            M4[q] = m;
            V4[q] = v;
        }
        for (int f = nq * 4 + lane; f < nf; f += 32) {  // ragged tail of the last warp
            float p = a.shN[o + f], m = a.m[5][o + f], v = a.v[5][o + f];
            shn_coeff<R>(f, p, m, v, sC, sY, sP, lr, b1, b2, eps);
            a.shN[o + f] = p;
            a.m[5][o + f] = m;
            a.v[5][o + f] = v;
        }
    }
    __syncwarp();

    float* pm = geo + geo_off(0) + lane * 3;  // means
    float* pq = geo + geo_off(1) + lane * 4;  // quats
    float* ps = geo + geo_off(2) + lane * 3;  // log-scales
    float* po = geo + geo_off(3) + lane;      // logit opacity
    float* p0 = geo + geo_off(4) + lane * 3;  // sh0
    constexpr int M = kGeoFloats, V = 2 * kGeoFloats;
    if (valid) {
        float g[16];
#pragma unroll
        for (int b = 0; b < 16; ++b) g[b] = 0.f;
        {
            float gb = 0.f;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                float p = p0[c], m = p0[M + c], v = p0[V + c];
                gb = __fadd_rn(gb, __fmul_rn(vcol[c], p));
                adam_update(p, m, v, Y[0] * vcol[c], a.lr[4], a.b1, a.b2, a.eps);
                p0[c] = p;
                p0[M + c] = m;
                p0[V + c] = v;
            }
            g[0] = gb;
        }
        if constexpr (R > 0) {
            const float* pr = sP + lane * R;
#pragma unroll
            for (int b = 1; b <= R / 3; ++b)
                g[b] = __fadd_rn(__fadd_rn(pr[(b - 1) * 3], pr[(b - 1) * 3 + 1]), pr[(b - 1) * 3 + 2]);
        }
        float vdir[3] = {0.f, 0.f, 0.f};
        if (deg >= 1) {
            float gx, gy, gz;
            sh_basis_vjp(deg, x, y, z, g, gx, gy, gz);
            const float dot = gx * x + gy * y + gz * z;
            vdir[0] = (gx - dot * x) * inorm;
            vdir[1] = (gy - dot * y) * inorm;
            vdir[2] = (gz - dot * z) * inorm;
        }

        // ---- projection backward (C = 1), activations recomputed
        const float mean[3] = {pm[0], pm[1], pm[2]};
        const float quat[4] = {pq[0], pq[1], pq[2], pq[3]};
        const float s[3] = {exp_cr(ps[0]), exp_cr(ps[1]), exp_cr(ps[2])};
        const float sig = sigmoid_cr(po[0]);
        float v_comp = 0.f;
        if (a.antialiased) {
            v_comp = vop * sig;
            vop = vop * comp;
        }
        ProjVjpIn pi;
        pi.mean_w = mean;
        pi.quat = quat;
        pi.scale = s;
        pi.covar6 = nullptr;
        pi.R = k.R;
        pi.t = k.t;
        pi.fx = k.fx; pi.fy = k.fy; pi.cx = k.cx; pi.cy = k.cy;
        pi.width = a.width;
        pi.height = a.height;
        pi.eps2d = a.eps2d;
        pi.conic = con;
        pi.v_m2x = vm2[0];
        pi.v_m2y = vm2[1];
        pi.v_depth = 0.f;
        pi.v_conic = vcon;
        pi.has_comp = a.antialiased != 0;
        pi.comp = comp;
        pi.v_comp = v_comp;
        ProjVjpOut o;
        projection_vjp(pi, o, false);

        // ---- chains, regularisers and Adam on the four geometric groups
        float gs[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            float gv = o.v_scale[c] * s[c];
            if (a.scale_reg_w > 0.0f) gv += a.scale_reg_w * s[c];
            gs[c] = gv;
        }
        float gop = vop * (sig * (1.0f - sig));
        if (a.opacity_reg_w > 0.0f) gop += a.opacity_reg_w * sig * (1.0f - sig);
#pragma unroll
        for (int c = 0; c < 3; ++c)
            adam_update(pm[c], pm[M + c], pm[V + c], o.v_mean[c] + vdir[c], a.lr[0], a.b1, a.b2, a.eps);
#pragma unroll
        for (int c = 0; c < 4; ++c)
            adam_update(pq[c], pq[M + c], pq[V + c], o.v_quat[c], a.lr[1], a.b1, a.b2, a.eps);
#pragma unroll
        for (int c = 0; c < 3; ++c)
            adam_update(ps[c], ps[M + c], ps[V + c], gs[c], a.lr[2], a.b1, a.b2, a.eps);
        adam_update(po[0], po[M], po[V], gop, a.lr[3], a.b1, a.b2, a.eps);
    }
    if (a.inject_noise && in_range) {
        const uint64_t nb0 = static_cast<uint64_t>(i) * 3;
        const float n3[3] = {normal_at(nb0, a.noise_seed, a.noise_offset),
                             normal_at(nb0 + 1, a.noise_seed, a.noise_offset),
                             normal_at(nb0 + 2, a.noise_seed, a.noise_offset)};
        float mean[3] = {pm[0], pm[1], pm[2]};
        perturb_one(mean, pq, ps, po[0], n3, a.noise_scale, 0.005f, 100.f);
        pm[0] = mean[0];
        pm[1] = mean[1];
        pm[2] = mean[2];
    }

    // ---- write the geometric slabs back
    if (bulk) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
            for (int g = 0; g < 5; ++g) {
                const int64_t o = static_cast<int64_t>(base) * geo_dim(g);
                const uint32_t bytes = 32u * geo_dim(g) * sizeof(float);
                bulk_store(gparam[g] + o, geo + geo_off(g), bytes);
                bulk_store(a.m[g] + o, geo + kGeoFloats + geo_off(g), bytes);
                bulk_store(a.v[g] + o, geo + 2 * kGeoFloats + geo_off(g), bytes);
            }
            bulk_commit();
            bulk_wait_all();
        }
    } else {
        __syncwarp();
#pragma unroll
        for (int g = 0; g < 5; ++g) {
            const int64_t o = static_cast<int64_t>(base) * geo_dim(g);
            for (int e = lane; e < ng * geo_dim(g); e += 32) {
                gparam[g][o + e] = geo[geo_off(g) + e];
                a.m[g][o + e] = geo[kGeoFloats + geo_off(g) + e];
                a.v[g][o + e] = geo[2 * kGeoFloats + geo_off(g) + e];
            }
        }
    }
}

template <int R>
void launch_bwd_gauss_t(const BwdGaussArgs& a, const BwdGaussConst& k, cudaStream_t s) {
    static bool configured = false;  // per template instance; the attribute is per function
    constexpr size_t bytes = BwdSmem<R>::kBytes;
    if (!configured) {
        cuda_check(cudaFuncSetAttribute(bwd_gauss_kernel<R>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(bytes)),
                   "bwd_gauss smem attribute");
        configured = true;
    }
    SX_LAUNCH(bwd_gauss_kernel<R>, blocks_for(a.count, kBwdWarps * 32), kBwdWarps * 32, bytes, s,
              a, k);
}

}  // namespace

void launch_adam(const SxAdamInputs& in, cudaStream_t s) {
    if (in.n_elems == 0) return;
    SX_LAUNCH(adam_kernel, blocks_for(in.n_elems, kThreads), kThreads, 0, s, in.param, in.grad,
              in.exp_avg, in.exp_avg_sq, in.valid, in.n_elems, in.n_elems / in.n_gauss, in.lr,
              in.b1, in.b2, in.eps);
}

void launch_projection_bwd(const SxProjectionFusedInputs& in, const SxProjectionFusedGradsIn& g,
                           const SxProjectionFusedGrads& out, cudaStream_t s) {
    const int64_t CN = in.N * in.C;
    auto zero = [&](float* p, int64_t n) {
        if (p && n > 0) cuda_check(cudaMemsetAsync(p, 0, sizeof(float) * n, s), "memset grads");
    };
    zero(out.v_means, in.N * 3);
    zero(out.v_covars, in.covars ? in.N * 6 : 0);
    zero(out.v_quats, in.covars ? 0 : in.N * 4);
    zero(out.v_scales, in.covars ? 0 : in.N * 3);
    zero(out.v_viewmats, g.viewmats_grad ? in.C * 16 : 0);
    if (CN == 0) return;
    SX_LAUNCH(projection_bwd_kernel, blocks_for(CN, kThreads), kThreads, 0, s, in, g, out);
}

void launch_sh_bwd(const SxShInputs& in, const float* v_colors, float* v_coeffs, float* v_dirs,
                   cudaStream_t s) {
    const int64_t BN = in.B * in.N;
    if (in.N * in.K * in.D > 0)
        cuda_check(cudaMemsetAsync(v_coeffs, 0, sizeof(float) * in.N * in.K * in.D, s),
                   "memset v_coeffs");
    if (in.compute_v_dirs && v_dirs && BN > 0)
        cuda_check(cudaMemsetAsync(v_dirs, 0, sizeof(float) * BN * 3, s), "memset v_dirs");
    if (BN == 0) return;
    SX_LAUNCH(sh_bwd_kernel, blocks_for(BN, kThreads), kThreads, 0, s, in.dirs, in.coeffs,
              in.masks, v_colors, static_cast<int>(in.degrees_to_use), BN, in.N, in.K,
              static_cast<int>(in.D), in.B > 1, v_coeffs, in.compute_v_dirs ? v_dirs : nullptr);
}

void launch_rng_normal(uint64_t seed, uint64_t offset, int64_t count, float* out, cudaStream_t s) {
    if (count == 0) return;
    SX_LAUNCH(rng_normal_kernel, blocks_for((count + 3) / 4, kThreads), kThreads, 0, s, out, count,
              seed, offset);
}

void launch_rng_u32(uint64_t seed, uint64_t offset, int64_t count, uint32_t* out, cudaStream_t s) {
    if (count == 0) return;
    SX_LAUNCH(rng_u32_kernel, blocks_for((count + 3) / 4, kThreads), kThreads, 0, s, out, count,
              seed, offset);
}

void launch_relocation(const SxRelocationInputs& in, float* new_op, float* new_sc, cudaStream_t s) {
    if (in.N == 0) return;
    SX_LAUNCH(relocation_kernel, blocks_for(in.N, kThreads), kThreads, 0, s, in.opacities,
              in.scales, in.ratios, in.binoms, in.N, in.n_max, in.min_opacity, new_op, new_sc);
}

void launch_perturb(const SxPerturbInputs& in, cudaStream_t s) {
    if (in.N == 0) return;
    SX_LAUNCH(perturb_kernel, blocks_for(in.N, kThreads), kThreads, 0, s, in);
}

void launch_bwd_gauss(const BwdGaussArgs& a, cudaStream_t s) {
    if (a.count <= 0) return;
    BwdGaussConst k;
    const float* vm = a.viewmat;
    const int rows[9] = {0, 1, 2, 4, 5, 6, 8, 9, 10};
    for (int i = 0; i < 9; ++i) k.R[i] = vm[rows[i]];
    k.t[0] = vm[3];
    k.t[1] = vm[7];
    k.t[2] = vm[11];
    for (int i = 0; i < 3; ++i)
        k.campos[i] = -(vm[0 * 4 + i] * vm[0 * 4 + 3] + vm[1 * 4 + i] * vm[1 * 4 + 3] +
                        vm[2 * 4 + i] * vm[2 * 4 + 3]);
    k.fx = a.Kmat[0];
    k.fy = a.Kmat[4];
    k.cx = a.Kmat[2];
    k.cy = a.Kmat[5];
    switch (a.K) {
        case 1: launch_bwd_gauss_t<0>(a, k, s); break;
        case 4: launch_bwd_gauss_t<9>(a, k, s); break;
        case 9: launch_bwd_gauss_t<24>(a, k, s); break;
        case 16: launch_bwd_gauss_t<45>(a, k, s); break;
        default: throw_invalid("bwd_gauss", "K must be 1, 4, 9 or 16");
    }
}

}  // namespace sx
