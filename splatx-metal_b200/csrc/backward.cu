// backward.cu — projection and SH backward (per-kernel API), fused Adam, Philox RNG, MCMC
// relocation / perturbation, and the executor's fused per-Gaussian backward + optimiser step.
#include <cfloat>

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

// The per-Gaussian backward runs as two kernels, one thread per Gaussian, over the executor's
// resident 32-Gaussian tiles (tile_index: a tile holds a group's d components as d runs of 32
// floats, so each warp-wide load or store is 128 contiguous bytes and a warp's footprint in a
// group is one contiguous d*128-byte run):
//   bwd_sh    the SH colour backward and Adam on sh0 / shN — about 80% of the step's parameter
//             bytes — at low register count and high occupancy; emits the direction gradient
//             v_dir (3 floats) for the second kernel.
//   bwd_geom  projection VJP, activation chains, regularisers, Adam on means / quats / scales /
//             opacities and the MCMC noise; the activations come from the forward pass.
constexpr int kBwdThreads = 128;

// The row of thread v: the identity, or with a row subset the rank-major enumeration of
// r * map_shard + [map_c0, map_c1).
__device__ __forceinline__ int64_t bwd_row(const BwdGaussArgs& a, int64_t v) {
    if (a.map_world == 0) return v;
    const int64_t len = a.map_c1 - a.map_c0;
    const int64_t r = v / len;
    return r < a.map_world ? r * a.map_shard + a.map_c0 + (v - r * len) : INT64_MAX;
}
inline int64_t bwd_threads(const BwdGaussArgs& a) {
    return a.map_world == 0 ? a.count : a.map_world * (a.map_c1 - a.map_c0);
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 4-byte global -> shared copy that holds no register while it is in flight.
__device__ __forceinline__ void cp_async4(float* smem, const float* gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
                 "l"(gmem)
                 : "memory");
}

// bwd_sh streams a Gaussian's SH bands (band 0 = sh0, bands 1.. = shN, three channels each) with
// the parameter and both Adam moments of kShStages - 1 bands ahead in flight: each thread copies
// its own band components into its own shared-memory slots with cp.async and reads back only
// those, so the pipeline needs no barrier and the loads in flight hold no registers. (A variant
// where each warp copies whole 128-byte runs with 16-byte copies, 2.25 per lane per band instead
// of 9, measured 10 us slower per step at config 2.)
constexpr int kShStages = 4;

// MODE: 0 Adam in place; 1 add the gradients to the accumulators; 2 write them (the step's
// first view: rows it does not see are zeroed) — BwdGaussArgs::accumulate.
template <int KM1, int MODE>
__global__ void __launch_bounds__(kBwdThreads, 8)
bwd_sh_kernel(BwdGaussArgs a) {
    constexpr bool ACCUM = MODE != 0;
    if (*a.skip_flag) return;  // uniform: the step overflowed
    // [stage][array: parameter, exp_avg (accumulated gradient), exp_avg_sq][channel][thread]
    __shared__ float st[kShStages][3][3][kBwdThreads];
    const StepParams& sp = *a.step;
    const BwdGaussConst& k = sp.bwd;
    const int64_t ri = bwd_row(a, blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x);
    if (ri >= a.count) return;
    const int i = static_cast<int>(ri);
    if (a.valid[i] == 0) {
        if constexpr (MODE == 2) {  // not seen by this view: its accumulated SH gradient is zero
            float* g0 = a.gacc[4] + tile_index(i, 3);
#pragma unroll
            for (int c = 0; c < 3; ++c) g0[32 * c] = 0.f;
            float* gN = a.gacc[5] + tile_index(i, 3 * KM1);
#pragma unroll
            for (int c = 0; c < 3 * KM1; ++c) gN[32 * c] = 0.f;
        }
        return;
    }
    const int t = threadIdx.x;
    constexpr int NB = 1 + KM1;  // bands
    // band b's channel-0 element in its group's tiled buffer (channel c at + 32 c)
    const int64_t off0 = tile_index(i, 3);
    const int64_t offN = tile_index(i, 3 * KM1);
    auto elem = [&](int b, int arr) -> float* {
        if (b == 0)
            return (arr == 0 ? a.sh0 : ACCUM ? a.gacc[4] : (arr == 1 ? a.m[4] : a.v[4])) + off0;
        const int64_t o = offN + static_cast<int64_t>(b - 1) * 3 * 32;
        return (arr == 0 ? a.shN : ACCUM ? a.gacc[5] : (arr == 1 ? a.m[5] : a.v[5])) + o;
    };
    auto issue = [&](int b) {
        if (b < NB) {
            const int sg = b % kShStages;
#pragma unroll
            for (int arr = 0; arr < (MODE == 0 ? 3 : MODE == 1 ? 2 : 1); ++arr) {
                const float* src = elem(b, arr);
#pragma unroll
                for (int c = 0; c < 3; ++c) cp_async4(&st[sg][arr][c][t], src + 32 * c);
            }
        }
        cp_async_commit();  // one group per band (empty past the end): uniform group counting
    };
#pragma unroll
    for (int b = 0; b < kShStages - 1; ++b) issue(b);

    const float* pmean = a.means + tile_index(i, 3);
    const float mean[3] = {pmean[0], pmean[32], pmean[64]};
    const int64_t i3 = static_cast<int64_t>(i) * 3;
    float vcol[3] = {a.v_colors[i3], a.v_colors[i3 + 1], a.v_colors[i3 + 2]};
    const uint8_t rm = a.relu_mask[i];
#pragma unroll
    for (int c = 0; c < 3; ++c)
        if (!(rm & (1u << c))) vcol[c] = 0.f;
    a.v_colors[i3] = 0.f;  // consumed: zero for the next step's raster backward
    a.v_colors[i3 + 1] = 0.f;
    a.v_colors[i3 + 2] = 0.f;

    const int deg = static_cast<int>(a.degree);
    const float dx = mean[0] - k.campos[0], dy = mean[1] - k.campos[1], dz = mean[2] - k.campos[2];
    float x = 0.f, y = 0.f, z = 0.f, inorm = 0.f;
    if (deg >= 1) {
        inorm = 1.0f / sqrtf(dx * dx + dy * dy + dz * dz);
        x = dx * inorm;
        y = dy * inorm;
        z = dz * inorm;
    }
    float Y[16];
#pragma unroll
    for (int b = 0; b < 16; ++b) Y[b] = 0.f;
    sh_basis(deg, x, y, z, Y);
    float g[16];
#pragma unroll
    for (int b = 0; b < 16; ++b) g[b] = 0.f;
    const float lr0 = sp.lr[4], lrN = sp.lr[5];

#pragma unroll
    for (int b = 0; b < NB; ++b) {
        issue(b + kShStages - 1);
        cp_async_wait<kShStages - 1>();  // this thread's copies of band b have landed
        const int sg = b % kShStages;
        float P[3], M[3], V[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            P[c] = st[sg][0][c][t];
            M[c] = MODE == 2 ? 0.f : st[sg][1][c][t];
            V[c] = ACCUM ? 0.f : st[sg][2][c][t];
        }
        float gb = 0.f;
#pragma unroll
        for (int c = 0; c < 3; ++c) gb = __fadd_rn(gb, __fmul_rn(vcol[c], P[c]));
        g[b] = gb;
        float* Pd = elem(b, 0);
        float* Md = elem(b, 1);
        if constexpr (MODE == 2) {
#pragma unroll
            for (int c = 0; c < 3; ++c) Md[32 * c] = Y[b] * vcol[c];  // the step's first view
        } else if constexpr (MODE == 1) {
#pragma unroll
            for (int c = 0; c < 3; ++c) Md[32 * c] = M[c] + Y[b] * vcol[c];  // running gradient sum
        } else {
            float* Vd = elem(b, 2);
            const float lr = b == 0 ? lr0 : lrN;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                adam_update(P[c], M[c], V[c], Y[b] * vcol[c], lr, a.b1, a.b2, a.eps);
                Pd[32 * c] = P[c];
                Md[32 * c] = M[c];
                Vd[32 * c] = V[c];
            }
        }
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
    float* pd = a.v_dir + tile_index(i, 3);
    pd[0] = vdir[0];
    pd[32] = vdir[1];
    pd[64] = vdir[2];
}

// Bounded to seven resident CTAs (72 registers, a little spilling to L1): with the Adam moments
// in shared memory the kernel spills less there than at six (80 registers); unbounded it takes 121.
template <int MODE>
__global__ void __launch_bounds__(kBwdThreads, 7)
bwd_geom_kernel(BwdGaussArgs a) {
    constexpr bool ACCUM = MODE != 0;
    __shared__ float s_mom[22][kBwdThreads];  // exp_avg x11 then exp_avg_sq x11 of this thread's row
    if (*a.skip_flag) return;  // uniform: the step overflowed
    const StepParams& sp = *a.step;
    const BwdGaussConst& k = sp.bwd;
    const int64_t ri = bwd_row(a, blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x);
    if (ri >= a.count) return;
    const int i = static_cast<int>(ri);
    const bool valid = a.valid[i] != 0;
    if (!valid && MODE == 2) {  // not seen by this view: zero gradients, zero visibility
        float* g0 = a.gacc[0] + tile_index(i, 3);
        float* g1 = a.gacc[1] + tile_index(i, 4);
        float* g2 = a.gacc[2] + tile_index(i, 3);
#pragma unroll
        for (int c = 0; c < 3; ++c) g0[c * 32] = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) g1[c * 32] = 0.f;
#pragma unroll
        for (int c = 0; c < 3; ++c) g2[c * 32] = 0.f;
        a.gacc[3][tile_index(i, 1)] = 0.f;
        a.gvis[tile_index(i, 1)] = 0.f;
        return;
    }
    if (!valid && (ACCUM || !sp.inject_noise)) return;
    float* pmean = a.means + tile_index(i, 3);
    float* pquat = a.quats + tile_index(i, 4);
    float* pscl = a.log_scales + tile_index(i, 3);
    float* popa = a.opac_logit + tile_index(i, 1);
    float mean[3] = {pmean[0], pmean[32], pmean[64]};
    float quat[4] = {pquat[0], pquat[32], pquat[64], pquat[96]};
    float lsc[3] = {pscl[0], pscl[32], pscl[64]};
    float olg = popa[0];

    if (valid) {
        const int64_t i3 = static_cast<int64_t>(i) * 3;
        const float vm2[2] = {a.v_means2d[i * 2], a.v_means2d[i * 2 + 1]};
        const float vcon[3] = {a.v_conics[i3], a.v_conics[i3 + 1], a.v_conics[i3 + 2]};
        float vop = a.v_opac[i];
        const float con[3] = {a.conics[i3], a.conics[i3 + 1], a.conics[i3 + 2]};
        const float comp = a.antialiased ? a.comps[i] : 0.f;
        const float* pd = a.v_dir + tile_index(i, 3);
        const float vdir[3] = {pd[0], pd[32], pd[64]};
        const float* pa = a.act + tile_index(i, 4);
        const float s[3] = {pa[0], pa[32], pa[64]};
        const float sig = pa[96];
        float* gm[4] = {a.m[0] + tile_index(i, 3), a.m[1] + tile_index(i, 4),
                        a.m[2] + tile_index(i, 3), a.m[3] + tile_index(i, 1)};
        float* gv[4] = {a.v[0] + tile_index(i, 3), a.v[1] + tile_index(i, 4),
                        a.v[2] + tile_index(i, 3), a.v[3] + tile_index(i, 1)};
        // both Adam moments of the four groups (11 components each) are copied into this
        // thread's shared-memory slots while the projection VJP runs, instead of holding 22
        // registers across it
        constexpr int kDimsG[4] = {3, 4, 3, 1};
        if constexpr (!ACCUM) {
            int j = 0;
#pragma unroll
            for (int g = 0; g < 4; ++g)
#pragma unroll
                for (int c = 0; c < kDimsG[g]; ++c, ++j) {
                    cp_async4(&s_mom[j][threadIdx.x], gm[g] + c * 32);
                    cp_async4(&s_mom[11 + j][threadIdx.x], gv[g] + c * 32);
                }
            cp_async_commit();
        }
        a.v_means2d[i * 2] = 0.f;  // consumed: zero for the next step's raster backward
        a.v_means2d[i * 2 + 1] = 0.f;
        a.v_conics[i3] = 0.f; a.v_conics[i3 + 1] = 0.f; a.v_conics[i3 + 2] = 0.f;
        a.v_opac[i] = 0.f;

        // ---- projection backward (C = 1)
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
            float gvs = o.v_scale[c] * s[c];
            if (!ACCUM && sp.scale_reg_w > 0.0f) gvs += sp.scale_reg_w * s[c];
            gs[c] = gvs;
        }
        float gop = vop * (sig * (1.0f - sig));
        if (!ACCUM && sp.opacity_reg_w > 0.0f) gop += sp.opacity_reg_w * sig * (1.0f - sig);
        float mm[3], mv[3], qm[4], qv[4], sm[3], sv[3], om = 0.f, ov = 0.f;
        if constexpr (!ACCUM) {
            cp_async_wait<0>();  // this thread's moment copies have landed
            const int t = threadIdx.x;
#pragma unroll
            for (int c = 0; c < 3; ++c) { mm[c] = s_mom[c][t]; mv[c] = s_mom[11 + c][t]; }
#pragma unroll
            for (int c = 0; c < 4; ++c) { qm[c] = s_mom[3 + c][t]; qv[c] = s_mom[14 + c][t]; }
#pragma unroll
            for (int c = 0; c < 3; ++c) { sm[c] = s_mom[7 + c][t]; sv[c] = s_mom[18 + c][t]; }
            om = s_mom[10][t];
            ov = s_mom[21][t];
        }
        if constexpr (ACCUM) {  // data-term gradients summed over the step's views
            float* g0 = a.gacc[0] + tile_index(i, 3);
            float* g1 = a.gacc[1] + tile_index(i, 4);
            float* g2 = a.gacc[2] + tile_index(i, 3);
            if constexpr (MODE == 2) {  // the step's first view writes
#pragma unroll
                for (int c = 0; c < 3; ++c) g0[c * 32] = o.v_mean[c] + vdir[c];
#pragma unroll
                for (int c = 0; c < 4; ++c) g1[c * 32] = o.v_quat[c];
#pragma unroll
                for (int c = 0; c < 3; ++c) g2[c * 32] = gs[c];
                a.gacc[3][tile_index(i, 1)] = gop;
                a.gvis[tile_index(i, 1)] = 1.0f;
            } else {
#pragma unroll
                for (int c = 0; c < 3; ++c) g0[c * 32] += o.v_mean[c] + vdir[c];
#pragma unroll
                for (int c = 0; c < 4; ++c) g1[c * 32] += o.v_quat[c];
#pragma unroll
                for (int c = 0; c < 3; ++c) g2[c * 32] += gs[c];
                a.gacc[3][tile_index(i, 1)] += gop;
                a.gvis[tile_index(i, 1)] += 1.0f;
            }
            return;
        }
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            adam_update(mean[c], mm[c], mv[c], o.v_mean[c] + vdir[c], sp.lr[0], a.b1, a.b2, a.eps);
            gm[0][c * 32] = mm[c];
            gv[0][c * 32] = mv[c];
            pmean[c * 32] = mean[c];
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            adam_update(quat[c], qm[c], qv[c], o.v_quat[c], sp.lr[1], a.b1, a.b2, a.eps);
            gm[1][c * 32] = qm[c];
            gv[1][c * 32] = qv[c];
            pquat[c * 32] = quat[c];
        }
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            adam_update(lsc[c], sm[c], sv[c], gs[c], sp.lr[2], a.b1, a.b2, a.eps);
            gm[2][c * 32] = sm[c];
            gv[2][c * 32] = sv[c];
            pscl[c * 32] = lsc[c];
        }
        adam_update(olg, om, ov, gop, sp.lr[3], a.b1, a.b2, a.eps);
        gm[3][0] = om;
        gv[3][0] = ov;
        popa[0] = olg;
    }
    if (sp.inject_noise) {
        const uint64_t nb0 = static_cast<uint64_t>(i) * 3;
        const float n3[3] = {normal_at(nb0, sp.noise_seed, sp.noise_offset),
                             normal_at(nb0 + 1, sp.noise_seed, sp.noise_offset),
                             normal_at(nb0 + 2, sp.noise_seed, sp.noise_offset)};
        perturb_one(mean, quat, lsc, olg, n3, sp.noise_scale, 0.005f, 100.f);
        pmean[0] = mean[0];
        pmean[32] = mean[1];
        pmean[64] = mean[2];
    }
}

// Row-major [n, d] staging rows <-> the resident 32-Gaussian tiles (rows r0 .. r0+n-1).
__global__ void __launch_bounds__(kThreads)
rows_to_tiles_kernel(const float* __restrict__ rows, float* __restrict__ tiles, int d, int64_t n,
                     int64_t r0) {
    const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (idx >= n * d) return;
    const int64_t r = idx / d;
    const int c = static_cast<int>(idx - r * d);
    tiles[tile_index(r0 + r, d) + c * 32] = rows[idx];
}

__global__ void __launch_bounds__(kThreads)
tiles_to_rows_kernel(const float* __restrict__ tiles, float* __restrict__ rows, int d, int64_t n,
                     int64_t r0) {
    const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (idx >= n * d) return;
    const int64_t r = idx / d;
    const int c = static_cast<int>(idx - r * d);
    rows[idx] = tiles[tile_index(r0 + r, d) + c * 32];
}

template <int KM1>
void launch_bwd_sh_t(const BwdGaussArgs& a, cudaStream_t s) {
    const unsigned blocks = blocks_for(bwd_threads(a), kBwdThreads);
    if (a.accumulate == 2)
        SX_LAUNCH((bwd_sh_kernel<KM1, 2>), blocks, kBwdThreads, 0, s, a);
    else if (a.accumulate == 1)
        SX_LAUNCH((bwd_sh_kernel<KM1, 1>), blocks, kBwdThreads, 0, s, a);
    else
        SX_LAUNCH((bwd_sh_kernel<KM1, 0>), blocks, kBwdThreads, 0, s, a);
}

// Adam over one shard of rows from accumulated gradients (view-parallel training): the mean over
// the step's views, the regularisers (recomputed activations, as in the fused backward), rows not
// visible in any view untouched, then the MCMC noise and the rows' accumulators re-zeroed.
template <int KM1>
__global__ void __launch_bounds__(kBwdThreads)
apply_grads_kernel(ApplyGradsArgs a) {
    const int64_t i = a.row_begin + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= a.row_end) return;
    constexpr int kDims[6] = {3, 4, 3, 1, 3, 3 * KM1};
    const bool upd = i < a.count && a.gvis[tile_index(i, 1)] > 0.f;
#pragma unroll
    for (int g = 0; g < 6; ++g) {
        if (kDims[g] == 0) continue;
        const int64_t b = tile_index(i, kDims[g]);
#pragma unroll
        for (int c = 0; c < kDims[g]; ++c) {
            const int64_t o = b + 32 * c;
            if (upd) {
                float grad = a.gacc[g][o] * a.inv_views;
                float p = a.p[g][o];
                if (g == 2 && a.scale_reg_w > 0.0f) grad += a.scale_reg_w * exp_cr(p);
                if (g == 3 && a.opacity_reg_w > 0.0f) {
                    const float sig = sigmoid_cr(p);
                    grad += a.opacity_reg_w * sig * (1.0f - sig);
                }
                float m = a.m[g][o], v = a.v[g][o];
                adam_update(p, m, v, grad, a.lr[g], a.b1, a.b2, a.eps);
                a.p[g][o] = p;
                a.m[g][o] = m;
                a.v[g][o] = v;
            }
            a.gacc[g][o] = 0.f;
        }
    }
    a.gvis[tile_index(i, 1)] = 0.f;
    if (a.inject_noise && i < a.count) {
        float* pmean = a.p[0] + tile_index(i, 3);
        const float* pquat = a.p[1] + tile_index(i, 4);
        const float* pscl = a.p[2] + tile_index(i, 3);
        float mean[3] = {pmean[0], pmean[32], pmean[64]};
        const float quat[4] = {pquat[0], pquat[32], pquat[64], pquat[96]};
        const float lsc[3] = {pscl[0], pscl[32], pscl[64]};
        const uint64_t nb0 = static_cast<uint64_t>(i) * 3;
        const float n3[3] = {normal_at(nb0, a.noise_seed, a.noise_offset),
                             normal_at(nb0 + 1, a.noise_seed, a.noise_offset),
                             normal_at(nb0 + 2, a.noise_seed, a.noise_offset)};
        perturb_one(mean, quat, lsc, a.p[3][tile_index(i, 1)], n3, a.noise_scale, 0.005f, 100.f);
        pmean[0] = mean[0];
        pmean[32] = mean[1];
        pmean[64] = mean[2];
    }
}

// Owner-shard reduce + Adam + broadcast over peer memory (launch_exchange_apply). A thread owns 4
// consecutive rows, i.e. one float4 of every 32-float component run of their tile, so each peer
// load or store moves 16 bytes and a warp's requests cover whole 128-byte lines. The W ranks'
// gradients of a chunk of components are all requested before the first is used: W x kChunk
// independent NVLink loads per thread are in flight instead of one round trip per component.
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, const float4& v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ float& el(float4& v, int k) { return reinterpret_cast<float*>(&v)[k]; }

template <int KM1, int W>
__global__ void __launch_bounds__(kBwdThreads)
exchange_apply_kernel(PeerApplyArgs x) {
    const ApplyGradsArgs& a = x.a;
    const int64_t i0 =
        a.row_begin + (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) * 4;
    if (i0 >= a.row_end) return;
    if (x.status && *x.status != 0) return;  // a wait of this step ran out: change nothing
    constexpr int kDims[6] = {3, 4, 3, 1, 3, 3 * KM1};
    constexpr int kChunk = W >= 16 ? 1 : 16 / W;
    float4 vis = ld4(x.gvis[0] + i0);  // the opacity-like layout: row i at float i
#pragma unroll
    for (int r = 1; r < W; ++r) {
        const float4 t = ld4(x.gvis[r] + i0);
        vis.x += t.x;
        vis.y += t.y;
        vis.z += t.z;
        vis.w += t.w;
    }
    bool upd[4];
    bool any = false;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        upd[k] = i0 + k < a.count && el(vis, k) > 0.f;
        any |= upd[k];
    }
    const int64_t bmean = tile_index(i0, 3);
    float4 mean4[3];
    if (any) {
#pragma unroll
        for (int g = 0; g < 6; ++g) {
            const int d = kDims[g];
            if (d == 0) continue;
            const int64_t base = tile_index(i0, d);
#pragma unroll
            for (int c0 = 0; c0 < d; c0 += kChunk) {
                float4 parts[kChunk][W];
#pragma unroll
                for (int cc = 0; cc < kChunk; ++cc)
                    if (c0 + cc < d) {
#pragma unroll
                        for (int r = 0; r < W; ++r)
                            parts[cc][r] = ld4(x.gacc[r][g] + base + 32 * (c0 + cc));
                    }
#pragma unroll
                for (int cc = 0; cc < kChunk; ++cc) {
                    const int c = c0 + cc;
                    if (c >= d) continue;
                    const int64_t o = base + 32 * c;
                    float4 sum = parts[cc][0];
#pragma unroll
                    for (int r = 1; r < W; ++r) {  // rank order
                        sum.x += parts[cc][r].x;
                        sum.y += parts[cc][r].y;
                        sum.z += parts[cc][r].z;
                        sum.w += parts[cc][r].w;
                    }
                    float4 p = ld4(a.p[g] + o), m = ld4(a.m[g] + o), v = ld4(a.v[g] + o);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if (!upd[k]) continue;
                        float grad = el(sum, k) * a.inv_views;
                        float& pk = el(p, k);
                        if (g == 2 && a.scale_reg_w > 0.0f) grad += a.scale_reg_w * exp_cr(pk);
                        if (g == 3 && a.opacity_reg_w > 0.0f) {
                            const float sig = sigmoid_cr(pk);
                            grad += a.opacity_reg_w * sig * (1.0f - sig);
                        }
                        adam_update(pk, el(m, k), el(v, k), grad, a.lr[g], a.b1, a.b2, a.eps);
                    }
                    st4(a.m[g] + o, m);
                    st4(a.v[g] + o, v);
                    if (g == 0) {  // the means go out after the noise
                        st4(a.p[0] + o, p);
                        mean4[c] = p;
                    } else {
#pragma unroll
                        for (int r = 0; r < W; ++r) st4(x.params[r][g] + o, p);
                    }
                }
            }
        }
    }
    bool noisy = false;
    if (a.inject_noise) {
        if (!any) {
#pragma unroll
            for (int c = 0; c < 3; ++c) mean4[c] = ld4(a.p[0] + bmean + 32 * c);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t i = i0 + k;
            if (i >= a.count) continue;
            noisy = true;
            const float* pquat = a.p[1] + tile_index(i, 4);
            const float* pscl = a.p[2] + tile_index(i, 3);
            float mean[3] = {el(mean4[0], k), el(mean4[1], k), el(mean4[2], k)};
            const float quat[4] = {pquat[0], pquat[32], pquat[64], pquat[96]};
            const float lsc[3] = {pscl[0], pscl[32], pscl[64]};
            const uint64_t nb0 = static_cast<uint64_t>(i) * 3;
            const float n3[3] = {normal_at(nb0, a.noise_seed, a.noise_offset),
                                 normal_at(nb0 + 1, a.noise_seed, a.noise_offset),
                                 normal_at(nb0 + 2, a.noise_seed, a.noise_offset)};
            perturb_one(mean, quat, lsc, a.p[3][tile_index(i, 1)], n3, a.noise_scale, 0.005f,
                        100.f);
#pragma unroll
            for (int c = 0; c < 3; ++c) el(mean4[c], k) = mean[c];
        }
    }
    if (any || noisy) {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int r = 0; r < W; ++r) st4(x.params[r][0] + bmean + 32 * c, mean4[c]);
    }
    // release this thread's peer stores at system scope before the caller's cross-rank barrier
    // (the peers' next kernels read these rows once the barrier has completed)
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

template <int KM1>
void launch_exchange_t(const PeerApplyArgs& x, unsigned blocks, cudaStream_t s) {
    void (*k)(PeerApplyArgs) = nullptr;
    switch (x.world) {
        case 1: k = exchange_apply_kernel<KM1, 1>; break;
        case 2: k = exchange_apply_kernel<KM1, 2>; break;
        case 3: k = exchange_apply_kernel<KM1, 3>; break;
        case 4: k = exchange_apply_kernel<KM1, 4>; break;
        case 5: k = exchange_apply_kernel<KM1, 5>; break;
        case 6: k = exchange_apply_kernel<KM1, 6>; break;
        case 7: k = exchange_apply_kernel<KM1, 7>; break;
        case 8: k = exchange_apply_kernel<KM1, 8>; break;
        default: throw_invalid("exchange_apply", "world must be in [1, 8]");
    }
    SX_LAUNCH(k, blocks, kBwdThreads, 0, s, x);
}

// Cross-GPU barrier (launch_peer_barrier): thread t signals rank t, then waits for rank t's
// signal in this rank's own array. Polls are bounded (kPeerBarrierPolls, ~1 s); a wait that runs
// out records kStatusPeerBarrierTimeout and returns.
constexpr uint32_t kPeerBarrierPolls = 1u << 23;

__global__ void peer_barrier_kernel(PeerBarrierArgs b) {
    const int t = threadIdx.x;
    if (t < b.world) {
        uint32_t* slot = b.flags[t] + b.rank;
        asm volatile("fence.acq_rel.sys;" ::: "memory");  // this rank's earlier writes first
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(slot), "r"(b.epoch) : "memory");
    }
    __syncwarp();
    if (t < b.world) {
        const uint32_t* mine = b.flags[b.rank] + t;
        uint32_t v = 0;
        uint32_t polls = 0;
        for (;;) {
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if (static_cast<int32_t>(v - b.epoch) >= 0) break;
            if (++polls >= kPeerBarrierPolls) {
                atomicOr(b.status, kStatusPeerBarrierTimeout);
                break;
            }
            __nanosleep(128);
        }
    }
}

// MCMC position noise on the resident rows [0, count) outside a step (the refine step's noise runs
// after the refine, on the grown count; Trainer.cpp:966 -> mcmc_inject_noise, Trainer.cpp:1396).
__global__ void __launch_bounds__(kThreads)
noise_rows_kernel(float* __restrict__ means, const float* __restrict__ quats,
                  const float* __restrict__ log_scales, const float* __restrict__ opac_logit,
                  int64_t count, uint64_t seed, uint64_t offset, float noise_scale) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= count) return;
    float* pmean = means + tile_index(i, 3);
    const float* pquat = quats + tile_index(i, 4);
    const float* pscl = log_scales + tile_index(i, 3);
    float mean[3] = {pmean[0], pmean[32], pmean[64]};
    const float quat[4] = {pquat[0], pquat[32], pquat[64], pquat[96]};
    const float lsc[3] = {pscl[0], pscl[32], pscl[64]};
    const uint64_t nb0 = static_cast<uint64_t>(i) * 3;
    const float n3[3] = {normal_at(nb0, seed, offset), normal_at(nb0 + 1, seed, offset),
                         normal_at(nb0 + 2, seed, offset)};
    perturb_one(mean, quat, lsc, opac_logit[tile_index(i, 1)], n3, noise_scale, 0.005f, 100.f);
    pmean[0] = mean[0];
    pmean[32] = mean[1];
    pmean[64] = mean[2];
}

// ---- MCMC refine surgery on the tiled arena (one thread per row or per row element) ----
__global__ void __launch_bounds__(kThreads)
gather_log_scales_kernel(const float* __restrict__ ls, const int64_t* __restrict__ idx, int64_t n,
                         float* __restrict__ out) {
    const int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (j >= n) return;
    const int64_t b = tile_index(idx[j], 3);
    out[j * 3] = ls[b];
    out[j * 3 + 1] = ls[b + 32];
    out[j * 3 + 2] = ls[b + 64];
}

__global__ void __launch_bounds__(kThreads)
write_sources_kernel(float* __restrict__ op, float* __restrict__ ls, const int64_t* __restrict__ idx,
                     const float* __restrict__ logits, const float* __restrict__ lsn, int64_t n) {
    const int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (j >= n) return;
    const int64_t r = idx[j];
    op[tile_index(r, 1)] = logits[j];
    const int64_t b = tile_index(r, 3);
    ls[b] = lsn[j * 3];
    ls[b + 32] = lsn[j * 3 + 1];
    ls[b + 64] = lsn[j * 3 + 2];
}

// thread (j, e): element e of the concatenated row (59 floats at SH degree 3)
__global__ void __launch_bounds__(kThreads)
copy_rows_kernel(RowCopyArgs a, const int64_t* __restrict__ dst, const int64_t* __restrict__ src,
                 int64_t n, int row_floats) {
    const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (t >= n * row_floats) return;
    const int64_t j = t / row_floats;
    int e = static_cast<int>(t - j * row_floats);
    int g = 0;
    while (e >= a.dims[g]) e -= a.dims[g++];
    const int d = a.dims[g];
    a.p[g][tile_index(dst[j], d) + 32 * e] = a.p[g][tile_index(src[j], d) + 32 * e];
}

__global__ void __launch_bounds__(kThreads)
zero_moment_rows_kernel(MomentRowsArgs a, const int64_t* __restrict__ idx, int64_t n,
                        int row_floats) {
    const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (t >= n * row_floats) return;
    const int64_t j = t / row_floats;
    int e = static_cast<int>(t - j * row_floats);
    int g = 0;
    while (e >= a.dims[g]) e -= a.dims[g++];
    const int64_t o = tile_index(idx[j], a.dims[g]) + 32 * e;
    a.m[g][o] = 0.f;
    a.v[g][o] = 0.f;
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

void launch_rows_to_tiles(const float* rows, float* tiles, int d, int64_t n, int64_t r0,
                          cudaStream_t s) {
    if (n * d == 0) return;
    SX_LAUNCH(rows_to_tiles_kernel, blocks_for(n * d, kThreads), kThreads, 0, s, rows, tiles, d, n,
              r0);
}

void launch_tiles_to_rows(const float* tiles, float* rows, int d, int64_t n, int64_t r0,
                          cudaStream_t s) {
    if (n * d == 0) return;
    SX_LAUNCH(tiles_to_rows_kernel, blocks_for(n * d, kThreads), kThreads, 0, s, tiles, rows, d, n,
              r0);
}

void launch_noise_rows(float* means, const float* quats, const float* log_scales,
                       const float* opac_logit, int64_t count, uint64_t seed, uint64_t offset,
                       float noise_scale, cudaStream_t s) {
    if (count <= 0) return;
    SX_LAUNCH(noise_rows_kernel, blocks_for(count, kThreads), kThreads, 0, s, means, quats,
              log_scales, opac_logit, count, seed, offset, noise_scale);
}

void launch_gather_log_scales(const float* log_scales, const int64_t* idx, int64_t n, float* out,
                              cudaStream_t s) {
    if (n <= 0) return;
    SX_LAUNCH(gather_log_scales_kernel, blocks_for(n, kThreads), kThreads, 0, s, log_scales, idx, n,
              out);
}

void launch_write_sources(float* opac_logit, float* log_scales, const int64_t* idx,
                          const float* logits, const float* log_scales_new, int64_t n,
                          cudaStream_t s) {
    if (n <= 0) return;
    SX_LAUNCH(write_sources_kernel, blocks_for(n, kThreads), kThreads, 0, s, opac_logit, log_scales,
              idx, logits, log_scales_new, n);
}

void launch_copy_rows(const RowCopyArgs& a, const int64_t* dst, const int64_t* src, int64_t n,
                      cudaStream_t s) {
    int row = 0;
    for (int g = 0; g < 6; ++g) row += a.dims[g];
    if (n <= 0 || row == 0) return;
    SX_LAUNCH(copy_rows_kernel, blocks_for(n * row, kThreads), kThreads, 0, s, a, dst, src, n, row);
}

void launch_zero_moment_rows(const MomentRowsArgs& a, const int64_t* idx, int64_t n, cudaStream_t s) {
    int row = 0;
    for (int g = 0; g < 6; ++g) row += a.dims[g];
    if (n <= 0 || row == 0) return;
    SX_LAUNCH(zero_moment_rows_kernel, blocks_for(n * row, kThreads), kThreads, 0, s, a, idx, n, row);
}

void launch_exchange_apply(const PeerApplyArgs& x, cudaStream_t s) {
    const int64_t n = x.a.row_end - x.a.row_begin;
    if (n <= 0) return;
    if (x.world < 1 || x.world > kMaxPeers || x.rank < 0 || x.rank >= x.world)
        throw_invalid("exchange_apply", "world must be in [1, 8] and rank in [0, world)");
    if (x.a.row_begin % 32 || x.a.row_end % 32)
        throw_invalid("exchange_apply", "rows must be whole 32-row tiles");
    const unsigned blocks = blocks_for(n / 4, kBwdThreads);
    switch (x.a.K) {
        case 1: launch_exchange_t<0>(x, blocks, s); break;
        case 4: launch_exchange_t<3>(x, blocks, s); break;
        case 9: launch_exchange_t<8>(x, blocks, s); break;
        case 16: launch_exchange_t<15>(x, blocks, s); break;
        default: throw_invalid("exchange_apply", "K must be 1, 4, 9 or 16");
    }
}

void launch_peer_barrier(const PeerBarrierArgs& b, cudaStream_t s) {
    if (b.world < 1 || b.world > kMaxPeers || b.rank < 0 || b.rank >= b.world)
        throw_invalid("peer_barrier", "world must be in [1, 8] and rank in [0, world)");
    if (!b.status) throw_invalid("peer_barrier", "null status word");
    for (int r = 0; r < b.world; ++r)
        if (!b.flags[r]) throw_invalid("peer_barrier", "a rank's flag array is not mapped");
    SX_LAUNCH(peer_barrier_kernel, 1, 32, 0, s, b);
}

uint32_t peer_barrier_selftest(int world, int* applied) {
    if (world < 1 || world > kMaxPeers) throw_invalid("peer_barrier_selftest", "world must be in [1, 8]");
    // one allocation: world flag arrays, the status word (padded to 16 bytes), then a 32-row SH
    // degree 0 arena — parameters, both moments and accumulated gradients of the five groups, and
    // the visibility
    constexpr int kRows = 32;
    constexpr int kDims[5] = {3, 4, 3, 1, 3};
    const size_t flag_words = static_cast<size_t>(world) * kMaxPeers;
    const size_t head = (flag_words + 1 + 3) / 4 * 4;  // floats after the flags + status
    size_t arena = 0;
    for (int d : kDims) arena += static_cast<size_t>(kRows) * d;
    const size_t words = head + 4 * arena + kRows;
    uint32_t* buf = nullptr;
    cuda_check(cudaMalloc(&buf, words * sizeof(uint32_t)), "selftest alloc");
    uint32_t status = 0;
    cudaStream_t s = nullptr;
    try {
        cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "selftest stream");
        cuda_check(cudaMemsetAsync(buf, 0, words * sizeof(uint32_t), s), "selftest zero");
        float* f = reinterpret_cast<float*>(buf + head);
        ApplyGradsArgs a{};
        size_t off = 0;
        for (int g = 0; g < 5; ++g) {
            const size_t n = static_cast<size_t>(kRows) * kDims[g];
            a.p[g] = f + off;
            a.m[g] = f + off + arena;
            a.v[g] = f + off + 2 * arena;
            a.gacc[g] = f + off + 3 * arena;
            off += n;
        }
        a.gvis = f + 4 * arena;
        std::vector<float> ones(arena + kRows, 1.0f);  // gradients and visibility 1
        cuda_check(cudaMemcpyAsync(a.gacc[0], ones.data(), ones.size() * sizeof(float),
                                   cudaMemcpyHostToDevice, s),
                   "selftest grads");
        a.K = 1;
        a.row_begin = 0;
        a.row_end = kRows;
        a.count = kRows;
        a.inv_views = 1.0f;
        for (int g = 0; g < 6; ++g) a.lr[g] = 1.0f;
        a.b1 = 0.9f;
        a.b2 = 0.999f;
        a.eps = 1e-15f;

        PeerBarrierArgs b{};
        b.world = world;
        b.rank = 0;
        b.epoch = 1;
        for (int r = 0; r < world; ++r) b.flags[r] = buf + static_cast<size_t>(r) * kMaxPeers;
        b.status = buf + flag_words;
        launch_peer_barrier(b, s);
        // what step_exchange enqueues after a barrier: this rank's exchange (a world of one: its
        // own buffers)
        PeerApplyArgs x{};
        x.a = a;
        x.world = 1;
        x.rank = 0;
        for (int g = 0; g < 5; ++g) {
            x.gacc[0][g] = a.gacc[g];
            x.params[0][g] = a.p[g];
        }
        x.gvis[0] = a.gvis;
        x.status = b.status;
        launch_exchange_apply(x, s);
        std::vector<float> back(arena * 4 + kRows);
        cuda_check(cudaMemcpyAsync(back.data(), f, back.size() * sizeof(float), cudaMemcpyDeviceToHost, s),
                   "selftest read");
        cuda_check(cudaMemcpyAsync(&status, b.status, sizeof(status), cudaMemcpyDeviceToHost, s),
                   "selftest status");
        cuda_check(cudaStreamSynchronize(s), "selftest sync");
        bool changed = false;
        for (size_t i = 0; i < arena; ++i) changed |= back[i] != 0.0f;
        if (applied) *applied = changed ? 1 : 0;
    } catch (...) {
        if (s) cudaStreamDestroy(s);
        cudaFree(buf);
        throw;
    }
    cudaStreamDestroy(s);
    cudaFree(buf);
    return status;
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
    switch (a.K) {
        case 1: launch_bwd_sh_t<0>(a, s); break;
        case 4: launch_bwd_sh_t<3>(a, s); break;
        case 9: launch_bwd_sh_t<8>(a, s); break;
        case 16: launch_bwd_sh_t<15>(a, s); break;
        default: throw_invalid("bwd_gauss", "K must be 1, 4, 9 or 16");
    }
    if (a.accumulate < 0 || a.accumulate > 2) throw_invalid("bwd_gauss", "accumulate mode must be 0, 1 or 2");
    const unsigned blocks = blocks_for(bwd_threads(a), kBwdThreads);
    if (a.accumulate == 2)
        SX_LAUNCH(bwd_geom_kernel<2>, blocks, kBwdThreads, 0, s, a);
    else if (a.accumulate == 1)
        SX_LAUNCH(bwd_geom_kernel<1>, blocks, kBwdThreads, 0, s, a);
    else
        SX_LAUNCH(bwd_geom_kernel<0>, blocks, kBwdThreads, 0, s, a);
}

void launch_apply_grads(const ApplyGradsArgs& a, cudaStream_t s) {
    const int64_t n = a.row_end - a.row_begin;
    if (n <= 0) return;
    const unsigned blocks = blocks_for(n, kBwdThreads);
    switch (a.K) {
        case 1: SX_LAUNCH(apply_grads_kernel<0>, blocks, kBwdThreads, 0, s, a); break;
        case 4: SX_LAUNCH(apply_grads_kernel<3>, blocks, kBwdThreads, 0, s, a); break;
        case 9: SX_LAUNCH(apply_grads_kernel<8>, blocks, kBwdThreads, 0, s, a); break;
        case 16: SX_LAUNCH(apply_grads_kernel<15>, blocks, kBwdThreads, 0, s, a); break;
        default: throw_invalid("apply_grads", "K must be 1, 4, 9 or 16");
    }
}

}  // namespace sx
