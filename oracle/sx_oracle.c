/*
 * sx_oracle.c — CPU oracle of the 3DGS training step. TEST INFRASTRUCTURE (see sx_oracle.h):
 * used only as the checker in tests/ and smoke(), and as the timed CPU reference in bench.py.
 *
 * Build: gcc -O2 -std=c11 -ffp-contract=off -fPIC -shared (no fast-math, no FMA contraction):
 * every expression rounds like the reference's x86-64 CPU build; std::fma becomes fmaf, and
 * std::exp/log/sqrt on floats become glibc expf/logf/sqrtf exactly as in the reference.
 * Float-to-int conversions of tile bounds saturate (the behaviour of arm64, where the reference's
 * goldens were produced, and of CUDA), instead of relying on C's undefined behaviour.
 */
#include "sx_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#define K_ALPHA_THRESHOLD (1.f / 255.f)
#define K_GAUSSIAN_EXTEND 3.33f
#define K_MIN_COMPENSATION 0.005f
#define K_MAX_ALPHA 0.99f
#define K_TRANSMITTANCE_THRESHOLD 1e-4f
#define K_MIN_ONE_MINUS_ALPHA 1e-6f
#define K_SSIM_C1 1e-4f
#define K_SSIM_C2 9e-4f

/* 11-tap Gaussian window, sigma 1.5, normalised in f64 then rounded to f32 (built at first use). */
static float g_ssim_taps[11];
static int g_taps_ready = 0;
static void ssim_taps(void) {
    if (g_taps_ready) return;
    double w[11], s = 0.0;
    for (int i = 0; i < 11; i++) {
        w[i] = exp(-((double)(i - 5) * (i - 5)) / 4.5);
        s += w[i];
    }
    for (int i = 0; i < 11; i++) g_ssim_taps[i] = (float)(w[i] / s);
    g_taps_ready = 1;
}

static inline float smin(float a, float b) { return (b < a) ? b : a; }
static inline float smax(float a, float b) { return (a < b) ? b : a; }
static inline int imin(int a, int b) { return a < b ? a : b; }
static inline int imax(int a, int b) { return a > b ? a : b; }

/* float -> int truncation with saturation (NaN -> 0). */
static inline int f2i(float x) {
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x <= -2147483648.0f) return INT32_MIN;
    return (int)x;
}

#ifdef _OPENMP
#include <omp.h>
#endif

int32_t sxo_set_threads(int32_t n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

uint32_t sxo_bits_for_count(int64_t count) {
    if (count <= 1) return 0u;
    uint32_t bits = 0;
    for (uint64_t v = (uint64_t)count - 1u; v != 0; v >>= 1) bits++;
    return bits;
}

/* ---------------------------------------------------------------------------------------------
 * fused_adam — CpuKernels.cpp:127-146 (AdamCUDA semantics: no bias correction, eps outside the
 * sqrt, rows with valid==0 skipped entirely).
 * ------------------------------------------------------------------------------------------- */
void sxo_fused_adam(float* p, const float* g, float* m, float* v, const uint8_t* valid,
                    int64_t n, int64_t n_gauss, float lr, float b1, float b2, float eps) {
    if (n == 0) return;
    const int64_t D = n / n_gauss;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        if (valid && valid[i / D] == 0) continue;
        const float gi = g[i];
        float mi = m[i], vi = v[i];
        mi = b1 * mi + (1.0f - b1) * gi;
        vi = b2 * vi + (1.0f - b2) * gi * gi;
        const float step = -lr * mi / (sqrtf(vi) + eps);
        p[i] += step;
        m[i] = mi;
        v[i] = vi;
    }
}

/* ---------------------------------------------------------------------------------------------
 * projection_fused_fwd — CpuKernels.cpp:168-273 with the quat/scale covariance of
 * Math.cpp:9-44 (normalise by division, R diag(s) (R diag(s))^T, sequential 3-term sums).
 * ------------------------------------------------------------------------------------------- */
static void mat3_mul(const float* a, const float* b, float* c) {
    for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++) {
            float s = 0.f;
            for (int k = 0; k < 3; k++) s += a[i * 3 + k] * b[k * 3 + j];
            c[i * 3 + j] = s;
        }
}
static void mat3_t(const float* a, float* t) {
    for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++) t[i * 3 + j] = a[j * 3 + i];
}
static void quat_scale_covar(const float* q, const float* s, float* C) {
    float w = q[0], x = q[1], y = q[2], z = q[3];
    const float n = sqrtf(w * w + x * x + y * y + z * z);
    if (n > 0.0f) {
        w /= n;
        x /= n;
        y /= n;
        z /= n;
    }
    float M[9];
    M[0] = 1 - 2 * (y * y + z * z); M[1] = 2 * (x * y - w * z); M[2] = 2 * (x * z + w * y);
    M[3] = 2 * (x * y + w * z); M[4] = 1 - 2 * (x * x + z * z); M[5] = 2 * (y * z - w * x);
    M[6] = 2 * (x * z - w * y); M[7] = 2 * (y * z + w * x); M[8] = 1 - 2 * (x * x + y * y);
    for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++) M[i * 3 + j] *= s[j];
    float Mt[9];
    mat3_t(M, Mt);
    mat3_mul(M, Mt, C);
}

void sxo_projection_fused_fwd(const float* means, const float* covars6, const float* quats,
                              const float* scales, const float* opacities, const float* viewmats,
                              const float* Ks, int64_t N, int64_t C, int32_t width, int32_t height,
                              float eps2d, float near_plane, float far_plane, float radius_clip,
                              int32_t calc_comp, int32_t* radii, float* means2d, float* depths,
                              float* conics, float* comps) {
    for (int64_t c = 0; c < C; c++) {
        const float* V = viewmats + c * 16;
        const float R[9] = {V[0], V[1], V[2], V[4], V[5], V[6], V[8], V[9], V[10]};
        const float t[3] = {V[3], V[7], V[11]};
        const float* K = Ks + c * 9;
        const float fx = K[0], fy = K[4], cx = K[2], cy = K[5];
        const float tan_fovx = 0.5f * (float)width / fx;
        const float tan_fovy = 0.5f * (float)height / fy;
        const float lim_x_pos = ((float)width - cx) / fx + 0.3f * tan_fovx;
        const float lim_x_neg = cx / fx + 0.3f * tan_fovx;
        const float lim_y_pos = ((float)height - cy) / fy + 0.3f * tan_fovy;
        const float lim_y_neg = cy / fy + 0.3f * tan_fovy;
        float Rt[9];
        mat3_t(R, Rt);
#pragma omp parallel for schedule(static)
        for (int64_t n = 0; n < N; n++) {
            const int64_t gi = c * N + n;
            const float* mw = means + n * 3;
            const float mx = R[0] * mw[0] + R[1] * mw[1] + R[2] * mw[2] + t[0];
            const float my = R[3] * mw[0] + R[4] * mw[1] + R[5] * mw[2] + t[1];
            const float mz = R[6] * mw[0] + R[7] * mw[1] + R[8] * mw[2] + t[2];
            if (mz < near_plane || mz > far_plane) continue;
            float Cw[9];
            if (covars6) {
                const float* cv = covars6 + n * 6;
                const float tmp[9] = {cv[0], cv[1], cv[2], cv[1], cv[3], cv[4], cv[2], cv[4], cv[5]};
                memcpy(Cw, tmp, sizeof(tmp));
            } else {
                quat_scale_covar(quats + n * 4, scales + n * 3, Cw);
            }
            float RC[9], Cc[9];
            mat3_mul(R, Cw, RC);
            mat3_mul(RC, Rt, Cc);
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
            c00 += eps2d;
            c11 += eps2d;
            const float det = c00 * c11 - c01 * c10;
            const float comp = sqrtf(smax(K_MIN_COMPENSATION * K_MIN_COMPENSATION, det_orig / det));
            if (det <= 0.0f) continue;
            const float rdet = 1.0f / det;
            float extend = K_GAUSSIAN_EXTEND;
            if (opacities) {
                float op = opacities[n];
                if (calc_comp) op *= comp;
                if (op < K_ALPHA_THRESHOLD) continue;
                extend = smin(K_GAUSSIAN_EXTEND, sqrtf(2.0f * logf(op / K_ALPHA_THRESHOLD)));
            }
            const float rx = ceilf(extend * sqrtf(c00));
            const float ry = ceilf(extend * sqrtf(c11));
            if (rx <= radius_clip && ry <= radius_clip) continue;
            if (m2x + rx <= 0.0f || m2x - rx >= (float)width || m2y + ry <= 0.0f ||
                m2y - ry >= (float)height)
                continue;
            radii[gi * 2] = (int32_t)rx;
            radii[gi * 2 + 1] = (int32_t)ry;
            means2d[gi * 2] = m2x;
            means2d[gi * 2 + 1] = m2y;
            depths[gi] = mz;
            conics[gi * 3] = c11 * rdet;
            conics[gi * 3 + 1] = -c10 * rdet;
            conics[gi * 3 + 2] = c00 * rdet;
            if (calc_comp) comps[gi] = comp;
        }
    }
}

/* ---------------------------------------------------------------------------------------------
 * projection_fused_bwd — restated from the gsplat VJP chain (ProjectionEWA.metal:186-560; the
 * reference has no CPU backward): conic inverse VJP, optional compensation VJP, perspective VJP
 * with the FOV clamp branch, world->camera VJPs, quaternion/scale covariance VJP with the
 * normalisation projection. Accumulates into zeroed outputs; culled (radii<=0) slots contribute 0.
 * ------------------------------------------------------------------------------------------- */
void sxo_projection_fused_bwd(const float* means, const float* covars6, const float* quats,
                              const float* scales, const float* viewmats, const float* Ks,
                              int64_t N, int64_t C, int32_t width, int32_t height, float eps2d,
                              const int32_t* radii, const float* conics, const float* comps,
                              const float* v_means2d, const float* v_depths, const float* v_conics,
                              const float* v_comps, float* v_means, float* v_covars,
                              float* v_quats, float* v_scales, float* v_viewmats) {
    for (int64_t c = 0; c < C; c++) {
        const float* V = viewmats + c * 16;
        const float R[9] = {V[0], V[1], V[2], V[4], V[5], V[6], V[8], V[9], V[10]};
        const float t[3] = {V[3], V[7], V[11]};
        const float* K = Ks + c * 9;
        const float fx = K[0], fy = K[4], cx = K[2], cy = K[5];
        const float Wf = (float)width, Hf = (float)height;
        const float tan_fovx = 0.5f * Wf / fx, tan_fovy = 0.5f * Hf / fy;
        const float lxp = (Wf - cx) / fx + 0.3f * tan_fovx, lxn = cx / fx + 0.3f * tan_fovx;
        const float lyp = (Hf - cy) / fy + 0.3f * tan_fovy, lyn = cy / fy + 0.3f * tan_fovy;
        /* rows are disjoint per Gaussian when there is one camera and no pose gradient */
#pragma omp parallel for schedule(static) if (C == 1 && v_viewmats == NULL)
        for (int64_t n = 0; n < N; n++) {
            const int64_t gi = c * N + n;
            if (!(radii[gi * 2] > 0 && radii[gi * 2 + 1] > 0)) continue;
            const float* cn = conics + gi * 3;
            const float* vc = v_conics + gi * 3;
            /* v_cov2d = -conic * [[va, vb/2], [vb/2, vc]] * conic */
            const float A[4] = {cn[0], cn[1], cn[1], cn[2]};
            const float Vv[4] = {vc[0], vc[1] * 0.5f, vc[1] * 0.5f, vc[2]};
            float P[4], vM[4];
            P[0] = A[0] * Vv[0] + A[1] * Vv[2]; P[1] = A[0] * Vv[1] + A[1] * Vv[3];
            P[2] = A[2] * Vv[0] + A[3] * Vv[2]; P[3] = A[2] * Vv[1] + A[3] * Vv[3];
            vM[0] = -(P[0] * A[0] + P[1] * A[2]); vM[1] = -(P[0] * A[1] + P[1] * A[3]);
            vM[2] = -(P[2] * A[0] + P[3] * A[2]); vM[3] = -(P[2] * A[1] + P[3] * A[3]);
            if (v_comps) {
                const float comp = comps[gi];
                const float det_cb = A[0] * A[3] - A[1] * A[2];
                const float vs = v_comps[gi] * 0.5f / (comp + 1e-6f);
                const float omc = 1.f - comp * comp;
                vM[0] += vs * (omc * A[0] - eps2d * det_cb);
                vM[1] += vs * (omc * A[1]);
                vM[2] += vs * (omc * A[2]);
                vM[3] += vs * (omc * A[3] - eps2d * det_cb);
            }
            /* forward recomputation */
            float Cw[9], Rq[9] = {0}, M[9] = {0}, qn[4] = {0}, inv_norm = 0.f;
            if (covars6) {
                const float* cv = covars6 + n * 6;
                const float tmp[9] = {cv[0], cv[1], cv[2], cv[1], cv[3], cv[4], cv[2], cv[4], cv[5]};
                memcpy(Cw, tmp, sizeof(tmp));
            } else {
                const float* q = quats + n * 4;
                float w = q[0], x = q[1], y = q[2], z = q[3];
                inv_norm = 1.0f / sqrtf(x * x + y * y + z * z + w * w);
                w *= inv_norm; x *= inv_norm; y *= inv_norm; z *= inv_norm;
                qn[0] = w; qn[1] = x; qn[2] = y; qn[3] = z;
                Rq[0] = 1.f - 2.f * (y * y + z * z); Rq[1] = 2.f * (x * y - w * z); Rq[2] = 2.f * (x * z + w * y);
                Rq[3] = 2.f * (x * y + w * z); Rq[4] = 1.f - 2.f * (x * x + z * z); Rq[5] = 2.f * (y * z - w * x);
                Rq[6] = 2.f * (x * z - w * y); Rq[7] = 2.f * (y * z + w * x); Rq[8] = 1.f - 2.f * (x * x + y * y);
                const float* s = scales + n * 3;
                for (int i = 0; i < 3; i++)
                    for (int j = 0; j < 3; j++) M[i * 3 + j] = Rq[i * 3 + j] * s[j];
                float Mt[9];
                mat3_t(M, Mt);
                mat3_mul(M, Mt, Cw);
            }
            const float* mw = means + n * 3;
            const float x = R[0] * mw[0] + R[1] * mw[1] + R[2] * mw[2] + t[0];
            const float y = R[3] * mw[0] + R[4] * mw[1] + R[5] * mw[2] + t[1];
            const float z = R[6] * mw[0] + R[7] * mw[1] + R[8] * mw[2] + t[2];
            float RC[9], Rt[9], Cc[9];
            mat3_mul(R, Cw, RC);
            mat3_t(R, Rt);
            mat3_mul(RC, Rt, Cc);
            const float rz = 1.f / z, rz2 = rz * rz, rz3 = rz2 * rz;
            const float tx = z * fminf(lxp, fmaxf(-lxn, x * rz));
            const float ty = z * fminf(lyp, fmaxf(-lyn, y * rz));
            const float J[6] = {fx * rz, 0.f, -fx * tx * rz2, 0.f, fy * rz, -fy * ty * rz2};
            /* v_Cc = J^T vM J */
            float vCc[9];
            for (int i = 0; i < 3; i++)
                for (int j = 0; j < 3; j++) {
                    float s = 0.f;
                    for (int a = 0; a < 2; a++)
                        for (int b = 0; b < 2; b++) s += J[a * 3 + i] * vM[a * 2 + b] * J[b * 3 + j];
                    vCc[i * 3 + j] = s;
                }
            float vmc[3] = {fx * rz * v_means2d[gi * 2], fy * rz * v_means2d[gi * 2 + 1],
                            -(fx * x * v_means2d[gi * 2] + fy * y * v_means2d[gi * 2 + 1]) * rz2};
            /* v_J = vM J Cc^T + vM^T J Cc */
            float vJ[6];
            for (int a = 0; a < 2; a++)
                for (int k = 0; k < 3; k++) {
                    float s = 0.f;
                    for (int b = 0; b < 2; b++)
                        for (int j = 0; j < 3; j++)
                            s += (vM[a * 2 + b] + vM[b * 2 + a]) * J[b * 3 + j] * Cc[j * 3 + k];
                    vJ[a * 3 + k] = s;
                }
            if (x * rz <= lxp && x * rz >= -lxn)
                vmc[0] += -fx * rz2 * vJ[2];
            else
                vmc[2] += -fx * rz3 * vJ[2] * tx;
            if (y * rz <= lyp && y * rz >= -lyn)
                vmc[1] += -fy * rz2 * vJ[5];
            else
                vmc[2] += -fy * rz3 * vJ[5] * ty;
            vmc[2] += -fx * rz2 * vJ[0] - fy * rz2 * vJ[4] + 2.f * fx * tx * rz3 * vJ[2] +
                      2.f * fy * ty * rz3 * vJ[5];
            vmc[2] += v_depths[gi];
            for (int i = 0; i < 3; i++)
                v_means[n * 3 + i] += R[i] * vmc[0] + R[3 + i] * vmc[1] + R[6 + i] * vmc[2];
            /* v_Cw = R^T vCc R */
            float tmp[9], vCw[9];
            mat3_mul(Rt, vCc, tmp);
            mat3_mul(tmp, R, vCw);
            if (v_viewmats) {
                float sC[9], a1[9], a2[9];
                for (int i = 0; i < 3; i++)
                    for (int j = 0; j < 3; j++) sC[i * 3 + j] = vCc[i * 3 + j] + vCc[j * 3 + i];
                mat3_mul(sC, R, a1);
                mat3_mul(a1, Cw, a2);
                for (int i = 0; i < 3; i++) {
                    for (int j = 0; j < 3; j++)
                        v_viewmats[c * 16 + i * 4 + j] += vmc[i] * mw[j] + a2[i * 3 + j];
                    v_viewmats[c * 16 + i * 4 + 3] += vmc[i];
                }
            }
            if (covars6) {
                v_covars[n * 6 + 0] += vCw[0];
                v_covars[n * 6 + 1] += vCw[1] + vCw[3];
                v_covars[n * 6 + 2] += vCw[2] + vCw[6];
                v_covars[n * 6 + 3] += vCw[4];
                v_covars[n * 6 + 4] += vCw[5] + vCw[7];
                v_covars[n * 6 + 5] += vCw[8];
                continue;
            }
            float sym[9], vMq[9], v[9];
            for (int i = 0; i < 3; i++)
                for (int j = 0; j < 3; j++) sym[i * 3 + j] = vCw[i * 3 + j] + vCw[j * 3 + i];
            mat3_mul(sym, M, vMq);
            const float* s = scales + n * 3;
            for (int i = 0; i < 3; i++)
                for (int j = 0; j < 3; j++) v[i * 3 + j] = vMq[i * 3 + j] * s[j];
            for (int j = 0; j < 3; j++)
                v_scales[n * 3 + j] += Rq[j] * vMq[j] + Rq[3 + j] * vMq[3 + j] + Rq[6 + j] * vMq[6 + j];
            const float w = qn[0], qx = qn[1], qy = qn[2], qz = qn[3];
            const float gw = 2.f * (qx * (v[7] - v[5]) + qy * (v[2] - v[6]) + qz * (v[3] - v[1]));
            const float gx = 2.f * (-2.f * qx * (v[4] + v[8]) + qy * (v[1] + v[3]) +
                                    qz * (v[2] + v[6]) + w * (v[7] - v[5]));
            const float gy = 2.f * (qx * (v[1] + v[3]) - 2.f * qy * (v[0] + v[8]) +
                                    qz * (v[5] + v[7]) + w * (v[2] - v[6]));
            const float gz = 2.f * (qx * (v[2] + v[6]) + qy * (v[5] + v[7]) -
                                    2.f * qz * (v[0] + v[4]) + w * (v[3] - v[1]));
            const float d = gw * w + gx * qx + gy * qy + gz * qz;
            v_quats[n * 4 + 0] += (gw - d * w) * inv_norm;
            v_quats[n * 4 + 1] += (gx - d * qx) * inv_norm;
            v_quats[n * 4 + 2] += (gy - d * qy) * inv_norm;
            v_quats[n * 4 + 3] += (gz - d * qz) * inv_norm;
        }
    }
}

/* ---------------------------------------------------------------------------------------------
 * Spherical harmonics (Sloan's hard-coded real basis, degrees 0..4) — forward follows
 * sh_fwd_cpu (CpuKernels.cpp:289-378); backward (no CPU reference exists) is the basis VJP
 * v_coeffs[k][c] = Y_k v_color[c] plus the normalisation VJP of the direction gradient.
 * ------------------------------------------------------------------------------------------- */
static void sh_basis_cpu(uint32_t deg, float x, float y, float z, float* Y) {
    Y[0] = 0.2820947917738781f;
    if (deg < 1) return;
    Y[1] = -0.48860251190292f * y;
    Y[2] = 0.48860251190292f * z;
    Y[3] = -0.48860251190292f * x;
    if (deg < 2) return;
    const float z2 = z * z, c1 = x * x - y * y, s1 = 2.f * x * y;
    Y[4] = 0.5462742152960395f * s1;
    Y[5] = -1.092548430592079f * z * y;
    Y[6] = 0.9461746957575601f * z2 - 0.3153915652525201f;
    Y[7] = -1.092548430592079f * z * x;
    Y[8] = 0.5462742152960395f * c1;
    if (deg < 3) return;
    const float c2 = x * c1 - y * s1, s2 = x * s1 + y * c1;
    const float p3 = -2.285228997322329f * z2 + 0.4570457994644658f;
    Y[9] = -0.5900435899266435f * s2;
    Y[10] = 1.445305721320277f * z * s1;
    Y[11] = p3 * y;
    Y[12] = z * (1.865881662950577f * z2 - 1.119528997770346f);
    Y[13] = p3 * x;
    Y[14] = 1.445305721320277f * z * c1;
    Y[15] = -0.5900435899266435f * c2;
    if (deg < 4) return;
    const float c3 = x * c2 - y * s2, s3 = x * s2 + y * c2;
    const float p4a = z * (-4.683325804901025f * z2 + 2.007139630671868f);
    const float p4b = 3.31161143515146f * z2 - 0.47308734787878f;
    Y[16] = 0.6258357354491763f * s3;
    Y[17] = -1.770130769779931f * z * s2;
    Y[18] = p4b * s1;
    Y[19] = p4a * y;
    Y[20] = 1.984313483298443f * z * Y[12] - 1.006230589874905f * Y[6];
    Y[21] = p4a * x;
    Y[22] = p4b * c1;
    Y[23] = -1.770130769779931f * z * c2;
    Y[24] = 0.6258357354491763f * c3;
}

/* d/d(x,y,z) of sum_k g[k] Y_k (normalised direction). */
static void sh_basis_vjp_cpu(uint32_t deg, float x, float y, float z, const float* g, float* out) {
    float gx = 0.f, gy = 0.f, gz = 0.f;
    if (deg >= 1) {
        gx += -0.48860251190292f * g[3];
        gy += -0.48860251190292f * g[1];
        gz += 0.48860251190292f * g[2];
    }
    if (deg >= 2) {
        const float a = 1.092548430592079f, cc = 0.5462742152960395f, b3 = 0.9461746957575601f;
        gx += g[4] * cc * 2.f * y + g[7] * (-a * z) + g[8] * cc * 2.f * x;
        gy += g[4] * cc * 2.f * x + g[5] * (-a * z) + g[8] * cc * -2.f * y;
        gz += g[5] * (-a * y) + g[6] * (2.f * b3 * z) + g[7] * (-a * x);
    }
    if (deg >= 3) {
        const float z2 = z * z, c1 = x * x - y * y, s1 = 2.f * x * y;
        const float c1x = 2.f * x, c1y = -2.f * y, s1x = 2.f * y, s1y = 2.f * x;
        const float s2 = x * s1 + y * c1, c2 = x * c1 - y * s1;
        const float c2x = c1 + x * c1x - y * s1x, c2y = x * c1y - s1 - y * s1y;
        const float s2x = s1 + x * s1x + y * c1x, s2y = x * s1y + c1 + y * c1y;
        const float A = 0.5900435899266435f, B = 1.445305721320277f;
        const float p3 = -2.285228997322329f * z2 + 0.4570457994644658f;
        const float p3z = -2.f * 2.285228997322329f * z;
        const float q3z = 3.f * 1.865881662950577f * z2 - 1.119528997770346f;
        gx += g[9] * (-A * s2x) + g[10] * (B * z * s1x) + g[13] * p3 + g[14] * (B * z * c1x) +
              g[15] * (-A * c2x);
        gy += g[9] * (-A * s2y) + g[10] * (B * z * s1y) + g[11] * p3 + g[14] * (B * z * c1y) +
              g[15] * (-A * c2y);
        gz += g[10] * (B * s1) + g[11] * (p3z * y) + g[12] * q3z + g[13] * (p3z * x) + g[14] * (B * c1);
        if (deg >= 4) {
            const float c3x = c2 + x * c2x - y * s2x, c3y = x * c2y - s2 - y * s2y;
            const float s3x = s2 + x * s2x + y * c2x, s3y = x * s2y + c2 + y * c2y;
            const float E = 0.6258357354491763f, F = 1.770130769779931f;
            const float p4a = z * (-4.683325804901025f * z2 + 2.007139630671868f);
            const float p4az = -3.f * 4.683325804901025f * z2 + 2.007139630671868f;
            const float p4b = 3.31161143515146f * z2 - 0.47308734787878f;
            const float p4bz = 2.f * 3.31161143515146f * z;
            const float q3 = z * (1.865881662950577f * z2 - 1.119528997770346f);
            const float y6z = 2.f * 0.9461746957575601f * z;
            gx += g[16] * (E * s3x) + g[17] * (-F * z * s2x) + g[18] * (p4b * s1x) + g[21] * p4a +
                  g[22] * (p4b * c1x) + g[23] * (-F * z * c2x) + g[24] * (E * c3x);
            gy += g[16] * (E * s3y) + g[17] * (-F * z * s2y) + g[18] * (p4b * s1y) + g[19] * p4a +
                  g[22] * (p4b * c1y) + g[23] * (-F * z * c2y) + g[24] * (E * c3y);
            gz += g[17] * (-F * s2) + g[18] * (p4bz * s1) + g[19] * (p4az * y) +
                  g[20] * (1.984313483298443f * (q3 + z * q3z) - 1.006230589874905f * y6z) +
                  g[21] * (p4az * x) + g[22] * (p4bz * c1) + g[23] * (-F * c2);
        }
    }
    out[0] = gx;
    out[1] = gy;
    out[2] = gz;
}

void sxo_sh_fwd(const float* dirs, const float* coeffs, const uint8_t* masks, uint32_t degree,
                int64_t B, int64_t N, int64_t K, uint32_t D, float* colors) {
    const int nb = (int)((degree + 1) * (degree + 1));
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < B * N; e++) {
        if (masks && masks[e] == 0) continue;
        const float* co = coeffs + (e % N) * K * D;
        float Y[25], x = 0.f, y = 0.f, z = 0.f;
        if (degree >= 1) {
            const float* d = dirs + e * 3;
            const float inorm = 1.0f / sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
            x = d[0] * inorm;
            y = d[1] * inorm;
            z = d[2] * inorm;
        }
        sh_basis_cpu(degree, x, y, z, Y);
        for (uint32_t c = 0; c < D; c++) {
            float acc = Y[0] * co[c];
            for (int k = 1; k < nb; k++) acc += Y[k] * co[k * D + c];
            colors[e * D + c] = acc;
        }
    }
}

void sxo_sh_bwd(const float* dirs, const float* coeffs, const uint8_t* masks, uint32_t degree,
                int64_t B, int64_t N, int64_t K, uint32_t D, const float* v_colors,
                float* v_coeffs, float* v_dirs) {
    const int nb = (int)((degree + 1) * (degree + 1));
    /* B == 1: each element owns its Gaussian's coefficient rows */
#pragma omp parallel for schedule(static) if (B == 1)
    for (int64_t e = 0; e < B * N; e++) {
        if (masks && masks[e] == 0) continue;
        const int64_t gid = e % N;
        const float* co = coeffs + gid * K * D;
        const float* vc = v_colors + e * D;
        float Y[25], g[25], x = 0.f, y = 0.f, z = 0.f, inorm = 0.f;
        const float* d = dirs + e * 3;
        if (degree >= 1) {
            inorm = 1.0f / sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
            x = d[0] * inorm;
            y = d[1] * inorm;
            z = d[2] * inorm;
        }
        sh_basis_cpu(degree, x, y, z, Y);
        for (int k = 0; k < nb; k++) {
            float gk = 0.f;
            for (uint32_t c = 0; c < D; c++) {
                v_coeffs[gid * K * D + k * D + c] += Y[k] * vc[c];
                gk += vc[c] * co[k * D + c];
            }
            g[k] = gk;
        }
        if (v_dirs && degree >= 1) {
            float vn[3];
            sh_basis_vjp_cpu(degree, x, y, z, g, vn);
            const float dot = vn[0] * x + vn[1] * y + vn[2] * z;
            v_dirs[e * 3 + 0] += (vn[0] - dot * x) * inorm;
            v_dirs[e * 3 + 1] += (vn[1] - dot * y) * inorm;
            v_dirs[e * 3 + 2] += (vn[2] - dot * z) * inorm;
        }
    }
}

/* ---------------------------------------------------------------------------------------------
 * Tile intersection — isect_tiles_cpu (CpuKernels.cpp:371-669): AABB rectangle (:371-393) or
 * AccuTile (SNUGBOX + strip sweep, :395-560; SpeedySplat arXiv:2412.00578), count then emit with
 * keys image<<(32+tile_bits) | tile<<32 | f32bits(depth), emit order idx -> sweep u -> v.
 * ------------------------------------------------------------------------------------------- */
typedef struct {
    uint64_t* ids;
    int32_t* flat;
    int64_t cur;
    uint64_t hi_enc, depth_enc;
    int32_t fid;
} Emit;

static inline void emit_one(Emit* e, uint32_t tile) {
    if (!e) return;
    e->ids[e->cur] = e->hi_enc | ((uint64_t)tile << 32) | e->depth_enc;
    e->flat[e->cur] = e->fid;
    e->cur++;
}

static uint32_t aabb(float mx, float my, float rx, float ry, float ts, int tw, int th, Emit* e) {
    const float trx = rx / ts, try_ = ry / ts, tx = mx / ts, ty = my / ts;
    const int x0 = imin(imax(0, f2i(floorf(tx - trx))), tw);
    const int y0 = imin(imax(0, f2i(floorf(ty - try_))), th);
    const int x1 = imin(imax(0, f2i(ceilf(tx + trx))), tw);
    const int y1 = imin(imax(0, f2i(ceilf(ty + try_))), th);
    if (e)
        for (int i = y0; i < y1; i++)
            for (int j = x0; j < x1; j++) emit_one(e, (uint32_t)(i * tw + j));
    return (uint32_t)((y1 - y0) * (x1 - x0));
}

static void line_isect(float A, float B, float C, float disc, float t, float px, float py, int isY,
                       float coord, float* lo, float* hi) {
    const float pu = isY ? py : px, pv = isY ? px : py;
    const float coeff = isY ? A : C;
    const float h = coord - pu;
    const float sq = sqrtf(disc * h * h + t * coeff);
    *lo = (-B * h - sq) / coeff + pv;
    *hi = (-B * h + sq) / coeff + pv;
}

static uint32_t accutile(const float* conic, float opacity, float mx, float my, float ts, int tw,
                         int th, Emit* e) {
    const float A = conic[0], B = conic[1], C = conic[2];
    const float disc = B * B - A * C;
    const float t = fminf(K_GAUSSIAN_EXTEND * K_GAUSSIAN_EXTEND,
                          2.0f * logf(opacity / K_ALPHA_THRESHOLD));
    if (t <= 0.f) return 0;
    const float ntd = -t / disc;
    const float xe = sqrtf(ntd * C), ye = sqrtf(ntd * A);
    float bmin_x = mx - xe, bmin_y = my - ye, bmax_x = mx + xe, bmax_y = my + ye;
    const float BxC = B * xe / C, ByA = B * ye / A;
    float amin_x = my + BxC, amin_y = mx + ByA, amax_x = my - BxC, amax_y = mx - ByA;
    int rminx = imax(0, imin(tw, f2i(bmin_x / ts)));
    int rminy = imax(0, imin(th, f2i(bmin_y / ts)));
    int rmaxx = imax(0, imin(tw, f2i(bmax_x / ts + 1.f)));
    int rmaxy = imax(0, imin(th, f2i(bmax_y / ts + 1.f)));
    const int ysp = rmaxy - rminy, xsp = rmaxx - rminx;
    if (ysp * xsp == 0) return 0;
    const int isY = ysp < xsp;
    if (isY) {
        int ti; float tf;
        ti = rminx; rminx = rminy; rminy = ti;
        ti = rmaxx; rmaxx = rmaxy; rmaxy = ti;
        tf = bmin_x; bmin_x = bmin_y; bmin_y = tf;
        tf = bmax_x; bmax_x = bmax_y; bmax_y = tf;
        tf = amin_x; amin_x = amin_y; amin_y = tf;
        tf = amax_x; amax_x = amax_y; amax_y = tf;
    }
    uint32_t count = 0;
    float lmax_lo = bmax_y, lmax_hi = bmin_y;
    float min_line = rminx * ts;
    float lmin_lo, lmin_hi;
    if (bmin_x <= min_line)
        line_isect(A, B, C, disc, t, mx, my, isY, min_line, &lmin_lo, &lmin_hi);
    else {
        lmin_lo = lmax_lo;
        lmin_hi = lmax_hi;
    }
    for (int u = rminx; u < rmaxx; u++) {
        const float max_line = min_line + ts;
        if (max_line <= bmax_x) line_isect(A, B, C, disc, t, mx, my, isY, max_line, &lmax_lo, &lmax_hi);
        const float emin = (min_line <= amin_y && amin_y < max_line) ? bmin_y : fminf(lmin_lo, lmax_lo);
        const float emax = (min_line <= amax_y && amax_y < max_line) ? bmax_y : fmaxf(lmin_hi, lmax_hi);
        const int v0 = imax(rminy, imin(rmaxy, f2i(emin / ts)));
        const int v1 = imin(rmaxy, imax(rminy, f2i(emax / ts + 1.f)));
        for (int v = v0; v < v1; v++) {
            count++;
            emit_one(e, (uint32_t)(isY ? u * tw + v : v * tw + u));
        }
        lmin_lo = lmax_lo;
        lmin_hi = lmax_hi;
        min_line = max_line;
    }
    return count;
}

int64_t sxo_isect_count(const float* means2d, const int32_t* radii, const float* conics,
                        const float* opacities, int64_t n, uint32_t tile_size, uint32_t tile_width,
                        uint32_t tile_height, int32_t* tiles) {
    int64_t total = 0;
    const float ts = (float)tile_size;
#pragma omp parallel for schedule(dynamic, 1024) reduction(+ : total)
    for (int64_t i = 0; i < n; i++) {
        const float rx = (float)radii[i * 2], ry = (float)radii[i * 2 + 1];
        uint32_t c = 0;
        if (rx > 0.f && ry > 0.f) {
            if (conics && opacities)
                c = accutile(conics + i * 3, opacities[i], means2d[i * 2], means2d[i * 2 + 1], ts,
                             (int)tile_width, (int)tile_height, NULL);
            else
                c = aabb(means2d[i * 2], means2d[i * 2 + 1], rx, ry, ts, (int)tile_width,
                         (int)tile_height, NULL);
        }
        tiles[i] = (int32_t)c;
        total += c;
    }
    return total;
}

void sxo_isect_emit(const float* means2d, const int32_t* radii, const float* depths,
                    const float* conics, const float* opacities, int64_t I, int64_t N,
                    uint32_t tile_size, uint32_t tile_width, uint32_t tile_height,
                    const int32_t* tiles, uint64_t* ids, int32_t* flat) {
    const uint32_t tb = sxo_bits_for_count((int64_t)tile_width * tile_height);
    const float ts = (float)tile_size;
    const int64_t n = I * N;
    int64_t* start = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    int64_t run = 0;
    for (int64_t i = 0; i < n; i++) {
        start[i] = run;
        run += tiles[i];
    }
#pragma omp parallel for schedule(dynamic, 1024)
    for (int64_t i = 0; i < n; i++) {
        const float rx = (float)radii[i * 2], ry = (float)radii[i * 2 + 1];
        if (!(rx > 0.f && ry > 0.f)) continue;
        uint32_t dbits;
        memcpy(&dbits, &depths[i], 4);
        Emit e = {ids, flat, start[i], (uint64_t)(i / N) << (32 + tb), (uint64_t)dbits, (int32_t)i};
        if (conics && opacities)
            accutile(conics + i * 3, opacities[i], means2d[i * 2], means2d[i * 2 + 1], ts,
                     (int)tile_width, (int)tile_height, &e);
        else
            aabb(means2d[i * 2], means2d[i * 2 + 1], rx, ry, ts, (int)tile_width, (int)tile_height, &e);
    }
    free(start);
}

/* sort_isect_cpu (CpuKernels.cpp:680-706): stable by key — here a stable LSD radix sort on
 * 16-bit digits over the key bits (equivalent to the reference's index std::stable_sort). */
int32_t sxo_sort_isect(const uint64_t* keys, const int32_t* values, int64_t n, uint32_t key_n_bits,
                       uint64_t* ko, int32_t* vo) {
    if (n <= 0) return 0;
    if (key_n_bits < 64)
        for (int64_t i = 0; i < n; i++)
            if (keys[i] >> key_n_bits) return -1;
    uint64_t* kt = (uint64_t*)malloc(sizeof(uint64_t) * n);
    int32_t* vt = (int32_t*)malloc(sizeof(int32_t) * n);
    int64_t* cnt = (int64_t*)malloc(sizeof(int64_t) * 65536);
    memcpy(ko, keys, sizeof(uint64_t) * n);
    memcpy(vo, values, sizeof(int32_t) * n);
    for (uint32_t shift = 0; shift < key_n_bits; shift += 16) {
        memset(cnt, 0, sizeof(int64_t) * 65536);
        for (int64_t i = 0; i < n; i++) cnt[(ko[i] >> shift) & 0xffff]++;
        int64_t run = 0;
        for (int d = 0; d < 65536; d++) {
            const int64_t c = cnt[d];
            cnt[d] = run;
            run += c;
        }
        for (int64_t i = 0; i < n; i++) {
            const int64_t p = cnt[(ko[i] >> shift) & 0xffff]++;
            kt[p] = ko[i];
            vt[p] = vo[i];
        }
        memcpy(ko, kt, sizeof(uint64_t) * n);
        memcpy(vo, vt, sizeof(int32_t) * n);
    }
    free(kt);
    free(vt);
    free(cnt);
    return 0;
}

/* isect_offset_encode_cpu (CpuKernels.cpp:715-747). */
void sxo_isect_offset_encode(const uint64_t* ids, int64_t n, int64_t I, uint32_t tile_width,
                             uint32_t tile_height, int32_t* offsets) {
    const int64_t n_tiles = (int64_t)tile_width * tile_height;
    const int64_t total = I * n_tiles;
    memset(offsets, 0, sizeof(int32_t) * (size_t)total);
    if (n == 0) return;
    const uint32_t tb = sxo_bits_for_count(n_tiles);
    const uint64_t mask = ((uint64_t)1 << tb) - 1;
#define FLAT(k) ((int64_t)(((k) >> 32) >> tb) * n_tiles + (int64_t)(((k) >> 32) & mask))
    for (int64_t i = 0; i < n; i++) {
        const int64_t cur = FLAT(ids[i]);
        if (i == 0)
            for (int64_t t = 0; t <= cur; t++) offsets[t] = 0;
        if (i == n - 1)
            for (int64_t t = cur + 1; t < total; t++) offsets[t] = (int32_t)n;
        if (i > 0) {
            if ((ids[i - 1] >> 32) == (ids[i] >> 32)) continue;
            const int64_t prev = FLAT(ids[i - 1]);
            for (int64_t t = prev + 1; t <= cur; t++) offsets[t] = (int32_t)i;
        }
    }
#undef FLAT
}

/* ---------------------------------------------------------------------------------------------
 * Rasterisation — forward follows rasterize_fwd_cpu (CpuKernels.cpp:776-851): per pixel,
 * front to back, sigma = 0.5(a dx^2 + c dy^2) + b dx dy, alpha = min(0.99, o expf(-sigma)),
 * skip on sigma<0 or alpha<1/255, exclusive stop at T(1-alpha) <= 1e-4, fmaf colour sums.
 * Backward (no CPU reference exists) restates Rasterize3DGSBwd.metal:70-298 sequentially:
 * back-to-front from T_final, T /= (1 - alpha) (floor 1e-6), the three v_alpha terms, the clamp
 * gate o*vis <= 0.99, gradients accumulated per Gaussian.
 * ------------------------------------------------------------------------------------------- */
static inline int64_t tile_end(const int32_t* off, int64_t img, int64_t I, int64_t tile,
                               int64_t n_tiles, int64_t n_isects) {
    return (img == I - 1 && tile == n_tiles - 1) ? n_isects : off[tile + 1];
}

void sxo_rasterize_fwd(const float* means2d, const float* conics, const float* colors,
                       const float* opacities, const float* bgs, const uint8_t* masks,
                       const int32_t* offsets, const int32_t* flatten_ids, int64_t I, int64_t N,
                       int64_t n_isects, uint32_t W, uint32_t H, uint32_t ts, uint32_t tw,
                       uint32_t th, float* rc, float* ra, int32_t* li) {
    (void)N;
    const int64_t n_tiles = (int64_t)tw * th;
    for (int64_t img = 0; img < I; img++) {
        const int32_t* off = offsets + img * n_tiles;
        const float* bg = bgs ? bgs + img * 3 : NULL;
        float* o_rc = rc + img * (int64_t)H * W * 3;
        float* o_ra = ra + img * (int64_t)H * W;
        int32_t* o_li = li + img * (int64_t)H * W;
#pragma omp parallel for schedule(dynamic, 4)
        for (int64_t tile = 0; tile < n_tiles; tile++) {
            const int64_t txi = tile % tw, tyi = tile / tw;
            const int masked = masks && masks[img * n_tiles + tile] == 0;
            const int64_t s = off[tile], e = tile_end(off, img, I, tile, n_tiles, n_isects);
            for (uint32_t yy = 0; yy < ts; yy++) {
                const int64_t py = tyi * ts + yy;
                if (py >= H) continue;
                for (uint32_t xx = 0; xx < ts; xx++) {
                    const int64_t px = txi * ts + xx;
                    if (px >= W) continue;
                    const int64_t pix = py * W + px;
                    if (masked) {
                        for (int k = 0; k < 3; k++) o_rc[pix * 3 + k] = bg ? bg[k] : 0.f;
                        o_ra[pix] = 0.f;
                        o_li[pix] = 0;
                        continue;
                    }
                    const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
                    float T = 1.0f, out[3] = {0.f, 0.f, 0.f};
                    uint32_t cur = 0;
                    for (int64_t idx = s; idx < e; idx++) {
                        const int32_t g = flatten_ids[idx];
                        const float dx = means2d[2 * g] - fx, dy = means2d[2 * g + 1] - fy;
                        const float* cn = conics + 3 * g;
                        const float sigma = 0.5f * (cn[0] * dx * dx + cn[2] * dy * dy) + cn[1] * dx * dy;
                        const float vis = expf(-sigma);
                        const float alpha = smin(K_MAX_ALPHA, opacities[g] * vis);
                        if (sigma < 0.f || alpha < K_ALPHA_THRESHOLD) continue;
                        const float nT = T * (1.0f - alpha);
                        if (nT <= K_TRANSMITTANCE_THRESHOLD) break;
                        const float w = alpha * T;
                        for (int k = 0; k < 3; k++) out[k] = fmaf(colors[g * 3 + k], w, out[k]);
                        cur = (uint32_t)idx;
                        T = nT;
                    }
                    o_ra[pix] = 1.0f - T;
                    for (int k = 0; k < 3; k++) o_rc[pix * 3 + k] = bg ? fmaf(T, bg[k], out[k]) : out[k];
                    o_li[pix] = (int32_t)cur;
                }
            }
        }
    }
}

void sxo_rasterize_bwd(const float* means2d, const float* conics, const float* colors,
                       const float* opacities, const float* bgs, const uint8_t* masks,
                       const int32_t* offsets, const int32_t* flatten_ids, int64_t I, int64_t N,
                       int64_t n_isects, uint32_t W, uint32_t H, uint32_t ts, uint32_t tw,
                       uint32_t th, const float* render_alphas, const int32_t* last_ids,
                       const float* v_rc, const float* v_ra, float* v_m2, float* v_con,
                       float* v_col, float* v_op, float* v_m2abs) {
    (void)N;
    if (n_isects == 0) return;
    const int64_t n_tiles = (int64_t)tw * th;
    /* One gradient slot per intersection: every (tile, Gaussian) pair accumulates over its tile's
     * pixels in pixel order, then slots are summed per Gaussian in sorted order — the result does
     * not depend on how many threads processed the tiles. */
    const int NV = v_m2abs ? 11 : 9;
    float* slot = (float*)calloc((size_t)n_isects * NV, sizeof(float));
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t bt = 0; bt < I * n_tiles; bt++) {
        const int64_t img = bt / n_tiles, tile = bt % n_tiles;
        if (masks && masks[img * n_tiles + tile] == 0) continue;
        const int32_t* off = offsets + img * n_tiles;
        const float* bg = bgs ? bgs + img * 3 : NULL;
        const int64_t base = img * (int64_t)H * W;
        const int64_t txi = tile % tw, tyi = tile / tw;
        const int64_t s = off[tile], e = tile_end(off, img, I, tile, n_tiles, n_isects);
        for (uint32_t yy = 0; yy < ts; yy++) {
            const int64_t py = tyi * ts + yy;
            if (py >= H) continue;
            for (uint32_t xx = 0; xx < ts; xx++) {
                const int64_t px = txi * ts + xx;
                if (px >= W) continue;
                const int64_t pix = base + py * W + px;
                const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
                const float T_final = 1.0f - render_alphas[pix];
                float T = T_final, acc[3] = {0.f, 0.f, 0.f};
                const int64_t bin_final = last_ids[pix];
                const float vc[3] = {v_rc[pix * 3], v_rc[pix * 3 + 1], v_rc[pix * 3 + 2]};
                const float va = v_ra[pix];
                float bg_dot = 0.f;
                if (bg) bg_dot = bg[0] * vc[0] + bg[1] * vc[1] + bg[2] * vc[2];
                for (int64_t idx = (bin_final < e - 1 ? bin_final : e - 1); idx >= s; idx--) {
                    const int32_t g = flatten_ids[idx];
                    const float dx = means2d[2 * g] - fx, dy = means2d[2 * g + 1] - fy;
                    const float* cn = conics + 3 * g;
                    const float op = opacities[g];
                    const float sigma = 0.5f * (cn[0] * dx * dx + cn[2] * dy * dy) + cn[1] * dx * dy;
                    const float vis = expf(-sigma);
                    const float alpha = smin(K_MAX_ALPHA, op * vis);
                    if (sigma < 0.f || alpha < K_ALPHA_THRESHOLD) continue;
                    const float ra = 1.0f / smax(K_MIN_ONE_MINUS_ALPHA, 1.0f - alpha);
                    T *= ra;
                    const float fac = alpha * T;
                    float* sl = slot + idx * NV;
                    float v_alpha = 0.f;
                    for (int k = 0; k < 3; k++) {
                        sl[k] += fac * vc[k];
                        v_alpha += (colors[g * 3 + k] * T - acc[k] * ra) * vc[k];
                    }
                    v_alpha += T_final * ra * va;
                    if (bg) v_alpha += -T_final * ra * bg_dot;
                    if (op * vis <= K_MAX_ALPHA) {
                        const float v_sigma = -op * vis * v_alpha;
                        sl[3] += 0.5f * v_sigma * dx * dx;
                        sl[4] += v_sigma * dx * dy;
                        sl[5] += 0.5f * v_sigma * dy * dy;
                        const float gx = v_sigma * (cn[0] * dx + cn[1] * dy);
                        const float gy = v_sigma * (cn[1] * dx + cn[2] * dy);
                        sl[6] += gx;
                        sl[7] += gy;
                        sl[8] += vis * v_alpha;
                        if (NV == 11) {
                            sl[9] += fabsf(gx);
                            sl[10] += fabsf(gy);
                        }
                    }
                    for (int k = 0; k < 3; k++) acc[k] += colors[g * 3 + k] * fac;
                }
            }
        }
    }
    for (int64_t idx = 0; idx < n_isects; idx++) {
        const int32_t g = flatten_ids[idx];
        const float* sl = slot + idx * NV;
        for (int k = 0; k < 3; k++) v_col[g * 3 + k] += sl[k];
        for (int k = 0; k < 3; k++) v_con[g * 3 + k] += sl[3 + k];
        v_m2[g * 2] += sl[6];
        v_m2[g * 2 + 1] += sl[7];
        v_op[g] += sl[8];
        if (NV == 11) {
            v_m2abs[g * 2] += sl[9];
            v_m2abs[g * 2 + 1] += sl[10];
        }
    }
    free(slot);
}

/* ---------------------------------------------------------------------------------------------
 * SSIM — forward follows ssim_fwd_cpu (CpuKernels.cpp:1019-1106): separable 11-tap window
 * (horizontal then vertical, fmaf accumulation, taps u = 0..10), map = SSIM at window START p,
 * coefficient maps Dmu/Dsigma/Dcross; mean in f64 in index order. Backward (no CPU reference):
 * v_img1(q) = G [ (w*Dmu)(q) + 2 x(q) (w*Dsig)(q) + y(q) (w*Dcross)(q) ], G = -v_loss/M, where
 * (w*D)(q) = sum_{u,v} w[u] w[v] D(q_y - v, q_x - u) over in-range map pixels.
 * ------------------------------------------------------------------------------------------- */
double sxo_ssim_fwd(const float* img1, const float* img2, int64_t I, int64_t H, int64_t W, int64_t C,
                    int32_t need, float* map, float* cmu, float* csg, float* ccr) {
    ssim_taps();
    const int64_t mh = H - 10, mw = W - 10;
    float* h[5];
    for (int k = 0; k < 5; k++) h[k] = (float*)malloc(sizeof(float) * (size_t)(H * mw));
    for (int64_t i = 0; i < I; i++)
        for (int64_t c = 0; c < C; c++) {
#pragma omp parallel for schedule(static)
            for (int64_t y = 0; y < H; y++)
                for (int64_t xw = 0; xw < mw; xw++) {
                    float m1 = 0.f, m2 = 0.f, e11 = 0.f, e22 = 0.f, e12 = 0.f;
                    for (int u = 0; u < 11; u++) {
                        const float w = g_ssim_taps[u];
                        const int64_t off = (((i * H + y) * W) + xw + u) * C + c;
                        const float x = img1[off], g = img2[off];
                        m1 = fmaf(w, x, m1);
                        m2 = fmaf(w, g, m2);
                        e11 = fmaf(w * x, x, e11);
                        e22 = fmaf(w * g, g, e22);
                        e12 = fmaf(w * x, g, e12);
                    }
                    const int64_t ho = y * mw + xw;
                    h[0][ho] = m1; h[1][ho] = m2; h[2][ho] = e11; h[3][ho] = e22; h[4][ho] = e12;
                }
#pragma omp parallel for schedule(static)
            for (int64_t my = 0; my < mh; my++)
                for (int64_t mx = 0; mx < mw; mx++) {
                    float mu1 = 0.f, mu2 = 0.f, e11 = 0.f, e22 = 0.f, e12 = 0.f;
                    for (int v = 0; v < 11; v++) {
                        const float w = g_ssim_taps[v];
                        const int64_t ho = (my + v) * mw + mx;
                        mu1 = fmaf(w, h[0][ho], mu1);
                        mu2 = fmaf(w, h[1][ho], mu2);
                        e11 = fmaf(w, h[2][ho], e11);
                        e22 = fmaf(w, h[3][ho], e22);
                        e12 = fmaf(w, h[4][ho], e12);
                    }
                    const float s1 = fmaf(-mu1, mu1, e11), s2 = fmaf(-mu2, mu2, e22);
                    const float s12 = fmaf(-mu1, mu2, e12);
                    const float A1 = 2.f * mu1 * mu2 + K_SSIM_C1;
                    const float B1 = mu1 * mu1 + mu2 * mu2 + K_SSIM_C1;
                    const float A2 = 2.f * s12 + K_SSIM_C2;
                    const float B2 = s1 + s2 + K_SSIM_C2;
                    const float den = B1 * B2;
                    const float S = (A1 * A2) / den;
                    const int64_t mo = (((i * mh + my) * mw) + mx) * C + c;
                    map[mo] = S;
                    if (need) {
                        const float d_mu1 = 2.f * (mu2 * A2 / den - mu1 * S / B1);
                        const float d_s1 = -S / B2;
                        const float d_s12 = 2.f * A1 / den;
                        cmu[mo] = d_mu1 - 2.f * mu1 * d_s1 - mu2 * d_s12;
                        csg[mo] = d_s1;
                        ccr[mo] = d_s12;
                    }
                }
        }
    for (int k = 0; k < 5; k++) free(h[k]);
    const int64_t cnt = I * mh * mw * C;
    double sum = 0.0;
    for (int64_t k = 0; k < cnt; k++) sum += (double)map[k];
    return sum / (double)cnt;
}

void sxo_ssim_bwd(const float* img1, const float* img2, int64_t I, int64_t H, int64_t W, int64_t C,
                  const float* cmu, const float* csg, const float* ccr, float v_loss, float* v_img1) {
    ssim_taps();
    const int64_t mh = H - 10, mw = W - 10;
    const float G = (float)(-(double)v_loss / ((double)I * C * mh * mw));
    float* hz = (float*)malloc(sizeof(float) * (size_t)(mh * W * 3));
    for (int64_t i = 0; i < I; i++)
        for (int64_t c = 0; c < C; c++) {
            /* horizontal adjoint: hz[py][qx] = sum_u w[u] D(py, qx - u) */
#pragma omp parallel for schedule(static)
            for (int64_t py = 0; py < mh; py++)
                for (int64_t qx = 0; qx < W; qx++) {
                    float s[3] = {0.f, 0.f, 0.f};
                    for (int u = 0; u < 11; u++) {
                        const int64_t px = qx - 10 + u;
                        if (px < 0 || px >= mw) continue;
                        const float w = g_ssim_taps[u];
                        const int64_t mo = (((i * mh + py) * mw) + px) * C + c;
                        s[0] = fmaf(w, cmu[mo], s[0]);
                        s[1] = fmaf(w, csg[mo], s[1]);
                        s[2] = fmaf(w, ccr[mo], s[2]);
                    }
                    for (int k = 0; k < 3; k++) hz[(py * W + qx) * 3 + k] = s[k];
                }
#pragma omp parallel for schedule(static)
            for (int64_t qy = 0; qy < H; qy++)
                for (int64_t qx = 0; qx < W; qx++) {
                    float s[3] = {0.f, 0.f, 0.f};
                    for (int v = 0; v < 11; v++) {
                        const int64_t py = qy - 10 + v;
                        if (py < 0 || py >= mh) continue;
                        const float w = g_ssim_taps[v];
                        for (int k = 0; k < 3; k++) s[k] = fmaf(w, hz[(py * W + qx) * 3 + k], s[k]);
                    }
                    const int64_t q = (((i * H + qy) * W) + qx) * C + c;
                    v_img1[q] = G * (s[0] + 2.f * img1[q] * s[1] + img2[q] * s[2]);
                }
        }
    free(hz);
}

/* ---------------------------------------------------------------------------------------------
 * RNG — Philox4x32-10 (Salmon et al., SC'11), counter (t, offset_lo, offset_hi, 0), key seed;
 * u32 -> (0,1] as (float(x)+1) 2^-32; Box-Muller with logf/sqrtf/cosf/sinf (CpuKernels.cpp:863-905).
 * ------------------------------------------------------------------------------------------- */
void sxo_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3], k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; r++) {
        if (r > 0) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        c0 = n0;
        c1 = (uint32_t)p1;
        c2 = n2;
        c3 = (uint32_t)p0;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

void sxo_rng_philox_u32(uint64_t seed, uint64_t offset, int64_t count, uint32_t* out) {
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    for (int64_t t = 0; t * 4 < count; t++) {
        const uint32_t ctr[4] = {(uint32_t)t, (uint32_t)offset, (uint32_t)(offset >> 32), 0u};
        uint32_t r[4];
        sxo_philox4x32_10(ctr, key, r);
        for (int j = 0; j < 4 && t * 4 + j < count; j++) out[t * 4 + j] = r[j];
    }
}

static void box_muller(uint32_t a, uint32_t b, float* z0, float* z1) {
    const float u1 = ((float)a + 1.0f) * (1.0f / 4294967296.0f);
    const float u2 = ((float)b + 1.0f) * (1.0f / 4294967296.0f);
    const float r = sqrtf(-2.0f * logf(u1));
    const float th = 6.28318530717958647692f * u2;
    *z0 = r * cosf(th);
    *z1 = r * sinf(th);
}

void sxo_rng_normal_f32(uint64_t seed, uint64_t offset, int64_t count, float* out) {
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    for (int64_t t = 0; t * 4 < count; t++) {
        const uint32_t ctr[4] = {(uint32_t)t, (uint32_t)offset, (uint32_t)(offset >> 32), 0u};
        uint32_t r[4];
        sxo_philox4x32_10(ctr, key, r);
        float z[4];
        box_muller(r[0], r[1], &z[0], &z[1]);
        box_muller(r[2], r[3], &z[2], &z[3]);
        for (int j = 0; j < 4 && t * 4 + j < count; j++) out[t * 4 + j] = z[j];
    }
}

/* make_binoms_lut (CpuKernels.cpp:906-917): exact Pascal rows in u64, cast to float. */
void sxo_make_binoms_lut(int32_t n_max, float* lut) {
    uint64_t* row = (uint64_t*)calloc((size_t)n_max, sizeof(uint64_t));
    for (int n = 0; n < n_max; n++) {
        for (int k = n; k >= 1; k--) row[k] += row[k - 1];
        row[0] = 1;
        for (int k = 0; k < n_max; k++) lut[(size_t)n * n_max + k] = k <= n ? (float)row[k] : 0.0f;
    }
    free(row);
}

/* mcmc_relocation_cpu (CpuKernels.cpp:924-963). */
int32_t sxo_mcmc_relocation(const float* op, const float* sc, const int32_t* ratios,
                            const float* binoms, int64_t N, int32_t n_max, float min_op,
                            float* new_op, float* new_sc) {
    for (int64_t i = 0; i < N; i++) {
        const int n = ratios[i];
        if (n < 1 || n > n_max) return -1;
        const float o = op[i];
        float no = 1.0f - powf(1.0f - o, 1.0f / (float)n);
        no = smin(smax(no, min_op), 1.0f - FLT_EPSILON);
        new_op[i] = no;
        float denom = 0.0f;
        for (int a = 1; a <= n; a++)
            for (int k = 0; k <= a - 1; k++) {
                const float bc = binoms[(size_t)(a - 1) * n_max + k];
                const float sign = (k & 1) ? -1.0f : 1.0f;
                const float term = (sign / sqrtf((float)(k + 1))) * powf(no, (float)(k + 1));
                denom += bc * term;
            }
        const float coeff = o / denom;
        for (int k = 0; k < 3; k++) new_sc[i * 3 + k] = coeff * sc[i * 3 + k];
    }
    return 0;
}

/* mcmc_perturb_positions_cpu (CpuKernels.cpp:969-1007). */
void sxo_mcmc_perturb_positions(float* pos, const float* quats, const float* scales_log,
                                const float* op_logit, const float* noise, int64_t N,
                                float noise_scale, float t, float k) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < N; i++) {
        const float* q = quats + i * 4;
        float w = q[0], x = q[1], y = q[2], z = q[3];
        const float inv = 1.0f / sqrtf(x * x + y * y + z * z + w * w);
        x *= inv; y *= inv; z *= inv; w *= inv;
        const float R[9] = {1.f - 2.f * (y * y + z * z), 2.f * (x * y - w * z), 2.f * (x * z + w * y),
                            2.f * (x * y + w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z - w * x),
                            2.f * (x * z - w * y), 2.f * (y * z + w * x), 1.f - 2.f * (x * x + y * y)};
        const float s[3] = {expf(scales_log[i * 3]), expf(scales_log[i * 3 + 1]), expf(scales_log[i * 3 + 2])};
        float M[9], Cv[9];
        for (int a = 0; a < 3; a++)
            for (int b = 0; b < 3; b++) M[a * 3 + b] = R[a * 3 + b] * s[b];
        for (int a = 0; a < 3; a++)
            for (int b = 0; b < 3; b++)
                Cv[a * 3 + b] = M[a * 3] * M[b * 3] + M[a * 3 + 1] * M[b * 3 + 1] + M[a * 3 + 2] * M[b * 3 + 2];
        const float density = 1.0f / (1.0f + expf(-op_logit[i]));
        const float gate = 1.0f / (1.0f + expf(k * (density - t)));
        const float wgt = gate * noise_scale;
        const float n0 = noise[i * 3] * wgt, n1 = noise[i * 3 + 1] * wgt, n2 = noise[i * 3 + 2] * wgt;
        pos[i * 3 + 0] += Cv[0] * n0 + Cv[1] * n1 + Cv[2] * n2;
        pos[i * 3 + 1] += Cv[3] * n0 + Cv[4] * n1 + Cv[5] * n2;
        pos[i * 3 + 2] += Cv[6] * n0 + Cv[7] * n1 + Cv[8] * n2;
    }
}

/* ---------------------------------------------------------------------------------------------
 * The host training step — Trainer::forward_pass (Trainer.cpp:716-832) + Trainer::step
 * (:974-1131): activations, projection, SH + post-op, AccuTile, stable sort, offsets, raster,
 * L1 (+ SSIM lerp), raster bwd, relu mask, SH bwd, projection bwd, v_means += v_dirs, chains +
 * regularisers, Adam x6 (valid-masked), MCMC noise (Trainer.cpp:1400-1420).
 * ------------------------------------------------------------------------------------------- */
#define ALLOC(T, n) ((T*)calloc((size_t)((n) > 0 ? (n) : 1), sizeof(T)))

/* The step's activations (train_exp / train_sigmoid, TrainStep.metal:23-45; host path
 * activate_scales / activate_opacities, Trainer.cpp:430-459): scales = exp(log-scales), opacity =
 * 1 / (1 + exp(-logit)), float expf. */
void sxo_train_activations(const float* log_scales, const float* logits, int64_t N, float* s_lin,
                           float* sig) {
    for (int64_t i = 0; i < N * 3; i++) s_lin[i] = expf(log_scales[i]);
    for (int64_t i = 0; i < N; i++) sig[i] = 1.0f / (1.0f + expf(-logits[i]));
}

/* The training loss and its gradient with respect to the render (host path Trainer.cpp:982-1016
 * with l1_loss_and_grad Trainer.cpp:330-345; resident path MetalBackend.cpp:2241-2263):
 * L1 = mean |r - gt| summed in f64, v = sign(r - gt) / n (sign(0) = 0, train_l1_grad,
 * TrainStep.metal:143); with lambda > 0, v = (1 - lambda) v + ssim_bwd(G = lambda) and
 * loss = (1 - lambda) L1 + lambda (1 - mean SSIM). */
float sxo_train_loss(const float* rc, const float* gt, int32_t H, int32_t W, float lam,
                     float* v) {
    const int64_t n = (int64_t)H * W * 3;
    const float g = 1.0f / (float)n;
    double acc = 0.0;
    for (int64_t i = 0; i < n; i++) {
        const float d = rc[i] - gt[i];
        acc += fabs((double)d);
        v[i] = d > 0.0f ? g : (d < 0.0f ? -g : 0.0f);
    }
    const float l1 = (float)(acc / (double)n);
    float loss = l1;
    if (lam > 0.0f) {
        const int64_t mc = (int64_t)(H - 10) * (W - 10) * 3;
        float* map = ALLOC(float, mc);
        float* cmu = ALLOC(float, mc);
        float* csg = ALLOC(float, mc);
        float* ccr = ALLOC(float, mc);
        float* vd = ALLOC(float, n);
        const double ss = sxo_ssim_fwd(rc, gt, 1, H, W, 3, 1, map, cmu, csg, ccr);
        sxo_ssim_bwd(rc, gt, 1, H, W, 3, cmu, csg, ccr, lam, vd);
        const float wl1 = 1.0f - lam;
        for (int64_t i = 0; i < n; i++) v[i] = wl1 * v[i] + vd[i];
        loss = wl1 * l1 + lam * (1.0f - (float)ss);
        free(map); free(cmu); free(csg); free(ccr); free(vd);
    }
    return loss;
}

int32_t sxo_train_step(float* const* P, float* const* M1, float* const* M2, int64_t N,
                       const float* vm, const float* Km, int32_t W, int32_t H, const float* gt,
                       const SxoStepConfig* cfg, float* loss_out, int64_t* n_isects_out,
                       float* render_out) {
    if (N < 1 || W < 1 || H < 1 || !cfg) return -1;
    const int64_t K = (int64_t)(cfg->sh_degree + 1) * (cfg->sh_degree + 1);
    const int64_t dims[6] = {3, 4, 3, 1, 3, (K - 1) * 3};
    const uint32_t deg = cfg->degrees_to_use;
    float* s_lin = ALLOC(float, N * 3);
    float* sig = ALLOC(float, N);
    sxo_train_activations(P[2], P[3], N, s_lin, sig);
    int32_t* radii = ALLOC(int32_t, N * 2);
    float* m2d = ALLOC(float, N * 2);
    float* dep = ALLOC(float, N);
    float* con = ALLOC(float, N * 3);
    float* comp = ALLOC(float, N);
    sxo_projection_fused_fwd(P[0], NULL, P[1], s_lin, sig, vm, Km, N, 1, W, H, cfg->eps2d,
                             cfg->near_plane, cfg->far_plane, cfg->radius_clip, cfg->antialiased,
                             radii, m2d, dep, con, comp);
    float* rop = sig;
    float* op_aa = NULL;
    if (cfg->antialiased) {
        op_aa = ALLOC(float, N);
        for (int64_t i = 0; i < N; i++) op_aa[i] = sig[i] * comp[i];
        rop = op_aa;
    }
    uint8_t* valid = ALLOC(uint8_t, N);
    for (int64_t i = 0; i < N; i++) valid[i] = (radii[i * 2] > 0 && radii[i * 2 + 1] > 0) ? 1 : 0;
    float campos[3];
    for (int i = 0; i < 3; i++)
        campos[i] = -(vm[0 * 4 + i] * vm[0 * 4 + 3] + vm[1 * 4 + i] * vm[1 * 4 + 3] +
                      vm[2 * 4 + i] * vm[2 * 4 + 3]);
    float* dirs = ALLOC(float, N * 3);
    for (int64_t i = 0; i < N; i++)
        for (int k = 0; k < 3; k++) dirs[i * 3 + k] = P[0][i * 3 + k] - campos[k];
    float* coeffs = ALLOC(float, N * K * 3);
    for (int64_t i = 0; i < N; i++) {
        for (int c = 0; c < 3; c++) coeffs[(i * K) * 3 + c] = P[4][i * 3 + c];
        for (int64_t k = 1; k < K; k++)
            for (int c = 0; c < 3; c++)
                coeffs[(i * K + k) * 3 + c] = P[5][(i * (K - 1) + (k - 1)) * 3 + c];
    }
    float* colors = ALLOC(float, N * 3);
    uint8_t* relu = ALLOC(uint8_t, N * 3);
    sxo_sh_fwd(dirs, coeffs, valid, deg, 1, N, K, 3, colors);
    for (int64_t i = 0; i < N * 3; i++) {
        const float pre = colors[i] + 0.5f;
        relu[i] = pre > 0.0f ? 1 : 0;
        colors[i] = smax(pre, 0.0f);
    }
    const uint32_t tw = (uint32_t)((W + 15) / 16), th = (uint32_t)((H + 15) / 16);
    int32_t* tiles = ALLOC(int32_t, N);
    const int64_t n_isects = sxo_isect_count(m2d, radii, con, rop, N, 16, tw, th, tiles);
    uint64_t* ids = ALLOC(uint64_t, n_isects);
    int32_t* fl = ALLOC(int32_t, n_isects);
    sxo_isect_emit(m2d, radii, dep, con, rop, 1, N, 16, tw, th, tiles, ids, fl);
    uint64_t* ids_s = ALLOC(uint64_t, n_isects);
    int32_t* fl_s = ALLOC(int32_t, n_isects);
    const uint32_t key_bits = 32 + sxo_bits_for_count((int64_t)tw * th) + sxo_bits_for_count(1);
    sxo_sort_isect(ids, fl, n_isects, key_bits, ids_s, fl_s);
    int32_t* off = ALLOC(int32_t, (int64_t)tw * th);
    sxo_isect_offset_encode(ids_s, n_isects, 1, tw, th, off);
    const int64_t npx = (int64_t)W * H;
    float* rc = ALLOC(float, npx * 3);
    float* ra = ALLOC(float, npx);
    int32_t* li = ALLOC(int32_t, npx);
    sxo_rasterize_fwd(m2d, con, colors, rop, NULL, NULL, off, fl_s, 1, N, n_isects, (uint32_t)W,
                      (uint32_t)H, 16, tw, th, rc, ra, li);
    if (render_out) memcpy(render_out, rc, sizeof(float) * (size_t)(npx * 3));
    *n_isects_out = n_isects;
    int32_t status = 0;
    if (!cfg->forward_only) {
        const int64_t n = npx * 3;
        float* v = ALLOC(float, n);
        *loss_out = sxo_train_loss(rc, gt, H, W, cfg->ssim_weight, v);
        float* v_ra = ALLOC(float, npx);
        float* vm2 = ALLOC(float, N * 2);
        float* vcon = ALLOC(float, N * 3);
        float* vcol = ALLOC(float, N * 3);
        float* vop = ALLOC(float, N);
        sxo_rasterize_bwd(m2d, con, colors, rop, NULL, NULL, off, fl_s, 1, N, n_isects,
                          (uint32_t)W, (uint32_t)H, 16, tw, th, ra, li, v, v_ra, vm2, vcon, vcol,
                          vop, NULL);
        for (int64_t i = 0; i < N * 3; i++)
            if (!relu[i]) vcol[i] = 0.0f;
        float* vco = ALLOC(float, N * K * 3);
        float* vdir = ALLOC(float, N * 3);
        sxo_sh_bwd(dirs, coeffs, valid, deg, 1, N, K, 3, vcol, vco, vdir);
        float* vcomp = NULL;
        if (cfg->antialiased) {
            vcomp = ALLOC(float, N);
            for (int64_t i = 0; i < N; i++) {
                const float a = vop[i];
                vcomp[i] = a * sig[i];
                vop[i] = a * comp[i];
            }
        }
        float* vzero = ALLOC(float, N);
        float* vmean = ALLOC(float, N * 3);
        float* vq = ALLOC(float, N * 4);
        float* vs = ALLOC(float, N * 3);
        sxo_projection_fused_bwd(P[0], NULL, P[1], s_lin, vm, Km, N, 1, W, H, cfg->eps2d, radii,
                                 con, comp, vm2, vzero, vcon, vcomp, vmean, NULL, vq, vs, NULL);
        for (int64_t i = 0; i < N * 3; i++) vmean[i] += vdir[i];
        for (int64_t i = 0; i < N * 3; i++) vs[i] *= s_lin[i];
        for (int64_t i = 0; i < N; i++) {
            const float s = sig[i];
            vop[i] *= s * (1.0f - s);
        }
        if (cfg->opacity_reg > 0.0f) {
            const float w = cfg->opacity_reg / (float)N;
            for (int64_t i = 0; i < N; i++) vop[i] += w * sig[i] * (1.0f - sig[i]);
        }
        if (cfg->scale_reg > 0.0f) {
            const float w = cfg->scale_reg / (float)(N * 3);
            for (int64_t i = 0; i < N * 3; i++) vs[i] += w * s_lin[i];
        }
        float* vsh0 = ALLOC(float, N * 3);
        float* vshN = ALLOC(float, N * (K - 1) * 3);
        for (int64_t i = 0; i < N; i++) {
            for (int c = 0; c < 3; c++) vsh0[i * 3 + c] = vco[(i * K) * 3 + c];
            for (int64_t k = 1; k < K; k++)
                for (int c = 0; c < 3; c++)
                    vshN[(i * (K - 1) + (k - 1)) * 3 + c] = vco[(i * K + k) * 3 + c];
        }
        float* grads[6] = {vmean, vq, vs, vop, vsh0, vshN};
        for (int g6 = 0; g6 < 6; g6++) {
            if (dims[g6] == 0) continue;
            sxo_fused_adam(P[g6], grads[g6], M1[g6], M2[g6], valid, N * dims[g6], N, cfg->lr[g6],
                           cfg->b1, cfg->b2, cfg->eps);
        }
        if (cfg->inject_noise) {
            float* noise = ALLOC(float, N * 3);
            sxo_rng_normal_f32(cfg->noise_seed, cfg->noise_offset, N * 3, noise);
            sxo_mcmc_perturb_positions(P[0], P[1], P[2], P[3], noise, N, cfg->noise_scale, 0.005f,
                                       100.f);
            free(noise);
        }
        free(v); free(v_ra); free(vm2); free(vcon); free(vcol); free(vop); free(vco); free(vdir);
        free(vcomp); free(vzero); free(vmean); free(vq); free(vs); free(vsh0); free(vshN);
    } else {
        *loss_out = 0.0f;
    }
    free(s_lin); free(sig); free(radii); free(m2d); free(dep); free(con); free(comp); free(op_aa);
    free(valid); free(dirs); free(coeffs); free(colors); free(relu); free(tiles); free(ids);
    free(fl); free(ids_s); free(fl_s); free(off); free(rc); free(ra); free(li);
    return status;
}

/* ===================== MCMC refine (Trainer.cpp:1195-1435) ===================== */

/* mt19937_64: w=64, n=312, m=156, r=31, the twist matrix a, tempering (u,d)=(29,0x5555...),
 * (s,b)=(17,0x71D6...), (t,c)=(37,0xFFF7...), l=43, and the initialisation multiplier f — the
 * published parameters of MT19937-64 as the C++ standard lists them. */
#define MT_N 312
#define MT_M 156
static const uint64_t kMtA = 0xB5026F5AA96619E9ULL;
static const uint64_t kMtUpper = 0xFFFFFFFF80000000ULL; /* the top w - r bits */
static const uint64_t kMtLower = 0x000000007FFFFFFFULL; /* the low r bits */

void sxo_mt64_seed(SxoMt64* g, uint64_t seed) {
    g->x[0] = seed;
    for (int k = 1; k < MT_N; k++)
        g->x[k] = 6364136223846793005ULL * (g->x[k - 1] ^ (g->x[k - 1] >> 62)) + (uint64_t)k;
    g->i = MT_N;
}

static void mt64_twist(SxoMt64* g) {
    for (int k = 0; k < MT_N; k++) {
        const uint64_t y = (g->x[k] & kMtUpper) | (g->x[(k + 1) % MT_N] & kMtLower);
        g->x[k] = g->x[(k + MT_M) % MT_N] ^ (y >> 1) ^ ((y & 1ULL) ? kMtA : 0ULL);
    }
    g->i = 0;
}

uint64_t sxo_mt64_next(SxoMt64* g) {
    if (g->i >= MT_N) mt64_twist(g);
    uint64_t y = g->x[g->i++];
    y ^= (y >> 29) & 0x5555555555555555ULL;
    y ^= (y << 17) & 0x71D67FFFEDA60000ULL;
    y ^= (y << 37) & 0xFFF7EEE000000000ULL;
    y ^= y >> 43;
    return y;
}

/* The weights' running sum in double (index order); u = (next >> 11) * 2^-53 * sum; the first
 * index whose running sum exceeds u, clamped to n - 1 (a zero weight is never chosen). */
int32_t sxo_multinomial(const float* w, int64_t n, int64_t n_samples, SxoMt64* rng, int64_t* out) {
    double* cdf = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
    double acc = 0.0;
    for (int64_t i = 0; i < n; i++) {
        if (!(w[i] >= 0.0f)) {
            free(cdf);
            return -1;
        }
        acc += (double)w[i];
        cdf[i] = acc;
    }
    if (!(acc > 0.0)) {
        free(cdf);
        return -1;
    }
    for (int64_t j = 0; j < n_samples; j++) {
        const double u = (double)(sxo_mt64_next(rng) >> 11) * 0x1.0p-53 * acc;
        int64_t lo = 0, hi = n; /* first index with cdf > u */
        while (lo < hi) {
            const int64_t mid = lo + (hi - lo) / 2;
            if (cdf[mid] > u) hi = mid;
            else lo = mid + 1;
        }
        out[j] = lo < n - 1 ? lo : n - 1;
    }
    free(cdf);
    return 0;
}

static float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

/* run_relocation_for + the source update (Trainer.cpp:1231-1257, :1313-1323, :1365-1375). */
static int32_t relocate_sources(float* const* P, const int64_t* src, int64_t n, const float* op_act,
                                float min_op, int32_t* counts) {
    static float lut[51 * 51];
    static int lut_ready = 0;
    if (!lut_ready) {
        sxo_make_binoms_lut(51, lut);
        lut_ready = 1;
    }
    float* g_op = (float*)malloc(sizeof(float) * (size_t)(n + 1));
    float* g_sc = (float*)malloc(sizeof(float) * (size_t)(3 * n + 1));
    float* n_op = (float*)malloc(sizeof(float) * (size_t)(n + 1));
    float* n_sc = (float*)malloc(sizeof(float) * (size_t)(3 * n + 1));
    int32_t* ratios = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + 1));
    int32_t rc = 0;
    for (int64_t j = 0; j < n; j++) counts[src[j]]++;
    for (int64_t j = 0; j < n; j++) {
        const int64_t s = src[j];
        g_op[j] = op_act[s];
        for (int k = 0; k < 3; k++) g_sc[j * 3 + k] = expf(P[2][s * 3 + k]);
        ratios[j] = counts[s] + 1 < 51 ? counts[s] + 1 : 51;
    }
    for (int64_t j = 0; j < n; j++) counts[src[j]] = 0;
    if (sxo_mcmc_relocation(g_op, g_sc, ratios, lut, n, 51, min_op, n_op, n_sc) != 0) rc = -1;
    for (int64_t j = 0; j < n && rc == 0; j++) {
        const float p = n_op[j];
        if (!(p > 0.0f && p < 1.0f)) { rc = -1; break; }
        P[3][src[j]] = logf(p / (1.0f - p));
        for (int k = 0; k < 3; k++) {
            if (!(n_sc[j * 3 + k] > 0.0f)) { rc = -1; break; }
            P[2][src[j] * 3 + k] = logf(n_sc[j * 3 + k]);
        }
    }
    free(g_op); free(g_sc); free(n_op); free(n_sc); free(ratios);
    return rc;
}

static void copy_rows(float* const* P, const int64_t* dims, const int64_t* dst, const int64_t* src,
                      int64_t n) {
    for (int g = 0; g < 6; g++) {
        const int64_t d = dims[g];
        if (d == 0) continue;
        for (int64_t j = 0; j < n; j++)
            memcpy(P[g] + dst[j] * d, P[g] + src[j] * d, sizeof(float) * (size_t)d);
    }
}

static void zero_moment_rows(float* const* m, float* const* v, const int64_t* dims,
                             const int64_t* rows, int64_t n) {
    for (int g = 0; g < 6; g++) {
        const int64_t d = dims[g];
        if (d == 0) continue;
        for (int64_t j = 0; j < n; j++) {
            memset(m[g] + rows[j] * d, 0, sizeof(float) * (size_t)d);
            memset(v[g] + rows[j] * d, 0, sizeof(float) * (size_t)d);
        }
    }
}

int32_t sxo_mcmc_refine(SxoMt64* rng, float* const* P, float* const* M, float* const* V,
                        const int64_t* dims, int64_t count, int64_t cap_max, float min_op,
                        int64_t* relocated_dead, int64_t* relocation_src, int64_t* added_src,
                        SxoMcmcResult* out) {
    if (count < 1 || cap_max < count || !(min_op > 0.0f && min_op < 1.0f)) return -1;
    const int64_t N = count;
    int32_t rc = 0;
    float* op_act = (float*)malloc(sizeof(float) * (size_t)N);
    int32_t* counts = (int32_t*)calloc((size_t)N, sizeof(int32_t));
    int64_t* dead = (int64_t*)malloc(sizeof(int64_t) * (size_t)N);
    int64_t* alive = (int64_t*)malloc(sizeof(int64_t) * (size_t)N);
    int64_t* local = (int64_t*)malloc(sizeof(int64_t) * (size_t)N);
    int64_t* sampled = (int64_t*)malloc(sizeof(int64_t) * (size_t)(N + 1));
    float* probs = (float*)malloc(sizeof(float) * (size_t)N);
    out->n_relocated = out->n_added = 0;

    /* relocate: dead = sigmoid(op) <= min_opacity, sources from the alive rows */
    for (int64_t i = 0; i < N; i++) op_act[i] = sigmoid_f(P[3][i]);
    int64_t nd = 0, na = 0;
    for (int64_t i = 0; i < N; i++) {
        if (op_act[i] <= min_op) dead[nd++] = i;
        else alive[na++] = i;
    }
    if (nd > 0 && na > 0) {
        for (int64_t j = 0; j < na; j++) probs[j] = op_act[alive[j]];
        rc = sxo_multinomial(probs, na, nd, rng, local);
        if (rc == 0) {
            for (int64_t j = 0; j < nd; j++) sampled[j] = alive[local[j]];
            rc = relocate_sources(P, sampled, nd, op_act, min_op, counts);
        }
        if (rc == 0) {
            copy_rows(P, dims, dead, sampled, nd);
            zero_moment_rows(M, V, dims, sampled, nd); /* the SOURCES (Trainer.cpp:1334) */
            memcpy(relocated_dead, dead, sizeof(int64_t) * (size_t)nd);
            memcpy(relocation_src, sampled, sizeof(int64_t) * (size_t)nd);
            out->n_relocated = nd;
        }
    }
    /* add: grow to min(cap_max, ceil(1.05 N)); sources from all rows (updated opacities) */
    const int64_t target = (N * 21 + 19) / 20 < cap_max ? (N * 21 + 19) / 20 : cap_max;
    const int64_t n_add = target - N;
    if (rc == 0 && n_add > 0) {
        for (int64_t i = 0; i < N; i++) op_act[i] = sigmoid_f(P[3][i]);
        int64_t* src = (int64_t*)malloc(sizeof(int64_t) * (size_t)n_add);
        int64_t* dst = (int64_t*)malloc(sizeof(int64_t) * (size_t)n_add);
        rc = sxo_multinomial(op_act, N, n_add, rng, src);
        if (rc == 0) rc = relocate_sources(P, src, n_add, op_act, min_op, counts);
        if (rc == 0) {
            for (int64_t j = 0; j < n_add; j++) dst[j] = N + j;
            copy_rows(P, dims, dst, src, n_add);
            zero_moment_rows(M, V, dims, dst, n_add); /* the NEW rows (Trainer.cpp:1389-1391) */
            memcpy(added_src, src, sizeof(int64_t) * (size_t)n_add);
            out->n_added = n_add;
        }
        free(src);
        free(dst);
    }
    out->count = N + out->n_added;
    free(op_act); free(counts); free(dead); free(alive); free(local); free(sampled); free(probs);
    return rc;
}
