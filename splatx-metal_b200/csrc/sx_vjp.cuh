// sx_vjp.cuh — vector-Jacobian products of the EWA projection (C=1 per thread), Philox4x32-10,
// and the small matrix helpers they use. Row-major 3x3 / 2x2 / 2x3 storage throughout.
//
// Math: gsplat's fused projection backward (restated in splatx-metal
// Sources/SplatXKernelSrc/ProjectionEWA.metal:186-560): inverse VJP of the conic, the optional
// compensation VJP, perspective-projection VJP with the FOV-clamp branch, world->camera VJPs and
// the quaternion/scale covariance VJP with the normalisation projection.
#pragma once

#include "sx_common.cuh"

namespace sx {

__device__ __forceinline__ void m3_mul(const float* a, const float* b, float* c) {
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            c[i * 3 + j] = a[i * 3] * b[j] + a[i * 3 + 1] * b[3 + j] + a[i * 3 + 2] * b[6 + j];
}
// c = a * b^T
__device__ __forceinline__ void m3_mul_bt(const float* a, const float* b, float* c) {
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            c[i * 3 + j] = a[i * 3] * b[j * 3] + a[i * 3 + 1] * b[j * 3 + 1] + a[i * 3 + 2] * b[j * 3 + 2];
}
// c = a^T * b
__device__ __forceinline__ void m3_mul_at(const float* a, const float* b, float* c) {
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            c[i * 3 + j] = a[i] * b[j] + a[3 + i] * b[3 + j] + a[6 + i] * b[6 + j];
}

// Rotation of the normalised quaternion [w,x,y,z] (1/sqrt of the x,y,z,w square sum).
__device__ __forceinline__ void quat_rotmat(const float* q, float* R, float* qn, float& inv_norm) {
    float w = q[0], x = q[1], y = q[2], z = q[3];
    inv_norm = 1.0f / sqrtf(x * x + y * y + z * z + w * w);
    w *= inv_norm;
    x *= inv_norm;
    y *= inv_norm;
    z *= inv_norm;
    qn[0] = w; qn[1] = x; qn[2] = y; qn[3] = z;
    R[0] = 1.f - 2.f * (y * y + z * z);
    R[1] = 2.f * (x * y - w * z);
    R[2] = 2.f * (x * z + w * y);
    R[3] = 2.f * (x * y + w * z);
    R[4] = 1.f - 2.f * (x * x + z * z);
    R[5] = 2.f * (y * z - w * x);
    R[6] = 2.f * (x * z - w * y);
    R[7] = 2.f * (y * z + w * x);
    R[8] = 1.f - 2.f * (x * x + y * y);
}

struct ProjVjpIn {
    const float* mean_w;  // [3]
    const float* quat;    // [4] (quat/scale path) or nullptr
    const float* scale;   // [3] linear
    const float* covar6;  // [6] triu (covars path) or nullptr
    const float* R;       // [9] row-major world->camera
    const float* t;       // [3]
    float fx, fy, cx, cy;
    int width, height;
    float eps2d;
    const float* conic;   // [3] forward output
    float v_m2x, v_m2y, v_depth;
    const float* v_conic; // [3]
    bool has_comp;
    float comp, v_comp;
};

struct ProjVjpOut {
    float v_mean[3];
    float v_covar[9];  // world covariance gradient (full)
    float v_quat[4];
    float v_scale[3];
    float v_R[9];
    float v_t[3];
};

__device__ __forceinline__ void projection_vjp(const ProjVjpIn& in, ProjVjpOut& o, bool want_pose) {
    // conic = inverse(cov2d + eps I): v_cov2d = -conic v_conic_sym conic
    const float c0 = in.conic[0], c1 = in.conic[1], c2 = in.conic[2];
    const float va = in.v_conic[0], vb = 0.5f * in.v_conic[1], vc = in.v_conic[2];
    // P = conic * V (symmetric 2x2 each)
    const float p00 = c0 * va + c1 * vb, p01 = c0 * vb + c1 * vc;
    const float p10 = c1 * va + c2 * vb, p11 = c1 * vb + c2 * vc;
    float vM00 = -(p00 * c0 + p01 * c1), vM01 = -(p00 * c1 + p01 * c2);
    float vM10 = -(p10 * c0 + p11 * c1), vM11 = -(p10 * c1 + p11 * c2);
    if (in.has_comp) {
        const float det_cb = c0 * c2 - c1 * c1;
        const float v_sqr = in.v_comp * 0.5f / (in.comp + 1e-6f);
        const float omc = 1.f - in.comp * in.comp;
        vM00 += v_sqr * (omc * c0 - in.eps2d * det_cb);
        vM01 += v_sqr * (omc * c1);
        vM10 += v_sqr * (omc * c1);
        vM11 += v_sqr * (omc * c2 - in.eps2d * det_cb);
    }

    // forward recomputation
    float Cw[9], Rq[9] = {0}, qn[4] = {0}, inv_norm = 0.f, M[9] = {0};
    if (in.covar6) {
        const float* cv = in.covar6;
        Cw[0] = cv[0]; Cw[1] = cv[1]; Cw[2] = cv[2];
        Cw[3] = cv[1]; Cw[4] = cv[3]; Cw[5] = cv[4];
        Cw[6] = cv[2]; Cw[7] = cv[4]; Cw[8] = cv[5];
    } else {
        quat_rotmat(in.quat, Rq, qn, inv_norm);
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) M[i * 3 + j] = Rq[i * 3 + j] * in.scale[j];
        m3_mul_bt(M, M, Cw);
    }
    const float* R = in.R;
    const float* mw = in.mean_w;
    const float x = R[0] * mw[0] + R[1] * mw[1] + R[2] * mw[2] + in.t[0];
    const float y = R[3] * mw[0] + R[4] * mw[1] + R[5] * mw[2] + in.t[1];
    const float z = R[6] * mw[0] + R[7] * mw[1] + R[8] * mw[2] + in.t[2];
    float RC[9], Cc[9];
    m3_mul(R, Cw, RC);
    m3_mul_bt(RC, R, Cc);

    const float fx = in.fx, fy = in.fy;
    const float Wf = static_cast<float>(in.width), Hf = static_cast<float>(in.height);
    const float tan_fovx = 0.5f * Wf / fx, tan_fovy = 0.5f * Hf / fy;
    const float lim_x_pos = (Wf - in.cx) / fx + 0.3f * tan_fovx;
    const float lim_x_neg = in.cx / fx + 0.3f * tan_fovx;
    const float lim_y_pos = (Hf - in.cy) / fy + 0.3f * tan_fovy;
    const float lim_y_neg = in.cy / fy + 0.3f * tan_fovy;
    const float rz = 1.f / z, rz2 = rz * rz, rz3 = rz2 * rz;
    const float tx = z * fminf(lim_x_pos, fmaxf(-lim_x_neg, x * rz));
    const float ty = z * fminf(lim_y_pos, fmaxf(-lim_y_neg, y * rz));
    // J (2x3): [J00 0 J02; 0 J11 J12]
    const float J00 = fx * rz, J02 = -fx * tx * rz2, J11 = fy * rz, J12 = -fy * ty * rz2;

    // v_Cc = J^T vM J
    // vM J (2x3)
    const float a00 = vM00 * J00, a01 = vM01 * J11, a02 = vM00 * J02 + vM01 * J12;
    const float a10 = vM10 * J00, a11 = vM11 * J11, a12 = vM10 * J02 + vM11 * J12;
    float vCc[9];
    vCc[0] = J00 * a00;            vCc[1] = J00 * a01;            vCc[2] = J00 * a02;
    vCc[3] = J11 * a10;            vCc[4] = J11 * a11;            vCc[5] = J11 * a12;
    vCc[6] = J02 * a00 + J12 * a10; vCc[7] = J02 * a01 + J12 * a11; vCc[8] = J02 * a02 + J12 * a12;

    float vmc[3] = {fx * rz * in.v_m2x, fy * rz * in.v_m2y,
                    -(fx * x * in.v_m2x + fy * y * in.v_m2y) * rz2};
    // v_J = vM J Cc^T + vM^T J Cc  (Cc symmetric) = (vM + vM^T) J Cc
    const float s00 = 2.f * vM00, s01 = vM01 + vM10, s11 = 2.f * vM11;
    // J Cc (2x3)
    const float jc0[3] = {J00 * Cc[0] + J02 * Cc[6], J00 * Cc[1] + J02 * Cc[7], J00 * Cc[2] + J02 * Cc[8]};
    const float jc1[3] = {J11 * Cc[3] + J12 * Cc[6], J11 * Cc[4] + J12 * Cc[7], J11 * Cc[5] + J12 * Cc[8]};
    float vJ[2][3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        vJ[0][k] = s00 * jc0[k] + s01 * jc1[k];
        vJ[1][k] = s01 * jc0[k] + s11 * jc1[k];
    }
    if (x * rz <= lim_x_pos && x * rz >= -lim_x_neg)
        vmc[0] += -fx * rz2 * vJ[0][2];
    else
        vmc[2] += -fx * rz3 * vJ[0][2] * tx;
    if (y * rz <= lim_y_pos && y * rz >= -lim_y_neg)
        vmc[1] += -fy * rz2 * vJ[1][2];
    else
        vmc[2] += -fy * rz3 * vJ[1][2] * ty;
    vmc[2] += -fx * rz2 * vJ[0][0] - fy * rz2 * vJ[1][1] + 2.f * fx * tx * rz3 * vJ[0][2] +
              2.f * fy * ty * rz3 * vJ[1][2];
    vmc[2] += in.v_depth;

    // world -> camera
#pragma unroll
    for (int i = 0; i < 3; ++i)
        o.v_mean[i] = R[i] * vmc[0] + R[3 + i] * vmc[1] + R[6 + i] * vmc[2];
    if (want_pose) {
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            o.v_t[i] = vmc[i];
#pragma unroll
            for (int j = 0; j < 3; ++j) o.v_R[i * 3 + j] = vmc[i] * mw[j];
        }
        // v_R += vCc R Cw^T + vCc^T R Cw = (vCc + vCc^T) R Cw  (Cw symmetric)
        float sC[9], tmp[9], add[9];
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) sC[i * 3 + j] = vCc[i * 3 + j] + vCc[j * 3 + i];
        m3_mul(sC, R, tmp);
        m3_mul(tmp, Cw, add);
#pragma unroll
        for (int k = 0; k < 9; ++k) o.v_R[k] += add[k];
    }
    // v_Cw = R^T vCc R
    float tmp2[9];
    m3_mul_at(R, vCc, tmp2);
    m3_mul(tmp2, R, o.v_covar);

    if (!in.covar6) {
        // v_M = (v_Cw + v_Cw^T) M
        float sym[9], vM[9];
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) sym[i * 3 + j] = o.v_covar[i * 3 + j] + o.v_covar[j * 3 + i];
        m3_mul(sym, M, vM);
        float v[9];  // d/dRq
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) v[i * 3 + j] = vM[i * 3 + j] * in.scale[j];
#pragma unroll
        for (int j = 0; j < 3; ++j)
            o.v_scale[j] = Rq[j] * vM[j] + Rq[3 + j] * vM[3 + j] + Rq[6 + j] * vM[6 + j];
        const float w = qn[0], qx = qn[1], qy = qn[2], qz = qn[3];
        const float gw = 2.f * (qx * (v[7] - v[5]) + qy * (v[2] - v[6]) + qz * (v[3] - v[1]));
        const float gx = 2.f * (-2.f * qx * (v[4] + v[8]) + qy * (v[1] + v[3]) + qz * (v[2] + v[6]) +
                                w * (v[7] - v[5]));
        const float gy = 2.f * (qx * (v[1] + v[3]) - 2.f * qy * (v[0] + v[8]) + qz * (v[5] + v[7]) +
                                w * (v[2] - v[6]));
        const float gz = 2.f * (qx * (v[2] + v[6]) + qy * (v[5] + v[7]) - 2.f * qz * (v[0] + v[4]) +
                                w * (v[3] - v[1]));
        const float d = gw * w + gx * qx + gy * qy + gz * qz;
        o.v_quat[0] = (gw - d * w) * inv_norm;
        o.v_quat[1] = (gx - d * qx) * inv_norm;
        o.v_quat[2] = (gy - d * qy) * inv_norm;
        o.v_quat[3] = (gz - d * qz) * inv_norm;
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) o.v_quat[k] = 0.f;
#pragma unroll
        for (int k = 0; k < 3; ++k) o.v_scale[k] = 0.f;
    }
}

// ---- Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel Random Numbers: As Easy as 1, 2, 3",
// SC'11): counter (c0..c3), key (k0,k1), ten rounds, Weyl key schedule between rounds.
struct Philox4 {
    uint32_t v[4];
};

__host__ __device__ __forceinline__ Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2,
                                                          uint32_t c3, uint32_t k0, uint32_t k1) {
    constexpr uint32_t kMul0 = 0xD2511F53u, kMul1 = 0xCD9E8D57u;
    constexpr uint32_t kWeyl0 = 0x9E3779B9u, kWeyl1 = 0xBB67AE85u;
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = static_cast<uint64_t>(kMul0) * c0;
        const uint64_t p1 = static_cast<uint64_t>(kMul1) * c2;
        const uint32_t n0 = static_cast<uint32_t>(p1 >> 32) ^ c1 ^ k0;
        const uint32_t n2 = static_cast<uint32_t>(p0 >> 32) ^ c3 ^ k1;
        c1 = static_cast<uint32_t>(p1);
        c3 = static_cast<uint32_t>(p0);
        c0 = n0;
        c2 = n2;
        k0 += kWeyl0;
        k1 += kWeyl1;
    }
    Philox4 o;
    o.v[0] = c0; o.v[1] = c1; o.v[2] = c2; o.v[3] = c3;
    return o;
}

// u32 -> (0,1]: (float(x) + 1) * 2^-32, computed in float so x = 0xffffffff gives exactly 1.
__device__ __forceinline__ float u32_to_unit(uint32_t x) {
    return (static_cast<float>(x) + 1.0f) * (1.0f / 4294967296.0f);
}

// Box-Muller pair from two words: r = sqrt(-2 ln u1), theta = 2 pi u2.
__device__ __forceinline__ void box_muller(uint32_t x0, uint32_t x1, float& z0, float& z1) {
    const float u1 = u32_to_unit(x0), u2 = u32_to_unit(x1);
    const float r = sqrtf(-2.0f * logf(u1));
    const float theta = 6.28318530717958647692f * u2;
    float s, c;
    sincosf(theta, &s, &c);
    z0 = r * c;
    z1 = r * s;
}

// Standard normal number `idx` of the stream (seed, offset): thread t = idx/4 of the reference's
// rng_normal_f32 produces normals 4t..4t+3 from one Philox block (Rng.metal:34-47).
__device__ __forceinline__ float normal_at(uint64_t idx, uint64_t seed, uint64_t offset) {
    const uint32_t t = static_cast<uint32_t>(idx >> 2);
    const Philox4 r = philox4x32_10(t, static_cast<uint32_t>(offset),
                                    static_cast<uint32_t>(offset >> 32), 0u,
                                    static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
    const int j = static_cast<int>(idx & 3);
    float z0, z1;
    if (j < 2)
        box_muller(r.v[0], r.v[1], z0, z1);
    else
        box_muller(r.v[2], r.v[3], z0, z1);
    return (j & 1) ? z1 : z0;
}

}  // namespace sx
