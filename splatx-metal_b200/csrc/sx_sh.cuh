// sx_sh.cuh — real spherical-harmonics basis (degrees 0..4) and its derivatives, in the
// hard-coded Sloan form ("Efficient Spherical Harmonic Evaluation", JCGT 2013) that gsplat and
// splatx-metal evaluate (Sources/SplatXKernelSrc/SphericalHarmonics.metal:35-389).
//
// Conventions of the contract: the direction is normalised inside with 1/sqrt (unguarded: a zero
// direction gives NaN, as in the reference), degree 0 never reads the direction, coefficients are
// [K][D] per Gaussian with band index k = l*l + l + m.
#pragma once

#include "sx_common.cuh"

namespace sx {

// Sloan's constants (rounded from their closed forms; the values every 3DGS implementation uses).
constexpr float kShC0 = 0.28209479177387814f;   // 1/(2 sqrt(pi))
constexpr float kShC1 = 0.4886025119029199f;    // sqrt(3/(4 pi))
constexpr float kShC2a = 1.0925484305920792f;   // degree-2 xy / yz / xz factor
constexpr float kShC2b = 0.31539156525252005f;  // degree-2 (3z^2-1) factor
constexpr float kShC2c = 0.5462742152960396f;   // degree-2 (x^2-y^2) factor
constexpr float kShC3a = 0.5900435899266435f;
constexpr float kShC3b = 1.445305721320277f;
constexpr float kShC3c = 2.285228997322329f;
constexpr float kShC3d = 0.4570457994644658f;
constexpr float kShC3e = 1.865881662950577f;
constexpr float kShC3f = 1.119528997770346f;
constexpr float kShC4a = 0.6258357354491763f;
constexpr float kShC4b = 1.770130769779931f;
constexpr float kShC4c = 3.31161143515146f;
constexpr float kShC4d = 0.47308734787878f;
constexpr float kShC4e = 4.683325804901025f;
constexpr float kShC4f = 2.007139630671868f;
constexpr float kShC4g = 1.984313483298443f;
constexpr float kShC4h = 1.006230589874905f;

__host__ __device__ constexpr int sh_bands(int degree) { return (degree + 1) * (degree + 1); }

// Basis values Y[0..(deg+1)^2) at the normalised direction (x,y,z).
__device__ __forceinline__ void sh_basis(int degree, float x, float y, float z, float* Y) {
    Y[0] = kShC0;
    if (degree < 1) return;
    Y[1] = -kShC1 * y;
    Y[2] = kShC1 * z;
    Y[3] = -kShC1 * x;
    if (degree < 2) return;
    const float z2 = z * z;
    const float c1 = x * x - y * y;  // cos(2 phi) r^2
    const float s1 = 2.f * x * y;    // sin(2 phi) r^2
    Y[4] = kShC2c * s1;
    Y[5] = -kShC2a * z * y;
    Y[6] = fmaf(3.f * kShC2b, z2, -kShC2b);
    Y[7] = -kShC2a * z * x;
    Y[8] = kShC2c * c1;
    if (degree < 3) return;
    const float c2 = x * c1 - y * s1;
    const float s2 = x * s1 + y * c1;
    const float p3 = fmaf(-kShC3c, z2, kShC3d);
    Y[9] = -kShC3a * s2;
    Y[10] = kShC3b * z * s1;
    Y[11] = p3 * y;
    Y[12] = z * fmaf(kShC3e, z2, -kShC3f);
    Y[13] = p3 * x;
    Y[14] = kShC3b * z * c1;
    Y[15] = -kShC3a * c2;
    if (degree < 4) return;
    const float c3 = x * c2 - y * s2;
    const float s3 = x * s2 + y * c2;
    const float p4a = z * fmaf(-kShC4e, z2, kShC4f);
    const float p4b = fmaf(kShC4c, z2, -kShC4d);
    Y[16] = kShC4a * s3;
    Y[17] = -kShC4b * z * s2;
    Y[18] = p4b * s1;
    Y[19] = p4a * y;
    Y[20] = fmaf(kShC4g * z, Y[12], -kShC4h * Y[6]);
    Y[21] = p4a * x;
    Y[22] = p4b * c1;
    Y[23] = -kShC4b * z * c2;
    Y[24] = kShC4a * c3;
}

// Gradient of sum_k g[k] * Y_k with respect to the normalised (x,y,z), where g[k] is the
// colour-weighted coefficient sum. Only bands 1.. contribute (Y_0 is constant).
__device__ __forceinline__ void sh_basis_vjp(int degree, float x, float y, float z, const float* g,
                                             float& gx, float& gy, float& gz) {
    gx = 0.f;
    gy = 0.f;
    gz = 0.f;
    if (degree < 1) return;
    gx = fmaf(-kShC1, g[3], gx);
    gy = fmaf(-kShC1, g[1], gy);
    gz = fmaf(kShC1, g[2], gz);
    if (degree < 2) return;
    const float z2 = z * z;
    const float c1 = x * x - y * y, s1 = 2.f * x * y;
    // partials of the helper polynomials
    const float c1x = 2.f * x, c1y = -2.f * y;
    const float s1x = 2.f * y, s1y = 2.f * x;
    // Y4 = C s1, Y5 = -a z y, Y6 = 3b z^2 - b, Y7 = -a z x, Y8 = C c1
    gx += g[4] * kShC2c * s1x + g[7] * (-kShC2a * z) + g[8] * kShC2c * c1x;
    gy += g[4] * kShC2c * s1y + g[5] * (-kShC2a * z) + g[8] * kShC2c * c1y;
    gz += g[5] * (-kShC2a * y) + g[6] * (6.f * kShC2b * z) + g[7] * (-kShC2a * x);
    if (degree < 3) return;
    const float c2 = x * c1 - y * s1, s2 = x * s1 + y * c1;
    const float c2x = c1 + x * c1x - y * s1x, c2y = x * c1y - s1 - y * s1y;
    const float s2x = s1 + x * s1x + y * c1x, s2y = x * s1y + c1 + y * c1y;
    const float p3 = fmaf(-kShC3c, z2, kShC3d), p3z = -2.f * kShC3c * z;
    const float q3 = z * fmaf(kShC3e, z2, -kShC3f), q3z = fmaf(3.f * kShC3e, z2, -kShC3f);
    // Y9 = -a s2, Y10 = b z s1, Y11 = p3 y, Y12 = q3, Y13 = p3 x, Y14 = b z c1, Y15 = -a c2
    gx += g[9] * (-kShC3a * s2x) + g[10] * (kShC3b * z * s1x) + g[13] * p3 +
          g[14] * (kShC3b * z * c1x) + g[15] * (-kShC3a * c2x);
    gy += g[9] * (-kShC3a * s2y) + g[10] * (kShC3b * z * s1y) + g[11] * p3 +
          g[14] * (kShC3b * z * c1y) + g[15] * (-kShC3a * c2y);
    gz += g[10] * (kShC3b * s1) + g[11] * (p3z * y) + g[12] * q3z + g[13] * (p3z * x) +
          g[14] * (kShC3b * c1);
    if (degree < 4) return;
    const float c3x = c2 + x * c2x - y * s2x, c3y = x * c2y - s2 - y * s2y;
    const float s3x = s2 + x * s2x + y * c2x, s3y = x * s2y + c2 + y * c2y;
    const float c3 = x * c2 - y * s2, s3 = x * s2 + y * c2;
    const float p4a = z * fmaf(-kShC4e, z2, kShC4f), p4az = fmaf(-3.f * kShC4e, z2, kShC4f);
    const float p4b = fmaf(kShC4c, z2, -kShC4d), p4bz = 2.f * kShC4c * z;
    const float y6 = fmaf(3.f * kShC2b, z2, -kShC2b), y6z = 6.f * kShC2b * z;
    // Y20 = g z q3 - h y6  ->  d/dz = g (q3 + z q3z) - h y6z
    gx += g[16] * (kShC4a * s3x) + g[17] * (-kShC4b * z * s2x) + g[18] * (p4b * s1x) +
          g[21] * p4a + g[22] * (p4b * c1x) + g[23] * (-kShC4b * z * c2x) + g[24] * (kShC4a * c3x);
    gy += g[16] * (kShC4a * s3y) + g[17] * (-kShC4b * z * s2y) + g[18] * (p4b * s1y) +
          g[19] * p4a + g[22] * (p4b * c1y) + g[23] * (-kShC4b * z * c2y) + g[24] * (kShC4a * c3y);
    gz += g[17] * (-kShC4b * s2) + g[18] * (p4bz * s1) + g[19] * (p4az * y) +
          g[20] * (kShC4g * (q3 + z * q3z) - kShC4h * y6z) + g[21] * (p4az * x) +
          g[22] * (p4bz * c1) + g[23] * (-kShC4b * c2);
    (void)c3;
    (void)s3;
}

}  // namespace sx
