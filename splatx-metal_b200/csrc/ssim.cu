// ssim.cu — SSIM forward/backward (11x11 Gaussian window, sigma 1.5, C1=1e-4, C2=9e-4, "valid"
// padding, gradient for img1 only; Ssim.metal:66-268 / spec 08) and the executor's fused
// L1+SSIM loss.
//
// Forward: a 16x16 map tile per CTA per (image, channel); the 26x26 apron of both images is staged
// in shared memory, the separable window runs horizontally (26 rows x 16 columns, five moments)
// then vertically. With need_coeffs the kernel also writes the three coefficient maps the
// backward needs:  Dmu = dS/dmu1 - 2 mu1 dS/dsigma1 - mu2 dS/dsigma12, Dsig = dS/dsigma1,
// Dcross = dS/dsigma12.
// Backward: v_img1(q) = G [ (w*Dmu)(q) + 2 x(q) (w*Dsig)(q) + y(q) (w*Dcross)(q) ], G = -v_loss/M,
// the adjoint of the valid correlation = a full correlation over zero-padded maps.
// Means are reduced on the device in f64 in a fixed tree order (bit-deterministic).
#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

constexpr int T = kSsimTile, A = kSsimApron, WIN = kSsimWin;

__device__ __forceinline__ int64_t ihwc(int64_t i, int64_t y, int64_t x, int64_t c, int64_t H,
                                        int64_t W, int64_t C) {
    return (((i * H + y) * W) + x) * C + c;
}

// Fixed-order block sum of one double per thread (256 threads, 1-D or 16x16) -> the thread of
// linear index 0 returns the total.
__device__ __forceinline__ double block_sum_f64(double v, double* sm) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
    const int tid = threadIdx.y * blockDim.x + threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    if (lane == 0) sm[warp] = v;
    __syncthreads();
    double t = 0.0;
    if (tid == 0)
        for (int w = 0; w < (T * T) / 32; ++w) t += sm[w];
    return t;
}

__global__ void __launch_bounds__(T* T)
ssim_fwd_kernel(const float* __restrict__ img1, const float* __restrict__ img2, int64_t H,
                int64_t W, int64_t C, int64_t map_h, int64_t map_w, bool need_coeffs,
                float* __restrict__ map, float* __restrict__ cmu, float* __restrict__ csg,
                float* __restrict__ ccr, double* __restrict__ partials) {
    __shared__ float tx[A * A], ty[A * A];
    __shared__ float h1[A * T], h2[A * T], h11[A * T], h22[A * T], h12[A * T];
    __shared__ double red[8];
    const int tid = threadIdx.y * T + threadIdx.x;
    const int64_t img = blockIdx.z / C, ch = blockIdx.z % C;
    const int64_t oy = static_cast<int64_t>(blockIdx.y) * T, ox = static_cast<int64_t>(blockIdx.x) * T;
    for (int i = tid; i < A * A; i += T * T) {
        const int64_t gy = oy + i / A, gx = ox + i % A;
        float a = 0.f, b = 0.f;
        if (gy < H && gx < W) {
            const int64_t off = ihwc(img, gy, gx, ch, H, W, C);
            a = img1[off];
            b = img2[off];
        }
        tx[i] = a;
        ty[i] = b;
    }
    __syncthreads();
    for (int i = tid; i < A * T; i += T * T) {
        const int r = i / T, cx = i % T;
        float m1 = 0.f, m2 = 0.f, e11 = 0.f, e22 = 0.f, e12 = 0.f;
#pragma unroll
        for (int u = 0; u < WIN; ++u) {
            const float w = kSsimTaps[u];
            const float x = tx[r * A + cx + u], y = ty[r * A + cx + u];
            m1 = fmaf(w, x, m1);
            m2 = fmaf(w, y, m2);
            e11 = fmaf(w * x, x, e11);
            e22 = fmaf(w * y, y, e22);
            e12 = fmaf(w * x, y, e12);
        }
        h1[i] = m1; h2[i] = m2; h11[i] = e11; h22[i] = e22; h12[i] = e12;
    }
    __syncthreads();
    const int64_t my = oy + threadIdx.y, mx = ox + threadIdx.x;
    double part = 0.0;
    if (my < map_h && mx < map_w) {
        float mu1 = 0.f, mu2 = 0.f, e11 = 0.f, e22 = 0.f, e12 = 0.f;
#pragma unroll
        for (int v = 0; v < WIN; ++v) {
            const float w = kSsimTaps[v];
            const int i = (threadIdx.y + v) * T + threadIdx.x;
            mu1 = fmaf(w, h1[i], mu1);
            mu2 = fmaf(w, h2[i], mu2);
            e11 = fmaf(w, h11[i], e11);
            e22 = fmaf(w, h22[i], e22);
            e12 = fmaf(w, h12[i], e12);
        }
        const float s1 = fmaf(-mu1, mu1, e11);
        const float s2 = fmaf(-mu2, mu2, e22);
        const float s12 = fmaf(-mu1, mu2, e12);
        const float A1 = 2.f * mu1 * mu2 + kSsimC1;
        const float B1 = mu1 * mu1 + mu2 * mu2 + kSsimC1;
        const float A2 = 2.f * s12 + kSsimC2;
        const float B2 = s1 + s2 + kSsimC2;
        const float den = B1 * B2;
        const float S = (A1 * A2) / den;
        const int64_t mo = ihwc(img, my, mx, ch, map_h, map_w, C);
        map[mo] = S;
        part = static_cast<double>(S);
        if (need_coeffs) {
            const float d_mu1 = 2.f * (mu2 * A2 / den - mu1 * S / B1);
            const float d_s1 = -S / B2;
            const float d_s12 = 2.f * A1 / den;
            cmu[mo] = d_mu1 - 2.f * mu1 * d_s1 - mu2 * d_s12;
            csg[mo] = d_s1;
            ccr[mo] = d_s12;
        }
    }
    const double t = block_sum_f64(part, red);
    if (tid == 0) {
        const int64_t b = (static_cast<int64_t>(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        partials[b] = t;
    }
}

// Backward, one thread per input pixel of one channel. With l1 != nullptr (executor) it also
// folds the L1 gradient w_l1 * sign(x - y) / n and the per-block sum of |x - y| (f64).
__global__ void __launch_bounds__(T* T)
ssim_bwd_kernel(const float* __restrict__ img1, const float* __restrict__ img2, int64_t H,
                int64_t W, int64_t C, int64_t map_h, int64_t map_w, const float* __restrict__ cmu,
                const float* __restrict__ csg, const float* __restrict__ ccr, float G,
                float* __restrict__ v_img1, bool with_l1, float w_l1, float l1_g,
                double* __restrict__ l1_partials) {
    __shared__ float t1[A * A], t2[A * A], t3[A * A];
    __shared__ float h1[A * T], h2[A * T], h3[A * T];
    __shared__ double red[8];
    const int tid = threadIdx.y * T + threadIdx.x;
    const int64_t img = blockIdx.z / C, ch = blockIdx.z % C;
    const int64_t oy = static_cast<int64_t>(blockIdx.y) * T, ox = static_cast<int64_t>(blockIdx.x) * T;
    constexpr int PAD = WIN - 1;
    for (int i = tid; i < A * A; i += T * T) {
        const int64_t py = oy + i / A - PAD, px = ox + i % A - PAD;
        float a = 0.f, b = 0.f, c = 0.f;
        if (py >= 0 && py < map_h && px >= 0 && px < map_w) {
            const int64_t off = ihwc(img, py, px, ch, map_h, map_w, C);
            a = cmu[off];
            b = csg[off];
            c = ccr[off];
        }
        t1[i] = a;
        t2[i] = b;
        t3[i] = c;
    }
    __syncthreads();
    for (int i = tid; i < A * T; i += T * T) {
        const int r = i / T, cx = i % T;
        float s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int u = 0; u < WIN; ++u) {
            const float w = kSsimTaps[u];
            s1 = fmaf(w, t1[r * A + cx + u], s1);
            s2 = fmaf(w, t2[r * A + cx + u], s2);
            s3 = fmaf(w, t3[r * A + cx + u], s3);
        }
        h1[i] = s1;
        h2[i] = s2;
        h3[i] = s3;
    }
    __syncthreads();
    const int64_t qy = oy + threadIdx.y, qx = ox + threadIdx.x;
    double part = 0.0;
    if (qy < H && qx < W) {
        float c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
        for (int v = 0; v < WIN; ++v) {
            const float w = kSsimTaps[v];
            const int i = (threadIdx.y + v) * T + threadIdx.x;
            c1 = fmaf(w, h1[i], c1);
            c2 = fmaf(w, h2[i], c2);
            c3 = fmaf(w, h3[i], c3);
        }
        const int64_t q = ihwc(img, qy, qx, ch, H, W, C);
        const float x = img1[q], y = img2[q];
        float out = G * (c1 + 2.f * x * c2 + y * c3);
        if (with_l1) {
            const float d = x - y;
            const float base = d > 0.0f ? l1_g : (d < 0.0f ? -l1_g : 0.0f);
            out = w_l1 * base + out;
            part = fabs(static_cast<double>(d));
        }
        v_img1[q] = out;
    }
    if (with_l1) {
        const double t = block_sum_f64(part, red);
        if (tid == 0) {
            const int64_t b = (static_cast<int64_t>(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
            l1_partials[b] = t;
        }
    }
}

// ---- the executor's fused loss: 32x16 tiles, all three channels per CTA -------------------
// Same arithmetic per output as ssim_fwd_kernel / ssim_bwd_kernel (tap order, fmaf chains,
// formulas), different work split: the interleaved image rows of the tile's apron load coalesced
// once for the three channels; the horizontal pass gives each thread four adjacent outputs read
// with float4 shared loads (8 loads per 4 outputs instead of 88); the vertical pass gives each
// thread two rows. Coefficient maps are planar [3][mh][mw] and no SSIM map is written.
constexpr int LX = 32, LY = 16;           // tile (map points forward, pixels backward)
constexpr int LAY = LY + WIN - 1;         // 26 apron rows
constexpr int LAX = LX + WIN - 1;         // 42 apron columns
constexpr int LAXP = LAX + 2;             // 44: rows padded to whole float4s
constexpr int LGROUPS = LAY * (LX / 4);   // 208 horizontal work items (4 outputs each)

// 4-byte asynchronous global -> shared copy; src_ok == false writes 0 without reading `src`.
__device__ __forceinline__ void cp_async_f32_zfill(float* dst, const float* src, bool src_ok) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src),
                 "r"(src_ok ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void load_row14(const float* row, int c0, float (&v)[16]) {
    const float4* p = reinterpret_cast<const float4*>(row + c0);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float4 q = p[k];
        v[4 * k] = q.x; v[4 * k + 1] = q.y; v[4 * k + 2] = q.z; v[4 * k + 3] = q.w;
    }
}

__global__ void __launch_bounds__(256, 3)
ssim_loss_fwd_kernel(const float* __restrict__ img1, const float* __restrict__ img2, int H, int W,
                     int mh, int mw, float* __restrict__ cmu, float* __restrict__ csg,
                     float* __restrict__ ccr, double* __restrict__ partials) {
    __shared__ __align__(16) float sx[3][LAY][LAXP];
    __shared__ __align__(16) float sy[3][LAY][LAXP];
    __shared__ __align__(16) float hm[5][LAY][LX];
    __shared__ double red[8];
    const int tid = threadIdx.x;
    const int ox = blockIdx.x * LX, oy = blockIdx.y * LY;
    {
        // warps over apron rows, lanes over a row's 126 interleaved floats (42 pixels x RGB),
        // which are contiguous in the image: element e of row r is (oy + r, ox + e / 3), channel
        // e % 3; the lane's four (pixel, channel) pairs are fixed, only the row base moves
        const int lane = tid & 31, warp = tid >> 5;
        for (int r = warp; r < LAY; r += 8) {
            const int gy = oy + r;
            const int64_t base = (static_cast<int64_t>(gy) * W + ox) * 3;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int e = lane + 32 * j;
                if (e >= LAX * 3) continue;
                const int col = e / 3, ch = e - 3 * col;
                const bool ok = gy < H && ox + col < W;
                const int64_t off = ok ? base + e : 0;
                cp_async_f32_zfill(&sx[ch][r][col], img1 + off, ok);
                cp_async_f32_zfill(&sy[ch][r][col], img2 + off, ok);
            }
        }
    }
    cp_async_commit();
    cp_async_wait<0>();
    if (tid < 3 * LAY * 2) {  // the two pad columns (read by the last float4, never used)
        const int ch = tid / (LAY * 2), r = (tid / 2) % LAY, c = LAX + (tid & 1);
        sx[ch][r][c] = 0.f;
        sy[ch][r][c] = 0.f;
    }
    __syncthreads();
    double part = 0.0;
    const int col = tid & 31, g = tid >> 5;
    for (int ch = 0; ch < 3; ++ch) {
        if (tid < LGROUPS) {
            const int r = tid / (LX / 4), c0 = (tid % (LX / 4)) * 4;
            float X[16], Y[16];
            load_row14(&sx[ch][r][0], c0, X);
            load_row14(&sy[ch][r][0], c0, Y);
            float o[5][4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float m1 = 0.f, m2 = 0.f, e11 = 0.f, e22 = 0.f, e12 = 0.f;
#pragma unroll
                for (int u = 0; u < WIN; ++u) {
                    const float w = kSsimTaps[u];
                    const float x = X[q + u], y = Y[q + u];
                    m1 = fmaf(w, x, m1);
                    m2 = fmaf(w, y, m2);
                    e11 = fmaf(w * x, x, e11);
                    e22 = fmaf(w * y, y, e22);
                    e12 = fmaf(w * x, y, e12);
                }
                o[0][q] = m1; o[1][q] = m2; o[2][q] = e11; o[3][q] = e22; o[4][q] = e12;
            }
#pragma unroll
            for (int k = 0; k < 5; ++k)
                *reinterpret_cast<float4*>(&hm[k][r][c0]) = make_float4(o[k][0], o[k][1], o[k][2], o[k][3]);
        }
        __syncthreads();
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int r = 2 * g + rr;
            const int my = oy + r, mx = ox + col;
            float mu1 = 0.f, mu2 = 0.f, e11 = 0.f, e22 = 0.f, e12 = 0.f;
#pragma unroll
            for (int v = 0; v < WIN; ++v) {
                const float w = kSsimTaps[v];
                mu1 = fmaf(w, hm[0][r + v][col], mu1);
                mu2 = fmaf(w, hm[1][r + v][col], mu2);
                e11 = fmaf(w, hm[2][r + v][col], e11);
                e22 = fmaf(w, hm[3][r + v][col], e22);
                e12 = fmaf(w, hm[4][r + v][col], e12);
            }
            if (my < mh && mx < mw) {
                const float s1 = fmaf(-mu1, mu1, e11);
                const float s2 = fmaf(-mu2, mu2, e22);
                const float s12 = fmaf(-mu1, mu2, e12);
                const float A1 = 2.f * mu1 * mu2 + kSsimC1;
                const float B1 = mu1 * mu1 + mu2 * mu2 + kSsimC1;
                const float A2 = 2.f * s12 + kSsimC2;
                const float B2 = s1 + s2 + kSsimC2;
                const float den = B1 * B2;
                const float S = (A1 * A2) / den;
                part += static_cast<double>(S);
                const float d_mu1 = 2.f * (mu2 * A2 / den - mu1 * S / B1);
                const float d_s1 = -S / B2;
                const float d_s12 = 2.f * A1 / den;
                const int64_t mo = (static_cast<int64_t>(ch) * mh + my) * mw + mx;
                cmu[mo] = d_mu1 - 2.f * mu1 * d_s1 - mu2 * d_s12;
                csg[mo] = d_s1;
                ccr[mo] = d_s12;
            }
        }
        __syncthreads();
    }
    const double t = block_sum_f64(part, red);
    if (tid == 0) partials[static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x] = t;
}

// Backward of the fused loss: v(q) = G [(w*Dmu)(q) + 2 x(q) (w*Dsig)(q) + y(q) (w*Dcross)(q)]
// (zero-padded coefficient maps) + w_l1 sign(x - y) / n, and per-CTA sums of |x - y| (f64).
__global__ void __launch_bounds__(256)
ssim_loss_bwd_kernel(const float* __restrict__ img1, const float* __restrict__ img2, int H, int W,
                     int mh, int mw, const float* __restrict__ cmu, const float* __restrict__ csg,
                     const float* __restrict__ ccr, float G, float w_l1, float l1_g,
                     float* __restrict__ v_img1, double* __restrict__ l1_partials) {
    extern __shared__ __align__(16) float dyn[];
    float (*tm)[3][LAY][LAXP] = reinterpret_cast<float (*)[3][LAY][LAXP]>(dyn);  // [ch][map]
    __shared__ __align__(16) float hb[3][LAY][LX];
    __shared__ double red[8];
    constexpr int PAD = WIN - 1;
    const int tid = threadIdx.x;
    const int ox = blockIdx.x * LX, oy = blockIdx.y * LY;
    const int col = tid & 31, g = tid >> 5;
    double part = 0.0;
    // the three channels' map aprons, one commit group per channel, all in flight at once:
    // warps over the 3 x 26 apron rows of a channel, lanes over a row's 44 (padded) columns
    {
        const int lane = tid & 31, warp = tid >> 5;
        const int px0 = ox - PAD + lane, px1 = px0 + 32;
        const bool c1_in = lane + 32 < LAXP;
        const bool x0_ok = px0 >= 0 && px0 < mw, x1_ok = lane + 32 < LAX && px1 >= 0 && px1 < mw;
        for (int ch = 0; ch < 3; ++ch) {
            for (int kr = warp; kr < 3 * LAY; kr += 8) {
                const int k = kr / LAY, r = kr - k * LAY;
                const int py = oy + r - PAD;
                const bool y_ok = py >= 0 && py < mh;
                const float* src = (k == 0 ? cmu : (k == 1 ? csg : ccr)) +
                                   (y_ok ? (static_cast<int64_t>(ch) * mh + py) * mw : 0);
                float* dst = &tm[ch][k][r][0];
                cp_async_f32_zfill(dst + lane, src + (y_ok && x0_ok ? px0 : 0), y_ok && x0_ok);
                if (c1_in)
                    cp_async_f32_zfill(dst + lane + 32, src + (y_ok && x1_ok ? px1 : 0),
                                       y_ok && x1_ok);
            }
            cp_async_commit();
        }
    }
    for (int ch = 0; ch < 3; ++ch) {
        if (ch == 0) cp_async_wait<2>();
        else if (ch == 1) cp_async_wait<1>();
        else cp_async_wait<0>();
        __syncthreads();
        if (tid < LGROUPS) {
            const int r = tid / (LX / 4), c0 = (tid % (LX / 4)) * 4;
            float o[3][4];
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                float T[16];
                load_row14(&tm[ch][k][r][0], c0, T);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float acc = 0.f;
#pragma unroll
                    for (int u = 0; u < WIN; ++u) acc = fmaf(kSsimTaps[u], T[q + u], acc);
                    o[k][q] = acc;
                }
            }
#pragma unroll
            for (int k = 0; k < 3; ++k)
                *reinterpret_cast<float4*>(&hb[k][r][c0]) = make_float4(o[k][0], o[k][1], o[k][2], o[k][3]);
        }
        __syncthreads();
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int r = 2 * g + rr;
            const int qy = oy + r, qx = ox + col;
            float c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
            for (int v = 0; v < WIN; ++v) {
                const float w = kSsimTaps[v];
                c1 = fmaf(w, hb[0][r + v][col], c1);
                c2 = fmaf(w, hb[1][r + v][col], c2);
                c3 = fmaf(w, hb[2][r + v][col], c3);
            }
            if (qy < H && qx < W) {
                const int64_t q = (static_cast<int64_t>(qy) * W + qx) * 3 + ch;
                const float x = img1[q], y = img2[q];
                float out = G * (c1 + 2.f * x * c2 + y * c3);
                const float d = x - y;
                const float base = d > 0.0f ? l1_g : (d < 0.0f ? -l1_g : 0.0f);
                out = w_l1 * base + out;
                part += fabs(static_cast<double>(d));
                v_img1[q] = out;
            }
        }
        __syncthreads();
    }
    const double t = block_sum_f64(part, red);
    if (tid == 0) l1_partials[static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x] = t;
}

// L1 only (ssim_weight == 0): v = sign(r - gt) / n, per-block sums of |r - gt|.
__global__ void __launch_bounds__(256)
l1_kernel(const float* __restrict__ r, const float* __restrict__ gt, int64_t n, float g,
          float* __restrict__ v, double* __restrict__ partials) {
    __shared__ double red[8];
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    double part = 0.0;
    if (i < n) {
        const float d = r[i] - gt[i];
        v[i] = d > 0.0f ? g : (d < 0.0f ? -g : 0.0f);
        part = fabs(static_cast<double>(d));
    }
    const double t = block_sum_f64(part, red);
    if (threadIdx.x == 0) partials[blockIdx.x] = t;
}

// Fixed-order sum of `n` partials by one CTA of 256 threads.
__device__ __forceinline__ double sum_partials(const double* p, int64_t n, double* sm) {
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += 256) s += p[i];
    return block_sum_f64(s, sm);
}

__global__ void __launch_bounds__(256)
mean_kernel(const double* __restrict__ partials, int64_t nparts, double denom,
            double* __restrict__ out) {
    __shared__ double red[8];
    const double t = sum_partials(partials, nparts, red);
    if (threadIdx.x == 0) *out = t / denom;
}

__global__ void __launch_bounds__(256)
loss_kernel(const double* __restrict__ l1_parts, int64_t n_l1, double n_px,
            const double* __restrict__ ssim_parts, int64_t n_ssim, double m_count, float lam,
            float* __restrict__ loss, const int32_t* skip_flag) {
    __shared__ double red[8];
    const double l1 = sum_partials(l1_parts, n_l1, red);
    __syncthreads();
    double ss = 0.0;
    if (n_ssim > 0) ss = sum_partials(ssim_parts, n_ssim, red);
    if (threadIdx.x == 0) {
        const float l1_loss = static_cast<float>(l1 / n_px);
        float out = l1_loss;
        if (n_ssim > 0) {
            const double ssim = ss / m_count;
            out = (1.0f - lam) * l1_loss + lam * (1.0f - static_cast<float>(ssim));
        }
        if (skip_flag && *skip_flag) out = __int_as_float(0x7fc00000);  // overflowed step
        *loss = out;
    }
}

size_t align_up(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

dim3 ssim_grid(int64_t rows, int64_t cols, int64_t planes) {
    return dim3(static_cast<unsigned>((cols + T - 1) / T), static_cast<unsigned>((rows + T - 1) / T),
                static_cast<unsigned>(planes));
}

}  // namespace

size_t ssim_fwd_workspace(int64_t I, int64_t H, int64_t W, int64_t C) {
    const dim3 g = ssim_grid(H - (WIN - 1), W - (WIN - 1), I * C);
    return align_up(sizeof(double) * static_cast<size_t>(g.x) * g.y * g.z);
}

void launch_ssim_fwd(const float* img1, const float* img2, int64_t I, int64_t H, int64_t W,
                     int64_t C, bool need_coeffs, float* map, float* cmu, float* csg, float* ccr,
                     double* mean_out, void* ws, cudaStream_t s) {
    const int64_t mh = H - (WIN - 1), mw = W - (WIN - 1);
    const dim3 g = ssim_grid(mh, mw, I * C);
    double* parts = static_cast<double*>(ws);
    SX_LAUNCH(ssim_fwd_kernel, g, dim3(T, T), 0, s, img1, img2, H, W, C, mh, mw, need_coeffs, map,
              cmu, csg, ccr, parts);
    const int64_t np = static_cast<int64_t>(g.x) * g.y * g.z;
    SX_LAUNCH(mean_kernel, 1, 256, 0, s, parts, np, static_cast<double>(I * C * mh * mw), mean_out);
}

void launch_ssim_bwd(const float* img1, const float* img2, int64_t I, int64_t H, int64_t W,
                     int64_t C, const float* cmu, const float* csg, const float* ccr, float G,
                     float* v_img1, cudaStream_t s) {
    const int64_t mh = H - (WIN - 1), mw = W - (WIN - 1);
    const dim3 g = ssim_grid(H, W, I * C);
    SX_LAUNCH(ssim_bwd_kernel, g, dim3(T, T), 0, s, img1, img2, H, W, C, mh, mw, cmu, csg, ccr, G,
              v_img1, false, 0.f, 0.f, static_cast<double*>(nullptr));
}

size_t loss_workspace(int64_t H, int64_t W) {
    const int64_t mh = H > WIN - 1 ? H - (WIN - 1) : 1, mw = W > WIN - 1 ? W - (WIN - 1) : 1;
    const int64_t gf = ((mw + LX - 1) / LX) * ((mh + LY - 1) / LY);
    const int64_t gb = ((W + LX - 1) / LX) * ((H + LY - 1) / LY);
    const int64_t n_l1 = (H * W * 3 + 255) / 256;
    const int64_t nb = gb > n_l1 ? gb : n_l1;
    return align_up(sizeof(double) * static_cast<size_t>(gf)) +
           align_up(sizeof(double) * static_cast<size_t>(nb));
}

void launch_train_loss(const float* render, const float* gt, int64_t H, int64_t W,
                       float ssim_weight, float* map, float* cmu, float* csg, float* ccr,
                       float* v_render, float* loss_out, void* ws, const int32_t* skip_flag,
                       cudaStream_t s) {
    (void)map;  // the executor needs no SSIM map
    const int64_t n_px = H * W * 3;
    const float l1_g = 1.0f / static_cast<float>(n_px);
    const int64_t gmh = H > WIN - 1 ? H - (WIN - 1) : 1, gmw = W > WIN - 1 ? W - (WIN - 1) : 1;
    const dim3 gf(static_cast<unsigned>((gmw + LX - 1) / LX), static_cast<unsigned>((gmh + LY - 1) / LY));
    const size_t off = align_up(sizeof(double) * static_cast<size_t>(gf.x) * gf.y);
    double* ssim_parts = static_cast<double*>(ws);
    double* l1_parts = reinterpret_cast<double*>(static_cast<unsigned char*>(ws) + off);
    if (ssim_weight > 0.0f) {
        const int mh = static_cast<int>(H - (WIN - 1)), mw = static_cast<int>(W - (WIN - 1));
        SX_LAUNCH(ssim_loss_fwd_kernel, gf, 256, 0, s, render, gt, static_cast<int>(H),
                  static_cast<int>(W), mh, mw, cmu, csg, ccr, ssim_parts);
        const dim3 gb(static_cast<unsigned>((W + LX - 1) / LX), static_cast<unsigned>((H + LY - 1) / LY));
        const float G = -ssim_weight / static_cast<float>(3 * static_cast<int64_t>(mh) * mw);
        constexpr size_t kBwdDyn = sizeof(float) * 3 * 3 * LAY * LAXP;  // 41 KB of map aprons
        smem_limit_once(reinterpret_cast<const void*>(ssim_loss_bwd_kernel), static_cast<int>(kBwdDyn),
                        "ssim loss smem attribute");
        SX_LAUNCH(ssim_loss_bwd_kernel, gb, 256, kBwdDyn, s, render, gt, static_cast<int>(H),
                  static_cast<int>(W), mh, mw, cmu, csg, ccr, G, 1.0f - ssim_weight, l1_g, v_render,
                  l1_parts);
        SX_LAUNCH(loss_kernel, 1, 256, 0, s, l1_parts, static_cast<int64_t>(gb.x) * gb.y,
                  static_cast<double>(n_px), ssim_parts, static_cast<int64_t>(gf.x) * gf.y,
                  static_cast<double>(3 * static_cast<int64_t>(mh) * mw), ssim_weight, loss_out,
                  skip_flag);
    } else {
        const int64_t nb = (n_px + 255) / 256;
        SX_LAUNCH(l1_kernel, static_cast<unsigned>(nb), 256, 0, s, render, gt, n_px, l1_g, v_render,
                  l1_parts);
        SX_LAUNCH(loss_kernel, 1, 256, 0, s, l1_parts, nb, static_cast<double>(n_px),
                  static_cast<const double*>(nullptr), int64_t(0), 0.0, 0.0f, loss_out, skip_flag);
    }
}

}  // namespace sx
