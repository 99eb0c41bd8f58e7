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
    const dim3 gf = ssim_grid(mh, mw, 3);
    const dim3 gb = ssim_grid(H, W, 3);
    const int64_t n_l1 = (H * W * 3 + 255) / 256;
    const int64_t nb = static_cast<int64_t>(gb.x) * gb.y * gb.z;
    return align_up(sizeof(double) * static_cast<size_t>(gf.x) * gf.y * gf.z) +
           align_up(sizeof(double) * static_cast<size_t>(nb > n_l1 ? nb : n_l1));
}

void launch_train_loss(const float* render, const float* gt, int64_t H, int64_t W,
                       float ssim_weight, float* map, float* cmu, float* csg, float* ccr,
                       float* v_render, float* loss_out, void* ws, const int32_t* skip_flag,
                       cudaStream_t s) {
    const int64_t n_px = H * W * 3;
    const float l1_g = 1.0f / static_cast<float>(n_px);
    const int64_t gmh = H > WIN - 1 ? H - (WIN - 1) : 1, gmw = W > WIN - 1 ? W - (WIN - 1) : 1;
    const dim3 gf = ssim_grid(gmh, gmw, 3);
    const size_t off = align_up(sizeof(double) * static_cast<size_t>(gf.x) * gf.y * gf.z);
    double* ssim_parts = static_cast<double*>(ws);
    double* l1_parts = reinterpret_cast<double*>(static_cast<unsigned char*>(ws) + off);
    if (ssim_weight > 0.0f) {
        const int64_t mh = H - (WIN - 1), mw = W - (WIN - 1);
        SX_LAUNCH(ssim_fwd_kernel, gf, dim3(T, T), 0, s, render, gt, H, W, int64_t(3), mh, mw,
                  true, map, cmu, csg, ccr, ssim_parts);
        const dim3 gb = ssim_grid(H, W, 3);
        const float G = -ssim_weight / static_cast<float>(3 * mh * mw);
        SX_LAUNCH(ssim_bwd_kernel, gb, dim3(T, T), 0, s, render, gt, H, W, int64_t(3), mh, mw, cmu,
                  csg, ccr, G, v_render, true, 1.0f - ssim_weight, l1_g, l1_parts);
        SX_LAUNCH(loss_kernel, 1, 256, 0, s, l1_parts,
                  static_cast<int64_t>(gb.x) * gb.y * gb.z, static_cast<double>(n_px), ssim_parts,
                  static_cast<int64_t>(gf.x) * gf.y * gf.z, static_cast<double>(3 * mh * mw),
                  ssim_weight, loss_out, skip_flag);
    } else {
        const int64_t nb = (n_px + 255) / 256;
        SX_LAUNCH(l1_kernel, static_cast<unsigned>(nb), 256, 0, s, render, gt, n_px, l1_g, v_render,
                  l1_parts);
        SX_LAUNCH(loss_kernel, 1, 256, 0, s, l1_parts, nb, static_cast<double>(n_px),
                  static_cast<const double*>(nullptr), int64_t(0), 0.0, 0.0f, loss_out, skip_flag);
    }
}

}  // namespace sx
