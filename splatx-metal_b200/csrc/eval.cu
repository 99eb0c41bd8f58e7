// eval.cu — device-side evaluation of a rendered view and frame quantisation.
//
// The reference evaluates on the host (TrainC.cpp:653-696): the render is clamped to [0, 1],
// PSNR = 10 log10(1 / mse) with the squared differences summed in double (psnr, Trainer.cpp:
// 349-360), an affine per-channel colour correction from four double moments per channel
// (color_correct_affine, Trainer.cpp:364-392) and SSIM of the clamped and the corrected render
// against the target (eval_ssim, Trainer.cpp:405-418). Here the same arithmetic runs on the device
// next to the render: sums are double per-block partials reduced in a fixed order (the metrics are
// bit-deterministic), and only four doubles come back. Frames for video (sx_render_session_frame,
// TrainC.cpp:1518-1572) are quantised on the device to RGBA8 (NaN -> 0, clamp, round half to even
// of v * 255, alpha 255), so a frame crosses PCIe as 4 bytes per pixel instead of 12.
#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

constexpr int kEvalThreads = 256;
constexpr int kEvalBlocks = 4 * 148;

__device__ __forceinline__ double block_sum(double v, double* sh) {
    sh[threadIdx.x] = v;
    __syncthreads();
#pragma unroll
    for (int s = kEvalThreads / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) sh[threadIdx.x] += sh[threadIdx.x + s];
        __syncthreads();
    }
    const double r = sh[0];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kEvalThreads) clamp01_kernel(float* __restrict__ x, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = x[i];
        x[i] = v < 0.0f ? 0.0f : (1.0f < v ? 1.0f : v);  // std::clamp: NaN stays NaN
    }
}

// parts[b] = sum over block b's grid-stride share of (a - b)^2 in double
__global__ void __launch_bounds__(kEvalThreads)
sqdiff_kernel(const float* __restrict__ a, const float* __restrict__ b, int64_t n,
              double* __restrict__ parts) {
    __shared__ double sh[kEvalThreads];
    double acc = 0.0;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const double d = static_cast<double>(a[i]) - static_cast<double>(b[i]);
        acc += d * d;
    }
    const double s = block_sum(acc, sh);
    if (threadIdx.x == 0) parts[blockIdx.x] = s;
}

// parts[b * 12 + 4c + {0..3}] = block b's sums of ref, img, ref*img, ref*ref of channel c
__global__ void __launch_bounds__(kEvalThreads)
cc_moments_kernel(const float* __restrict__ img, const float* __restrict__ ref, int64_t n_px,
                  double* __restrict__ parts) {
    __shared__ double sh[kEvalThreads];
    double m[12] = {};
    for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < n_px;
         p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const double r = static_cast<double>(ref[p * 3 + c]);
            const double v = static_cast<double>(img[p * 3 + c]);
            m[4 * c] += r;
            m[4 * c + 1] += v;
            m[4 * c + 2] += r * v;
            m[4 * c + 3] += r * r;
        }
    }
#pragma unroll 1
    for (int k = 0; k < 12; ++k) {
        const double s = block_sum(m[k], sh);
        if (threadIdx.x == 0) parts[blockIdx.x * 12 + k] = s;
    }
}

// out[k] = sum over b of parts[b * width + k], each thread a fixed strided subset, then a tree
__global__ void __launch_bounds__(kEvalThreads)
reduce_parts_kernel(const double* __restrict__ parts, int nparts, int width, double* __restrict__ out) {
    __shared__ double sh[kEvalThreads];
    for (int k = 0; k < width; ++k) {
        double acc = 0.0;
        for (int b = threadIdx.x; b < nparts; b += kEvalThreads) acc += parts[b * width + k];
        const double s = block_sum(acc, sh);
        if (threadIdx.x == 0) out[k] = s;
    }
}

// color_correct_affine's per-channel map, out = clip((img - b) / a, 0, 1)
__global__ void __launch_bounds__(kEvalThreads)
cc_apply_kernel(const float* __restrict__ img, const double* __restrict__ mom, int64_t n_px,
                float* __restrict__ out) {
    const double n = static_cast<double>(n_px);
    double a[3], b[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const double ref_mean = mom[4 * c] / n;
        const double img_mean = mom[4 * c + 1] / n;
        const double var_ref = fmax(mom[4 * c + 3] / n - ref_mean * ref_mean, 1e-8);
        double ac = (mom[4 * c + 2] / n - ref_mean * img_mean) / var_ref;
        b[c] = img_mean - ac * ref_mean;  // from a before the guard, as the reference
        if (fabs(ac) < 1e-8) ac = 1.0;
        a[c] = ac;
    }
    for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < n_px;
         p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const double v = (static_cast<double>(img[p * 3 + c]) - b[c]) / a[c];
            out[p * 3 + c] = static_cast<float>(fmin(fmax(v, 0.0), 1.0));
        }
    }
}

__global__ void __launch_bounds__(kEvalThreads)
rgba8_kernel(const float* __restrict__ rgb, int64_t n_px, uchar4* __restrict__ out) {
    for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < n_px;
         p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        unsigned char q[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            float v = rgb[p * 3 + c];
            if (!(v > 0.0f)) v = 0.0f;  // NaN included
            if (v > 1.0f) v = 1.0f;
            q[c] = static_cast<unsigned char>(__float2int_rn(v * 255.0f));
        }
        out[p] = make_uchar4(q[0], q[1], q[2], 255);
    }
}

unsigned grid_for(int64_t n) {
    const int64_t b = (n + kEvalThreads - 1) / kEvalThreads;
    return static_cast<unsigned>(b < 1 ? 1 : (b > kEvalBlocks ? kEvalBlocks : b));
}

}  // namespace

size_t eval_workspace() { return sizeof(double) * static_cast<size_t>(kEvalBlocks) * 12; }

void launch_clamp01(float* x, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    SX_LAUNCH(clamp01_kernel, grid_for(n), kEvalThreads, 0, s, x, n);
}

void launch_sum_sqdiff(const float* a, const float* b, int64_t n, double* parts, double* out,
                       cudaStream_t s) {
    const unsigned g = grid_for(n);
    SX_LAUNCH(sqdiff_kernel, g, kEvalThreads, 0, s, a, b, n, parts);
    SX_LAUNCH(reduce_parts_kernel, 1, kEvalThreads, 0, s, parts, static_cast<int>(g), 1, out);
}

void launch_color_correct(const float* img, const float* ref, int64_t n_px, double* parts,
                          double* moments, float* out, cudaStream_t s) {
    const unsigned g = grid_for(n_px);
    SX_LAUNCH(cc_moments_kernel, g, kEvalThreads, 0, s, img, ref, n_px, parts);
    SX_LAUNCH(reduce_parts_kernel, 1, kEvalThreads, 0, s, parts, static_cast<int>(g), 12, moments);
    SX_LAUNCH(cc_apply_kernel, grid_for(n_px), kEvalThreads, 0, s, img, moments, n_px, out);
}

void launch_rgba8(const float* rgb, int64_t n_px, uint8_t* out, cudaStream_t s) {
    if (n_px <= 0) return;
    SX_LAUNCH(rgba8_kernel, grid_for(n_px), kEvalThreads, 0, s, rgb, n_px,
              reinterpret_cast<uchar4*>(out));
}

}  // namespace sx
