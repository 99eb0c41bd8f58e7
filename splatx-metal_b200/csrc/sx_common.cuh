// sx_common.cuh — constants, error plumbing and numeric helpers shared by every sm_100a kernel of
// the 3DGS training step.
//
// Constants are the values of the gsplat/splatx contract (Sources/SplatXKernelSrc/
// KernelConstants.h:17-37 in splatx-metal); they are restated here because the kernels' integer
// outputs (radii, tile sets, last_ids) depend on them bit for bit.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace sx {

// ---- contract constants ----
constexpr float kAlphaThreshold = 1.f / 255.f;  // minimum alpha that contributes
constexpr float kGaussianExtend = 3.33f;        // sigma multiple of the screen-space radius
constexpr float kMinCompensation = 0.005f;      // floor of the anti-aliasing compensation
constexpr float kMaxAlpha = 0.99f;              // alpha clamp
constexpr float kTransmittanceThreshold = 1e-4f;  // exclusive early-stop threshold on T
constexpr float kMinOneMinusAlpha = 1e-6f;      // floor of 1-alpha when T is walked back
constexpr float kSsimC1 = 1e-4f;                // (0.01)^2
constexpr float kSsimC2 = 9e-4f;                // (0.03)^2
constexpr int kTile = 16;                       // raster tile edge (the only instantiation)
constexpr int kTileThreads = kTile * kTile;     // one thread per pixel
constexpr int kSsimWin = 11;                    // 11x11 Gaussian window, sigma 1.5
constexpr int kSsimTile = 16;
constexpr int kSsimApron = kSsimTile + kSsimWin - 1;  // 26

// 1-D SSIM taps: g(i) = exp(-(i-5)^2 / (2*1.5^2)), normalised in f64, rounded to f32 (the same
// table the reference stores; hex floats so the derivation is reproducible bit for bit).
__device__ __constant__ static const float kSsimTaps[kSsimWin] = {
    0x1.0d956cp-10f, 0x1.f1fe02p-8f, 0x1.26eb18p-5f, 0x1.bff0fep-4f, 0x1.b43c40p-3f,
    0x1.106560p-2f,  0x1.b43c40p-3f, 0x1.bff0fep-4f, 0x1.26eb18p-5f, 0x1.f1fe02p-8f,
    0x1.0d956cp-10f};

// ---- errors ----
struct InvalidArgument : std::invalid_argument {
    using std::invalid_argument::invalid_argument;
};
struct RuntimeError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

[[noreturn]] inline void throw_invalid(const char* what, const std::string& msg) {
    throw InvalidArgument(std::string(what) + ": " + msg);
}

inline void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        throw RuntimeError(std::string(what) + ": CUDA error " + cudaGetErrorName(e) + " (" +
                           cudaGetErrorString(e) + ")");
}

// Every kernel launch of the library goes through SX_LAUNCH so that launches can be counted.
void note_launch();
// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current device, once per
// (kernel, device) — the attribute is per device, so a process driving several GPUs needs it on
// each.
void smem_limit_once(const void* kernel, int bytes, const char* what);
int64_t launch_count();

#define SX_LAUNCH(kernel, grid, block, smem, stream, ...)                                  \
    do {                                                                                   \
        kernel<<<(grid), (block), (smem), (stream)>>>(__VA_ARGS__);                        \
        ::sx::note_launch();                                                               \
        ::sx::cuda_check(cudaGetLastError(), #kernel);                                     \
    } while (0)

// Bits of the executor's device status word (read back with every step's results): a bounded
// device-side wait that ran out sets its bit and the kernel finishes without waiting further.
constexpr uint32_t kStatusSortLookbackTimeout = 1u;
constexpr uint32_t kStatusPeerBarrierTimeout = 2u;

// The executor's resident parameter layout: Gaussians in tiles of 32; within a tile a group's d
// components are d runs of 32 floats. Component c of Gaussian i lives at tile_index(i, d) + 32*c.
__host__ __device__ __forceinline__ int64_t tile_index(int64_t i, int d) {
    return (i >> 5) * (32 * static_cast<int64_t>(d)) + (i & 31);
}

inline unsigned blocks_for(int64_t n, int threads) {
    return static_cast<unsigned>((n + threads - 1) / threads);
}

inline uint32_t bits_for_count(int64_t count) {
    if (count <= 1) return 0u;
    uint32_t bits = 0;
    for (uint64_t v = static_cast<uint64_t>(count) - 1u; v != 0; v >>= 1) bits++;
    return bits;
}

// ---- device numeric helpers ----
// std::min / std::max semantics (b<a ? b : a) — differ from fminf/fmaxf only on NaN, and the CPU
// contract is written with std::min/std::max.
__device__ __forceinline__ float smin(float a, float b) { return (b < a) ? b : a; }
__device__ __forceinline__ float smax(float a, float b) { return (a < b) ? b : a; }

// Correctly rounded (to within a 2^-29 chance) single-precision exp/log, computed through the
// double-precision library functions and rounded once. Used wherever a transcendental feeds an
// integer output (radii, tile sets), so that the GPU and a CPU reference agree bit for bit
// whenever the CPU's libm is itself correctly rounded.
__device__ __forceinline__ float exp_cr(float x) { return static_cast<float>(exp(static_cast<double>(x))); }
__device__ __forceinline__ float log_cr(float x) { return static_cast<float>(log(static_cast<double>(x))); }

__device__ __forceinline__ float sigmoid_cr(float x) { return 1.0f / (1.0f + exp_cr(-x)); }

constexpr unsigned kFullMask = 0xffffffffu;

// Warp "transpose" reduction of K values (K <= 16): after the call, every even lane whose slot
// (transpose_reduce_slot<K>) is >= 0 holds the warp-wide sum of value[slot]. It takes
// ceil(K/2)+ceil(K/4)+... + 1 shuffles instead of 5*K for K independent butterflies.
template <int K>
__device__ __forceinline__ float warp_transpose_reduce(const float (&v)[K], int lane) {
    static_assert(K >= 2 && K <= 16, "transpose reduce supports 2..16 values");
    constexpr int H1 = (K + 1) / 2, H2 = (H1 + 1) / 2, H3 = (H2 + 1) / 2, H4 = (H3 + 1) / 2;
    static_assert(H4 == 1, "four halving rounds must reach one value");
    float a1[H1], a2[H2], a3[H3];
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
    for (int i = 0; i < H1; ++i) {
        const float lo = v[i];
        const float hi = (i + H1 < K) ? v[i + H1] : 0.f;
        const float send = b4 ? lo : hi;
        a1[i] = (b4 ? hi : lo) + __shfl_xor_sync(kFullMask, send, 16);
    }
#pragma unroll
    for (int i = 0; i < H2; ++i) {
        const float lo = a1[i];
        const float hi = (i + H2 < H1) ? a1[i + H2] : 0.f;
        const float send = b3 ? lo : hi;
        a2[i] = (b3 ? hi : lo) + __shfl_xor_sync(kFullMask, send, 8);
    }
#pragma unroll
    for (int i = 0; i < H3; ++i) {
        const float lo = a2[i];
        const float hi = (i + H3 < H2) ? a2[i + H3] : 0.f;
        const float send = b2 ? lo : hi;
        a3[i] = (b2 ? hi : lo) + __shfl_xor_sync(kFullMask, send, 4);
    }
    float a4;
    {
        const float lo = a3[0];
        const float hi = (1 < H3) ? a3[1] : 0.f;
        const float send = b1 ? lo : hi;
        a4 = (b1 ? hi : lo) + __shfl_xor_sync(kFullMask, send, 2);
    }
    return a4 + __shfl_xor_sync(kFullMask, a4, 1);
}

// Which value index the lane holds after warp_transpose_reduce<K>, or -1 (padding / odd lane).
template <int K>
__device__ __forceinline__ int transpose_reduce_slot(int lane) {
    constexpr int H1 = (K + 1) / 2, H2 = (H1 + 1) / 2, H3 = (H2 + 1) / 2;
    if (lane & 1) return -1;
    int i = (lane & 2) ? 1 : 0;
    if (i >= H3) return -1;
    i += (lane & 4) ? H3 : 0;
    if (i >= H2) return -1;
    i += (lane & 8) ? H2 : 0;
    if (i >= H1) return -1;
    i += (lane & 16) ? H1 : 0;
    if (i >= K) return -1;
    return i;
}

}  // namespace sx
