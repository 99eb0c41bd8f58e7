// sort.cu — prefix scans and the stable LSD radix sort used by the intersection pipeline.
//
// The sort contract (KernelBackend.h:130-153, sort_isect): ascending unsigned keys, STABLE (ties
// keep input order — emit order), only the low key_n_bits significant. This is a
// reduce-then-scan radix sort with 8-bit digits: per pass an upsweep (per-CTA digit counts), a
// digit-parallel scan of those counts, and a downsweep that ranks keys stably inside the CTA with
// warp match_any (rank = earlier peers in the same warp round + the warp's earlier rounds + the
// earlier warps) and writes them out through shared memory so global stores are contiguous per
// digit. No CTA ever waits on another CTA, so nothing can spin.
#include <algorithm>
#include <mutex>

#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

constexpr int kRsThreads = 256;
constexpr int kRsWarps = kRsThreads / 32;
constexpr int kRadix = 256;
constexpr uint32_t kNoDigit = 0xffffffffu;

template <typename K>
struct RadixCfg;
template <>
struct RadixCfg<uint32_t> {
    static constexpr int kItems = 16;
};
template <>
struct RadixCfg<uint64_t> {
    static constexpr int kItems = 8;
};
template <typename K>
constexpr int radix_tile() {
    return kRsThreads * RadixCfg<K>::kItems;
}

__device__ __forceinline__ int64_t resolve_n(int64_t n_host, const int64_t* n_dev) {
    if (!n_dev) return n_host;
    const int64_t v = *n_dev;
    return v < n_host ? v : n_host;  // never beyond the buffers the grid was sized for
}

// Block-wide exclusive scan of one uint32 per thread (blockDim.x == 256 or 1024, multiple of 32).
template <int THREADS>
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* warp_sums,
                                                    uint32_t& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(kFullMask, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    constexpr int NW = THREADS / 32;
    if (warp == 0) {
        uint32_t w = lane < NW ? warp_sums[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(kFullMask, w, o);
            if (lane >= o) w += y;
        }
        if (lane < NW) warp_sums[lane] = w;  // inclusive warp prefix
    }
    __syncthreads();
    const uint32_t warp_excl = warp == 0 ? 0u : warp_sums[warp - 1];
    total = warp_sums[NW - 1];
    __syncthreads();
    return warp_excl + x - v;
}

template <typename K>
__global__ void __launch_bounds__(kRsThreads)
rs_upsweep(const K* __restrict__ keys, int64_t n_host, const int64_t* n_dev, int shift,
           uint32_t mask, uint32_t* __restrict__ hist, int64_t nb_cap) {
    constexpr int ITEMS = RadixCfg<K>::kItems;
    constexpr int TILE = radix_tile<K>();
    const int64_t n = resolve_n(n_host, n_dev);
    const int64_t base = static_cast<int64_t>(blockIdx.x) * TILE;
    if (base >= n) return;
    __shared__ uint32_t cnt[kRsWarps][kRadix];
    for (int i = threadIdx.x; i < kRsWarps * kRadix; i += kRsThreads) (&cnt[0][0])[i] = 0;
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t wbase = base + static_cast<int64_t>(warp) * 32 * ITEMS;
#pragma unroll 4
    for (int r = 0; r < ITEMS; ++r) {
        const int64_t pos = wbase + r * 32 + lane;
        const uint32_t d = pos < n ? static_cast<uint32_t>(keys[pos] >> shift) & mask : kNoDigit;
        const unsigned peers = __match_any_sync(kFullMask, d);
        if (d != kNoDigit && lane == __ffs(peers) - 1) cnt[warp][d] += __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    for (int d = threadIdx.x; d < kRadix; d += kRsThreads) {
        uint32_t s = 0;
#pragma unroll
        for (int w = 0; w < kRsWarps; ++w) s += cnt[w][d];
        hist[static_cast<int64_t>(d) * nb_cap + blockIdx.x] = s;
    }
}

// One CTA per digit: exclusive scan of that digit's per-CTA counts, digit total to totals[d].
__global__ void __launch_bounds__(1024)
rs_scan(uint32_t* __restrict__ hist, uint32_t* __restrict__ totals, int64_t n_host,
        const int64_t* n_dev, int tile, int64_t nb_cap) {
    __shared__ uint32_t warp_sums[32];
    const int64_t n = resolve_n(n_host, n_dev);
    const int64_t nb = (n + tile - 1) / tile;
    uint32_t* h = hist + static_cast<int64_t>(blockIdx.x) * nb_cap;
    uint32_t carry = 0;
    for (int64_t b0 = 0; b0 < nb; b0 += 1024) {
        const int64_t i = b0 + threadIdx.x;
        const uint32_t v = i < nb ? h[i] : 0u;
        uint32_t tot;
        const uint32_t ex = block_excl_scan<1024>(v, warp_sums, tot);
        if (i < nb) h[i] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) totals[blockIdx.x] = carry;
}

template <typename K>
struct DownsweepSmem {
    K keys[radix_tile<K>()];
    int32_t vals[radix_tile<K>()];
    uint32_t cnt[kRsWarps][kRadix];
    uint32_t bexcl[kRadix];
    uint32_t gbase[kRadix];
    uint32_t warp_sums[32];
};

template <typename K>
__global__ void __launch_bounds__(kRsThreads)
rs_downsweep(const K* __restrict__ keys_in, const int32_t* __restrict__ vals_in,
             K* __restrict__ keys_out, int32_t* __restrict__ vals_out, int64_t n_host,
             const int64_t* n_dev, int shift, uint32_t mask, const uint32_t* __restrict__ hist,
             const uint32_t* __restrict__ totals, int64_t nb_cap) {
    constexpr int ITEMS = RadixCfg<K>::kItems;
    constexpr int TILE = radix_tile<K>();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    DownsweepSmem<K>& sm = *reinterpret_cast<DownsweepSmem<K>*>(smem_raw);
    const int64_t n = resolve_n(n_host, n_dev);
    const int64_t base = static_cast<int64_t>(blockIdx.x) * TILE;
    if (base >= n) return;
    const int tile_n = static_cast<int>(min(static_cast<int64_t>(TILE), n - base));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wofs = warp * 32 * ITEMS;

    for (int i = threadIdx.x; i < kRsWarps * kRadix; i += kRsThreads) (&sm.cnt[0][0])[i] = 0;
    K k[ITEMS];
    int32_t v[ITEMS];
    uint32_t dg[ITEMS];
#pragma unroll
    for (int r = 0; r < ITEMS; ++r) {
        const int off = wofs + r * 32 + lane;
        if (off < tile_n) {
            k[r] = keys_in[base + off];
            v[r] = vals_in[base + off];
            dg[r] = static_cast<uint32_t>(k[r] >> shift) & mask;
        } else {
            k[r] = 0;
            v[r] = 0;
            dg[r] = kNoDigit;
        }
    }
    __syncthreads();
    const unsigned lt_mask = (1u << lane) - 1u;
    uint32_t loc[ITEMS];
#pragma unroll
    for (int r = 0; r < ITEMS; ++r) {
        const uint32_t d = dg[r];
        const unsigned peers = __match_any_sync(kFullMask, d);
        const int leader = __ffs(peers) - 1;
        uint32_t old = 0;
        if (lane == leader && d != kNoDigit) {
            old = sm.cnt[warp][d];
            sm.cnt[warp][d] = old + __popc(peers);
        }
        old = __shfl_sync(kFullMask, old, leader);
        loc[r] = old + __popc(peers & lt_mask);
        __syncwarp();
    }
    __syncthreads();
    // per digit: exclusive prefix over warps, then over digits (block), then the global base
    const int t = threadIdx.x;  // kRsThreads == kRadix
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < kRsWarps; ++w) {
        const uint32_t c = sm.cnt[w][t];
        sm.cnt[w][t] = run;
        run += c;
    }
    uint32_t tot;
    const uint32_t bex = block_excl_scan<kRsThreads>(run, sm.warp_sums, tot);
    sm.bexcl[t] = bex;
    const uint32_t dex = block_excl_scan<kRsThreads>(totals[t], sm.warp_sums, tot);
    sm.gbase[t] = dex + hist[static_cast<int64_t>(t) * nb_cap + blockIdx.x];
    __syncthreads();
#pragma unroll
    for (int r = 0; r < ITEMS; ++r) {
        const uint32_t d = dg[r];
        if (d == kNoDigit) continue;
        const uint32_t p = sm.bexcl[d] + sm.cnt[warp][d] + loc[r];
        sm.keys[p] = k[r];
        sm.vals[p] = v[r];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < tile_n; i += kRsThreads) {
        const K key = sm.keys[i];
        const uint32_t d = static_cast<uint32_t>(key >> shift) & mask;
        const int64_t dst = static_cast<int64_t>(sm.gbase[d]) + (i - static_cast<int64_t>(sm.bexcl[d]));
        keys_out[dst] = key;
        vals_out[dst] = sm.vals[i];
    }
}

size_t align_up(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

template <typename K>
size_t radix_ws_bytes(int64_t n) {
    const int64_t nb = (n + radix_tile<K>() - 1) / radix_tile<K>();
    return align_up(sizeof(K) * static_cast<size_t>(n)) + align_up(sizeof(int32_t) * n) +
           align_up(sizeof(uint32_t) * kRadix * static_cast<size_t>(nb > 0 ? nb : 1)) +
           align_up(sizeof(uint32_t) * kRadix);
}

template <typename K>
void radix_sort_impl(const K* keys_in, const int32_t* vals_in, K* keys_out, int32_t* vals_out,
                     int64_t n, const int64_t* n_dev, uint32_t key_bits, void* ws,
                     cudaStream_t s) {
    if (n <= 0 || key_bits == 0) return;
    constexpr int TILE = radix_tile<K>();
    const int64_t nb = (n + TILE - 1) / TILE;
    unsigned char* p = static_cast<unsigned char*>(ws);
    K* tk = reinterpret_cast<K*>(p);
    p += align_up(sizeof(K) * static_cast<size_t>(n));
    int32_t* tv = reinterpret_cast<int32_t*>(p);
    p += align_up(sizeof(int32_t) * n);
    uint32_t* hist = reinterpret_cast<uint32_t*>(p);
    p += align_up(sizeof(uint32_t) * kRadix * static_cast<size_t>(nb));
    uint32_t* totals = reinterpret_cast<uint32_t*>(p);

    const int passes = static_cast<int>((key_bits + 7) / 8);
    const size_t smem = sizeof(DownsweepSmem<K>);
    smem_limit_once(reinterpret_cast<const void*>(rs_downsweep<K>), static_cast<int>(smem),
                    "radix smem attribute");
    const K* src_k = keys_in;
    const int32_t* src_v = vals_in;
    for (int pass = 0; pass < passes; ++pass) {
        const int shift = pass * 8;
        const uint32_t bits = key_bits - shift >= 8 ? 8u : key_bits - shift;
        const uint32_t mask = (1u << bits) - 1u;
        // the last pass lands in the output; earlier passes alternate so src != dst
        const bool to_out = ((passes - 1 - pass) % 2) == 0;
        K* dk = to_out ? keys_out : tk;
        int32_t* dv = to_out ? vals_out : tv;
        SX_LAUNCH(rs_upsweep<K>, static_cast<unsigned>(nb), kRsThreads, 0, s, src_k, n, n_dev,
                  shift, mask, hist, nb);
        SX_LAUNCH(rs_scan, kRadix, 1024, 0, s, hist, totals, n, n_dev, TILE, nb);
        SX_LAUNCH(rs_downsweep<K>, static_cast<unsigned>(nb), kRsThreads, smem, s, src_k, src_v,
                  dk, dv, n, n_dev, shift, mask, hist, totals, nb);
        src_k = dk;
        src_v = dv;
    }
}

// ------------------------------------------------------------------ single-sweep sort --------
// The executor's u32 sorts: one histogram kernel for every pass, then ONE kernel per pass (keys and
// values read once, written once). A CTA claims its tile in launch order from a counter, ranks the
// tile's keys stably (warp match_any, as above), publishes its per-digit counts, and finds its
// global digit offsets by looking back over the tiles before it (decoupled look-back: a tile's
// slot holds its count flagged AGGREGATE, then its inclusive prefix flagged INCLUSIVE). Every
// claimed predecessor is already running and never waits on a later tile, so the look-back always
// ends; it is nevertheless bounded, and a wait that runs out sets kStatusSortLookbackTimeout in
// the caller's status word. Counts and prefixes are 30-bit (n < 2^30).
constexpr uint32_t kLbAggregate = 1u << 30;
constexpr uint32_t kLbInclusive = 2u << 30;
constexpr uint32_t kLbValue = (1u << 30) - 1u;
constexpr int kLbSpinLimit = 1 << 22;
constexpr int kLbWindow = 16;  // predecessor slots read per look-back step
constexpr int kOsMaxPasses = 4;
constexpr int kOsHistThreads = 512;
constexpr int kOsHistMaxCtas = 148;  // one per SM: few partial histograms to merge

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
    return *reinterpret_cast<const volatile uint32_t*>(p);
}
__device__ __forceinline__ void st_volatile(uint32_t* p, uint32_t v) {
    *reinterpret_cast<volatile uint32_t*>(p) = v;
}

// Digit histograms of every pass, plus (full_hist != null) the histogram of the whole key.
__global__ void __launch_bounds__(kOsHistThreads)
os_hist(const uint32_t* __restrict__ keys, int64_t n_host, const int64_t* n_dev, int passes,
        int bits, uint32_t* __restrict__ ghist, uint32_t* __restrict__ full_hist, int full_bins) {
    extern __shared__ uint32_t hsm[];  // [passes][256] then [full_bins]
    uint32_t* fh = hsm + kOsMaxPasses * kRadix;
    const int64_t n = resolve_n(n_host, n_dev);
    for (int i = threadIdx.x; i < kOsMaxPasses * kRadix + (full_hist ? full_bins : 0); i += kOsHistThreads)
        hsm[i] = 0;
    __syncthreads();
    const uint32_t mask = (1u << bits) - 1u;
    // with the whole-key histogram, the passes' digit counts are derived from it in os_scan
    auto count = [&](uint32_t k) {
        if (full_hist) {
            atomicAdd(&fh[k], 1u);
        } else {
            for (int p = 0; p < passes; ++p) atomicAdd(&hsm[p * kRadix + ((k >> (p * bits)) & mask)], 1u);
        }
    };
    // four keys per 16-byte load, two loads in flight per thread
    const uint4* k4 = reinterpret_cast<const uint4*>(keys);
    const int64_t n4 = n / 4;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kOsHistThreads;
    int64_t i = static_cast<int64_t>(blockIdx.x) * kOsHistThreads + threadIdx.x;
    for (; i + stride < n4; i += 2 * stride) {
        const uint4 a = k4[i], b = k4[i + stride];
        count(a.x); count(a.y); count(a.z); count(a.w);
        count(b.x); count(b.y); count(b.z); count(b.w);
    }
    for (; i < n4; i += stride) {
        const uint4 a = k4[i];
        count(a.x); count(a.y); count(a.z); count(a.w);
    }
    for (int64_t r = n4 * 4 + static_cast<int64_t>(blockIdx.x) * kOsHistThreads + threadIdx.x; r < n;
         r += stride)
        count(keys[r]);
    __syncthreads();
    if (full_hist) {
        for (int i = threadIdx.x; i < full_bins; i += kOsHistThreads)
            if (fh[i]) atomicAdd(&full_hist[i], fh[i]);
    } else {
        for (int i = threadIdx.x; i < passes * kRadix; i += kOsHistThreads)
            if (hsm[i]) atomicAdd(&ghist[i], hsm[i]);
    }
}

// Exclusive scans: block p < passes scans pass p's digit counts in place (with the whole-key
// histogram, it first sums them from it: digit d of pass p counts the keys t with
// (t >> p*bits) & mask == d); block `passes` (when offsets != null) scans the whole-key histogram
// into int32 offsets (the tile ranges).
__global__ void __launch_bounds__(1024)
os_scan(uint32_t* __restrict__ ghist, int passes, int bits, const uint32_t* __restrict__ full_hist,
        int full_bins, int32_t* __restrict__ offsets) {
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t derived[kRadix];
    if (static_cast<int>(blockIdx.x) < passes) {
        uint32_t* h = ghist + blockIdx.x * kRadix;
        if (full_hist) {
            const uint32_t mask = (1u << bits) - 1u;
            const int shift = static_cast<int>(blockIdx.x) * bits;
            if (threadIdx.x < kRadix) derived[threadIdx.x] = 0u;
            __syncthreads();
            for (int t = threadIdx.x; t < full_bins; t += 1024) {
                const uint32_t c = full_hist[t];
                if (c) atomicAdd(&derived[(static_cast<uint32_t>(t) >> shift) & mask], c);
            }
            __syncthreads();
        }
        const uint32_t v = threadIdx.x < kRadix ? (full_hist ? derived[threadIdx.x] : h[threadIdx.x]) : 0u;
        uint32_t tot;
        const uint32_t ex = block_excl_scan<1024>(v, warp_sums, tot);
        if (threadIdx.x < kRadix) h[threadIdx.x] = ex;
        return;
    }
    uint32_t carry = 0;
    for (int b0 = 0; b0 < full_bins; b0 += 1024) {
        const int i = b0 + static_cast<int>(threadIdx.x);
        const uint32_t v = i < full_bins ? full_hist[i] : 0u;
        uint32_t tot;
        const uint32_t ex = block_excl_scan<1024>(v, warp_sums, tot);
        if (i < full_bins) offsets[i] = static_cast<int32_t>(carry + ex);
        carry += tot;
    }
}

// Lanes of the warp holding the same digit as this lane: one ballot per digit bit (plus one for
// validity) instead of match_any, whose cost grows with the number of distinct values.
__device__ __forceinline__ unsigned digit_peers(uint32_t d, bool valid, int bits) {
    unsigned peers = __ballot_sync(kFullMask, valid);
    if (!valid) peers = ~peers;
    for (int b = 0; b < bits; ++b) {
        const bool set = (d >> b) & 1u;
        const unsigned m = __ballot_sync(kFullMask, set);
        peers &= set ? m : ~m;
    }
    return peers;
}

struct OnesweepSmem {
    uint32_t keys[radix_tile<uint32_t>()];
    int32_t vals[radix_tile<uint32_t>()];
    int32_t vals_in[radix_tile<uint32_t>()];  // the tile's values in input order (async copy)
    uint32_t cnt[kRsWarps][kRadix];
    uint32_t bexcl[kRadix];
    uint32_t gbase[kRadix];
    uint32_t warp_sums[32];
    uint32_t tile;
};

// 4-byte global -> shared copy that holds no register until it lands (cp.async, L2 only).
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__global__ void __launch_bounds__(kRsThreads, 3)
os_pass(const uint32_t* __restrict__ keys_in, const int32_t* __restrict__ vals_in,
        uint32_t* __restrict__ keys_out, int32_t* __restrict__ vals_out, int64_t n_host,
        const int64_t* n_dev, int shift, int bits, const uint32_t* __restrict__ digit_off,
        uint32_t* __restrict__ lookback, uint32_t* __restrict__ tile_ctr,
        uint32_t* __restrict__ status) {
    constexpr int ITEMS = RadixCfg<uint32_t>::kItems;
    constexpr int TILE = radix_tile<uint32_t>();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    OnesweepSmem& sm = *reinterpret_cast<OnesweepSmem*>(smem_raw);
    const int64_t n = resolve_n(n_host, n_dev);
    // A CTA claims tiles until they run out: a claimed tile's predecessors were claimed earlier by
    // CTAs that are running or done, so the look-back below never waits on an unstarted tile.
    for (;;) {
    __syncthreads();  // the previous tile's shared memory is no longer read
    if (threadIdx.x == 0) sm.tile = atomicAdd(tile_ctr, 1u);
    for (int i = threadIdx.x; i < kRsWarps * kRadix; i += kRsThreads) (&sm.cnt[0][0])[i] = 0;
    __syncthreads();
    const uint32_t tile = sm.tile;
    const int64_t base = static_cast<int64_t>(tile) * TILE;
    if (base >= n) return;  // uniform; no tile after the last real one is ever waited on
    const int tile_n = static_cast<int>(min(static_cast<int64_t>(TILE), n - base));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wofs = warp * 32 * ITEMS;
    const uint32_t mask = (1u << bits) - 1u;

    uint32_t k[ITEMS];
    uint32_t loc[ITEMS];
#pragma unroll
    for (int r = 0; r < ITEMS; ++r) {
        const int off = wofs + r * 32 + lane;
        k[r] = off < tile_n ? keys_in[base + off] : 0u;
        if (off < tile_n) cp_async4(&sm.vals_in[off], vals_in + base + off);
    }
    const unsigned lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int r = 0; r < ITEMS; ++r) {
        const int off = wofs + r * 32 + lane;
        const bool ok = off < tile_n;
        const uint32_t d = ok ? (k[r] >> shift) & mask : kNoDigit;
        const unsigned peers = digit_peers(d, ok, bits);
        const int leader = __ffs(peers) - 1;
        uint32_t old = 0;
        if (lane == leader && ok) {
            old = sm.cnt[warp][d];
            sm.cnt[warp][d] = old + __popc(peers);
        }
        old = __shfl_sync(kFullMask, old, leader);
        loc[r] = old + __popc(peers & lt_mask);
        __syncwarp();
    }
    __syncthreads();
    const int t = threadIdx.x;  // one thread per digit (kRsThreads == kRadix)
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < kRsWarps; ++w) {
        const uint32_t c = sm.cnt[w][t];
        sm.cnt[w][t] = run;
        run += c;
    }
    // publish this tile's counts first, then do the local work (block scan, scatter into shared
    // memory) before looking back: the predecessors get that time to publish their prefixes
    uint32_t* slot = lookback + static_cast<int64_t>(tile) * kRadix + t;
    const bool used_digit = t < (1 << bits);
    if (used_digit) st_volatile(slot, (tile == 0 ? kLbInclusive : kLbAggregate) | run);
    uint32_t tot;
    cp_async_wait_all();  // this thread's value copies have landed (the barrier below shares them)
    sm.bexcl[t] = block_excl_scan<kRsThreads>(run, sm.warp_sums, tot);
    __syncthreads();
#pragma unroll
    for (int r = 0; r < ITEMS; ++r) {
        const int off = wofs + r * 32 + lane;
        if (off >= tile_n) continue;
        const uint32_t d = (k[r] >> shift) & mask;
        const uint32_t p = sm.bexcl[d] + sm.cnt[warp][d] + loc[r];
        sm.keys[p] = k[r];
        sm.vals[p] = sm.vals_in[off];
    }
    if (!used_digit) {
        sm.gbase[t] = 0;  // digit not used by this pass: nothing to publish or find
    } else if (tile == 0) {
        sm.gbase[t] = digit_off[t];
    } else {
        // windowed look-back: kLbWindow predecessor slots read at once, consumed in order until an
        // inclusive prefix; a slot not yet published stops the window and is polled again
        uint32_t excl = 0;
        int64_t j = static_cast<int64_t>(tile) - 1;
        int spins = 0;
        while (true) {
            uint32_t v[kLbWindow];
#pragma unroll
            for (int w = 0; w < kLbWindow; ++w)
                v[w] = j - w >= 0 ? ld_volatile(lookback + (j - w) * kRadix + t) : kLbInclusive;
            uint32_t acc = 0;
            int used = 0;
            bool stop = false, blocked = false;
#pragma unroll
            for (int w = 0; w < kLbWindow; ++w) {
                if (stop || blocked) continue;
                const uint32_t flag = v[w] & ~kLbValue;
                if (flag == 0u) {
                    blocked = true;
                    continue;
                }
                acc += v[w] & kLbValue;
                ++used;
                stop = flag == kLbInclusive;
            }
            excl += acc;
            j -= used;
            if (stop) break;
            if (blocked) {
                if (++spins > kLbSpinLimit) {
                    if (status) atomicOr(status, kStatusSortLookbackTimeout);
                    break;
                }
                __nanosleep(32);
            }
        }
        st_volatile(slot, kLbInclusive | (excl + run));
        sm.gbase[t] = digit_off[t] + excl;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < tile_n; i += kRsThreads) {
        const uint32_t key = sm.keys[i];
        const uint32_t d = (key >> shift) & mask;
        const int64_t dst = static_cast<int64_t>(sm.gbase[d]) + (i - static_cast<int64_t>(sm.bexcl[d]));
        if (keys_out) keys_out[dst] = key;
        vals_out[dst] = sm.vals[i];
    }
    }  // next tile
}

struct OnesweepLayout {
    int passes = 0, bits = 0, full_bins = 0;
    int64_t tiles = 0;
    size_t off_tk = 0, off_tk2 = 0, off_tv = 0, off_zero = 0, zero_bytes = 0;
    size_t off_ghist = 0, off_full = 0, off_ctr = 0, off_lb = 0, total = 0;
};

OnesweepLayout onesweep_layout(int64_t n, uint32_t key_bits, int full_bins) {
    OnesweepLayout L;
    L.passes = static_cast<int>((key_bits + 7) / 8);
    if (L.passes < 1) L.passes = 1;
    L.bits = static_cast<int>((key_bits + L.passes - 1) / L.passes);
    L.full_bins = full_bins;
    L.tiles = (n + radix_tile<uint32_t>() - 1) / radix_tile<uint32_t>();
    if (L.tiles < 1) L.tiles = 1;
    size_t o = 0;
    L.off_tk = o; o += align_up(sizeof(uint32_t) * static_cast<size_t>(n > 0 ? n : 1));
    // a second key buffer only when intermediate passes must alternate without keys_out
    L.off_tk2 = o; o += L.passes >= 3 ? align_up(sizeof(uint32_t) * static_cast<size_t>(n > 0 ? n : 1)) : 0;
    L.off_tv = o; o += align_up(sizeof(int32_t) * static_cast<size_t>(n > 0 ? n : 1));
    L.off_zero = o;
    L.off_ghist = o; o += align_up(sizeof(uint32_t) * kOsMaxPasses * kRadix);
    L.off_full = o; o += align_up(sizeof(uint32_t) * static_cast<size_t>(full_bins > 0 ? full_bins : 1));
    L.off_ctr = o; o += align_up(sizeof(uint32_t) * kOsMaxPasses);
    L.off_lb = o; o += align_up(sizeof(uint32_t) * kRadix * static_cast<size_t>(L.tiles) * L.passes);
    L.zero_bytes = o - L.off_zero;
    L.total = o;
    return L;
}

// ------------------------------------------------------------------ scans ----------------------
constexpr int kScanThreads = 256;
constexpr int kScanItems = 16;
constexpr int kScanTile = kScanThreads * kScanItems;  // 4096

struct LoadI32 {
    using value_type = int32_t;
    const int32_t* p;
    __device__ __forceinline__ int32_t operator()(int64_t i) const { return p[i]; }
};
struct LoadGather {
    using value_type = int32_t;
    const int32_t* p;
    const int32_t* idx;
    __device__ __forceinline__ int32_t operator()(int64_t i) const { return p[idx[i]]; }
};
// All kScanItems loads of a lane are issued before the first is used: with the gathered load
// (counts in depth order) each is an L2 round trip, and a tile has few warps per SM.
template <typename Load>
__device__ __forceinline__ int64_t warp_segment_sum(Load load, int64_t wbase, int64_t n) {
    const int lane = threadIdx.x & 31;
    typename Load::value_type v[kScanItems];
#pragma unroll
    for (int r = 0; r < kScanItems; ++r) {
        const int64_t pos = wbase + r * 32 + lane;
        v[r] = pos < n ? load(pos) : 0;
    }
    int64_t s = 0;
#pragma unroll
    for (int r = 0; r < kScanItems; ++r) s += v[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFullMask, s, o);
    return s;
}

// Per-CTA totals of a 4096-element tile; with `side`, also the tile's sum of side[i] (plain
// order), in side_sums.
template <typename Load>
__global__ void __launch_bounds__(kScanThreads)
scan_reduce(Load load, int64_t n, int64_t* __restrict__ block_sums, const int32_t* __restrict__ side,
            int64_t* __restrict__ side_sums) {
    __shared__ int64_t ws[2][kScanThreads / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t wbase = static_cast<int64_t>(blockIdx.x) * kScanTile + warp * 32 * kScanItems;
    const int64_t s = warp_segment_sum(load, wbase, n);
    const int64_t s2 = side ? warp_segment_sum(LoadI32{side}, wbase, n) : 0;
    if (lane == 0) {
        ws[0][warp] = s;
        ws[1][warp] = s2;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int64_t t = 0, t2 = 0;
        for (int w = 0; w < kScanThreads / 32; ++w) {
            t += ws[0][w];
            t2 += ws[1][w];
        }
        block_sums[blockIdx.x] = t;
        if (side) side_sums[blockIdx.x] = t2;
    }
}

// Single CTA: exclusive scan of block sums in place; the grand total to *total. With `side`, the
// same CTA then sums side[0..nb) into *side_total.
__global__ void __launch_bounds__(1024)
scan_blocks(int64_t* __restrict__ sums, int64_t nb, int64_t* __restrict__ total,
            const int64_t* __restrict__ side = nullptr, int64_t* __restrict__ side_total = nullptr) {
    __shared__ int64_t warp_tot[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int64_t carry = 0;
    for (int64_t b0 = 0; b0 < nb; b0 += 1024) {
        const int64_t i = b0 + threadIdx.x;
        const int64_t v = i < nb ? sums[i] : 0;
        int64_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t y = __shfl_up_sync(kFullMask, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_tot[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int64_t w = warp_tot[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t y = __shfl_up_sync(kFullMask, w, o);
                if (lane >= o) w += y;
            }
            warp_tot[lane] = w;
        }
        __syncthreads();
        const int64_t wex = warp == 0 ? 0 : warp_tot[warp - 1];
        if (i < nb) sums[i] = carry + wex + x - v;
        carry += warp_tot[31];
        __syncthreads();
    }
    if (threadIdx.x == 0 && total) *total = carry;
    if (!side) return;  // uniform
    int64_t s = 0;
    for (int64_t i = threadIdx.x; i < nb; i += 1024) s += side[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFullMask, s, o);
    if (lane == 0) warp_tot[warp] = s;  // the scan loop ended on a barrier
    __syncthreads();
    if (threadIdx.x == 0) {
        int64_t t = 0;
        for (int w = 0; w < 32; ++w) t += warp_tot[w];
        *side_total = t;
    }
}

// Scan output: element pos of the prefix to out[pos].
template <typename OutT>
struct StorePlain {
    OutT* out;
    __device__ __forceinline__ void operator()(int64_t pos, int64_t v) const {
        out[pos] = static_cast<OutT>(v);
    }
};

// Re-scan each tile with its block offset; INCLUSIVE selects inclusive/exclusive output.
template <typename Load, typename Store, bool INCLUSIVE>
__global__ void __launch_bounds__(kScanThreads)
scan_down(Load load, int64_t n, const int64_t* __restrict__ block_offsets, Store store) {
    __shared__ int64_t ws[kScanThreads / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t wbase = static_cast<int64_t>(blockIdx.x) * kScanTile + warp * 32 * kScanItems;
    const int64_t wsum = warp_segment_sum(load, wbase, n);
    if (lane == 0) ws[warp] = wsum;
    __syncthreads();
    int64_t carry = block_offsets[blockIdx.x];
    for (int w = 0; w < warp; ++w) carry += ws[w];
    typename Load::value_type vals[kScanItems];  // loaded again (L2), all in flight at once
#pragma unroll
    for (int r = 0; r < kScanItems; ++r) {
        const int64_t pos = wbase + r * 32 + lane;
        vals[r] = pos < n ? load(pos) : 0;
    }
#pragma unroll
    for (int r = 0; r < kScanItems; ++r) {
        const int64_t pos = wbase + r * 32 + lane;
        const int64_t v = vals[r];
        int64_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t y = __shfl_up_sync(kFullMask, x, o);
            if (lane >= o) x += y;
        }
        if (pos < n) store(pos, carry + (INCLUSIVE ? x : x - v));
        carry += __shfl_sync(kFullMask, x, 31);
    }
}

__global__ void tile_offsets_u32_kernel(const uint32_t* __restrict__ keys, const int64_t* n_dev,
                                        int64_t cap, int64_t n_tiles,
                                        int32_t* __restrict__ offsets) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    const int64_t n = resolve_n(cap, n_dev);
    if (n == 0) {
        for (int64_t t = i; t < n_tiles; t += static_cast<int64_t>(gridDim.x) * blockDim.x)
            offsets[t] = 0;
        return;
    }
    if (i >= n) return;
    const int64_t cur = keys[i];
    if (i == 0)
        for (int64_t t = 0; t <= cur; ++t) offsets[t] = 0;
    if (i == n - 1)
        for (int64_t t = cur + 1; t < n_tiles; ++t) offsets[t] = static_cast<int32_t>(n);
    if (i > 0) {
        const int64_t prev = keys[i - 1];
        for (int64_t t = prev + 1; t <= cur; ++t) offsets[t] = static_cast<int32_t>(i);
    }
}

}  // namespace

size_t scan_i64_workspace(int64_t n) {
    const int64_t nb = (n + kScanTile - 1) / kScanTile;
    return align_up(sizeof(int64_t) * static_cast<size_t>(nb > 0 ? nb : 1));
}

void launch_scan_i64(const int32_t* in, int64_t* out, int64_t n, void* ws, cudaStream_t s) {
    if (n <= 0) return;
    const int64_t nb = (n + kScanTile - 1) / kScanTile;
    int64_t* sums = static_cast<int64_t*>(ws);
    LoadI32 ld{in};
    SX_LAUNCH(scan_reduce<LoadI32>, static_cast<unsigned>(nb), kScanThreads, 0, s, ld, n, sums, nullptr, nullptr);
    SX_LAUNCH(scan_blocks, 1, 1024, 0, s, sums, nb, static_cast<int64_t*>(nullptr));
    SX_LAUNCH((scan_down<LoadI32, StorePlain<int64_t>, true>), static_cast<unsigned>(nb),
              kScanThreads, 0, s, ld, n, sums, StorePlain<int64_t>{out});
}

// Block totals, then (with `side`) the side sums.
size_t scan_gather_workspace(int64_t n) { return 2 * scan_i64_workspace(n); }

void launch_scan_gather_excl(const int32_t* in, const int32_t* gather, int32_t* out,
                             int64_t* total, int64_t n, void* ws, cudaStream_t s,
                             const int32_t* side, int64_t* side_total) {
    if (n <= 0) {
        cuda_check(cudaMemsetAsync(total, 0, sizeof(int64_t), s), "memset total");
        if (side_total) cuda_check(cudaMemsetAsync(side_total, 0, sizeof(int64_t), s), "memset total");
        return;
    }
    const int64_t nb = (n + kScanTile - 1) / kScanTile;
    int64_t* sums = static_cast<int64_t*>(ws);
    int64_t* side_sums = reinterpret_cast<int64_t*>(static_cast<unsigned char*>(ws) + scan_i64_workspace(n));
    if (gather) {
        LoadGather ld{in, gather};
        SX_LAUNCH(scan_reduce<LoadGather>, static_cast<unsigned>(nb), kScanThreads, 0, s, ld, n, sums,
                  side, side ? side_sums : nullptr);
        SX_LAUNCH(scan_blocks, 1, 1024, 0, s, sums, nb, total, side ? side_sums : nullptr,
                  side_total);
        SX_LAUNCH((scan_down<LoadGather, StorePlain<int32_t>, false>), static_cast<unsigned>(nb),
                  kScanThreads, 0, s, ld, n, sums, StorePlain<int32_t>{out});
    } else {
        LoadI32 ld{in};
        SX_LAUNCH(scan_reduce<LoadI32>, static_cast<unsigned>(nb), kScanThreads, 0, s, ld, n, sums, nullptr, nullptr);
        SX_LAUNCH(scan_blocks, 1, 1024, 0, s, sums, nb, total);
        SX_LAUNCH((scan_down<LoadI32, StorePlain<int32_t>, false>), static_cast<unsigned>(nb),
                  kScanThreads, 0, s, ld, n, sums, StorePlain<int32_t>{out});
    }
}

size_t onesweep_u32_workspace(int64_t n, uint32_t key_bits, int64_t full_bins) {
    return onesweep_layout(n, key_bits, static_cast<int>(full_bins)).total;
}

void onesweep_sort_u32(const uint32_t* keys_in, const int32_t* vals_in, uint32_t* keys_out,
                       int32_t* vals_out, int64_t n, const int64_t* n_dev, uint32_t key_bits,
                       int32_t* full_offsets, int64_t full_bins, void* ws, uint32_t* status,
                       cudaStream_t s) {
    if (n <= 0 || key_bits == 0) return;
    if (n >= (int64_t{1} << 30)) throw_invalid("sort", "single-sweep sort needs n < 2^30");
    if (reinterpret_cast<uintptr_t>(keys_in) % 16 != 0)
        throw_invalid("sort", "single-sweep sort needs 16-byte aligned keys");
    if (full_offsets && (full_bins < 1 || full_bins > 16384 || (int64_t{1} << key_bits) < full_bins))
        throw_invalid("sort", "whole-key histogram needs 1 <= bins <= 16384 covering the keys");
    const int fb = full_offsets ? static_cast<int>(full_bins) : 0;
    const OnesweepLayout L = onesweep_layout(n, key_bits, fb);
    unsigned char* base = static_cast<unsigned char*>(ws);
    uint32_t* tk = reinterpret_cast<uint32_t*>(base + L.off_tk);
    int32_t* tv = reinterpret_cast<int32_t*>(base + L.off_tv);
    uint32_t* ghist = reinterpret_cast<uint32_t*>(base + L.off_ghist);
    uint32_t* fhist = reinterpret_cast<uint32_t*>(base + L.off_full);
    uint32_t* ctr = reinterpret_cast<uint32_t*>(base + L.off_ctr);
    uint32_t* lb = reinterpret_cast<uint32_t*>(base + L.off_lb);
    cuda_check(cudaMemsetAsync(base + L.off_zero, 0, L.zero_bytes, s), "sort workspace reset");

    smem_limit_once(reinterpret_cast<const void*>(os_pass), static_cast<int>(sizeof(OnesweepSmem)),
                    "sort smem attribute");
    smem_limit_once(reinterpret_cast<const void*>(os_hist),
                    static_cast<int>(sizeof(uint32_t) * (kOsMaxPasses * kRadix + 16384)),
                    "sort smem attribute");
    const unsigned hist_blocks = static_cast<unsigned>(
        std::min<int64_t>(kOsHistMaxCtas, (n + kOsHistThreads * 8 - 1) / (kOsHistThreads * 8)));
    const size_t hsm = sizeof(uint32_t) * (kOsMaxPasses * kRadix + fb);
    SX_LAUNCH(os_hist, hist_blocks, kOsHistThreads, hsm, s, keys_in, n, n_dev, L.passes, L.bits,
              ghist, full_offsets ? fhist : nullptr, fb);
    SX_LAUNCH(os_scan, static_cast<unsigned>(L.passes + (full_offsets ? 1 : 0)), 1024, 0, s, ghist,
              L.passes, L.bits, full_offsets ? fhist : nullptr, fb, full_offsets);
    const uint32_t* src_k = keys_in;
    const int32_t* src_v = vals_in;
    uint32_t* tk2 = reinterpret_cast<uint32_t*>(base + L.off_tk2);
    // at most three resident CTAs per SM (the pass's launch bound), each looping over tiles: a
    // grid sized by the capacity would mostly start CTAs that find no keys
    const unsigned pass_grid = static_cast<unsigned>(std::min<int64_t>(L.tiles, 148 * 3));
    for (int pass = 0; pass < L.passes; ++pass) {
        const int shift = pass * L.bits;
        const int bits = std::min<int>(L.bits, static_cast<int>(key_bits) - shift);
        const bool last = pass == L.passes - 1;
        // the last pass lands in the outputs; earlier passes alternate so src != dst
        const bool to_out = ((L.passes - 1 - pass) % 2) == 0;
        int32_t* dv = to_out ? vals_out : tv;
        uint32_t* dk;
        if (last) dk = keys_out;                       // may be null: keys not needed
        else if (keys_out) dk = to_out ? keys_out : tk;
        else dk = to_out ? tk2 : tk;                   // passes >= 3 without keys_out
        SX_LAUNCH(os_pass, pass_grid, kRsThreads, sizeof(OnesweepSmem), s,
                  src_k, src_v, dk, dv, n, n_dev, shift, bits, ghist + pass * kRadix,
                  lb + static_cast<int64_t>(pass) * L.tiles * kRadix, ctr + pass, status);
        src_k = dk;
        src_v = dv;
    }
}

size_t radix_sort_u64_workspace(int64_t n) { return radix_ws_bytes<uint64_t>(n); }
size_t radix_sort_u32_workspace(int64_t n) { return radix_ws_bytes<uint32_t>(n); }

void radix_sort_u64(const uint64_t* keys_in, const int32_t* vals_in, uint64_t* keys_out,
                    int32_t* vals_out, int64_t n, uint32_t key_bits, void* ws, cudaStream_t s) {
    radix_sort_impl<uint64_t>(keys_in, vals_in, keys_out, vals_out, n, nullptr, key_bits, ws, s);
}

void radix_sort_u32(const uint32_t* keys_in, const int32_t* vals_in, uint32_t* keys_out,
                    int32_t* vals_out, int64_t n, const int64_t* n_dev, uint32_t key_bits,
                    void* ws, cudaStream_t s) {
    radix_sort_impl<uint32_t>(keys_in, vals_in, keys_out, vals_out, n, n_dev, key_bits, ws, s);
}

// ------------------------------------------------------------------ allocation-free scan --------
// Fixed scratch for sxcuda_prefix_scan_i64_noalloc: one int64 block total per 4096-element tile.
// 65,536 entries (512 KiB per device, held from the library's first use on that device until the
// process exits) bound n at 65,536 * 4,096 = 268,435,456 elements.
constexpr int64_t kNoAllocScanSlots = 65536;
constexpr int64_t kNoAllocScanMaxN = kNoAllocScanSlots * kScanTile;
static __device__ __align__(256) int64_t g_noalloc_scan_scratch[kNoAllocScanSlots];

int64_t noalloc_scan_max_n() { return kNoAllocScanMaxN; }

// Device address of the scratch array for the current device. In host code
// g_noalloc_scan_scratch is only a host-side stand-in for the symbol, so the real address is
// looked up once per device (with that device current) and cached.
static int64_t* noalloc_scan_scratch() {
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static int64_t* cached[kMaxDevices] = {};
    if (dev < 0 || dev >= kMaxDevices) throw RuntimeError("prefix_scan_i64_noalloc: device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!cached[dev]) {
        void* p = nullptr;
        cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scan_scratch),
                   "prefix_scan_i64_noalloc: cudaGetSymbolAddress");
        cached[dev] = static_cast<int64_t*>(p);
    }
    return cached[dev];
}

// Same kernels as launch_scan_i64; the block totals go to the fixed scratch instead of a
// caller-provided workspace. Every slot the scan reads is written earlier in the same call, so
// nothing needs clearing first.
void launch_scan_i64_noalloc(const int32_t* in, int64_t* out, int64_t n, cudaStream_t s) {
    if (n > kNoAllocScanMaxN)
        throw_invalid("prefix_scan_i64_noalloc",
                      "n exceeds the fixed scratch capacity of 268435456 elements");
    if (n <= 0) return;
    launch_scan_i64(in, out, n, noalloc_scan_scratch(), s);
}

void launch_tile_offsets_u32(const uint32_t* sorted_tiles, const int64_t* n_dev, int64_t cap,
                             int64_t n_tiles, int32_t* offsets, cudaStream_t s) {
    const unsigned grid = blocks_for(cap > n_tiles ? cap : n_tiles, 256);
    SX_LAUNCH(tile_offsets_u32_kernel, grid, 256, 0, s, sorted_tiles, n_dev, cap, n_tiles, offsets);
}

}  // namespace sx
