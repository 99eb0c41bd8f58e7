// Supertile binning: the executor's tile-sorted intersection list (flatten_ids and the tile
// offsets) from the supertile entries that launch_emit_supertiles wrote and a stable sort put in
// supertile order. Integer work only.
//
// The list is the one the reference builds by sorting (tile, depth) keys (sort_isect,
// KernelBackend.h:164-176; isect_offset_encode, KernelBackend.h:178-190): tile-major, each
// tile's Gaussians in depth order. Here the order comes from the entries: a supertile's sorted
// run lists its Gaussians in depth order, so tile T's slots go to the entries whose mask holds T,
// in run order. The run is cut into chunks of kStChunk entries, a warp's rounds of 32:
//   st_chunks   the first chunk of every supertile (one CTA: a scan of the chunk counts);
//   st_count    per chunk, how many of its entries hold each of the supertile's 64 tiles;
//   st_prefix   per supertile, each chunk's exclusive prefix of those counts and each tile's total;
//               the CTA that finishes last scans the tile totals into tile_offsets;
//   st_write    per chunk and round, the Gaussian ids into their tiles' slots in entry order.
// A warp takes a chunk at a time with both rounds' loads issued first. A round's 32 masks,
// transposed as a 32 x 64 bit matrix, give lane k the round's entries holding tile bits k and
// k + 32, whose counters live in lane k's registers.
#include <algorithm>

#include "sx_internal.h"

namespace sx {
namespace {

constexpr int kBinThreads = 256;
constexpr int kBinWarps = kBinThreads / 32;
constexpr int kScanBlock = 1024;

// Exclusive scan of one value per thread over a 1024-thread block; `total` gets the block sum.
__device__ __forceinline__ uint32_t excl_scan_1024(uint32_t v, uint32_t* warp_sums, uint32_t& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(kFullMask, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = warp_sums[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(kFullMask, w, o);
            if (lane >= o) w += y;
        }
        warp_sums[lane] = w;
    }
    __syncthreads();
    const uint32_t before = warp == 0 ? 0u : warp_sums[warp - 1];
    total = warp_sums[31];
    __syncthreads();
    return before + x - v;
}

// The tile of bit `bit` of supertile `st`, or -1 beyond the grid's right or bottom edge.
__device__ __forceinline__ int64_t st_tile(const StBinArgs& a, int st, int bit) {
    const int tx = (st % a.st_width) * kStTiles + (bit % kStTiles);
    const int ty = (st / a.st_width) * kStTiles + (bit / kStTiles);
    if (tx >= static_cast<int>(a.tile_width) || ty >= static_cast<int>(a.tile_height)) return -1;
    return static_cast<int64_t>(ty) * a.tile_width + tx;
}

__global__ void __launch_bounds__(kScanBlock) st_chunks_kernel(StBinArgs a) {
    __shared__ uint32_t warp_sums[32];
    const int64_t n = *a.n_entries;
    uint32_t carry = 0;
    for (int s0 = 0; s0 < a.n_st; s0 += kScanBlock) {
        const int st = s0 + static_cast<int>(threadIdx.x);
        int64_t len = 0;
        if (st < a.n_st) len = (st + 1 < a.n_st ? a.st_offsets[st + 1] : n) - a.st_offsets[st];
        const uint32_t nch = static_cast<uint32_t>((len + kStChunk - 1) / kStChunk);
        uint32_t tot;
        const uint32_t ex = excl_scan_1024(nch, warp_sums, tot);
        if (st < a.n_st) a.st_chunk0[st] = static_cast<int32_t>(carry + ex);
        carry += tot;
    }
    if (threadIdx.x == 0) {
        a.st_chunk0[a.n_st] = static_cast<int32_t>(carry);
        *a.n_chunks = static_cast<int32_t>(carry);
    }
}

// Chunk c's supertile and entry range [b, e) of the sorted array. The supertile is the last one
// whose first chunk is <= c (supertiles without entries repeat their successor's first chunk).
struct ChunkRange {
    int st;
    int64_t b, e;
};
__device__ __forceinline__ ChunkRange chunk_range(const StBinArgs& a, int c, int64_t n) {
    int lo = 0, hi = a.n_st - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.st_chunk0[mid] <= c) lo = mid;
        else hi = mid - 1;
    }
    ChunkRange r;
    r.st = lo;
    const int64_t st_end = lo + 1 < a.n_st ? a.st_offsets[lo + 1] : n;
    r.b = a.st_offsets[lo] + static_cast<int64_t>(c - a.st_chunk0[lo]) * kStChunk;
    r.e = min(r.b + kStChunk, st_end);
    return r;
}

constexpr int kRounds = kStChunk / 32;

// 32 x 32 bit-matrix transpose over the warp: lane l holds row l, afterwards lane k holds column k
// (bit i = bit k of row i). Five butterfly stages, each swapping the off-diagonal blocks of the
// 2s x 2s blocks between lanes l and l ^ s.
__device__ __forceinline__ uint32_t warp_transpose32(uint32_t x) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
        const uint32_t lo = s == 16 ? 0x0000ffffu
                          : s == 8  ? 0x00ff00ffu
                          : s == 4  ? 0x0f0f0f0fu
                          : s == 2  ? 0x33333333u
                                    : 0x55555555u;
        const uint32_t y = __shfl_xor_sync(kFullMask, x, s);
        x = (lane & s) ? ((x & ~lo) | ((y & ~lo) >> s)) : ((x & lo) | ((y & lo) << s));
    }
    return x;
}

__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(kFullMask, v, o);
        if (lane >= o) v += y;
    }
    return v;
}

// The chunk's entry records in rounds of 32 (lane = entry): all rounds' sorted indices, then all
// their records, loads in flight together; zero records past the chunk.
__device__ __forceinline__ void chunk_entries(const StBinArgs& a, const ChunkRange& r,
                                              uint4 (&m)[kRounds]) {
    const int lane = threadIdx.x & 31;
    int32_t idx[kRounds];
#pragma unroll
    for (int k = 0; k < kRounds; ++k) {
        const int64_t i = r.b + k * 32 + lane;
        idx[k] = i < r.e ? a.sorted[i] : -1;
    }
#pragma unroll
    for (int k = 0; k < kRounds; ++k) m[k] = idx[k] >= 0 ? a.entry[idx[k]] : make_uint4(0u, 0u, 0u, 0u);
}

// Per chunk, the count of its entries holding each tile bit: the round's masks transposed give
// lane k the entries holding bit k (low word) and bit k + 32 (high word).
__global__ void __launch_bounds__(kBinThreads) st_count_kernel(StBinArgs a) {
    const int nch = *a.n_chunks;
    const int64_t n = *a.n_entries;
    const int lane = threadIdx.x & 31;
    const int warps = static_cast<int>(gridDim.x) * kBinWarps;
    for (int c = blockIdx.x * kBinWarps + (threadIdx.x >> 5); c < nch; c += warps) {  // per warp
        const ChunkRange r = chunk_range(a, c, n);
        uint4 m[kRounds];
        chunk_entries(a, r, m);
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int k = 0; k < kRounds; ++k) {
            lo += __popc(warp_transpose32(m[k].x));
            hi += __popc(warp_transpose32(m[k].y));
        }
        a.chunk_counts[static_cast<int64_t>(c) * 64 + lane] = lo;
        a.chunk_counts[static_cast<int64_t>(c) * 64 + 32 + lane] = hi;
    }
}

// Per chunk and round: the transposed masks give each tile its entries of the round; lane k
// lists the slots of tile k (then k + 32) in a per-warp shared list ordered by tile and, within a
// tile, by entry, and the warp then stores the list 32 items at a time, so consecutive lanes
// write consecutive slots of a tile. Items past the list's kRoundList capacity (rounds whose 32
// entries hold more pairs) are stored by the listing lane itself.
constexpr int kRoundList = 512;

__global__ void __launch_bounds__(kBinThreads) st_write_kernel(StBinArgs a) {
    __shared__ uint32_t s_slot[kBinWarps][kRoundList];
    __shared__ uint8_t s_ent[kBinWarps][kRoundList];
    __shared__ int32_t s_gid[kBinWarps][32];
    if (*a.overflow) return;  // uniform
    const int nch = *a.n_chunks;
    const int64_t n = *a.n_entries;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int warps = static_cast<int>(gridDim.x) * kBinWarps;
    for (int c = blockIdx.x * kBinWarps + w; c < nch; c += warps) {  // per warp
        const ChunkRange r = chunk_range(a, c, n);
        // next slot of tile bits lane and lane + 32 (bits beyond the grid are never set)
        const int64_t Tlo = st_tile(a, r.st, lane), Thi = st_tile(a, r.st, lane + 32);
        uint32_t slot_lo = Tlo >= 0 ? static_cast<uint32_t>(a.tile_offsets[Tlo]) +
                                          a.chunk_counts[static_cast<int64_t>(c) * 64 + lane]
                                    : 0u;
        uint32_t slot_hi = Thi >= 0 ? static_cast<uint32_t>(a.tile_offsets[Thi]) +
                                          a.chunk_counts[static_cast<int64_t>(c) * 64 + 32 + lane]
                                    : 0u;
        uint4 m[kRounds];  // (mask lo, mask hi, Gaussian id, 0)
        chunk_entries(a, r, m);
#pragma unroll
        for (int k = 0; k < kRounds; ++k) {
            const uint32_t tlo = warp_transpose32(m[k].x);
            const uint32_t thi = warp_transpose32(m[k].y);
            const uint32_t clo = __popc(tlo), chi = __popc(thi);
            const uint32_t ilo = warp_incl_scan(clo), ihi = warp_incl_scan(chi);
            const uint32_t tot_lo = __shfl_sync(kFullMask, ilo, 31);
            const uint32_t total = tot_lo + __shfl_sync(kFullMask, ihi, 31);
            s_gid[w][lane] = static_cast<int32_t>(m[k].z);
            __syncwarp();
            auto list = [&](uint32_t col, uint32_t o, uint32_t slot) {
                while (col) {
                    const int j = __ffs(col) - 1;
                    col &= col - 1u;
                    if (o < kRoundList) {
                        s_slot[w][o] = slot;
                        s_ent[w][o] = static_cast<uint8_t>(j);
                    } else {
                        a.flatten_ids[slot] = s_gid[w][j];
                    }
                    ++o;
                    ++slot;
                }
            };
            list(tlo, ilo - clo, slot_lo);
            list(thi, tot_lo + ihi - chi, slot_hi);
            slot_lo += clo;
            slot_hi += chi;
            __syncwarp();
            const uint32_t listed = min(total, static_cast<uint32_t>(kRoundList));
            for (uint32_t i = lane; i < listed; i += 32) a.flatten_ids[s_slot[w][i]] = s_gid[w][s_ent[w][i]];
            __syncwarp();  // the next round rewrites the list
        }
    }
}

// One CTA per supertile: thread (segment, bit) of 16 x 64 sums its segment of the supertile's
// chunks (16 loads in flight), the segment sums are scanned in shared memory, and each segment
// rewrites its chunk counts as exclusive prefixes; the last segment's end is the tile's total.
// The CTA that finishes last (a device counter, reset by that CTA for the next step) then scans
// the tile totals into tile_offsets.
constexpr int kPrefixSegs = 16;
static_assert(kPrefixSegs * 64 == kScanBlock, "the last CTA runs the 1024-thread tile scan");

__device__ __forceinline__ void scan_tile_totals(const StBinArgs& a, uint32_t* warp_sums) {
    const int64_t n_tiles = static_cast<int64_t>(a.tile_width) * a.tile_height;
    uint32_t carry = 0;
    for (int64_t t0 = 0; t0 < n_tiles; t0 += kScanBlock) {
        const int64_t T = t0 + threadIdx.x;
        const uint32_t v = T < n_tiles ? static_cast<uint32_t>(a.tile_counts[T]) : 0u;
        uint32_t tot;
        const uint32_t ex = excl_scan_1024(v, warp_sums, tot);
        if (T < n_tiles) a.tile_offsets[T] = static_cast<int32_t>(carry + ex);
        carry += tot;
    }
}

__global__ void __launch_bounds__(kPrefixSegs * 64) st_prefix_kernel(StBinArgs a) {
    __shared__ uint32_t s_seg[kPrefixSegs][64];
    const int st = blockIdx.x, bit = threadIdx.x & 63, seg = threadIdx.x >> 6;
    const int c0 = a.st_chunk0[st], c1 = a.st_chunk0[st + 1];
    const int per = (c1 - c0 + kPrefixSegs - 1) / kPrefixSegs;
    const int s0 = min(c0 + seg * per, c1), s1 = min(s0 + per, c1);
    uint32_t* col = a.chunk_counts + bit;
    constexpr int B = 16;  // loads in flight per thread
    uint32_t sum = 0;
    for (int c = s0; c < s1; c += B) {
        uint32_t v[B];
#pragma unroll
        for (int k = 0; k < B; ++k) v[k] = c + k < s1 ? col[static_cast<int64_t>(c + k) * 64] : 0u;
#pragma unroll
        for (int k = 0; k < B; ++k) sum += v[k];
    }
    s_seg[seg][bit] = sum;
    __syncthreads();
    uint32_t run = 0;
    for (int q = 0; q < seg; ++q) run += s_seg[q][bit];
    for (int c = s0; c < s1; c += B) {
        uint32_t v[B];
#pragma unroll
        for (int k = 0; k < B; ++k) v[k] = c + k < s1 ? col[static_cast<int64_t>(c + k) * 64] : 0u;
#pragma unroll
        for (int k = 0; k < B; ++k) {
            if (c + k < s1) col[static_cast<int64_t>(c + k) * 64] = run;
            run += v[k];
        }
    }
    if (seg == kPrefixSegs - 1) {
        const int64_t T = st_tile(a, st, bit);
        if (T >= 0) a.tile_counts[T] = static_cast<int32_t>(run);
    }
    // the last CTA to get here scans the tile totals
    __shared__ uint32_t s_last;
    __shared__ uint32_t warp_sums[32];
    __threadfence();  // this CTA's totals are visible before it is counted
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(a.done, 1u) == static_cast<uint32_t>(a.n_st) - 1u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();  // every other CTA's totals are read after their count
    scan_tile_totals(a, warp_sums);
    if (threadIdx.x == 0) *a.done = 0u;  // ready for the next step
}

}  // namespace

int64_t st_chunk_capacity(int64_t capacity, int64_t n_st) {
    return capacity / kStChunk + n_st + 1;
}

void launch_bin_supertiles(const StBinArgs& a, cudaStream_t s) {
    if (a.n_st <= 0) return;
    if (a.n_st > kStMaxSupertiles) throw_invalid("bin_supertiles", "too many supertiles");
    // eight CTAs per SM of the 148 (the grid is fixed for graph capture; warps stride the chunks)
    const unsigned grid = static_cast<unsigned>(std::max<int64_t>(
        1, std::min<int64_t>((a.max_chunks + kBinWarps - 1) / kBinWarps, 148 * 8)));
    SX_LAUNCH(st_chunks_kernel, 1, kScanBlock, 0, s, a);
    SX_LAUNCH(st_count_kernel, grid, kBinThreads, 0, s, a);
    SX_LAUNCH(st_prefix_kernel, static_cast<unsigned>(a.n_st), kPrefixSegs * 64, 0, s, a);
    SX_LAUNCH(st_write_kernel, grid, kBinThreads, 0, s, a);
}

}  // namespace sx
