// Device-wide exclusive scan and stable LSD radix sort of (u64 key, u32 value)
// pairs, written for sm_100a.  They replace CUB DeviceScan::InclusiveSum and
// DeviceRadixSort::SortPairs of the reference (gutRenderer.cu:1323, :1527).
//
// Radix sort: 8-bit digits, one pass per digit over [begin_bit, end_bit).
// Each pass is three kernels: per-block digit histograms, an exclusive scan
// of the digit-major histogram table, and a stable scatter.  The scatter
// ranks a block's 4096 items warp by warp in input order (match.any peer
// groups), stages them in shared memory in digit order and writes each digit
// run contiguously.  Equal keys keep their input order, as CUB's does.
//
// Everything here has internal linkage (anonymous namespace) so that every
// translation unit that includes this header gets its own kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gf {
namespace {

constexpr int kScanThreads = 512;
constexpr int kScanItems = 8;  // items per thread
constexpr int kScanTile = kScanThreads * kScanItems;

template <typename T>
__device__ __forceinline__ T warp_inclusive_scan(T v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Block-wide exclusive scan of one value per thread; returns the exclusive
// prefix and the block total.
template <typename T, int THREADS>
__device__ __forceinline__ T block_exclusive_scan(T v, T& total) {
    __shared__ T warpSums[THREADS / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const T inc = warp_inclusive_scan(v);
    if (lane == 31) warpSums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        T s = lane < THREADS / 32 ? warpSums[lane] : T(0);
        s = warp_inclusive_scan(s);
        if (lane < THREADS / 32) warpSums[lane] = s;
    }
    __syncthreads();
    total = warpSums[THREADS / 32 - 1];
    const T warpPrefix = warp == 0 ? T(0) : warpSums[warp - 1];
    __syncthreads();
    return warpPrefix + inc - v;
}

// Phase 1: per-tile sums.
template <typename In, typename Out>
__global__ __launch_bounds__(kScanThreads) void k_scan_reduce(const In* __restrict__ in, uint64_t n,
                                                              Out* __restrict__ tileSums) {
    const uint64_t base = uint64_t(blockIdx.x) * kScanTile;
    Out s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const uint64_t i = base + uint64_t(k) * kScanThreads + threadIdx.x;
        if (i < n) s += Out(in[i]);
    }
    Out total;
    block_exclusive_scan<Out, kScanThreads>(s, total);
    if (threadIdx.x == 0) tileSums[blockIdx.x] = total;
}

// Phase 2: exclusive scan of the tile sums in one block (loops over chunks).
template <typename Out>
__global__ __launch_bounds__(kScanThreads) void k_scan_tiles(Out* __restrict__ tileSums, uint32_t numTiles,
                                                             Out* __restrict__ grandTotal) {
    Out carry = 0;
    for (uint32_t base = 0; base < numTiles; base += kScanThreads) {
        const uint32_t i = base + threadIdx.x;
        const Out v = i < numTiles ? tileSums[i] : Out(0);
        Out total;
        const Out ex = block_exclusive_scan<Out, kScanThreads>(v, total);
        if (i < numTiles) tileSums[i] = carry + ex;
        carry += total;
    }
    if (threadIdx.x == 0 && grandTotal != nullptr) *grandTotal = carry;
}

// Phase 3: exclusive scan within each tile, offset by the tile prefix.  Items
// are processed thread-contiguously (thread t owns items t*8 .. t*8+7).
template <typename In, typename Out>
__global__ __launch_bounds__(kScanThreads) void k_scan_downsweep(const In* __restrict__ in, uint64_t n,
                                                                 const Out* __restrict__ tilePrefix,
                                                                 Out* __restrict__ out) {
    const uint64_t base = uint64_t(blockIdx.x) * kScanTile + uint64_t(threadIdx.x) * kScanItems;
    Out v[kScanItems];
    Out s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const uint64_t i = base + k;
        v[k] = i < n ? Out(in[i]) : Out(0);
        s += v[k];
    }
    Out total;
    Out run = block_exclusive_scan<Out, kScanThreads>(s, total) + tilePrefix[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const uint64_t i = base + k;
        if (i < n) out[i] = run;
        run += v[k];
    }
}

// ------------------------------------------------------------ radix sort
constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItemsPerThread = 16;
constexpr int kSortTile = kSortThreads * kSortItemsPerThread;  // 4096
constexpr int kSortWarpItems = 32 * kSortItemsPerThread;       // 512 contiguous items per warp
constexpr int kRadixBins = 256;

__device__ __forceinline__ uint32_t digit_of(uint64_t key, int shift) { return uint32_t(key >> shift) & 0xffu; }

// Per-block digit counts, stored digit-major: hist[digit * numBlocks + block].
// With nDev the item count is read from device memory (at most n, the count
// the grid was sized for); blocks past it store zero counts.
__global__ __launch_bounds__(kSortThreads) void k_radix_histogram(const uint64_t* __restrict__ keys, uint32_t n,
                                                                  int shift, uint32_t numBlocks,
                                                                  uint32_t* __restrict__ hist,
                                                                  const uint32_t* __restrict__ nDev = nullptr) {
    __shared__ uint32_t h[kSortWarps][kRadixBins];
    if (nDev != nullptr) n = min(n, *nDev);
    for (int i = threadIdx.x; i < kSortWarps * kRadixBins; i += kSortThreads) (&h[0][0])[i] = 0u;
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t base = blockIdx.x * kSortTile + warp * kSortWarpItems;
    // all loads first, so that their latencies overlap
    uint64_t key[kSortItemsPerThread];
#pragma unroll
    for (int k = 0; k < kSortItemsPerThread; ++k) {
        const uint32_t i = base + k * 32 + lane;
        key[k] = i < n ? __ldg(keys + i) : 0ull;
    }
#pragma unroll
    for (int k = 0; k < kSortItemsPerThread; ++k) {
        if (base + k * 32 + lane < n) atomicAdd(&h[warp][digit_of(key[k], shift)], 1u);
    }
    __syncthreads();
    for (int d = threadIdx.x; d < kRadixBins; d += kSortThreads) {
        uint32_t s = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) s += h[w][d];
        hist[uint64_t(d) * numBlocks + blockIdx.x] = s;
    }
}

// A warp ranks its 16 items per lane as kSortChains independent chains of
// kSortChainItems items (item k in chain k / kSortChainItems), each with its
// own digit counters, advanced together: item order (warp, chain, item, lane)
// is the input order, so the ranks stay stable, and the chains' shared-memory
// round trips overlap instead of following one another.
constexpr int kSortChains = 4;
constexpr int kSortChainItems = kSortItemsPerThread / kSortChains;
constexpr int kSortCounters = kSortWarps * kSortChains;

struct SortScatterSmem {
    uint64_t keys[kSortTile];
    uint32_t vals[kSortTile];
    uint32_t warpHist[kSortCounters][kRadixBins];  // running counts per (warp, chain), then their offsets
    uint32_t blockStart[kRadixBins];            // first block-local position of each digit
    uint32_t globalStart[kRadixBins];           // first global position of this block's digit run
};

__global__ __launch_bounds__(kSortThreads, 2) void k_radix_scatter(const uint64_t* __restrict__ keysIn,
                                                                const uint32_t* __restrict__ valsIn,
                                                                uint64_t* __restrict__ keysOut,
                                                                uint32_t* __restrict__ valsOut, uint32_t n,
                                                                int shift, uint32_t numBlocks,
                                                                const uint32_t* __restrict__ histScanned,
                                                                const uint32_t* __restrict__ nDev = nullptr) {
    extern __shared__ __align__(16) unsigned char smemRaw[];
    if (nDev != nullptr) n = min(n, *nDev);
    if (blockIdx.x * uint32_t(kSortTile) >= n) return;  // block-uniform: nothing of this block to move
    SortScatterSmem& sm = *reinterpret_cast<SortScatterSmem*>(smemRaw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < kSortCounters * kRadixBins; i += kSortThreads) (&sm.warpHist[0][0])[i] = 0u;
    for (int d = threadIdx.x; d < kRadixBins; d += kSortThreads)
        sm.globalStart[d] = histScanned[uint64_t(d) * numBlocks + blockIdx.x];
    __syncthreads();

    const uint32_t base = blockIdx.x * kSortTile + warp * kSortWarpItems;
    const uint32_t lanesBelow = (1u << lane) - 1u;
    uint64_t key[kSortItemsPerThread];
    uint32_t val[kSortItemsPerThread];
    uint32_t rank[kSortItemsPerThread];
    // All loads first: the ranking below synchronises the warp per item, and
    // a load issued inside that loop would wait out its full latency each time.
#pragma unroll
    for (int k = 0; k < kSortItemsPerThread; ++k) {
        const uint32_t i = base + k * 32 + lane;
        const bool valid = i < n;
        key[k] = valid ? __ldg(keysIn + i) : ~0ull;
        val[k] = valid ? __ldg(valsIn + i) : 0u;
    }
    // Chain-local stable ranks, item order = (k, lane) within the warp's 512-item run.
#pragma unroll
    for (int j = 0; j < kSortChainItems; ++j) {
        uint32_t dig[kSortChains], cnt[kSortChains];
        bool lead[kSortChains];
#pragma unroll
        for (int c = 0; c < kSortChains; ++c) {
            const int k = c * kSortChainItems + j;
            const bool valid = base + k * 32 + lane < n;
            dig[c] = digit_of(key[k], shift);
            const uint32_t peers = __match_any_sync(0xffffffffu, dig[c]) & __ballot_sync(0xffffffffu, valid);
            const uint32_t before = sm.warpHist[warp * kSortChains + c][dig[c]];
            rank[k] = before + __popc(peers & lanesBelow);
            cnt[c] = before + __popc(peers);
            lead[c] = valid && (peers & lanesBelow) == 0u;
        }
        __syncwarp();
#pragma unroll
        for (int c = 0; c < kSortChains; ++c)
            if (lead[c]) sm.warpHist[warp * kSortChains + c][dig[c]] = cnt[c];
        __syncwarp();
    }
    __syncthreads();
    // Per digit: exclusive prefix over (warp, chain) in item order (in place)
    // and the block-local digit start.
    if (threadIdx.x < kRadixBins) {
        const int d = threadIdx.x;
        uint32_t s = 0;
#pragma unroll
        for (int w = 0; w < kSortCounters; ++w) {
            const uint32_t c = sm.warpHist[w][d];
            sm.warpHist[w][d] = s;
            s += c;
        }
        sm.blockStart[d] = s;  // digit total for now
    }
    __syncthreads();
    {
        uint32_t total;
        const uint32_t v = threadIdx.x < kRadixBins ? sm.blockStart[threadIdx.x] : 0u;
        const uint32_t ex = block_exclusive_scan<uint32_t, kSortThreads>(v, total);
        if (threadIdx.x < kRadixBins) sm.blockStart[threadIdx.x] = ex;
    }
    __syncthreads();
    // Stage in shared memory in digit order.
#pragma unroll
    for (int k = 0; k < kSortItemsPerThread; ++k) {
        const uint32_t i = base + k * 32 + lane;
        if (i < n) {
            const uint32_t d = digit_of(key[k], shift);
            const uint32_t pos = sm.blockStart[d] + sm.warpHist[warp * kSortChains + k / kSortChainItems][d] + rank[k];
            sm.keys[pos] = key[k];
            sm.vals[pos] = val[k];
        }
    }
    __syncthreads();
    const uint32_t blockCount = min(uint32_t(kSortTile), n - blockIdx.x * kSortTile);
    for (uint32_t p = threadIdx.x; p < blockCount; p += kSortThreads) {
        const uint64_t k = sm.keys[p];
        const uint32_t d = digit_of(k, shift);
        const uint32_t g = sm.globalStart[d] + (p - sm.blockStart[d]);
        keysOut[g] = k;
        valsOut[g] = sm.vals[p];
    }
}

}  // namespace
}  // namespace gf
