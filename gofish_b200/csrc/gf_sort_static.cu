// Tile-key sort that allocates no device memory.
//
// Some callers of this library cannot allocate device memory while they
// render: renderers embedded in a host application that hands the library a
// fixed device budget and forbids allocation on its frame path, real-time
// loops in which a cudaMalloc (which can synchronize the device) would stall
// a frame, and allocator-less tools that only pass preallocated buffers.
// gf_sort_tile_keys_static gives them the tracer's (tile | depth) key sort
// with all of its scratch in one file-scope device array of fixed size.
//
// The scratch array (GF_STATIC_SORT_MAX_PAIRS pairs of ping-pong storage plus
// the digit histograms, about 3.1 MiB) is part of the library image: every
// GPU that loads the library holds it until the process exits.  Host code
// cannot use the array's name as a device address, so the first call on each
// device looks the address up with cudaGetSymbolAddress while that device is
// current; make that first call before any stream capture.  The address is
// kept for the life of the process, so cudaDeviceReset is not supported while
// the library is loaded (the array would move).  Every call on a
// device shares the one array: calls whose GPU work overlaps (on different
// streams, or from different threads) race on it and must be serialized by
// the caller.  Nothing in the array needs to start at zero: each pass
// rewrites every histogram entry it reads.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/gofish_b200.h"
#include "gf_sort.cuh"

int gf_record_error(int code, const char* message);

namespace {

constexpr uint32_t kMaxPairs = GF_STATIC_SORT_MAX_PAIRS;
constexpr uint32_t kMaxBlocks = (kMaxPairs + gf::kSortTile - 1) / gf::kSortTile;
constexpr uint32_t kHistEntries = kMaxBlocks * gf::kRadixBins;
constexpr uint32_t kMaxScanTiles = (kHistEntries + gf::kScanTile - 1) / gf::kScanTile;

struct StaticSortScratch {
    uint64_t keys[kMaxPairs];
    uint32_t ids[kMaxPairs];
    uint32_t hist[kHistEntries + 1];  // digit-major histogram table + grand total
    uint32_t scanTiles[kMaxScanTiles];
};

__device__ __align__(256) unsigned char g_sortScratch[sizeof(StaticSortScratch)];

constexpr int kMaxDevices = 64;
std::mutex g_setupMutex;
StaticSortScratch* g_scratchAddress[kMaxDevices] = {};

int fail_cuda(const char* what, cudaError_t e) {
    char buf[512];
    snprintf(buf, sizeof(buf), "gf_sort_tile_keys_static: %s failed: %s", what, cudaGetErrorString(e));
    return gf_record_error(GF_ERR_CUDA, buf);
}

}  // namespace

extern "C" int gf_sort_tile_keys_static(const uint64_t* keys_in, const uint32_t* ids_in, uint64_t* keys_out,
                                        uint32_t* ids_out, uint32_t n, int end_bit, void* stream) {
    if (n > kMaxPairs) {
        char buf[256];
        snprintf(buf, sizeof(buf),
                 "gf_sort_tile_keys_static: %u pairs exceed the fixed scratch of %u pairs (GF_STATIC_SORT_MAX_PAIRS)",
                 n, kMaxPairs);
        return gf_record_error(GF_ERR_CAPACITY, buf);
    }
    if (end_bit < 0 || end_bit > 64) return gf_record_error(GF_ERR_BAD_INPUT, "gf_sort_tile_keys_static: end_bit must be in [0, 64]");
    if (n > 0 && (keys_in == nullptr || ids_in == nullptr || keys_out == nullptr || ids_out == nullptr))
        return gf_record_error(GF_ERR_BAD_INPUT, "gf_sort_tile_keys_static: NULL buffer");
    if (n > 0 && (static_cast<const void*>(keys_in) == keys_out || static_cast<const void*>(ids_in) == ids_out))
        return gf_record_error(GF_ERR_BAD_INPUT, "gf_sort_tile_keys_static: inputs must not alias the outputs");
    // an error left by earlier work is reported as such, not as this sort's launch failure
    cudaError_t e = cudaPeekAtLastError();
    if (e != cudaSuccess) return fail_cuda("a CUDA call made before this sort", e);
    int device = -1;
    e = cudaGetDevice(&device);
    if (e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
    if (device < 0 || device >= kMaxDevices) return gf_record_error(GF_ERR_STATE, "gf_sort_tile_keys_static: device index out of range");
    StaticSortScratch* scratch = nullptr;
    {
        // Once per device, with that device current: the device address of the array.
        std::lock_guard<std::mutex> lock(g_setupMutex);
        if (g_scratchAddress[device] == nullptr) {
            void* ptr = nullptr;
            e = cudaGetSymbolAddress(&ptr, g_sortScratch);
            if (e != cudaSuccess) return fail_cuda("cudaGetSymbolAddress", e);
            e = cudaFuncSetAttribute(gf::k_radix_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     int(sizeof(gf::SortScatterSmem)));
            if (e != cudaSuccess) return fail_cuda("cudaFuncSetAttribute", e);
            g_scratchAddress[device] = static_cast<StaticSortScratch*>(ptr);
        }
        scratch = g_scratchAddress[device];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (n == 0) return GF_OK;
    const uint32_t blocks = (n + gf::kSortTile - 1) / gf::kSortTile;
    const uint64_t histN = uint64_t(blocks) * gf::kRadixBins;
    const uint32_t scanTiles = uint32_t((histN + gf::kScanTile - 1) / gf::kScanTile);
    int passes = 0;
    for (int shift = 0; shift < end_bit; shift += 8) ++passes;
    if (passes == 0) {
        e = cudaMemcpyAsync(keys_out, keys_in, sizeof(uint64_t) * n, cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(ids_out, ids_in, sizeof(uint32_t) * n, cudaMemcpyDeviceToDevice, s);
        return e == cudaSuccess ? GF_OK : fail_cuda("cudaMemcpyAsync", e);
    }
    // Ping-pong between the caller's output and the scratch so the last pass
    // lands in the output; the input is never written.
    const uint64_t* srcK = keys_in;
    const uint32_t* srcV = ids_in;
    bool toOutput = (passes % 2) == 1;
    int shift = 0;
    for (int p = 0; p < passes; ++p, shift += 8) {
        uint64_t* dstK = toOutput ? keys_out : scratch->keys;
        uint32_t* dstV = toOutput ? ids_out : scratch->ids;
        gf::k_radix_histogram<<<blocks, gf::kSortThreads, 0, s>>>(srcK, n, shift, blocks, scratch->hist);
        gf::k_scan_reduce<uint32_t, uint32_t><<<scanTiles, gf::kScanThreads, 0, s>>>(scratch->hist, histN,
                                                                                   scratch->scanTiles);
        gf::k_scan_tiles<uint32_t><<<1, gf::kScanThreads, 0, s>>>(scratch->scanTiles, scanTiles,
                                                                  scratch->hist + histN);
        gf::k_scan_downsweep<uint32_t, uint32_t><<<scanTiles, gf::kScanThreads, 0, s>>>(
            scratch->hist, histN, scratch->scanTiles, scratch->hist);
        gf::k_radix_scatter<<<blocks, gf::kSortThreads, sizeof(gf::SortScatterSmem), s>>>(
            srcK, srcV, dstK, dstV, n, shift, blocks, scratch->hist);
        e = cudaGetLastError();
        if (e != cudaSuccess) return fail_cuda("kernel launch", e);
        srcK = dstK;
        srcV = dstV;
        toOutput = !toOutput;
    }
    return GF_OK;
}
