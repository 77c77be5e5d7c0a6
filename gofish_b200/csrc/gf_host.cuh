// Host-side helpers shared by the library's translation units: error
// recording, stream-ordered device buffers, pose preparation and the host
// drivers of the device-wide scan and radix sort (gf_sort.cuh).
//
// Everything has internal linkage; the error string itself lives in
// gf_tracer.cu behind gf_record_error so that gf_last_error() reports the
// last failure of any entry point.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "../../include/gofish_b200.h"
#include "gf_device.cuh"
#include "gf_sort.cuh"

// Records an error for gf_last_error(); defined in gf_tracer.cu.
int gf_record_error(int code, const char* message);

namespace {

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return gf_record_error(code, buf);
}

#define GF_CUDA(call)                                                                                     \
    do {                                                                                                  \
        const cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess) return fail(GF_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

#define GF_LAUNCH_CHECK()                                                                                  \
    do {                                                                                                   \
        const cudaError_t e_ = cudaGetLastError();                                                         \
        if (e_ != cudaSuccess) return fail(GF_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e_)); \
    } while (0)

// Device allocation that grows geometrically, stream-ordered, so that steady
// state calls allocate nothing.
struct DeviceBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    int ensure(size_t need, cudaStream_t stream) {
        if (need <= bytes) return GF_OK;
        if (ptr != nullptr) {
            GF_CUDA(cudaFreeAsync(ptr, stream));
            ptr = nullptr;
            bytes = 0;
        }
        const size_t grown = need + need / 4 + 256;
        GF_CUDA(cudaMallocAsync(&ptr, grown, stream));
        bytes = grown;
        return GF_OK;
    }
    void release() {
        if (ptr != nullptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
    template <typename T>
    T* as() const {
        return static_cast<T*>(ptr);
    }
};

uint32_t bit_length(uint64_t n) {
    uint32_t b = 0;
    while (n != 0u) {
        ++b;
        n >>= 1;
    }
    return b;
}

// World->sensor rotation of the quaternion (x, y, z, w) of a [t, q] pose, its
// transpose and the sensor centre c = -R^T t, built in double precision and
// rounded once (the oracle's oracle_prepare_pose makes the same floats).
void prepare_pose(const float* pose7, gf::Pose& out) {
    const double tx = pose7[0], ty = pose7[1], tz = pose7[2];
    const double x = pose7[3], y = pose7[4], z = pose7[5], w = pose7[6];
    double R[9];
    R[0] = 1.0 - 2.0 * (y * y + z * z);
    R[1] = 2.0 * (x * y - w * z);
    R[2] = 2.0 * (x * z + w * y);
    R[3] = 2.0 * (x * y + w * z);
    R[4] = 1.0 - 2.0 * (x * x + z * z);
    R[5] = 2.0 * (y * z - w * x);
    R[6] = 2.0 * (x * z - w * y);
    R[7] = 2.0 * (y * z + w * x);
    R[8] = 1.0 - 2.0 * (x * x + y * y);
    for (int i = 0; i < 9; ++i) out.R[i] = float(R[i]);
    out.t[0] = float(tx);
    out.t[1] = float(ty);
    out.t[2] = float(tz);
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c) out.Rinv[3 * r + c] = out.R[3 * c + r];
    for (int r = 0; r < 3; ++r) out.c[r] = float(-(R[0 * 3 + r] * tx + R[1 * 3 + r] * ty + R[2 * 3 + r] * tz));
}

// Exclusive scan of n values; grandTotal receives the sum.  `tiles` is the
// per-tile partial-sum scratch; `launches` counts the kernels issued.
template <typename In, typename Out>
int scan_exclusive(DeviceBuffer& tiles, uint32_t& launches, const In* in, uint64_t n, Out* out, Out* grandTotal,
                   cudaStream_t stream) {
    const uint32_t count = uint32_t((n + gf::kScanTile - 1) / gf::kScanTile);
    if (count == 0) {
        GF_CUDA(cudaMemsetAsync(grandTotal, 0, sizeof(Out), stream));
        return GF_OK;
    }
    if (int e = tiles.ensure(sizeof(Out) * count, stream)) return e;
    Out* ts = tiles.as<Out>();
    gf::k_scan_reduce<In, Out><<<count, gf::kScanThreads, 0, stream>>>(in, n, ts);
    gf::k_scan_tiles<Out><<<1, gf::kScanThreads, 0, stream>>>(ts, count, grandTotal);
    gf::k_scan_downsweep<In, Out><<<count, gf::kScanThreads, 0, stream>>>(in, n, ts, out);
    launches += 3;
    GF_LAUNCH_CHECK();
    return GF_OK;
}

// Stable LSD radix sort of (u64 key, u32 value) pairs held in keys[0]/ids[0]
// over the key bits [beginBit, endBit), ping-ponging with keys[1]/ids[1];
// *finalBuf names the buffer that holds the result.  With nDev the number of
// pairs is read on the device (at most n, which sizes the grids), so the host
// need not know it.
int sort_pairs(DeviceBuffer& hist, DeviceBuffer& tiles, uint32_t& launches, DeviceBuffer* keys, DeviceBuffer* ids,
               uint32_t n, int beginBit, int endBit, int* finalBuf, cudaStream_t stream,
               const uint32_t* nDev = nullptr) {
    *finalBuf = 0;
    if (n == 0) return GF_OK;
    const uint32_t blocks = (n + gf::kSortTile - 1) / gf::kSortTile;
    if (int e = hist.ensure(sizeof(uint32_t) * (size_t(blocks) * gf::kRadixBins + 1), stream)) return e;
    uint32_t* h = hist.as<uint32_t>();
    const int smem = int(sizeof(gf::SortScatterSmem));
    GF_CUDA(cudaFuncSetAttribute(gf::k_radix_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    int src = 0;
    for (int shift = beginBit; shift < endBit; shift += 8) {
        gf::k_radix_histogram<<<blocks, gf::kSortThreads, 0, stream>>>(keys[src].as<uint64_t>(), n, shift, blocks, h,
                                                                      nDev);
        launches += 1;
        GF_LAUNCH_CHECK();
        if (int e = scan_exclusive<uint32_t, uint32_t>(tiles, launches, h, uint64_t(blocks) * gf::kRadixBins, h,
                                                        h + size_t(blocks) * gf::kRadixBins, stream))
            return e;
        gf::k_radix_scatter<<<blocks, gf::kSortThreads, smem, stream>>>(keys[src].as<uint64_t>(),
                                                                        ids[src].as<uint32_t>(),
                                                                        keys[src ^ 1].as<uint64_t>(),
                                                                        ids[src ^ 1].as<uint32_t>(), n, shift, blocks, h,
                                                                        nDev);
        launches += 1;
        GF_LAUNCH_CHECK();
        src ^= 1;
    }
    *finalBuf = src;
    return GF_OK;
}

}  // namespace
