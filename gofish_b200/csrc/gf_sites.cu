// Tetrahedralization sites on sm_100a (reference gofish/mesh/sites.py:43-83,
// where it runs in numpy on the host).
//
// Every Gaussian with opacity o > 1/255 contributes nine sites: its centre,
// then the eight corners mu + B (r s) of its support box, s in {-1,+1}^3 with
// x the slowest sign and z the fastest, where r = min(sqrt(-2 ln 0.0113f),
// sqrt(2 ln(255 o))) is the opacity-adaptive support radius.  Sites keep the
// Gaussians' order (a stable compaction by an exclusive scan of the kept
// flags), each carries its owner's index and the scale sigma_max r.
//
// Arithmetic: float64 throughout, rounded once to float32, with the
// contraction order of the numpy restatement: each corner coordinate is
// mu_i + ((B_i0 o_0 + B_i1 o_1) + B_i2 o_2) with o = r s, every product and
// sum rounded separately (-fmad=false).  r uses the double-precision log and
// square root.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/gofish_b200.h"
#include "gf_host.cuh"

namespace {

constexpr double kDeadOpacity = 1.0 / 255.0;

__global__ void k_site_flags(const float* __restrict__ density, uint32_t n, uint32_t* __restrict__ keep) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) keep[i] = double(density[i]) > kDeadOpacity ? 1u : 0u;
}

// One thread per Gaussian; slot = its position among the kept ones.
__global__ void k_sites(const float* __restrict__ positions, const float* __restrict__ factor,
                        const float* __restrict__ density, const float* __restrict__ sigmaMax, uint32_t n,
                        const uint32_t* __restrict__ keep, const uint32_t* __restrict__ slot, double radiusCap,
                        float* __restrict__ points, float* __restrict__ scale, int64_t* __restrict__ owner,
                        uint32_t* __restrict__ status) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || keep[i] == 0u) return;
    const double o = double(density[i]);
    const double r = fmin(radiusCap, sqrt(2.0 * log(255.0 * o)));
    if (!(isfinite(r) && r > 0.0)) {
        atomicOr(status, 1u);
        return;
    }
    const size_t base = size_t(slot[i]) * 9;
    const double mu[3] = {double(positions[3 * size_t(i)]), double(positions[3 * size_t(i) + 1]),
                          double(positions[3 * size_t(i) + 2])};
    double B[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) B[k] = double(factor[9 * size_t(i) + k]);
    float* out = points + 3 * base;
    out[0] = float(mu[0]);
    out[1] = float(mu[1]);
    out[2] = float(mu[2]);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const double off[3] = {(c & 4) ? r : -r, (c & 2) ? r : -r, (c & 1) ? r : -r};
#pragma unroll
        for (int row = 0; row < 3; ++row) {
            const double sum = (B[3 * row] * off[0] + B[3 * row + 1] * off[1]) + B[3 * row + 2] * off[2];
            out[3 * (1 + c) + row] = float(mu[row] + sum);
        }
    }
    const float s = float(double(sigmaMax[i]) * r);
#pragma unroll
    for (int k = 0; k < 9; ++k) {
        scale[base + k] = s;
        owner[base + k] = int64_t(i);
    }
}

}  // namespace

extern "C" int gf_mesh_sites(const float* positions, const float* factor, const float* density,
                             const float* sigma_max, uint32_t num_gaussians, float* points, float* scale,
                             int64_t* owner, uint32_t* count, uint32_t* status, void* stream) {
    if (num_gaussians > 0 && (positions == nullptr || factor == nullptr || density == nullptr || sigma_max == nullptr ||
                              points == nullptr || scale == nullptr || owner == nullptr))
        return fail(GF_ERR_BAD_INPUT, "NULL argument");
    if (count == nullptr || status == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL count or status");
    if (num_gaussians > 0xffffffffu / 9u) return fail(GF_ERR_CAPACITY, "too many Gaussians for 32-bit site indices");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GF_CUDA(cudaMemsetAsync(status, 0, sizeof(uint32_t), s));
    if (num_gaussians == 0) {
        GF_CUDA(cudaMemsetAsync(count, 0, sizeof(uint32_t), s));
        return GF_OK;
    }
    const uint32_t n = num_gaussians;
    // radius cap of the renderer's minimum kernel response, 0.0113 as float32
    const double radiusCap = std::sqrt(-2.0 * std::log(double(0.0113f)));
    DeviceBuffer keep, slot, tiles;
    if (int e = keep.ensure(sizeof(uint32_t) * n, s)) return e;
    if (int e = slot.ensure(sizeof(uint32_t) * n, s)) {
        keep.release();
        return e;
    }
    uint32_t launches = 0;
    int rc = GF_OK;
    k_site_flags<<<(n + 255) / 256, 256, 0, s>>>(density, n, keep.as<uint32_t>());
    if (cudaGetLastError() != cudaSuccess) rc = fail(GF_ERR_CUDA, "site flag launch failed");
    if (rc == GF_OK) rc = scan_exclusive<uint32_t, uint32_t>(tiles, launches, keep.as<uint32_t>(), n,
                                                             slot.as<uint32_t>(), count, s);
    if (rc == GF_OK) {
        k_sites<<<(n + 127) / 128, 128, 0, s>>>(positions, factor, density, sigma_max, n, keep.as<uint32_t>(),
                                                slot.as<uint32_t>(), radiusCap, points, scale, owner, status);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) rc = fail(GF_ERR_CUDA, "site launch failed: %s", cudaGetErrorString(e));
    }
    // stream-ordered frees: the kernels above finish before the memory is reused
    for (DeviceBuffer* b : {&keep, &slot, &tiles}) {
        if (b->ptr != nullptr) cudaFreeAsync(b->ptr, s);
        b->ptr = nullptr;
    }
    return rc;
}
