// Physical-mip 3-D filter search on sm_100a (reference
// threedgrut/physical_mip_csrc/fused_refresh_cuda.cu:40-219 best_rate_kernel,
// camera_local_validity.cuh, bindings.cpp:34-101).
//
// For every point, over every training frame whose calibrated support holds
// the projected point, the sampling rate is the smallest singular value of
// the 2x3 world pixel Jacobian; the finest rate wins, ties going to the
// smallest frame rank.  Double precision throughout, no contraction
// (-fmad=false), IEEE division and square root, atan2/hypot from
// gf_elementary.h (shared with the oracle, so results are bit-identical).
//
// Layout: one thread per point; the frame table (rotation, centre, camera,
// index, rank: 112 B per frame) is staged through shared memory in chunks of
// kFrameChunk frames, and the camera table (model, raster, 12 parameters,
// angular cap) sits in shared memory for the whole launch.  Every thread of
// a block reads the same frame record at the same time (broadcast), so the
// loop is FP64-issue bound.
#include <cuda_runtime.h>

#include <cfloat>
#include <climits>
#include <cstdint>

#include "../../include/gofish_b200.h"
#include "gf_elementary.h"

int gf_record_error(int code, const char* message);

namespace {

constexpr int kThreads = 128;
constexpr int kFrameChunk = 128;
constexpr int kMaxCameras = 64;
constexpr int kParams = 12;
constexpr double kCenterEps = 1.0e-12;  // fused_refresh_cuda.cu:22
constexpr double kNear = 0.2;           // camera_local_validity.cuh:15

struct FrameRecord {
    double R[9];  // camera-to-world rotation, row-major
    double c[3];  // camera centre
    int32_t camera, index;
    int64_t rank;
};

struct CameraRecord {
    double P[kParams];
    double maxAngle;
    int32_t model, width, height, pad;
};

struct Projection {
    double u, v, J[6];
    bool ok;
};

__device__ __forceinline__ Projection project_pinhole(const double* P, double x, double y, double z) {
    Projection o{};
    const double fx = P[0], fy = P[1], cx = P[2], cy = P[3];
    const double zs = fabs(z) > DBL_MIN ? z : 1.0;
    o.u = fx * x / zs + cx;
    o.v = fy * y / zs + cy;
    o.J[0] = fx / zs;
    o.J[2] = -fx * x / (zs * zs);
    o.J[4] = fy / zs;
    o.J[5] = -fy * y / (zs * zs);
    o.ok = z > 0.0;
    return o;
}

__device__ __forceinline__ Projection project_radial(int model, const double* P, double x, double y, double z) {
    Projection o{};
    const double fx = P[0], fy = P[1], cx = P[2], cy = P[3], k1 = P[4];
    const double k2 = model >= 4 ? P[5] : 0.0;
    const double p1 = model >= 5 ? P[6] : 0.0;
    const double p2 = model >= 5 ? P[7] : 0.0;
    const double k3 = model == 6 ? P[8] : 0.0;
    const double k4 = model == 6 ? P[9] : 0.0;
    const double k5 = model == 6 ? P[10] : 0.0;
    const double k6 = model == 6 ? P[11] : 0.0;
    const double zs = fabs(z) > DBL_MIN ? z : 1.0;
    const double a = x / zs, b = y / zs;
    const double r2 = a * a + b * b;
    const double r4 = r2 * r2, r6 = r4 * r2;
    const double num = 1.0 + k1 * r2 + k2 * r4 + k3 * r6;
    const double den = 1.0 + k4 * r2 + k5 * r4 + k6 * r6;
    const double dens = fabs(den) > DBL_MIN ? den : 1.0;
    const double g = num / dens;
    const double gp = ((k1 + 2.0 * k2 * r2 + 3.0 * k3 * r4) * dens - num * (k4 + 2.0 * k5 * r2 + 3.0 * k6 * r4)) /
                      (dens * dens);
    const double xd = a * g + 2.0 * p1 * a * b + p2 * (r2 + 2.0 * a * a);
    const double yd = b * g + p1 * (r2 + 2.0 * b * b) + 2.0 * p2 * a * b;
    o.u = fx * xd + cx;
    o.v = fy * yd + cy;
    const double xa = g + 2.0 * a * a * gp + 2.0 * p1 * b + 6.0 * p2 * a;
    const double xb = 2.0 * a * b * gp + 2.0 * p1 * a + 2.0 * p2 * b;
    const double ya = 2.0 * a * b * gp + 2.0 * p1 * a + 2.0 * p2 * b;
    const double yb = g + 2.0 * b * b * gp + 6.0 * p1 * b + 2.0 * p2 * a;
    const double iz = 1.0 / zs;
    o.J[0] = fx * xa * iz;
    o.J[1] = fx * xb * iz;
    o.J[2] = -fx * (xa * a + xb * b) * iz;
    o.J[3] = fy * ya * iz;
    o.J[4] = fy * yb * iz;
    o.J[5] = -fy * (ya * a + yb * b) * iz;
    o.ok = z > 0.0 && fabs(den) > DBL_MIN;
    return o;
}

__device__ __forceinline__ Projection project_fisheye(const double* P, double x, double y, double z, double dist,
                                                      double rho, double theta) {
    Projection o{};
    const double fx = P[0], fy = P[1], cx = P[2], cy = P[3];
    const double k1 = P[4], k2 = P[5], k3 = P[6], k4 = P[7];
    const double t2 = theta * theta;
    const double q = theta * (1.0 + t2 * (k1 + t2 * (k2 + t2 * (k3 + t2 * k4))));
    const double dq = 1.0 + t2 * (3.0 * k1 + t2 * (5.0 * k2 + t2 * (7.0 * k3 + t2 * 9.0 * k4)));
    const double rs = fmax(rho, sqrt(DBL_MIN));
    const double d2 = fmax(dist * dist, DBL_MIN);
    const double c = x / rs, s = y / rs;
    o.u = fx * q * c + cx;
    o.v = fy * q * s + cy;
    const double dth[3] = {z * x / (rs * d2), z * y / (rs * d2), -rho / d2};
    const double dph[3] = {-y / (rs * rs), x / (rs * rs), 0.0};
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        o.J[k] = fx * (dq * c * dth[k] - q * s * dph[k]);
        o.J[3 + k] = fy * (dq * s * dth[k] + q * c * dph[k]);
    }
    if (rho <= kCenterEps && z > 0.0) {
        o.u = cx;
        o.v = cy;
#pragma unroll
        for (int k = 0; k < 6; ++k) o.J[k] = 0.0;
        o.J[0] = fx / dist;
        o.J[4] = fy / dist;
    }
    o.ok = (rho > kCenterEps || z > 0.0) && dq > 0.0;
    return o;
}

struct MipArgs {
    const double* positions;
    int64_t N;
    const double* rotations;
    const double* centers;
    const int32_t* frameCamera;
    const int32_t* frameIndex;
    const int64_t* frameRank;
    int64_t F;
    const int32_t* cameraModel;
    const int32_t* cameraWidth;
    const int32_t* cameraHeight;
    const double* cameraParams;
    const double* cameraMaxAngle;
    int32_t C;
    const int32_t* rowLo;
    const int32_t* rowHi;
    int64_t rowStride;
    double* best;
    int32_t* owner;
    uint8_t* observed;
    double* direction;
};

__global__ __launch_bounds__(kThreads) void k_mip_best_rate(MipArgs a) {
    __shared__ FrameRecord sFrames[kFrameChunk];
    __shared__ CameraRecord sCams[kMaxCameras];
    for (int c = threadIdx.x; c < a.C; c += kThreads) {
        for (int k = 0; k < kParams; ++k) sCams[c].P[k] = a.cameraParams[kParams * c + k];
        sCams[c].maxAngle = a.cameraMaxAngle[c];
        sCams[c].model = a.cameraModel[c];
        sCams[c].width = a.cameraWidth[c];
        sCams[c].height = a.cameraHeight[c];
    }
    const int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x;
    const bool live = i < a.N;
    const double px = live ? a.positions[3 * i] : 0.0, py = live ? a.positions[3 * i + 1] : 0.0,
                 pz = live ? a.positions[3 * i + 2] : 0.0;
    double bestRate = 0.0, bx = 0.0, by = 0.0, bz = 0.0;
    int64_t bestRank = LLONG_MAX;
    int32_t bestFrame = -1;
    for (int64_t base = 0; base < a.F; base += kFrameChunk) {
        __syncthreads();
        for (int k = threadIdx.x; k < kFrameChunk && base + k < a.F; k += kThreads) {
            const int64_t f = base + k;
            for (int e = 0; e < 9; ++e) sFrames[k].R[e] = a.rotations[9 * f + e];
            for (int e = 0; e < 3; ++e) sFrames[k].c[e] = a.centers[3 * f + e];
            sFrames[k].camera = a.frameCamera[f];
            sFrames[k].index = a.frameIndex[f];
            sFrames[k].rank = a.frameRank[f];
        }
        __syncthreads();
        if (!live) continue;
        const int n = int(min(int64_t(kFrameChunk), a.F - base));
        for (int k = 0; k < n; ++k) {
            const FrameRecord& fr = sFrames[k];
            if (fr.camera < 0 || fr.camera >= a.C) continue;  // malformed table: never read past it
            const CameraRecord& cr = sCams[fr.camera];
            const double* R = fr.R;
            const double dx = px - fr.c[0], dy = py - fr.c[1], dz = pz - fr.c[2];
            const double x = dx * R[0] + dy * R[3] + dz * R[6];
            const double y = dx * R[1] + dy * R[4] + dz * R[7];
            const double z = dx * R[2] + dy * R[5] + dz * R[8];
            const double dist = sqrt(x * x + y * y + z * z);
            const double rho = gf::gf_hypotd(x, y);
            const double theta = gf::gf_atan2d(rho, z);
            const int model = cr.model;
            Projection pr;
            if (model == 0 || model == 1) pr = project_pinhole(cr.P, x, y, z);
            else if (model >= 3 && model <= 6) pr = project_radial(model, cr.P, x, y, z);
            else if (model == 2) pr = project_fisheye(cr.P, x, y, z, dist, rho, theta);
            else continue;
            const double local = model == 2 ? dist : z;
            bool ok = local > kNear && pr.ok;
#pragma unroll
            for (int e = 0; e < 6; ++e) ok = ok && gf::isfinite_d(pr.J[e]);
            ok = ok && gf::isfinite_d(pr.u) && gf::isfinite_d(pr.v);
            ok = ok && pr.u >= 0.0 && pr.u < cr.width && pr.v >= 0.0 && pr.v < cr.height;
            if (cr.maxAngle >= 0.0) ok = ok && theta < cr.maxAngle;
            if (ok) {
                const int64_t ix = int64_t(floor(pr.u)), iy = int64_t(floor(pr.v));
                ok = iy >= 0 && iy < cr.height && iy < a.rowStride && ix >= a.rowLo[fr.camera * a.rowStride + iy] &&
                     ix < a.rowHi[fr.camera * a.rowStride + iy];
            }
            if (!ok) continue;
            double w0[3], w1[3];
#pragma unroll
            for (int e = 0; e < 3; ++e) {
                w0[e] = pr.J[0] * R[3 * e] + pr.J[1] * R[3 * e + 1] + pr.J[2] * R[3 * e + 2];
                w1[e] = pr.J[3] * R[3 * e] + pr.J[4] * R[3 * e + 1] + pr.J[5] * R[3 * e + 2];
            }
            const double qa = w0[0] * w0[0] + w0[1] * w0[1] + w0[2] * w0[2];
            const double qb = w0[0] * w1[0] + w0[1] * w1[1] + w0[2] * w1[2];
            const double qc = w1[0] * w1[0] + w1[1] * w1[1] + w1[2] * w1[2];
            const double lmax = 0.5 * (qa + qc + gf::gf_hypotd(qa - qc, 2.0 * qb));
            const double lmin = (qa * qc - qb * qb) / lmax;
            if (!gf::isfinite_d(lmax) || !gf::isfinite_d(lmin) || !(lmax > 0.0) || !(lmin > 0.0)) continue;
            const double rate = sqrt(lmin);
            if (rate > bestRate || (rate == bestRate && fr.rank < bestRank)) {
                bestRate = rate;
                bestRank = fr.rank;
                bestFrame = fr.index;
                bx = dx;
                by = dy;
                bz = dz;
            }
        }
    }
    if (!live) return;
    a.best[i] = bestRate;
    a.owner[i] = bestFrame;
    a.observed[i] = bestFrame >= 0 ? 1u : 0u;
    if (bestFrame >= 0) {
        const double n = sqrt(bx * bx + by * by + bz * bz);
        a.direction[3 * i] = bx / n;
        a.direction[3 * i + 1] = by / n;
        a.direction[3 * i + 2] = bz / n;
    } else {
        a.direction[3 * i] = 0.0;
        a.direction[3 * i + 1] = 0.0;
        a.direction[3 * i + 2] = 0.0;
    }
}

}  // namespace

extern "C" int gf_mip_best_rate(const double* positions, int64_t num_points, const double* rotations,
                                const double* centers, const int32_t* frame_camera, const int32_t* frame_index,
                                const int64_t* frame_rank, int64_t num_frames, const int32_t* camera_model,
                                const int32_t* camera_width, const int32_t* camera_height,
                                const double* camera_params, const double* camera_max_angle, int32_t num_cameras,
                                const int32_t* row_lo, const int32_t* row_hi, int64_t row_stride, double* best_rate,
                                int32_t* owner, uint8_t* observed, double* direction, void* stream) {
    if (num_points <= 0 || num_frames <= 0)
        return gf_record_error(GF_ERR_BAD_INPUT, "point and frame inventories must be nonempty");
    if (num_cameras <= 0 || num_cameras > kMaxCameras)
        return gf_record_error(GF_ERR_CAPACITY, "between 1 and 64 cameras are supported");
    if (row_stride <= 0) return gf_record_error(GF_ERR_BAD_INPUT, "row-run stride must be positive");
    if (positions == nullptr || rotations == nullptr || centers == nullptr || frame_camera == nullptr ||
        frame_index == nullptr || frame_rank == nullptr || camera_model == nullptr || camera_width == nullptr ||
        camera_height == nullptr || camera_params == nullptr || camera_max_angle == nullptr || row_lo == nullptr ||
        row_hi == nullptr || best_rate == nullptr || owner == nullptr || observed == nullptr || direction == nullptr)
        return gf_record_error(GF_ERR_BAD_INPUT, "buffers must not be NULL");
    MipArgs a{positions,     num_points,   rotations,    centers,    frame_camera,     frame_index, frame_rank,
              num_frames,    camera_model, camera_width, camera_height, camera_params, camera_max_angle,
              num_cameras,   row_lo,       row_hi,       row_stride, best_rate,        owner,       observed,
              direction};
    const int64_t blocks = (num_points + kThreads - 1) / kThreads;
    if (blocks > 0x7fffffffll) return gf_record_error(GF_ERR_CAPACITY, "too many points");
    k_mip_best_rate<<<unsigned(blocks), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return gf_record_error(GF_ERR_CUDA, cudaGetErrorString(e));
    return GF_OK;
}
