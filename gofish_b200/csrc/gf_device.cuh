// Device math of the fisheye tracer: camera projection, unscented transform,
// conic/extent, tile admission, sort-key depth, SH radiance and the
// ray/particle hit test.  Compiled with -fmad=false: every a*b+c below is
// two roundings unless written as fmaf_rn, so the integer outputs (tile
// counts, keys, hit counts) are reproducible on the CPU.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "gf_elementary.h"
#include "../../include/gofish_b200.h"

namespace gf {

// Renderer constants (reference configs/render/3dgut.yaml and
// include/3dgut/threedgut.cuh:41-78).
constexpr float kAlphaThreshold = 0.00392156862745098f;
constexpr float kMinKernelResponse = 0.0113f;
constexpr float kMaxAlpha = 0.99f;
constexpr float kMinTransmittance = 0.0001f;
constexpr float kCovarianceDilation = 0.3f;
constexpr float kParticleMinSensorZ = 0.2f;
constexpr float kMaxDepthValue = 3.4028235e+38f;
constexpr float kUtDelta = 1.7320508075688772f;
constexpr float kUtWeightI = 1.0f / 6.0f;
constexpr float kUtWeight0 = 2.0f;
constexpr float kAabbHalfExtent = 1e06f;
constexpr int kTile = 16;
constexpr int kTileThreads = kTile * kTile;
constexpr uint32_t kInvalidParticle = 0xffffffffu;
// exp(-g/2) < kMinKernelResponse for every g > kResponseCutoff2 (exp(-4.5) =
// 0.01111 < 0.0113), so such candidates are rejected without evaluating exp.
constexpr float kResponseCutoff2 = 9.0f;

// Prepared pose (host-computed, see gf_pose_prepare in gf_tracer.cu).
struct Pose {
    float R[9];     // world -> sensor, row-major
    float t[3];
    float Rinv[9];  // sensor -> world
    float c[3];     // sensor centre in the world
};

struct V3 {
    float x, y, z;
};
__device__ __forceinline__ V3 v3(float x, float y, float z) { return {x, y, z}; }
__device__ __forceinline__ V3 operator+(V3 a, V3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
__device__ __forceinline__ V3 operator-(V3 a, V3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
__device__ __forceinline__ V3 operator*(float s, V3 a) { return {s * a.x, s * a.y, s * a.z}; }
__device__ __forceinline__ float dot3(V3 a, V3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ V3 mat3(const float* m, V3 v) {
    return {m[0] * v.x + m[1] * v.y + m[2] * v.z, m[3] * v.x + m[4] * v.y + m[5] * v.z,
            m[6] * v.x + m[7] * v.y + m[8] * v.z};
}
// Fused forms used by the per-pixel hit test (identical on the CPU oracle).
__device__ __forceinline__ float fdot3(V3 a, V3 b) { return __fmaf_rn(a.z, b.z, __fmaf_rn(a.y, b.y, a.x * b.x)); }

__device__ __forceinline__ int f2i_sat(float f) { return __float2int_rz(f); }  // saturating, NaN -> 0
__device__ __forceinline__ float saturate_f(float x) { return __saturatef(x); }

// ---------------------------------------------------------------- camera
__device__ __forceinline__ float stable_norm2(float x, float y) {
    const float ax = fabsf(x), ay = fabsf(y);
    const float mn = fminf(ax, ay), mx = fmaxf(ax, ay);
    if (mx <= 0.0f) return 0.0f;
    const float r = mn / mx;
    return mx * __fsqrt_rn(1.0f + r * r);
}

__device__ __forceinline__ bool project_fisheye(const gf_camera& cam, V3 p, float& u, float& v) {
    float rho = stable_norm2(p.x, p.y);
    if (rho <= 0.0f) rho = 1.1920928955078125e-07f;  // FLT_EPSILON
    const float thetaFull = gf_atan2f(rho, p.z);
    const float theta = fminf(thetaFull, cam.max_angle);
    const float theta2 = theta * theta;
    float poly = cam.radial[3];
    poly = theta2 * poly + cam.radial[2];
    poly = theta2 * poly + cam.radial[1];
    poly = theta2 * poly + cam.radial[0];
    const float delta = (theta * (poly * theta2 + 1.0f)) / rho;
    u = cam.focal_length[0] * p.x * delta + cam.principal_point[0];
    v = cam.focal_length[1] * p.y * delta + cam.principal_point[1];
    return theta < cam.max_angle && isfinite_f(u) && isfinite_f(v);
}

__device__ __forceinline__ bool project_pinhole(const gf_camera& cam, V3 p, float& pu, float& pv) {
    if (p.z <= 0.0f) {
        pu = 0.0f;
        pv = 0.0f;
        return false;
    }
    const float u = p.x / p.z, v = p.y / p.z;
    const float uu = u * u, vv = v * v;
    const float r2 = uu + vv;
    const float a1 = 2.0f * u * v;
    const float a2 = r2 + 2.0f * uu;
    const float a3 = r2 + 2.0f * vv;
    const float* k = cam.radial;
    const float num = 1.0f + r2 * (k[0] + r2 * (k[1] + r2 * k[2]));
    const float den = 1.0f + r2 * (k[3] + r2 * (k[4] + r2 * k[5]));
    const float icD = num / den;
    const float* tg = cam.tangential;
    const float* tp = cam.thin_prism;
    const float dx = tg[0] * a1 + tg[1] * a2 + r2 * (tp[0] + r2 * tp[1]);
    const float dy = tg[0] * a3 + tg[1] * a1 + r2 * (tp[2] + r2 * tp[3]);
    const bool validRadial = icD > 0.8f && icD < 1.2f;
    if (validRadial) {
        pu = (icD * u + dx) * cam.focal_length[0] + cam.principal_point[0];
        pv = (icD * v + dy) * cam.focal_length[1] + cam.principal_point[1];
    } else {
        pu = 0.0f;  // an out-of-range distortion never yields a valid projection
        pv = 0.0f;
    }
    return validRadial && isfinite_f(pu) && isfinite_f(pv);
}

__device__ __forceinline__ bool project_world(const gf_camera& cam, const Pose& pose, V3 pw, float& u, float& v) {
    const V3 ps = mat3(pose.R, pw) + v3(pose.t[0], pose.t[1], pose.t[2]);
    if (cam.model == GF_CAMERA_OPENCV_FISHEYE) return project_fisheye(cam, ps, u, v);
    return project_pinhole(cam, ps, u, v);
}

// ---------------------------------------------------------------- UT + conic
struct Projected {
    float cx, cy;
    float conic0, conic1, conic2;
    float opacity;
    float ex, ey;
};

// partialScale2 > 0 enables the partial UT (gutProjector.cuh:470-499): with
// the mean projected and, on every axis, one of its two sigma points valid,
// each invalid point becomes the reflection 2 p0 - p of its mirror, the mean
// is re-accumulated over the repaired points in index order and the
// covariance is scaled by partialScale2.
__device__ __forceinline__ bool unscented_projection(const gf_camera& cam, const Pose& pose, V3 mu, float density,
                                                     const float* B, float& cx, float& cy, float cov[3],
                                                     float partialScale2 = 0.0f) {
    if (density < kAlphaThreshold) return false;
    const bool fisheye = cam.model == GF_CAMERA_OPENCV_FISHEYE;
    if (fisheye) {
        const V3 ray = mu - v3(pose.c[0], pose.c[1], pose.c[2]);
        const float r2 = dot3(ray, ray);
        if (!(isfinite_f(r2) && r2 >= kParticleMinSensorZ * kParticleMinSensorZ)) return false;
    } else {
        const float z = mu.x * pose.R[6] + mu.y * pose.R[7] + mu.z * pose.R[8] + pose.t[2];
        if (z < kParticleMinSensorZ) return false;
    }
    float su[7], sv[7];
    bool ok[7];
    int numValid = 0;
    const bool c0 = project_world(cam, pose, mu, su[0], sv[0]);
    if (fisheye && !c0) return false;
    numValid += c0 ? 1 : 0;
    cx = su[0] * 0.0f;
    cy = sv[0] * 0.0f;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const V3 delta = kUtDelta * v3(B[i], B[3 + i], B[6 + i]);
        ok[i + 1] = project_world(cam, pose, mu + delta, su[i + 1], sv[i + 1]);
        numValid += ok[i + 1] ? 1 : 0;
        cx = cx + kUtWeightI * su[i + 1];
        cy = cy + kUtWeightI * sv[i + 1];
        ok[i + 4] = project_world(cam, pose, mu - delta, su[i + 4], sv[i + 4]);
        numValid += ok[i + 4] ? 1 : 0;
        cx = cx + kUtWeightI * su[i + 4];
        cy = cy + kUtWeightI * sv[i + 4];
    }
    float covScale = 1.0f;
    if (numValid != 7) {
        if (!(partialScale2 > 0.0f) || !c0) return false;
#pragma unroll
        for (int i = 0; i < 3; ++i)
            if (!ok[i + 1] && !ok[i + 4]) return false;
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            if (!ok[i + 1]) {
                su[i + 1] = 2.0f * su[0] - su[i + 4];
                sv[i + 1] = 2.0f * sv[0] - sv[i + 4];
            }
            if (!ok[i + 4]) {
                su[i + 4] = 2.0f * su[0] - su[i + 1];
                sv[i + 4] = 2.0f * sv[0] - sv[i + 1];
            }
        }
        cx = su[0] * 0.0f;
        cy = sv[0] * 0.0f;
#pragma unroll
        for (int k = 1; k < 7; ++k) {
            cx = cx + kUtWeightI * su[k];
            cy = cy + kUtWeightI * sv[k];
        }
        covScale = partialScale2;
    }
    {
        const float dx = su[0] - cx, dy = sv[0] - cy;
        cov[0] = kUtWeight0 * (dx * dx);
        cov[1] = kUtWeight0 * (dx * dy);
        cov[2] = kUtWeight0 * (dy * dy);
    }
#pragma unroll
    for (int i = 0; i < 6; ++i) {
        const float dx = su[i + 1] - cx, dy = sv[i + 1] - cy;
        cov[0] = cov[0] + kUtWeightI * (dx * dx);
        cov[1] = cov[1] + kUtWeightI * (dx * dy);
        cov[2] = cov[2] + kUtWeightI * (dy * dy);
    }
    if (covScale != 1.0f) {
        cov[0] = cov[0] * covScale;
        cov[1] = cov[1] * covScale;
        cov[2] = cov[2] * covScale;
    }
    return true;
}

__device__ __forceinline__ bool conic_extent(const float cov[3], float opacity, Projected& p) {
    const float dx = cov[0] + kCovarianceDilation, dy = cov[1], dz = cov[2] + kCovarianceDilation;
    const float det = dx * dz - dy * dy;
    if (det == 0.0f) return false;
    p.conic0 = dz / det;
    p.conic1 = -dy / det;
    p.conic2 = dx / det;
    p.opacity = opacity;
    if (opacity < kAlphaThreshold) return false;
    const float maxPower = gf_logf(opacity / kAlphaThreshold);
    const float extentFactor = fminf(3.33f, __fsqrt_rn(2.0f * maxPower));
    const float mid = 0.5f * (dx + dz);
    const float lambda = mid + __fsqrt_rn(fmaxf(0.01f, mid * mid - det));
    const float radius = extentFactor * __fsqrt_rn(lambda);
    p.ex = fminf(extentFactor * __fsqrt_rn(dx), radius);
    p.ey = fminf(extentFactor * __fsqrt_rn(dz), radius);
    return radius > 0.0f;
}

__device__ __forceinline__ bool fast_ut_valid(const Projected& p) {
    return p.ex > 1e-06f && p.opacity >= kAlphaThreshold;
}

struct TileBox {
    int x0, y0, x1, y1;
};

__device__ __forceinline__ TileBox tile_bbox(int gx, int gy, float cx, float cy, float ex, float ey) {
    TileBox b;
    b.x0 = min(gx, max(0, f2i_sat(floorf(((cx - 0.5f) - ex) / 16.0f))));
    b.y0 = min(gy, max(0, f2i_sat(floorf(((cy - 0.5f) - ey) / 16.0f))));
    b.x1 = min(gx, max(0, f2i_sat(ceilf(((cx - 0.5f) + ex) / 16.0f))));
    b.y1 = min(gy, max(0, f2i_sat(ceilf(((cy - 0.5f) + ey) / 16.0f))));
    return b;
}

// Minimum of the projected conic's power over one 16x16 tile.
__device__ __forceinline__ float tile_min_power(int tx, int ty, const Projected& p) {
    const float tminx = 16.0f * float(tx), tminy = 16.0f * float(ty);
    const float tmaxx = 16.0f + tminx, tmaxy = 16.0f + tminy;
    const float ox = tminx - p.cx, oy = tminy - p.cy;
    const float lax = ox > 0.0f ? 1.0f : 0.0f, lay = oy > 0.0f ? 1.0f : 0.0f;
    const float nirx = lax + (p.cx > tmaxx ? 1.0f : 0.0f);
    const float niry = lay + (p.cy > tmaxy ? 1.0f : 0.0f);
    if ((nirx + niry) > 0.0f) {
        const float px = lax != 0.0f ? tminx : tmaxx;
        const float py = lay != 0.0f ? tminy : tmaxy;
        const float dxx = copysignf(16.0f, ox), dxy = copysignf(16.0f, oy);
        const float diffx = p.cx - px, diffy = p.cy - py;
        const float rcpx = __frcp_rn(256.0f * p.conic0);
        const float rcpy = __frcp_rn(256.0f * p.conic2);
        const float tx_ = niry * saturate_f((dxx * p.conic0 * diffx + dxx * p.conic1 * diffy) * rcpx);
        const float ty_ = nirx * saturate_f((dxy * p.conic1 * diffx + dxy * p.conic2 * diffy) * rcpy);
        const float mx = p.cx - (px + tx_ * dxx), my = p.cy - (py + ty_ * dxy);
        return 0.5f * (p.conic0 * mx * mx + p.conic2 * my * my) + p.conic1 * mx * my;
    }
    return 0.0f;
}

// ---------------------------------------------------------------- sort key depth
__device__ __forceinline__ float finite_nonneg(float v, float fallbackMax) {
    if (isfinite_f(v) && v >= 0.0f) return v;
    return (isfinite_f(fallbackMax) && fallbackMax >= 0.0f) ? fallbackMax : 0.0f;
}

// tileRay: float4 {origin.xyz, usable flag}, float4 {direction.xyz, 0}.
__device__ __forceinline__ uint32_t depth_key_per_tile(V3 mu, const float* Binv, float camRadial, float4 to,
                                                       float4 td) {
    const V3 wo = v3(to.x, to.y, to.z);
    const V3 u = mu - wo;
    const float tileRadial = finite_nonneg(__fsqrt_rn(dot3(u, u)), camRadial);
    if (to.w == 0.0f) return __float_as_uint(finite_nonneg(tileRadial, camRadial));
    const V3 wd = v3(td.x, td.y, td.z);
    const V3 co = mat3(Binv, wo - mu);
    const V3 cd = mat3(Binv, wd);
    const float den = dot3(cd, cd);
    if (!(den > 0.0f) || !isfinite_f(den)) return __float_as_uint(finite_nonneg(tileRadial, 0.0f));
    const float t = -dot3(co, cd) / den;
    if (!isfinite_f(t)) return __float_as_uint(finite_nonneg(tileRadial, 0.0f));
    return __float_as_uint(fmaxf(0.0f, t));
}

// ---------------------------------------------------------------- SH
constexpr float SH_C0 = 0.28209479177387814f;
constexpr float SH_C1 = 0.4886025119029199f;
constexpr float SH_C2_0 = 1.0925484305920792f, SH_C2_1 = -1.0925484305920792f, SH_C2_2 = 0.31539156525252005f,
                SH_C2_3 = -1.0925484305920792f, SH_C2_4 = 0.5462742152960396f;
constexpr float SH_C3_0 = -0.5900435899266435f, SH_C3_1 = 2.890611442640554f, SH_C3_2 = -0.4570457994644658f,
                SH_C3_3 = 0.3731763325901154f, SH_C3_4 = -0.4570457994644658f, SH_C3_5 = 1.445305721320277f,
                SH_C3_6 = -0.5900435899266435f;

__device__ __forceinline__ void sh_basis(int deg, V3 d, float b[16]) {
#pragma unroll
    for (int i = 0; i < 16; ++i) b[i] = 0.0f;
    b[0] = SH_C0;
    if (deg > 0) {
        const float x = d.x, y = d.y, z = d.z;
        b[1] = -SH_C1 * y;
        b[2] = SH_C1 * z;
        b[3] = -SH_C1 * x;
        if (deg > 1) {
            const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
            b[4] = SH_C2_0 * xy;
            b[5] = SH_C2_1 * yz;
            b[6] = SH_C2_2 * (2.0f * zz - xx - yy);
            b[7] = SH_C2_3 * xz;
            b[8] = SH_C2_4 * (xx - yy);
            if (deg > 2) {
                b[9] = SH_C3_0 * y * (3.0f * xx - yy);
                b[10] = SH_C3_1 * xy * z;
                b[11] = SH_C3_2 * y * (4.0f * zz - xx - yy);
                b[12] = SH_C3_3 * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
                b[13] = SH_C3_4 * x * (4.0f * zz - xx - yy);
                b[14] = SH_C3_5 * z * (xx - yy);
                b[15] = SH_C3_6 * x * (xx - 3.0f * yy);
            }
        }
    }
}

__device__ __forceinline__ void sh_basis_grad(int deg, V3 d, float gx[16], float gy[16], float gz[16]) {
#pragma unroll
    for (int i = 0; i < 16; ++i) gx[i] = gy[i] = gz[i] = 0.0f;
    if (deg < 1) return;
    const float x = d.x, y = d.y, z = d.z;
    gy[1] = -SH_C1;
    gz[2] = SH_C1;
    gx[3] = -SH_C1;
    if (deg < 2) return;
    gx[4] = SH_C2_0 * y; gy[4] = SH_C2_0 * x;
    gy[5] = SH_C2_1 * z; gz[5] = SH_C2_1 * y;
    gx[6] = SH_C2_2 * (-2.0f * x); gy[6] = SH_C2_2 * (-2.0f * y); gz[6] = SH_C2_2 * (4.0f * z);
    gx[7] = SH_C2_3 * z; gz[7] = SH_C2_3 * x;
    gx[8] = SH_C2_4 * (2.0f * x); gy[8] = SH_C2_4 * (-2.0f * y);
    if (deg < 3) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    gx[9] = SH_C3_0 * (6.0f * x * y); gy[9] = SH_C3_0 * (3.0f * xx - 3.0f * yy);
    gx[10] = SH_C3_1 * (y * z); gy[10] = SH_C3_1 * (x * z); gz[10] = SH_C3_1 * (x * y);
    gx[11] = SH_C3_2 * (-2.0f * x * y); gy[11] = SH_C3_2 * (4.0f * zz - xx - 3.0f * yy); gz[11] = SH_C3_2 * (8.0f * y * z);
    gx[12] = SH_C3_3 * (-6.0f * x * z); gy[12] = SH_C3_3 * (-6.0f * y * z);
    gz[12] = SH_C3_3 * (6.0f * zz - 3.0f * xx - 3.0f * yy);
    gx[13] = SH_C3_4 * (4.0f * zz - 3.0f * xx - yy); gy[13] = SH_C3_4 * (-2.0f * x * y); gz[13] = SH_C3_4 * (8.0f * x * z);
    gx[14] = SH_C3_5 * (2.0f * x * z); gy[14] = SH_C3_5 * (-2.0f * y * z); gz[14] = SH_C3_5 * (xx - yy);
    gx[15] = SH_C3_6 * (3.0f * xx - 3.0f * yy); gy[15] = SH_C3_6 * (-6.0f * x * y);
}

__device__ __forceinline__ int sh_count(int deg) { return deg >= 3 ? 16 : (deg == 2 ? 9 : (deg == 1 ? 4 : 1)); }

// ---------------------------------------------------------------- rays + hit test
struct Ray {
    V3 o, d;
    float tmin, tmax;
    bool valid;
};

__device__ __forceinline__ void swapf(float& a, float& b) {
    const float t = a;
    a = b;
    b = t;
}

__device__ __forceinline__ Ray make_ray(const Pose& pose, V3 os, V3 ds) {
    Ray r;
    r.o = mat3(pose.Rinv, os) + v3(pose.c[0], pose.c[1], pose.c[2]);
    r.d = mat3(pose.Rinv, ds);
    const float lo = -kAabbHalfExtent, hi = kAabbHalfExtent;
    float tmin = (lo - r.o.x) / r.d.x, tmax = (hi - r.o.x) / r.d.x;
    if (tmin > tmax) swapf(tmin, tmax);
    float tymin = (lo - r.o.y) / r.d.y, tymax = (hi - r.o.y) / r.d.y;
    if (tymin > tymax) swapf(tymin, tymax);
    if (tmin > tymax || tymin > tmax) {
        tmin = 3.402823466e+38f;
        tmax = 3.402823466e+38f;
    } else {
        if (tymin > tmin) tmin = tymin;
        if (tymax < tmax) tmax = tymax;
        float tzmin = (lo - r.o.z) / r.d.z, tzmax = (hi - r.o.z) / r.d.z;
        if (tzmin > tzmax) swapf(tzmin, tzmax);
        if (tmin > tzmax || tzmin > tmax) {
            tmin = 3.402823466e+38f;
            tmax = 3.402823466e+38f;
        } else {
            if (tzmin > tmin) tmin = tzmin;
            if (tzmax < tmax) tmax = tzmax;
        }
    }
    r.tmin = fmaxf(tmin, 0.0f);
    r.tmax = tmax;
    r.valid = r.tmax > r.tmin;
    return r;
}

// Particle render record (64 B): pos.xyz, density | Binv row0, row1.x | row1.yz, row2.xy | row2.z, rgb.
struct Record {
    float4 a, b, c, d;
};

struct HalfRay {
    V3 gro, grdu, p;
    float denom, num, tauLine, tau;
    bool interior, valid;
};

__device__ __forceinline__ HalfRay half_ray(const Ray& r, const Record& q) {
    HalfRay h;
    const V3 g = v3(r.o.x - q.a.x, r.o.y - q.a.y, r.o.z - q.a.z);
    h.gro = v3(__fmaf_rn(q.b.z, g.z, __fmaf_rn(q.b.y, g.y, q.b.x * g.x)),
               __fmaf_rn(q.c.y, g.z, __fmaf_rn(q.c.x, g.y, q.b.w * g.x)),
               __fmaf_rn(q.d.x, g.z, __fmaf_rn(q.c.w, g.y, q.c.z * g.x)));
    h.grdu = v3(__fmaf_rn(q.b.z, r.d.z, __fmaf_rn(q.b.y, r.d.y, q.b.x * r.d.x)),
                __fmaf_rn(q.c.y, r.d.z, __fmaf_rn(q.c.x, r.d.y, q.b.w * r.d.x)),
                __fmaf_rn(q.d.x, r.d.z, __fmaf_rn(q.c.w, r.d.y, q.c.z * r.d.x)));
    h.denom = fdot3(h.grdu, h.grdu);
    h.valid = h.denom > 0.0f && isfinite_f(h.denom) && isfinite_f(r.tmin) && r.tmax > r.tmin;
    if (!h.valid) {
        h.num = 0.0f;
        h.tauLine = 0.0f;
        h.tau = 0.0f;
        h.p = h.gro;
        h.interior = false;
        return h;
    }
    h.num = fdot3(h.gro, h.grdu);
    h.tauLine = -h.num / h.denom;
    h.tau = fminf(fmaxf(h.tauLine, r.tmin), r.tmax);
    h.interior = h.tauLine > r.tmin && h.tauLine < r.tmax;
    h.p = v3(__fmaf_rn(h.tau, h.grdu.x, h.gro.x), __fmaf_rn(h.tau, h.grdu.y, h.gro.y),
             __fmaf_rn(h.tau, h.grdu.z, h.gro.z));
    return h;
}

// Radius of a sphere around mu that contains the particle's 3-sigma ellipsoid
// {x : |B^-1 (x - mu)| <= 3}: 3 / sigma_min(B^-1), from the smallest
// eigenvalue of B^-T B^-1 (closed-form trigonometric solution, double
// precision), inflated by 1%.  Returns +inf when the bound is not reliable.
__device__ __forceinline__ float support_radius(const float* Binv) {
    double m[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) m[i] = double(Binv[i]);
    // S = M^T M
    double s00 = 0, s01 = 0, s02 = 0, s11 = 0, s12 = 0, s22 = 0;
#pragma unroll
    for (int r = 0; r < 3; ++r) {
        const double a = m[3 * r], b = m[3 * r + 1], c = m[3 * r + 2];
        s00 += a * a; s01 += a * b; s02 += a * c; s11 += b * b; s12 += b * c; s22 += c * c;
    }
    const double q = (s00 + s11 + s22) / 3.0;
    const double p1 = s01 * s01 + s02 * s02 + s12 * s12;
    const double p2 = (s00 - q) * (s00 - q) + (s11 - q) * (s11 - q) + (s22 - q) * (s22 - q) + 2.0 * p1;
    double lmin, lmax;
    if (p2 <= 1e-30 * q * q) {
        lmin = lmax = q;
    } else {
        const double pp = sqrt(p2 / 6.0);
        const double b00 = (s00 - q) / pp, b11 = (s11 - q) / pp, b22 = (s22 - q) / pp;
        const double b01 = s01 / pp, b02 = s02 / pp, b12 = s12 / pp;
        const double det = b00 * (b11 * b22 - b12 * b12) - b01 * (b01 * b22 - b12 * b02) + b02 * (b01 * b12 - b11 * b02);
        const double r = fmin(1.0, fmax(-1.0, 0.5 * det));
        const double phi = acos(r) / 3.0;
        lmax = q + 2.0 * pp * cos(phi);
        lmin = q + 2.0 * pp * cos(phi + 2.0943951023931957);  // + 2 pi / 3
    }
    if (!(lmin > 1e-9 * lmax) || !(lmax < 1e300)) return __int_as_float(0x7f800000);
    return float(3.03 / sqrt(lmin)) * 1.0001f + 1e-6f;
}

}  // namespace gf
