// SOF's exact-crossing opacity field and its gradient on sm_100a (reference
// gutRenderer.cuh:297-430 sofExactCrossingOpacityForward / Backward,
// particleSofIntrinsicOpacitySample / Vjp in gaussianParticles.cuh:496-588).
//
// For each valid ray, rho* is the exact depth where the composited opacity
// crosses 1/2 (the quantile channel's crossing, 0 when there is none); the
// field replays the tile's candidates on [tmin, min(rho*, tmax)] (the whole
// ray without a crossing) with the intrinsic Gaussian of each candidate --
// rotation, physical scale and peak opacity of the packed row (slots 4-11),
// not the per-view footprint of image formation: p = s^-1 (R^T (w - mu)) at
// the segment's closest point, alpha = min(0.99, rho exp(-|p|^2 / 2)),
// accepted when the response exceeds 0.0113 and alpha exceeds 1/255; the
// field is 1 - prod(1 - alpha) over the accepted candidates in list order.
// The backward differentiates the product through each accepted alpha, with
// the segment end and the closest-point parameter detached: dO/dalpha_i is
// the product of the other factors (the full product over max(1 - alpha_i,
// 0.01)), and the gradient reaches the position, the quaternion, the scale
// and the intrinsic density.
//
// One CTA per tile, one thread per pixel; the tile's candidates are staged
// 256 at a time as (mean, intrinsic density), the rows of R^T and 1/s
// (64 bytes), so each pixel's loop reads shared memory only.  All threads
// walk every candidate in step, so the gradient merge of a candidate is the
// warp-uniform reduce-scatter of accumulate_grad.
#pragma once

#include "gf_render.cuh"

namespace gf {

struct SofIntrinsic {
    float4 mu;      // mean, intrinsic density
    float4 r0, r1;  // rows of R^T (xyz), 1/s (w of r0, r1, r2)
    float4 r2;
};

// Rows of R^T from the quaternion (w, x, y, z), as rotate_transpose, and 1/s.
__device__ __forceinline__ SofIntrinsic sof_intrinsic(const float* __restrict__ row) {
    const float4 p = __ldg(reinterpret_cast<const float4*>(row));
    const float4 q = __ldg(reinterpret_cast<const float4*>(row + 4));
    const float4 sc = __ldg(reinterpret_cast<const float4*>(row + 8));
    const float r = q.x, x = q.y, y = q.z, z = q.w;
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z, rx = r * x, ry = r * y,
                rz = r * z;
    SofIntrinsic out;
    out.mu = make_float4(p.x, p.y, p.z, sc.w);
    out.r0 = make_float4(1.0f - 2.0f * (yy + zz), 2.0f * (xy + rz), 2.0f * (xz - ry), 1.0f / sc.x);
    out.r1 = make_float4(2.0f * (xy - rz), 1.0f - 2.0f * (xx + zz), 2.0f * (yz + rx), 1.0f / sc.y);
    out.r2 = make_float4(2.0f * (xz + ry), 2.0f * (yz - rx), 1.0f - 2.0f * (xx + yy), 1.0f / sc.z);
    return out;
}

struct SofSample {
    bool accepted;
    float alpha, response, argument, depth;
    V3 p;
};

// s^-1 (R^T v)
__device__ __forceinline__ V3 sof_local(const SofIntrinsic& g, V3 v) {
    return v3(fdot3(v3(g.r0.x, g.r0.y, g.r0.z), v) * g.r0.w, fdot3(v3(g.r1.x, g.r1.y, g.r1.z), v) * g.r1.w,
              fdot3(v3(g.r2.x, g.r2.y, g.r2.z), v) * g.r2.w);
}

__device__ __forceinline__ SofSample sof_sample(const SofIntrinsic& g, const Ray& ray, float tmin, float tmax) {
    SofSample s{};
    s.accepted = false;
    if (!(tmax >= tmin)) return s;
    const V3 gro = sof_local(g, v3(ray.o.x - g.mu.x, ray.o.y - g.mu.y, ray.o.z - g.mu.z));
    const V3 grdu = sof_local(g, ray.d);
    float tau;
    if (tmax == tmin) {
        tau = tmin;
    } else {
        const float denom = fdot3(grdu, grdu);
        if (!(denom > 0.0f && isfinite_f(denom) && isfinite_f(tmin))) return s;
        const float tauLine = -fdot3(gro, grdu) / denom;
        tau = fminf(fmaxf(tauLine, tmin), tmax);
    }
    s.depth = tau;
    s.p = v3(__fmaf_rn(tau, grdu.x, gro.x), __fmaf_rn(tau, grdu.y, gro.y), __fmaf_rn(tau, grdu.z, gro.z));
    s.argument = fmaxf(fdot3(s.p, s.p), 0.0f);
    s.response = gf_expf(-0.5f * s.argument);
    s.alpha = fminf(kMaxAlpha, s.response * g.mu.w);
    s.accepted = s.response > kMinKernelResponse && s.alpha > kAlphaThreshold;
    return s;
}

// The replay segment's end: min(rho*, tmax) with a crossing, tmax without.
__device__ __forceinline__ float sof_replay_end(const float* __restrict__ quant, size_t pix, const Ray& ray) {
    const float rho = quant[size_t(kQuantStride) * pix + kQuantiles + 1];
    return (rho > 0.0f && isfinite_f(rho)) ? fminf(rho, ray.tmax) : ray.tmax;
}

struct SofOpacityArgs {
    FrameArgs f;
    const uint8_t* mask;
    const uint2* ranges;
    const uint32_t* sortedIds;
    const float* particles;  // packed [N,32] rows
    const float* rayO;
    const float* rayD;
    const float* quant;
    float* opacity;           // forward output
    const float* opacityIn;   // backward: forward value
    const float* gradOpacity; // backward: dL/dO
    float4* gradIntrinsic;    // backward: [N,4] float4: pos.xyz, intrinsic density | quat wxyz | scale.xyz, 0 | 0
};

template <bool kBackward>
__global__ __launch_bounds__(kTileThreads) void k_sof_opacity(SofOpacityArgs a) {
    __shared__ SofIntrinsic sG[kTileThreads];
    if (a.mask[blockIdx.x] == 0u) return;  // block-uniform
    const FrameArgs& f = a.f;
    const uint32_t tile = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int px = int(tile % uint32_t(f.gx)) * kTile + (warp & 1) * 8 + (lane & 7);
    const int py = int(tile / uint32_t(f.gx)) * kTile + (warp >> 1) * 4 + (lane >> 3);
    const bool inImage = px < f.W && py < f.H;
    const size_t pix = size_t(px) + size_t(f.W) * size_t(py);
    Ray ray;
    ray.valid = false;
    ray.o = v3(0.0f, 0.0f, 0.0f);
    ray.d = v3(0.0f, 0.0f, 1.0f);
    ray.tmin = ray.tmax = 0.0f;
    if (inImage)
        ray = make_ray(f.pose, v3(a.rayO[3 * pix], a.rayO[3 * pix + 1], a.rayO[3 * pix + 2]),
                       v3(a.rayD[3 * pix], a.rayD[3 * pix + 1], a.rayD[3 * pix + 2]));
    bool active = ray.valid;
    float end = 0.0f;
    if (active) {
        end = sof_replay_end(a.quant, pix, ray);
        if (!(end >= ray.tmin)) {
            if constexpr (!kBackward) a.opacity[pix] = 0.0f;
            active = false;
        }
    }
    float upstream = 0.0f, full = 0.0f;
    if constexpr (kBackward) {
        if (active) {
            upstream = a.gradOpacity[pix];
            full = fminf(fmaxf(1.0f - a.opacityIn[pix], 0.0f), 1.0f);
            if (upstream == 0.0f) active = false;
        }
        if (__syncthreads_and(!active)) return;
    }
    const uint2 range = a.ranges[tile];
    float product = 1.0f;
    for (uint32_t base = range.x; base < range.y; base += kTileThreads) {
        const uint32_t s = base + threadIdx.x;
        __syncthreads();
        if (s < range.y) sG[threadIdx.x] = sof_intrinsic(a.particles + 32 * size_t(__ldg(a.sortedIds + s)));
        __syncthreads();
        const int cnt = int(min(uint32_t(kTileThreads), range.y - base));
        for (int j = 0; j < cnt; ++j) {
            const SofIntrinsic& g = sG[j];
            if constexpr (!kBackward) {
                if (active) {
                    const SofSample smp = sof_sample(g, ray, ray.tmin, end);
                    if (smp.accepted) product = product * (1.0f - smp.alpha);
                }
            } else {
                bool have = false;
                float4 gr[4] = {};
                uint32_t idx = kInvalidParticle;
                if (active) {
                    const SofSample smp = sof_sample(g, ray, ray.tmin, end);
                    if (smp.accepted) {
                        idx = __ldg(a.sortedIds + base + uint32_t(j));
                        const float exclusive = fminf(fmaxf(full / fmaxf(1.0f - smp.alpha, 1.0f - kMaxAlpha), 0.0f), 1.0f);
                        const float dAlpha = upstream * exclusive;
                        const float cap = smp.response * g.mu.w < kMaxAlpha ? 1.0f : 0.0f;
                        const float gDensity = cap * dAlpha * smp.response;
                        const float dResp = cap * dAlpha * g.mu.w;
                        const float dArg = dResp * (-0.5f * smp.response);
                        const V3 lpg = v3(2.0f * dArg * smp.p.x, 2.0f * dArg * smp.p.y, 2.0f * dArg * smp.p.z);
                        const V3 rpg = v3(g.r0.w * lpg.x, g.r1.w * lpg.y, g.r2.w * lpg.z);
                        const V3 w = v3(__fmaf_rn(smp.depth, ray.d.x, ray.o.x) - g.mu.x,
                                        __fmaf_rn(smp.depth, ray.d.y, ray.o.y) - g.mu.y,
                                        __fmaf_rn(smp.depth, ray.d.z, ray.o.z) - g.mu.z);
                        const V3 rot = v3(fdot3(v3(g.r0.x, g.r0.y, g.r0.z), w), fdot3(v3(g.r1.x, g.r1.y, g.r1.z), w),
                                          fdot3(v3(g.r2.x, g.r2.y, g.r2.z), w));
                        // position: -R rpg (columns of R are the rows of R^T)
                        const V3 gp = v3(-(g.r0.x * rpg.x + g.r1.x * rpg.y + g.r2.x * rpg.z),
                                         -(g.r0.y * rpg.x + g.r1.y * rpg.y + g.r2.y * rpg.z),
                                         -(g.r0.z * rpg.x + g.r1.z * rpg.y + g.r2.z * rpg.z));
                        // scale: d(p_k)/d(s_k) = -rot_k / s_k^2
                        const V3 gs = v3(-rot.x * g.r0.w * g.r0.w * lpg.x, -rot.y * g.r1.w * g.r1.w * lpg.y,
                                         -rot.z * g.r2.w * g.r2.w * lpg.z);
                        const float* row = a.particles + 32 * size_t(idx);
                        const float4 gq = rotate_transpose_vjp(__ldg(reinterpret_cast<const float4*>(row + 4)), w, rpg);
                        gr[0] = make_float4(gp.x, gp.y, gp.z, gDensity);
                        gr[1] = gq;
                        gr[2] = make_float4(gs.x, gs.y, gs.z, 0.0f);
                        have = true;
                    }
                }
                accumulate_grad(a.gradIntrinsic, have, idx, gr);
            }
        }
    }
    if constexpr (!kBackward) {
        if (active) a.opacity[pix] = 1.0f - product;
    }
}

}  // namespace gf
