// Kernels of the fisheye tracer forward and backward passes.
#pragma once

#include "gf_device.cuh"

namespace gf {

struct FrameArgs {
    gf_camera cam;
    Pose pose;
    int W, H;
    int gx, gy;  // tile grid
    uint32_t N;
    int shDegree;
    uint32_t shCoeffs;
    int keyMode;
};

// ------------------------------------------------------------ per-tile rays
// Central ray of each tile for the per-tile depth key: the mean of the four
// pixel rays around the tile centre, in the world frame, normalized twice
// (reference gutProjector.cuh:364-409).
__global__ void k_tile_rays(FrameArgs f, const float* __restrict__ rayO, const float* __restrict__ rayD,
                            float4* __restrict__ tileRays) {
    const int tile = blockIdx.x * blockDim.x + threadIdx.x;
    if (tile >= f.gx * f.gy) return;
    const int tx = tile % f.gx, ty = tile / f.gx;
    const int xb = tx * kTile, yb = ty * kTile;
    const int xe = min(f.W - 1, (tx + 1) * kTile - 1), ye = min(f.H - 1, (ty + 1) * kTile - 1);
    const int xlo = (xb + xe) / 2, xhi = (xb + xe + 1) / 2, ylo = (yb + ye) / 2, yhi = (yb + ye + 1) / 2;
    const size_t p[4] = {size_t(xlo) + size_t(f.W) * ylo, size_t(xhi) + size_t(f.W) * ylo,
                         size_t(xlo) + size_t(f.W) * yhi, size_t(xhi) + size_t(f.W) * yhi};
    V3 so = v3(0.0f, 0.0f, 0.0f), sd = v3(0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        so = so + v3(rayO[3 * p[k]], rayO[3 * p[k] + 1], rayO[3 * p[k] + 2]);
        sd = sd + v3(rayD[3 * p[k]], rayD[3 * p[k] + 1], rayD[3 * p[k] + 2]);
    }
    so = 0.25f * so;
    sd = 0.25f * sd;
    const V3 wo = mat3(f.pose.Rinv, so) + v3(f.pose.c[0], f.pose.c[1], f.pose.c[2]);
    float4 o = make_float4(wo.x, wo.y, wo.z, 0.0f);
    float4 d = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float n2 = dot3(sd, sd);
    if (n2 > 0.0f && isfinite_f(n2)) {
        sd = __frcp_rn(__fsqrt_rn(n2)) * sd;
        V3 wd = mat3(f.pose.Rinv, sd);
        const float m2 = dot3(wd, wd);
        if (m2 > 0.0f && isfinite_f(m2)) {
            wd = __frcp_rn(__fsqrt_rn(m2)) * wd;
            o.w = 1.0f;
            d = make_float4(wd.x, wd.y, wd.z, 0.0f);
        }
    }
    tileRays[2 * tile] = o;
    tileRays[2 * tile + 1] = d;
}

// ------------------------------------------------------------ projection
__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Number of admitted tiles of one projected particle (fast UT admission,
// reference gutProjector.cuh:186-210); visit(x, y, k) is called in y-major order.
template <typename Visit>
__device__ __forceinline__ uint32_t for_admitted_tiles(const FrameArgs& f, const uint8_t* __restrict__ mask,
                                                       const Projected& p, Visit&& visit) {
    if (!fast_ut_valid(p)) return 0u;
    const TileBox b = tile_bbox(f.gx, f.gy, p.cx, p.cy, p.ex, p.ey);
    const float maxPower = gf_logf(p.opacity / kAlphaThreshold) * 1.0f;
    uint32_t n = 0;
    for (int y = b.y0; y < b.y1; ++y) {
        for (int x = b.x0; x < b.x1; ++x) {
            if (mask[y * f.gx + x] == 0u) continue;
            if (!(tile_min_power(x, y, p) < maxPower)) continue;
            visit(x, y, n);
            ++n;
        }
    }
    return n;
}

// One thread per particle: UT projection, conic, admitted-tile count, SH
// radiance, and the 64-byte render record (reference projectOnTiles,
// gutProjector.cuh:653-945).
__global__ __launch_bounds__(256) void k_project(FrameArgs f, const float* __restrict__ particles,
                                                 const float* __restrict__ features,
                                                 const uint8_t* __restrict__ mask, float4* __restrict__ proj,
                                                 float4* __restrict__ records, uint32_t* __restrict__ counts,
                                                 uint32_t* __restrict__ visibility, float* __restrict__ bounds) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= f.N) return;
    const float* row = particles + 32 * size_t(i);
    const float4 r0 = ldg4(row + 0);    // pos.xyz, density
    const float4 r3 = ldg4(row + 12);   // B00 B01 B02 B10
    const float4 r4 = ldg4(row + 16);   // B11 B12 B20 B21
    const float4 r5 = ldg4(row + 20);   // B22 | Binv00 Binv01 Binv02
    const float4 r6 = ldg4(row + 24);   // Binv10 Binv11 Binv12 Binv20
    const float4 r7 = ldg4(row + 28);   // Binv21 Binv22 pad pad
    const V3 mu = v3(r0.x, r0.y, r0.z);
    const float density = r0.w;
    const float B[9] = {r3.x, r3.y, r3.z, r3.w, r4.x, r4.y, r4.z, r4.w, r5.x};

    Projected p{};
    float cx = 0.0f, cy = 0.0f, cov[3] = {0.0f, 0.0f, 0.0f};
    bool valid = unscented_projection(f.cam, f.pose, mu, density, B, cx, cy, cov);
    if (valid) {
        p.cx = cx;
        p.cy = cy;
        valid = conic_extent(cov, density, p);
    }
    if (!valid) p = Projected{};
    proj[2 * i] = make_float4(p.cx, p.cy, p.conic0, p.conic1);
    proj[2 * i + 1] = make_float4(p.conic2, p.opacity, p.ex, p.ey);

    // SH radiance at the incident direction (mu - camera)/|mu - camera|.
    const V3 v = mu - v3(f.pose.c[0], f.pose.c[1], f.pose.c[2]);
    const float dist = __fsqrt_rn(dot3(v, v));
    const V3 dir = v3(v.x / dist, v.y / dist, v.z / dist);
    float basis[16];
    sh_basis(f.shDegree, dir, basis);
    const float* c = features + size_t(i) * 3 * f.shCoeffs;
    const int nb = min(sh_count(f.shDegree), int(f.shCoeffs));
    float rgb[3];
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
        float acc = basis[0] * __ldg(c + ch);
        for (int k = 1; k < nb; ++k) acc = __fmaf_rn(basis[k], __ldg(c + 3 * k + ch), acc);
        rgb[ch] = fmaxf(acc + 0.5f, 0.0f);
    }
    float4* rec = records + 4 * size_t(i);
    rec[0] = r0;
    rec[1] = make_float4(r5.y, r5.z, r5.w, r6.x);
    rec[2] = make_float4(r6.y, r6.z, r6.w, r7.x);
    rec[3] = make_float4(r7.y, rgb[0], rgb[1], rgb[2]);

    const uint32_t n = for_admitted_tiles(f, mask, p, [](int, int, uint32_t) {});
    counts[i] = n;
    if (visibility != nullptr) visibility[i] = n ? 1u : 0u;
    if (n != 0u) {
        const float Binv[9] = {r5.y, r5.z, r5.w, r6.x, r6.y, r6.z, r6.w, r7.x, r7.y};
        bounds[i] = support_radius(Binv);
    }
}

// Emits (tile << 32 | depth bits) keys and particle ids at the scanned offsets
// (reference expandTileProjections, gutProjector.cuh:947-1113).
__global__ __launch_bounds__(256) void k_emit(FrameArgs f, const float4* __restrict__ proj,
                                              const float4* __restrict__ records, const uint8_t* __restrict__ mask,
                                              const float4* __restrict__ tileRays, const uint64_t* __restrict__ offsets,
                                              const uint32_t* __restrict__ counts, uint64_t* __restrict__ keys,
                                              uint32_t* __restrict__ ids) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= f.N) return;
    const float4 p0 = proj[2 * i], p1 = proj[2 * i + 1];
    Projected p;
    p.cx = p0.x; p.cy = p0.y; p.conic0 = p0.z; p.conic1 = p0.w;
    p.conic2 = p1.x; p.opacity = p1.y; p.ex = p1.z; p.ey = p1.w;
    if (!fast_ut_valid(p)) return;
    const float4 a = records[4 * size_t(i)], b = records[4 * size_t(i) + 1], c = records[4 * size_t(i) + 2],
                 d = records[4 * size_t(i) + 3];
    const V3 mu = v3(a.x, a.y, a.z);
    const float Binv[9] = {b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x};
    const V3 cv = mu - v3(f.pose.c[0], f.pose.c[1], f.pose.c[2]);
    const float camRadial = finite_nonneg(__fsqrt_rn(dot3(cv, cv)), kMaxDepthValue);
    const uint64_t begin = offsets[i];
    const uint32_t reserved = counts[i];  // the emit walk repeats the count walk; never write past its slots
    const int keyMode = f.keyMode;
    for_admitted_tiles(f, mask, p, [&](int x, int y, uint32_t k) {
        if (k >= reserved) return;
        const uint32_t tile = uint32_t(y * f.gx + x);
        uint32_t depth;
        if (keyMode == GF_KEY_GLOBAL_DEPTH) {
            depth = __float_as_uint(camRadial);
        } else {
            depth = depth_key_per_tile(mu, Binv, camRadial, tileRays[2 * tile], tileRays[2 * tile + 1]);
        }
        keys[begin + k] = (uint64_t(tile) << 32) | depth;
        ids[begin + k] = i;
    });
}

// Per-tile [begin, end) of the sorted keys (reference gutRenderer.cu:114-144).
__global__ void k_tile_ranges(const uint64_t* __restrict__ keys, uint32_t n, uint2* __restrict__ ranges) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t tile = uint32_t(keys[i] >> 32);
    if (i == 0 || uint32_t(keys[i - 1] >> 32) != tile) ranges[tile].x = i;
    if (i == n - 1 || uint32_t(keys[i + 1] >> 32) != tile) ranges[tile].y = i + 1;
}

// Projection backward: record gradients to the reference's [N,32] density
// gradient and [N,3*C] SH gradient (reference projectBackward,
// gutProjector.cuh:1171-1222; radianceFromSpHBwd, gaussianParticles.cuh:234-310).
__global__ __launch_bounds__(256) void k_project_bwd(FrameArgs f, const float* __restrict__ particles,
                                                     const float* __restrict__ features,
                                                     const uint32_t* __restrict__ counts,
                                                     const float4* __restrict__ gradRecords,
                                                     float* __restrict__ gradParticles,
                                                     float* __restrict__ gradFeatures) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= f.N) return;
    const float4 g0 = gradRecords[4 * size_t(i)], g1 = gradRecords[4 * size_t(i) + 1],
                 g2 = gradRecords[4 * size_t(i) + 2], g3 = gradRecords[4 * size_t(i) + 3];
    float gp0 = g0.x, gp1 = g0.y, gp2 = g0.z;
    float* gs = gradFeatures + size_t(i) * 3 * f.shCoeffs;
    if (counts[i] != 0u) {
        const float4 r0 = ldg4(particles + 32 * size_t(i));
        const V3 mu = v3(r0.x, r0.y, r0.z);
        const V3 v = mu - v3(f.pose.c[0], f.pose.c[1], f.pose.c[2]);
        const float dist = __fsqrt_rn(dot3(v, v));
        const V3 dir = v3(v.x / dist, v.y / dist, v.z / dist);
        float basis[16], bx[16], by[16], bz[16];
        sh_basis(f.shDegree, dir, basis);
        sh_basis_grad(f.shDegree, dir, bx, by, bz);
        const int nb = min(sh_count(f.shDegree), int(f.shCoeffs));
        const float* c = features + size_t(i) * 3 * f.shCoeffs;
        const float gr[3] = {g3.y, g3.z, g3.w};
        V3 dg = v3(0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            float acc = basis[0] * __ldg(c + ch);
            for (int k = 1; k < nb; ++k) acc = __fmaf_rn(basis[k], __ldg(c + 3 * k + ch), acc);
            const float m = (acc + 0.5f) > 0.0f ? gr[ch] : 0.0f;
            for (int k = 0; k < nb; ++k) gs[3 * k + ch] = basis[k] * m;
            for (int k = 1; k < nb; ++k) {
                const float ck = __ldg(c + 3 * k + ch) * m;
                dg.x += bx[k] * ck;
                dg.y += by[k] * ck;
                dg.z += bz[k] * ck;
            }
        }
        for (int k = nb; k < int(f.shCoeffs); ++k) {
            gs[3 * k] = 0.0f;
            gs[3 * k + 1] = 0.0f;
            gs[3 * k + 2] = 0.0f;
        }
        const float ndg = dot3(dir, dg);
        gp0 += (dg.x - dir.x * ndg) / dist;
        gp1 += (dg.y - dir.y * ndg) / dist;
        gp2 += (dg.z - dir.z * ndg) / dist;
    } else {
        for (uint32_t k = 0; k < 3 * f.shCoeffs; ++k) gs[k] = 0.0f;
    }
    float4* out = reinterpret_cast<float4*>(gradParticles + 32 * size_t(i));
    out[0] = make_float4(gp0, gp1, gp2, g0.w);                      // pos, density
    out[1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);                   // rotation
    out[2] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);                   // scale, intrinsic density
    out[3] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);                   // factor 0..3
    out[4] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);                   // factor 4..7
    out[5] = make_float4(0.0f, g1.x, g1.y, g1.z);                   // factor 8 | Binv 0..2
    out[6] = make_float4(g1.w, g2.x, g2.y, g2.z);                   // Binv 3..6
    out[7] = make_float4(g2.w, g3.x, 0.0f, 0.0f);                   // Binv 7..8 | padding
}

}  // namespace gf
