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
// gutProjector.cuh:653-286).
__global__ __launch_bounds__(256) void k_project(FrameArgs f, const float* __restrict__ particles,
                                                 const float* __restrict__ features,
                                                 const uint8_t* __restrict__ mask, float4* __restrict__ proj,
                                                 float4* __restrict__ records, uint32_t* __restrict__ counts,
                                                 uint32_t* __restrict__ visibility) {
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

// ------------------------------------------------------------ k-buffer
template <int K>
struct KBuffer {
    float t[K];
    float a[K];
    uint32_t id[K];
    uint32_t n;
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int i = 0; i < K; ++i) {
            t[i] = -1.0f;
            a[i] = 0.0f;
            id[i] = kInvalidParticle;
        }
        n = 0;
    }
    __device__ __forceinline__ bool full() const { return n == uint32_t(K); }
    // Reference HitParticleKBufferT::insert (gutKBufferRenderer.cuh:132-147):
    // the new hit sinks from the top by compare-and-swap; when full, slot 0 was
    // composited and is overwritten.
    __device__ __forceinline__ void insert(float ht, float ha, uint32_t hid) {
        if (full()) {
            t[0] = -1.0f;
        } else {
            ++n;
        }
#pragma unroll
        for (int i = K - 1; i >= 0; --i) {
            const bool sw = ht > t[i];
            const float tt = t[i], ta = a[i];
            const uint32_t ti = id[i];
            t[i] = sw ? ht : tt;
            a[i] = sw ? ha : ta;
            id[i] = sw ? hid : ti;
            ht = sw ? tt : ht;
            ha = sw ? ta : ha;
            hid = sw ? ti : hid;
        }
    }
    // Entry i of the drain order: slot K - n + i.
    __device__ __forceinline__ void drainEntry(uint32_t i, float& ht, float& ha, uint32_t& hid) const {
        const uint32_t s = uint32_t(K) - n + i;
        ht = 0.0f;
        ha = 0.0f;
        hid = kInvalidParticle;
#pragma unroll
        for (int k = 0; k < K; ++k) {
            if (uint32_t(k) == s) {
                ht = t[k];
                ha = a[k];
                hid = id[k];
            }
        }
    }
};

template <>
struct KBuffer<0> {
    uint32_t n;
    __device__ __forceinline__ void init() { n = 0; }
    __device__ __forceinline__ bool full() const { return true; }
    __device__ __forceinline__ void insert(float, float, uint32_t) {}
    __device__ __forceinline__ void drainEntry(uint32_t, float& ht, float& ha, uint32_t& hid) const {
        ht = 0.0f;
        ha = 0.0f;
        hid = kInvalidParticle;
    }
};

__device__ __forceinline__ Record load_record(const float4* __restrict__ records, uint32_t idx) {
    const float4* r = records + 4 * size_t(idx);
    Record q;
    q.a = __ldg(r);
    q.b = __ldg(r + 1);
    q.c = __ldg(r + 2);
    q.d = __ldg(r + 3);
    return q;
}

struct RenderArgs {
    FrameArgs f;
    const uint8_t* mask;
    const uint2* ranges;
    const uint32_t* sortedIds;
    const float4* records;
    const float* rayO;
    const float* rayD;
};

struct PixelFwd {
    float T, hitT;
    float r, g, b;
    uint32_t hitN;
    bool alive;
};

// Front-to-back composite of one hit (reference gutKBufferRenderer.cuh:307-416).
__device__ __forceinline__ void composite_fwd(PixelFwd& s, float ht, float ha, uint32_t hid,
                                              const float4* __restrict__ records) {
    const float w = ha * s.T;
    s.hitT = s.hitT + ht * w;
    s.T = s.T * (1.0f - ha);
    if (w > 0.0f) {
        const float4 c = __ldg(records + 4 * size_t(hid) + 3);
        s.r = __fmaf_rn(fmaxf(c.y, 0.0f), w, s.r);
        s.g = __fmaf_rn(fmaxf(c.z, 0.0f), w, s.g);
        s.b = __fmaf_rn(fmaxf(c.w, 0.0f), w, s.b);
        s.hitN++;
    }
    if (s.T < kMinTransmittance) s.alive = false;
}

// Hit test of one candidate against one ray (reference gaussianParticles.slang:293-338).
__device__ __forceinline__ bool hit_candidate(const Ray& ray, const Record& q, float& alpha, float& hitT) {
    const HalfRay h = half_ray(ray, q);
    if (!h.valid) return false;
    const float g = fdot3(h.p, h.p);
    if (g > kResponseCutoff2) return false;
    const float resp = gf_expf(-0.5f * g);
    alpha = fminf(kMaxAlpha, resp * q.a.w);
    hitT = h.tau;
    return resp > kMinKernelResponse && alpha > kAlphaThreshold && hitT >= ray.tmin && hitT <= ray.tmax;
}

constexpr int kBatch = kTileThreads;

// One CTA per 16x16 tile, one thread per pixel.  Candidates are staged in
// shared memory 256 at a time; each pixel keeps a K-entry k-buffer in
// registers (reference render kernel, gutRenderer.cuh:217-265 and
// evalKBuffer, gutKBufferRenderer.cuh:614-700).
template <int K>
__global__ __launch_bounds__(kTileThreads) void k_render_fwd(RenderArgs a, float* __restrict__ rgba,
                                                             float* __restrict__ hitDistance,
                                                             float* __restrict__ hitCount) {
    __shared__ Record srec[kBatch];
    const FrameArgs& f = a.f;
    const int tile = blockIdx.x;
    const int tx = tile % f.gx, ty = tile / f.gx;
    const int px = tx * kTile + (threadIdx.x & 15), py = ty * kTile + (threadIdx.x >> 4);
    const bool inImage = px < f.W && py < f.H;
    const size_t pix = size_t(px) + size_t(f.W) * py;
    const bool retained = a.mask[tile] != 0u;
    Ray ray;
    ray.valid = false;
    if (inImage && retained) {
        ray = make_ray(f.pose, v3(a.rayO[3 * pix], a.rayO[3 * pix + 1], a.rayO[3 * pix + 2]),
                       v3(a.rayD[3 * pix], a.rayD[3 * pix + 1], a.rayD[3 * pix + 2]));
    }
    PixelFwd s{1.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0u, ray.valid};
    KBuffer<K> kb;
    kb.init();
    if (retained) {
        const uint2 range = a.ranges[tile];
        for (uint32_t base = range.x; base < range.y; base += kBatch) {
            if (__syncthreads_and(!s.alive)) break;
            const uint32_t sIdx = base + threadIdx.x;
            if (sIdx < range.y) srec[threadIdx.x] = load_record(a.records, __ldg(a.sortedIds + sIdx));
            __syncthreads();
            const int cnt = min(uint32_t(kBatch), range.y - base);
            for (int j = 0; j < cnt && s.alive; ++j) {
                const Record q = srec[j];
                float alpha, ht;
                if (hit_candidate(ray, q, alpha, ht)) {
                    const uint32_t hid = __ldg(a.sortedIds + base + j);
                    if constexpr (K == 0) {
                        composite_fwd(s, ht, alpha, hid, a.records);
                    } else {
                        if (kb.full()) composite_fwd(s, kb.t[0], kb.a[0], kb.id[0], a.records);
                        kb.insert(ht, alpha, hid);
                    }
                }
            }
        }
        if constexpr (K > 0) {
            for (uint32_t i = 0; s.alive && i < kb.n; ++i) {
                float ht, ha;
                uint32_t hid;
                kb.drainEntry(i, ht, ha, hid);
                composite_fwd(s, ht, ha, hid, a.records);
            }
        }
    }
    if (!inImage) return;
    float4 out = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float hd = 1e06f, hc = 0.0f;
    if (ray.valid) {
        out = make_float4(s.r, s.g, s.b, 1.0f - s.T);
        hd = s.hitT;
        hc = float(s.hitN);
    }
    reinterpret_cast<float4*>(rgba)[pix] = out;
    hitDistance[pix] = hd;
    if (hitCount != nullptr) hitCount[pix] = hc;
}

// ------------------------------------------------------------ backward
struct RenderBwdArgs {
    RenderArgs r;
    const float* rgba;
    const float* hitDistance;
    const float* gradRgba;
    const float* gradHitDistance;
    float4* gradRecords;  // [N,4] float4: pos.xyz+density | Binv row0 + row1.x | row1.yz + row2.xy | row2.z + rgb
};

struct PixelBwd {
    float T, depth;
    float r, g, b;
    float featB[3], featG[3];
    float TB, TG, hitTB, hitTG;
    bool alive;
};

// Gradient of one composited hit (reference processHitBwd,
// gaussianParticles.cuh:736-1155, geometric channels inactive).  Returns
// false when the hit is rejected by the re-test.
__device__ __forceinline__ bool hit_vjp(PixelBwd& s, const Ray& ray, const Record& q, float4 g[4]) {
    const HalfRay h = half_ray(ray, q);
    if (!h.valid) return false;
    const float grayDist = fdot3(h.p, h.p);
    const float gres = gf_expf(-0.5f * grayDist);
    const float density = q.a.w;
    const float galphaU = gres * density;
    const float galpha = fminf(kMaxAlpha, galphaU);
    if (!(gres > kMinKernelResponse && galpha > kAlphaThreshold)) return false;
    const float gdist = h.tau;
    const float weight = galpha * s.T;
    const float nextT = (1.0f - galpha) * s.T;
    s.depth = s.depth + gdist * weight;
    const bool tail = nextT <= kMinTransmittance;
    const float residualHitT = fmaxf(tail ? 0.0f : (s.hitTB - s.depth) / nextT, 0.0f);
    const float galphaRayHitGrd = (gdist - residualHitT) * s.T * s.hitTG;
    const float residualTrm = galpha < 0.999999f ? s.TB / (1.0f - galpha) : s.T;
    const float galphaRayDnsGrd = residualTrm * -s.TG;
    const float cr = fmaxf(q.d.y, 0.0f), cg = fmaxf(q.d.z, 0.0f), cb = fmaxf(q.d.w, 0.0f);
    s.r = __fmaf_rn(cr, weight, s.r);
    s.g = __fmaf_rn(cg, weight, s.g);
    s.b = __fmaf_rn(cb, weight, s.b);
    const float rr = fmaxf(tail ? 0.0f : (s.featB[0] - s.r) / nextT, 0.0f);
    const float rg = fmaxf(tail ? 0.0f : (s.featB[1] - s.g) / nextT, 0.0f);
    const float rb = fmaxf(tail ? 0.0f : (s.featB[2] - s.b) / nextT, 0.0f);
    float comp = galphaRayHitGrd + galphaRayDnsGrd;
    comp += s.T * (cr - rr) * s.featG[0];
    comp += s.T * (cg - rg) * s.featG[1];
    comp += s.T * (cb - rb) * s.featG[2];
    const float gU = (galphaU < kMaxAlpha ? 1.0f : 0.0f) * comp;
    const float gDensity = gres * gU;
    const float gresGrd = density * gU;
    const float grayDistGrd = -0.5f * gres * gresGrd;
    const float tauGrad = weight * s.hitTG;
    // Closest-point VJP (reference gutHalfRayResponse.cuh:39-62).
    const V3 pointGrad = (2.0f * grayDistGrd) * h.p;
    V3 groGrd = pointGrad;
    V3 grduGrd = h.tau * pointGrad;
    const float totalTauGrad = tauGrad + dot3(pointGrad, h.grdu);
    if (h.interior) {
        const float inv = -1.0f / h.denom;
        const V3 tauOriginGrad = inv * h.grdu;
        const V3 tauDirectionGrad = inv * h.gro + ((2.0f * h.num) / (h.denom * h.denom)) * h.grdu;
        groGrd = groGrd + totalTauGrad * tauOriginGrad;
        grduGrd = grduGrd + totalTauGrad * tauDirectionGrad;
    }
    // Binv rows: r0 = (b.x b.y b.z), r1 = (b.w c.x c.y), r2 = (c.z c.w d.x).
    const float gpx = -(groGrd.x * q.b.x + groGrd.y * q.b.w + groGrd.z * q.c.z);
    const float gpy = -(groGrd.x * q.b.y + groGrd.y * q.c.x + groGrd.z * q.c.w);
    const float gpz = -(groGrd.x * q.b.z + groGrd.y * q.c.y + groGrd.z * q.d.x);
    const V3 gp = v3(ray.o.x - q.a.x, ray.o.y - q.a.y, ray.o.z - q.a.z);
    const float m00 = groGrd.x * gp.x + grduGrd.x * ray.d.x, m01 = groGrd.x * gp.y + grduGrd.x * ray.d.y,
                m02 = groGrd.x * gp.z + grduGrd.x * ray.d.z;
    const float m10 = groGrd.y * gp.x + grduGrd.y * ray.d.x, m11 = groGrd.y * gp.y + grduGrd.y * ray.d.y,
                m12 = groGrd.y * gp.z + grduGrd.y * ray.d.z;
    const float m20 = groGrd.z * gp.x + grduGrd.z * ray.d.x, m21 = groGrd.z * gp.y + grduGrd.z * ray.d.y,
                m22 = groGrd.z * gp.z + grduGrd.z * ray.d.z;
    g[0] = make_float4(gpx, gpy, gpz, gDensity);
    g[1] = make_float4(m00, m01, m02, m10);
    g[2] = make_float4(m11, m12, m20, m21);
    g[3] = make_float4(m22, s.featG[0] * weight, s.featG[1] * weight, s.featG[2] * weight);
    s.T = nextT;
    return true;
}

__device__ __forceinline__ float4 shfl_down4(float4 v, int o) {
    return make_float4(__shfl_down_sync(0xffffffffu, v.x, o), __shfl_down_sync(0xffffffffu, v.y, o),
                       __shfl_down_sync(0xffffffffu, v.z, o), __shfl_down_sync(0xffffffffu, v.w, o));
}
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// Warp-aggregated accumulation of one gradient per lane: when every active
// lane of the warp holds the same particle the 16 components are reduced
// with shuffles and written by one lane, otherwise each lane adds its own.
__device__ __forceinline__ void accumulate_grad(float4* __restrict__ gradRecords, bool have, uint32_t idx,
                                                float4 g[4]) {
    const uint32_t hm = __ballot_sync(0xffffffffu, have);
    if (hm == 0u) return;
    const int lane = threadIdx.x & 31;
    const int leader = __ffs(hm) - 1;
    const uint32_t leaderIdx = __shfl_sync(0xffffffffu, idx, leader);
    const bool uniform = __all_sync(0xffffffffu, !have || idx == leaderIdx);
    if (uniform && __popc(hm) > 1) {
        float4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = have ? g[k] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = add4(v[k], shfl_down4(v[k], o));
        }
        if (lane == 0) {
            float4* dst = gradRecords + 4 * size_t(leaderIdx);
#pragma unroll
            for (int k = 0; k < 4; ++k) atomicAdd(dst + k, v[k]);
        }
    } else if (have) {
        float4* dst = gradRecords + 4 * size_t(idx);
#pragma unroll
        for (int k = 0; k < 4; ++k) atomicAdd(dst + k, g[k]);
    }
}

// Backward replay: the identical traversal and k-buffer, each composited hit
// back-propagated from the final pixel values (reference renderBackward,
// gutRenderer.cuh:555-626).  Loops are warp-uniform so the gradient
// reduction can use full-warp shuffles.
template <int K>
__global__ __launch_bounds__(kTileThreads) void k_render_bwd(RenderBwdArgs a) {
    __shared__ Record srec[kBatch];
    const FrameArgs& f = a.r.f;
    const int tile = blockIdx.x;
    if (a.r.mask[tile] == 0u) return;  // block-uniform
    const int tx = tile % f.gx, ty = tile / f.gx;
    const int px = tx * kTile + (threadIdx.x & 15), py = ty * kTile + (threadIdx.x >> 4);
    const bool inImage = px < f.W && py < f.H;
    const size_t pix = size_t(px) + size_t(f.W) * py;
    Ray ray;
    ray.valid = false;
    PixelBwd s;
    s.T = 1.0f;
    s.depth = 0.0f;
    s.r = s.g = s.b = 0.0f;
    if (inImage) {
        ray = make_ray(f.pose, v3(a.r.rayO[3 * pix], a.r.rayO[3 * pix + 1], a.r.rayO[3 * pix + 2]),
                       v3(a.r.rayD[3 * pix], a.r.rayD[3 * pix + 1], a.r.rayD[3 * pix + 2]));
    }
    s.alive = ray.valid;
    if (ray.valid) {
        const float4 fo = reinterpret_cast<const float4*>(a.rgba)[pix];
        const float4 go = reinterpret_cast<const float4*>(a.gradRgba)[pix];
        s.featB[0] = fo.x; s.featB[1] = fo.y; s.featB[2] = fo.z;
        s.featG[0] = go.x; s.featG[1] = go.y; s.featG[2] = go.z;
        s.TB = 1.0f - fo.w;
        s.TG = -1.0f * go.w;
        s.hitTB = a.hitDistance[pix];
        s.hitTG = a.gradHitDistance[pix];
    }
    KBuffer<K> kb;
    kb.init();
    const uint2 range = a.r.ranges[tile];
    for (uint32_t base = range.x; base < range.y; base += kBatch) {
        if (__syncthreads_and(!s.alive)) break;
        const uint32_t sIdx = base + threadIdx.x;
        if (sIdx < range.y) srec[threadIdx.x] = load_record(a.r.records, __ldg(a.r.sortedIds + sIdx));
        __syncthreads();
        const int cnt = min(uint32_t(kBatch), range.y - base);
        for (int j = 0; j < cnt; ++j) {
            if (!__any_sync(0xffffffffu, s.alive)) break;
            bool have = false;
            uint32_t cid = kInvalidParticle;
            float4 g[4] = {};
            if (s.alive) {
                const Record q = srec[j];
                float alpha, ht;
                if (hit_candidate(ray, q, alpha, ht)) {
                    const uint32_t hid = __ldg(a.r.sortedIds + base + j);
                    if constexpr (K == 0) {
                        have = hit_vjp(s, ray, q, g);
                        cid = hid;
                    } else {
                        if (kb.full()) {
                            cid = kb.id[0];
                            have = hit_vjp(s, ray, load_record(a.r.records, cid), g);
                        }
                        kb.insert(ht, alpha, hid);
                    }
                    if (s.T < kMinTransmittance) s.alive = false;
                }
            }
            accumulate_grad(a.gradRecords, have, cid, g);
        }
    }
    if constexpr (K > 0) {
        for (uint32_t i = 0; i < uint32_t(K); ++i) {
            if (!__any_sync(0xffffffffu, s.alive && i < kb.n)) break;
            bool have = false;
            uint32_t cid = kInvalidParticle;
            float4 g[4] = {};
            if (s.alive && i < kb.n) {
                float ht, ha;
                kb.drainEntry(i, ht, ha, cid);
                have = hit_vjp(s, ray, load_record(a.r.records, cid), g);
                if (s.T < kMinTransmittance) s.alive = false;
            }
            accumulate_grad(a.gradRecords, have, cid, g);
        }
    }
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
