// Per-pixel k-buffer compositing, forward and backward (reference render /
// renderBackward kernels, gutRenderer.cuh:217-265, :555-626; evalKBuffer,
// gutKBufferRenderer.cuh:614-700; processHitParticle, :207-416;
// processHitBwd, gaussianParticles.cuh:736-1155).
//
// One CTA per 16x16 tile, one thread per pixel.  Tile candidates are staged
// in shared memory 256 at a time.  When every ray of the tile starts at the
// same point (a central camera) the canonical ray origin B^-1 (o - mu) of
// each candidate is computed once per tile instead of once per pixel.
//
// The k-buffer lives in shared memory as a per-pixel ring of K entries
// (hit distance, alpha, particle) kept sorted by hit distance.  It reproduces
// the reference's register network exactly: HitParticleKBufferT::insert
// (gutKBufferRenderer.cuh:132-147) sinks the new hit from the top with
// compare-and-swap (`hit > entry` strict).  For a sorted buffer that network
// (a) keeps every entry whose distance is >= the new hit's in place, (b)
// places the new hit below them, (c) moves every entry below it down by one
// slot, except that inside a run of equal distances only the run's top entry
// moves -- to the bottom of the run -- while the others stay.  The ring
// keeps a count of adjacent equal pairs; with no equal pairs (the usual case)
// an insertion is a plain sorted insert from the top, O(entries moved), and
// otherwise a general path applies rule (c) explicitly.
#pragma once

#include "gf_tracer_kernels.cuh"

namespace gf {

// Composite log of a training forward: for every pixel, the candidates the
// k-buffer composited, in order, as positions in the tile's sorted candidate
// list (relative to the tile's range start), so that the backward
// re-evaluates only the composited hits instead of replaying every candidate
// through the k-buffer.  Entry i of the pixel at thread p of tile t is
// ids[(i * tiles + t) * kTileThreads + p] (coalesced across a warp).  A pixel
// that composites more than `capacity` hits marks its tile in `overflow`; the
// backward replays such tiles.  Entries are 16-bit, so a tile of more than
// kLogTileCandidates candidates is marked the same way.  ids == nullptr: no
// log (inference).
struct CompositeLog {
    uint16_t* ids;       // [capacity][tiles][kTileThreads] candidate positions within the tile
    uint32_t* count;     // [tiles][kTileThreads] entries logged, at most capacity
    uint32_t* overflow;  // [tiles] 1 when a pixel of the tile exceeded the capacity
    uint32_t* overflowList;   // the flagged tiles, in no particular order
    uint32_t* overflowCount;  // their number (zeroed before the forward)
    uint32_t capacity;
    uint32_t tiles;
};

// Geometric training channels (rayPayload.cuh:242-322), written by the
// forward of a tracer created with enable_normals; any pointer may be NULL.
struct GeoOut {
    float* normal;    // [H,W,3]
    float* depthVar;  // [H,W,1]
    float* quant;     // [H,W,10]
    float* extent;    // [H,W,1]
    float* invD;      // [H,W,1]
    float* invD2;     // [H,W,1]
    const float* particles;  // packed [N,32] rows: quaternion (slots 4-7), intrinsic scale (8-10)
};

struct RenderArgs {
    FrameArgs f;
    const uint8_t* mask;
    const uint2* ranges;
    const uint32_t* sortedIds;
    const float4* records;
    const float* bounds;  // per-particle support radius (sphere around the mean containing the 3-sigma ellipsoid)
    const float* rayO;
    const float* rayD;
    CompositeLog log;
    GeoOut geo;
};

// Forward values and output gradients of the geometric channels in a backward
// (NULL pairs: the channel has no gradient).
struct GeoBwd {
    const float* normal;
    const float* gradNormal;
    const float* depthVar;
    const float* gradDepthVar;
    const float* extent;
    const float* gradExtent;
    const float* invD;
    const float* gradInvD;
    const float* invD2;
    const float* gradInvD2;
    const float* particles;    // packed [N,32] rows: quaternion (slots 4-7), intrinsic scale (8-10)
    float4* gradShape;         // [N,2] float4: quaternion (w, x, y, z) | scale.xyz, 0  (extent gradient)
    const float* quant;        // forward quantile channels [H*W, 10] (crossing depth 8, crossing rate 9)
    const float* gradQuant;    // dL/d quant (channel 8 read) or NULL
};

struct RenderBwdArgs {
    RenderArgs r;
    const float* rgba;
    const float* hitDistance;
    const float* gradRgba;
    const float* gradHitDistance;
    float4* gradRecords;  // [N,4] float4: pos.xyz+density | Binv row0 + row1.x | row1.yz + row2.xy | row2.z + rgb
    GeoBwd geo;
    float* absGrad;       // densification statistic (gf_trace_grads.position_abs_grad) or NULL
    int absMode;          // GF_ABS_GRAD_SCREEN ([N,8]: map 0-5, sums 6-7) or GF_ABS_GRAD_WORLD ([N,3])
};

constexpr int kBatch = kTileThreads;
// The forward stages 32 candidates at a time into one of two buffers: the
// records of the next batch are copied asynchronously (cp.async) by the
// block's first warp while every warp composites the current one, so no warp
// waits out a global-memory latency at the batch barrier.  With the K = 16
// ring (48 KiB) its block needs 54.5 KiB of shared memory, so four blocks
// (32 warps) fit on an SM.  The two-block kernels use the same room as one
// batch of 64, staged synchronously.
constexpr int kFwdBatch = 32;
constexpr int kFwdBuffers = 2;

// A staged candidate: the 64-byte render record, its canonical ray origin for
// the tile's common ray origin, and the cone from that origin that contains
// its support sphere (used to skip warps whose rays all miss the sphere).
struct Staged {
    float4 a, b, c, d;  // pos.xyz density | Binv r0, r1.x | r1.yz, r2.xy | r2.z, rgb
    float4 g;           // B^-1 (o - mu) | sin of the cone half-angle
    float4 u;           // unit direction o -> mu | cos of the cone half-angle (-3: never skipped)
};

// Warp-level culling.  Each warp covers an 8x4 pixel block; its rays (central
// tile only) lie in a cone (axis, half-angle theta).  A ray that misses a
// candidate's support sphere has g > 9 everywhere along it (the sphere
// contains the 3-sigma ellipsoid), so the hit test would reject it: a warp
// whose cone does not reach the candidate's cone skips the candidate.  The
// test adds 1e-3 rad to theta, far above its rounding error, so it never
// skips a hit and the outputs are unchanged.
constexpr float kCullMarginRad = 1e-3f;
constexpr int kMaskWords = kBatch / 32;

struct WarpCone {
    float ax, ay, az;
    float cosT, sinT;
    bool enabled;
};

// Shared memory of a render CTA: the staged batch, its particle ids, and the
// per-pixel rings (hit distance + alpha, sorted candidate position).
__host__ __device__ constexpr size_t render_smem_bytes(int K, int batch = kBatch) {
    return (sizeof(Staged) + sizeof(uint32_t)) * batch +
           size_t(K > 0 ? K : 1) * kTileThreads * (sizeof(float2) + sizeof(uint32_t));
}

__device__ __forceinline__ Record load_record(const float4* __restrict__ records, uint32_t idx) {
    const float4* r = records + 4 * size_t(idx);
    Record q;
    q.a = __ldg(r);
    q.b = __ldg(r + 1);
    q.c = __ldg(r + 2);
    q.d = __ldg(r + 3);
    return q;
}

__device__ __forceinline__ V3 binv_times(const float4& b, const float4& c, const float4& d, V3 v) {
    return v3(__fmaf_rn(b.z, v.z, __fmaf_rn(b.y, v.y, b.x * v.x)), __fmaf_rn(c.y, v.z, __fmaf_rn(c.x, v.y, b.w * v.x)),
              __fmaf_rn(d.x, v.z, __fmaf_rn(c.w, v.y, c.z * v.x)));
}

// Hit test of one candidate with a given canonical ray origin `gro`
// (reference gaussianParticles.slang:293-338; identical arithmetic to half_ray).
//
// With `pretest`, `miss` = A - (G + 1e-5 A) rounded, where A = |gro|^2 and G
// = min(9.001, 2 ln(255 rho) + 1e-3) is the squared canonical distance
// beyond which the hit test cannot pass (response below the 0.0113 cut-off,
// or alpha below 1/255).  The candidate is rejected before the division when
// denom * miss > num^2, i.e. when the squared distance of the ray's line to
// the centre, A - num^2/denom, exceeds G.  With unit roundoff u the rounding
// of A, denom, num and the products changes that quantity by less than 15u A,
// inside the 1e-5 A margin, and the squared distance the full test computes
// at the clamped closest point is at least (1 - 6u) times the line's (the
// point is one FMA per coordinate); G carries the 1e-3 margin against the
// rounding of exp and of the alpha product.  So a rejected candidate always
// fails the full test: the outputs do not change.
__device__ __forceinline__ bool hit_with_origin(const Ray& ray, V3 gro, const float4& b, const float4& c,
                                                const float4& d, float density, float& alpha, float& hitT,
                                                bool pretest = false, float miss = 0.0f) {
    const V3 grdu = binv_times(b, c, d, ray.d);
    const float denom = fdot3(grdu, grdu);
    // callers test valid rays only, and make_ray's valid (tmax > tmin, tmin =
    // max(., 0)) already means a finite tmin below tmax
    if (!(denom > 0.0f && isfinite_f(denom))) return false;
    const float num = fdot3(gro, grdu);
    if (pretest && __fmul_rn(denom, miss) > __fmul_rn(num, num)) return false;
    const float tauLine = -num / denom;
    const float tau = fminf(fmaxf(tauLine, ray.tmin), ray.tmax);
    const V3 p = v3(__fmaf_rn(tau, grdu.x, gro.x), __fmaf_rn(tau, grdu.y, gro.y), __fmaf_rn(tau, grdu.z, gro.z));
    const float g = fdot3(p, p);
    if (g > kResponseCutoff2) return false;
    const float resp = gf_expf(-0.5f * g);
    alpha = fminf(kMaxAlpha, resp * density);
    hitT = tau;
    return resp > kMinKernelResponse && alpha > kAlphaThreshold && hitT >= ray.tmin && hitT <= ray.tmax;
}

// ------------------------------------------------------------------ ring k-buffer
template <int K>
struct RingKBuffer {
    float2* ta;    // [K][kTileThreads] (hit distance, alpha)
    uint32_t* id;  // [K][kTileThreads] sorted position of the candidate in the tile list
    int tid;
    int head;
    int n;
    int ties;  // adjacent entries with equal hit distance

    __device__ __forceinline__ void init(float2* ta_, uint32_t* id_, int tid_) {
        ta = ta_;
        id = id_;
        tid = tid_;
        head = 0;
        n = 0;
        ties = 0;
    }
    __device__ __forceinline__ bool full() const { return n == K; }
    // ring slot of entry i (head + i < 2K); a mask when K is a power of two
    __device__ __forceinline__ int slot(int i) const {
        const int s = head + i;
        if constexpr ((K & (K - 1)) == 0) return s & (K - 1);
        return s >= K ? s - K : s;
    }
    __device__ __forceinline__ float2 getTA(int s) const { return ta[s * kTileThreads + tid]; }
    __device__ __forceinline__ uint32_t getId(int s) const { return id[s * kTileThreads + tid]; }
    __device__ __forceinline__ void put(int s, float2 v, uint32_t i) {
        ta[s * kTileThreads + tid] = v;
        id[s * kTileThreads + tid] = i;
    }
    // Removes the nearest entry (the reference's kb[0], composited when full).
    __device__ __forceinline__ void pop_front(float& t, float& a, uint32_t& idx) {
        const float2 v = getTA(head);
        t = v.x;
        a = v.y;
        idx = getId(head);
        if (n > 1 && getTA(slot(1)).x == t) --ties;
        head = slot(1);
        --n;
    }
    // Entry i in drain order (nearest first).
    __device__ __forceinline__ void entry(int i, float& t, float& a, uint32_t& idx) const {
        const int s = slot(i);
        const float2 v = getTA(s);
        t = v.x;
        a = v.y;
        idx = getId(s);
    }
    // Insert with the reference network's semantics; requires n < K.
    __device__ __forceinline__ void insert(float t, float a, uint32_t idx) {
        if (ties != 0) {
            insert_general(t, a, idx);
            return;
        }
        int i = n - 1;
        float above = -1.0f;
        while (i >= 0) {
            const int s = slot(i);
            const float2 v = getTA(s);
            if (!(v.x >= t)) break;
            put(slot(i + 1), v, getId(s));
            above = v.x;
            --i;
        }
        put(slot(i + 1), make_float2(t, a), idx);
        if (i + 1 < n && above == t) ++ties;
        ++n;
    }
    __device__ __forceinline__ void insert_general(float t, float a, uint32_t idx) {
        int p = 0;
        while (p < n && getTA(slot(p)).x < t) ++p;
        // Entries below the new hit: every run of equal distances moves its top entry to its bottom.
        int r = 0;
        while (r < p) {
            const float tr = getTA(slot(r)).x;
            int e = r + 1;
            while (e < p && getTA(slot(e)).x == tr) ++e;
            if (e - r >= 2) {
                const int top = slot(e - 1);
                const float2 topTA = getTA(top);
                const uint32_t topId = getId(top);
                for (int q = e - 1; q > r; --q) {
                    const int src = slot(q - 1);
                    put(slot(q), getTA(src), getId(src));
                }
                put(slot(r), topTA, topId);
            }
            r = e;
        }
        for (int q = n; q > p; --q) {
            const int src = slot(q - 1);
            put(slot(q), getTA(src), getId(src));
        }
        put(slot(p), make_float2(t, a), idx);
        if (p < n && getTA(slot(p + 1)).x == t) ++ties;
        ++n;
    }
};

// ------------------------------------------------------------------ shared set-up
struct TileSetup {
    int tile, px, py;
    bool inImage;
    size_t pix;
    Ray ray;
    bool central;  // every in-image ray of the tile starts at the same point
    V3 origin;     // that point
    WarpCone cone;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Initializes the pixel's ray and decides whether the tile is central (block-uniform).
__device__ __forceinline__ TileSetup tile_setup(const RenderArgs& a, bool retained, int tile) {
    __shared__ float sOrigin[3];
    TileSetup ts;
    const FrameArgs& f = a.f;
    ts.tile = tile;
    const int tx = ts.tile % f.gx, ty = ts.tile / f.gx;
    // warp w covers the 8x4 block (w & 1, w >> 1) of the tile; lane -> (lane & 7, lane >> 3)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    ts.px = tx * kTile + (warp & 1) * 8 + (lane & 7);
    ts.py = ty * kTile + (warp >> 1) * 4 + (lane >> 3);
    ts.inImage = ts.px < f.W && ts.py < f.H;
    ts.pix = size_t(ts.px) + size_t(f.W) * ts.py;
    ts.ray.valid = false;
    ts.ray.o = v3(0.0f, 0.0f, 0.0f);
    if (ts.inImage && retained) {
        ts.ray = make_ray(f.pose, v3(a.rayO[3 * ts.pix], a.rayO[3 * ts.pix + 1], a.rayO[3 * ts.pix + 2]),
                          v3(a.rayD[3 * ts.pix], a.rayD[3 * ts.pix + 1], a.rayD[3 * ts.pix + 2]));
    }
    if (threadIdx.x == 0) {
        sOrigin[0] = ts.ray.o.x;
        sOrigin[1] = ts.ray.o.y;
        sOrigin[2] = ts.ray.o.z;
    }
    __syncthreads();
    ts.origin = v3(sOrigin[0], sOrigin[1], sOrigin[2]);
    const bool same = !ts.inImage ||
                      (__float_as_uint(ts.ray.o.x) == __float_as_uint(ts.origin.x) &&
                       __float_as_uint(ts.ray.o.y) == __float_as_uint(ts.origin.y) &&
                       __float_as_uint(ts.ray.o.z) == __float_as_uint(ts.origin.z));
    // thread 0 is always in the image for a non-empty tile
    ts.central = __syncthreads_and(same) != 0;
    // Cone of the warp's valid rays.
    const bool valid = ts.ray.valid;
    const float sx = warp_sum(valid ? ts.ray.d.x : 0.0f);
    const float sy = warp_sum(valid ? ts.ray.d.y : 0.0f);
    const float sz = warp_sum(valid ? ts.ray.d.z : 0.0f);
    const float sn = sqrtf(sx * sx + sy * sy + sz * sz);
    ts.cone.enabled = false;
    ts.cone.ax = ts.cone.ay = ts.cone.az = 0.0f;
    ts.cone.cosT = 1.0f;
    ts.cone.sinT = 0.0f;
    if (__any_sync(0xffffffffu, valid) && ts.central && sn > 0.0f) {
        ts.cone.ax = sx / sn;
        ts.cone.ay = sy / sn;
        ts.cone.az = sz / sn;
        const float dl = sqrtf(dot3(ts.ray.d, ts.ray.d));
        const float c = valid ? (ts.cone.ax * ts.ray.d.x + ts.cone.ay * ts.ray.d.y + ts.cone.az * ts.ray.d.z) / dl : 1.0f;
        const float cmin = warp_min(fminf(1.0f, fmaxf(-1.0f, c)));
        const float theta = acosf(cmin) + kCullMarginRad;
        if (theta < 1.5f) {
            ts.cone.cosT = cosf(theta);
            ts.cone.sinT = sinf(theta);
            ts.cone.enabled = true;
        }
    }
    return ts;
}

// Bit i: candidate k*32+i of the staged batch may reach a ray of this warp.
__device__ __forceinline__ uint32_t warp_mask(const TileSetup& ts, const Staged* sRec, int cnt, int k) {
    const int j = k * 32 + (threadIdx.x & 31);
    bool pass = j < cnt;
    if (pass && ts.cone.enabled) {
        const float4 u = sRec[j].u;
        const float sinB = sRec[j].g.w;
        const float lhs = ts.cone.ax * u.x + ts.cone.ay * u.y + ts.cone.az * u.z;
        const float rhs = ts.cone.cosT * u.w - ts.cone.sinT * sinB;
        pass = !(lhs < rhs);
    }
    return __ballot_sync(0xffffffffu, pass);
}

__device__ __forceinline__ uint32_t idxOf(const RenderArgs& a, uint32_t sIdx) { return __ldg(a.sortedIds + sIdx); }

// Squared canonical distance beyond which a particle of density rho cannot
// pass the hit test, with margin (see hit_with_origin): min(9.001,
// 2 ln(255 rho) + 1e-3); -1 for rho <= 0 (never a hit).
__device__ __forceinline__ float miss_distance2(float density) {
    if (!(density > 0.0f)) return -1.0f;
    return fminf(9.001f, __fadd_rn(__fmul_rn(2.0f, gf_logf(__fmul_rn(255.0f, density))), 1e-3f));
}

// Stages candidate sIdx into shared memory (thread-private slot).  The
// forward (kFwd) of a central tile does not read the position again and
// keeps there the pre-test threshold of hit_with_origin.
template <bool kFwd = false>
__device__ __forceinline__ void stage(const RenderArgs& a, const TileSetup& ts, uint32_t sIdx, Staged& out) {
    const Record q = load_record(a.records, idxOf(a, sIdx));
    out.a = q.a;
    out.b = q.b;
    out.c = q.c;
    out.d = q.d;
    if (ts.central) {
        const V3 gro = binv_times(q.b, q.c, q.d, v3(ts.origin.x - q.a.x, ts.origin.y - q.a.y, ts.origin.z - q.a.z));
        if constexpr (kFwd) {
            const float A = fdot3(gro, gro);
            out.a.x = __fsub_rn(A, __fadd_rn(miss_distance2(q.a.w), __fmul_rn(1e-5f, A)));
        }
        const V3 v = v3(q.a.x - ts.origin.x, q.a.y - ts.origin.y, q.a.z - ts.origin.z);
        const float dist = sqrtf(dot3(v, v));
        const float radius = __ldg(a.bounds + idxOf(a, sIdx));
        float sinB = 0.0f, cosB = -3.0f;
        float4 u = make_float4(0.0f, 0.0f, 0.0f, cosB);
        if (dist > radius && isfinite_f(dist) && isfinite_f(radius)) {
            sinB = radius / dist;
            cosB = sqrtf(fmaxf(0.0f, 1.0f - sinB * sinB));
            u = make_float4(v.x / dist, v.y / dist, v.z / dist, cosB);
        }
        out.g = make_float4(gro.x, gro.y, gro.z, sinB);
        out.u = u;
    }
}

// The forward's staging, in two halves: the raw record of candidate sIdx is
// copied asynchronously into `out.a..d` (and its id and support radius into
// `id`, `bound`), then, once the copies have landed, derive() adds the
// fields that stage<true>() computes from them.
__device__ __forceinline__ void cp_async16(void* smemDst, const void* gmemSrc) {
    const uint32_t dst = uint32_t(__cvta_generic_to_shared(smemDst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(gmemSrc) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smemDst, const void* gmemSrc) {
    const uint32_t dst = uint32_t(__cvta_generic_to_shared(smemDst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(gmemSrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

__device__ __forceinline__ void fetch_async(const RenderArgs& a, uint32_t id, Staged& out, float& bound) {
    const float4* r = a.records + 4 * size_t(id);
    cp_async16(&out.a, r);
    cp_async16(&out.b, r + 1);
    cp_async16(&out.c, r + 2);
    cp_async16(&out.d, r + 3);
    cp_async4(&bound, a.bounds + id);
}

// The fields stage<true>() derives for a central tile, from the landed record.
__device__ __forceinline__ void derive(const TileSetup& ts, Staged& out, float radius) {
    if (!ts.central) return;
    const float4 qa = out.a;
    const V3 gro = binv_times(out.b, out.c, out.d, v3(ts.origin.x - qa.x, ts.origin.y - qa.y, ts.origin.z - qa.z));
    const float A = fdot3(gro, gro);
    out.a.x = __fsub_rn(A, __fadd_rn(miss_distance2(qa.w), __fmul_rn(1e-5f, A)));
    const V3 v = v3(qa.x - ts.origin.x, qa.y - ts.origin.y, qa.z - ts.origin.z);
    const float dist = sqrtf(dot3(v, v));
    float sinB = 0.0f, cosB = -3.0f;
    float4 u = make_float4(0.0f, 0.0f, 0.0f, cosB);
    if (dist > radius && isfinite_f(dist) && isfinite_f(radius)) {
        sinB = radius / dist;
        cosB = sqrtf(fmaxf(0.0f, 1.0f - sinB * sinB));
        u = make_float4(v.x / dist, v.y / dist, v.z / dist, cosB);
    }
    out.g = make_float4(gro.x, gro.y, gro.z, sinB);
    out.u = u;
}

template <bool kFwd = false>
__device__ __forceinline__ bool hit_staged(const TileSetup& ts, const Staged& q, float& alpha, float& ht) {
    if (ts.central) {
        return hit_with_origin(ts.ray, v3(q.g.x, q.g.y, q.g.z), q.b, q.c, q.d, q.a.w, alpha, ht, kFwd, q.a.x);
    }
    const V3 gro = binv_times(q.b, q.c, q.d, v3(ts.ray.o.x - q.a.x, ts.ray.o.y - q.a.y, ts.ray.o.z - q.a.z));
    return hit_with_origin(ts.ray, gro, q.b, q.c, q.d, q.a.w, alpha, ht);
}

// ------------------------------------------------------------------ forward
struct PixelFwd {
    float T, hitT;
    float r, g, b;
    uint32_t hitN;
    bool alive;
};

// The staged batch in shared memory: candidates [base, base + cnt) of the tile's sorted list.
struct Batch {
    const Staged* rec;
    const uint32_t* ids;
    uint32_t base, cnt;
};

// Render record of the candidate at sorted position sp: from the staged batch
// when it is there, else from global memory.
__device__ __forceinline__ Record record_at(const RenderArgs& a, const Batch& b, uint32_t sp, uint32_t& idx) {
    const uint32_t j = sp - b.base;
    Record q;
    if (j < b.cnt) {
        const Staged& st = b.rec[j];
        q.a = st.a;
        q.b = st.b;
        q.c = st.c;
        q.d = st.d;
        idx = b.ids[j];
    } else {
        idx = __ldg(a.sortedIds + sp);
        q = load_record(a.records, idx);
    }
    return q;
}

__device__ __forceinline__ float4 color_at(const RenderArgs& a, const Batch& b, uint32_t sp) {
    const uint32_t j = sp - b.base;
    if (j < b.cnt) return b.rec[j].d;
    return __ldg(a.records + 4 * size_t(__ldg(a.sortedIds + sp)) + 3);
}

// Candidates a logged tile may hold: log entries are 16-bit positions.
constexpr uint32_t kLogTileCandidates = 65536u;

// Appends one composited candidate (its position in the tile's list) to the
// pixel's log; entries past the capacity are counted, not stored.
__device__ __forceinline__ void log_composite(const CompositeLog& lg, uint32_t tile, uint32_t& n, uint32_t local) {
    if (lg.ids == nullptr) return;
    if (n < lg.capacity) lg.ids[(size_t(n) * lg.tiles + tile) * kTileThreads + threadIdx.x] = uint16_t(local);
    ++n;
}

// Ends the pixel's log: stores its entry count and marks the tile for the
// backward's replay when a pixel composited more hits than the log holds or
// the tile holds more candidates (`candidates`) than a 16-bit entry can name.
__device__ __forceinline__ void log_finish(const CompositeLog& lg, uint32_t tile, uint32_t nlog, uint32_t candidates) {
    lg.count[size_t(tile) * kTileThreads + threadIdx.x] = min(nlog, lg.capacity);
    const int over = __syncthreads_or(nlog > lg.capacity || candidates > kLogTileCandidates);
    if (threadIdx.x == 0) {
        lg.overflow[tile] = over ? 1u : 0u;
        if (over) lg.overflowList[atomicAdd(lg.overflowCount, 1u)] = tile;
    }
}

// Front-to-back composite of one hit (reference gutKBufferRenderer.cuh:307-416);
// c.yzw is the particle's colour.
__device__ __forceinline__ void composite_fwd(PixelFwd& s, float ht, float ha, float4 c) {
    const float w = ha * s.T;
    s.hitT = s.hitT + ht * w;
    s.T = s.T * (1.0f - ha);
    if (w > 0.0f) {
        s.r = __fmaf_rn(fmaxf(c.y, 0.0f), w, s.r);
        s.g = __fmaf_rn(fmaxf(c.z, 0.0f), w, s.g);
        s.b = __fmaf_rn(fmaxf(c.w, 0.0f), w, s.b);
        s.hitN++;
    }
    if (s.T < kMinTransmittance) s.alive = false;
}

// ------------------------------------------------------------------ geometric channels
// Per-hit terms of the training channels, accumulated for every composited
// hit in composite order (reference processHitParticle,
// gutKBufferRenderer.cuh:330-392): w = alpha T_before,
//   normal    += w n,  n = -normalize(B^-T normalize(B^-1 d))
//                      (canonicalRayNormal, gaussianParticles.slang:254-265)
//   depth var += (w t) t
//   extent    += w |s * (R^T d)|   (intrinsic rotation and scale of the row,
//                      gaussianParticles.cuh:131-141; R from the quaternion)
//   inv depth += w / max(t s_d, 0.2), inv depth2 += w / max(t s_d, 0.2)^2
//                      (sofDistortionCoordinate, sensorConstants.cuh:28-42;
//                      s_d = sensor ray z for a pinhole, 1 for a fisheye)
//   quantiles: the first hit depth at which 1 - T_after reaches each of
//              0.05 .. 0.50; max-weight hit depth; the exact 0.5 crossing
//              (finiteIntervalExactCrossing.cuh:42-109) inside the Gaussian
//              that carries T across 0.5.
// Sums use explicit fused multiply-adds; exp, log, division and square root
// are the shared IEEE/elementary ones, so the oracle reproduces every value.
constexpr int kQuantiles = 7;
constexpr int kQuantStride = kQuantiles + 3;

__device__ __forceinline__ float quantile_threshold(int i) {
    return i == 0 ? 0.05f : i == 1 ? 0.10f : i == 2 ? 0.15f : i == 3 ? 0.20f : i == 4 ? 0.30f : i == 5 ? 0.40f : 0.50f;
}

struct PixelGeo {
    float n[3];
    float sumWD2, sumExt, sumInvD, sumInvD2;
    float q[kQuantiles];
    float tauMaxW, tauMaxD, exactDepth, exactRate;
    float dscale;
};

__device__ __forceinline__ void geo_init(PixelGeo& g, float dscale) {
    g.n[0] = g.n[1] = g.n[2] = 0.0f;
    g.sumWD2 = g.sumExt = g.sumInvD = g.sumInvD2 = 0.0f;
#pragma unroll
    for (int i = 0; i < kQuantiles; ++i) g.q[i] = 0.0f;
    g.tauMaxW = g.tauMaxD = g.exactDepth = g.exactRate = 0.0f;
    g.dscale = dscale;
}

// Along-ray standard deviation of the intrinsic shape: |s * (R^T d)|, with
// R^T rows from the quaternion (w, x, y, z) as quaternionWXYZToMatrix
// (gaussianParticles.cuh:55-75).
__device__ __forceinline__ V3 rotate_transpose(float4 q, V3 d) {
    const float r = q.x, x = q.y, y = q.z, z = q.w;
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z, rx = r * x, ry = r * y,
                rz = r * z;
    const V3 r0 = v3(1.0f - 2.0f * (yy + zz), 2.0f * (xy + rz), 2.0f * (xz - ry));
    const V3 r1 = v3(2.0f * (xy - rz), 1.0f - 2.0f * (xx + zz), 2.0f * (yz + rx));
    const V3 r2 = v3(2.0f * (xz + ry), 2.0f * (yz - rx), 1.0f - 2.0f * (xx + yy));
    return v3(fdot3(r0, d), fdot3(r1, d), fdot3(r2, d));
}

__device__ __forceinline__ float extent_sigma(float4 q, float4 sc, V3 d) {
    const V3 rd = rotate_transpose(q, d);
    const V3 sd = v3(sc.x * rd.x, sc.y * rd.y, sc.z * rd.z);
    return __fsqrt_rn(fdot3(sd, sd) + 1e-18f);
}

__device__ __forceinline__ float crossing_alpha(float AA, float BB, float CC, float density, float t) {
    const float qd = fmaxf(__fmaf_rn(__fmaf_rn(AA, t, BB), t, CC), 0.0f);
    return fminf(kMaxAlpha, density * gf_expf(-0.5f * qd));
}

// The 0.5-opacity crossing inside one Gaussian on the closed ray interval
// (finiteIntervalExactCrossing.cuh:42-109): alpha(t) = rho exp(-q(t)/2),
// q(t) = AA t^2 + BB t + CC, and T_before (1 - alpha(t)) = 0.5 at the near
// root; the rate is dO/dt there.  False when there is no crossing.
__device__ __forceinline__ bool exact_crossing(float AA, float BB, float CC, float density, float tBefore, float tmin,
                                               float tmax, float& depth, float& rate) {
    const float threshold = 0.5f;
    if (!(isfinite_f(AA) && isfinite_f(BB) && isfinite_f(CC) && isfinite_f(density) && isfinite_f(tBefore) &&
          isfinite_f(tmin) && isfinite_f(tmax)))
        return false;
    if (!(AA > 0.0f) || !(density > 0.0f) || !(tmax > tmin) || !(tBefore > threshold) || !(tBefore <= 1.0f))
        return false;
    const float tLine = -BB / (2.0f * AA);
    const float tPeak = fminf(fmaxf(tLine, tmin), tmax);
    const float peakAlpha = crossing_alpha(AA, BB, CC, density, tPeak);
    const float required = 1.0f - threshold / tBefore;
    if (!(required > 0.0f) || !(required < kMaxAlpha) || !(peakAlpha >= required)) return false;
    const float level = required / density;
    if (!(level > 0.0f) || !(level <= 1.0f) || !isfinite_f(level)) return false;
    const float con = CC + 2.0f * gf_logf(level);
    const float disc = BB * BB - (4.0f * AA) * con;
    if (!(disc >= 0.0f) || !isfinite_f(disc)) return false;
    const float nearRoot = (-BB - __fsqrt_rn(disc)) / (2.0f * AA);
    if (!isfinite_f(nearRoot)) return false;
    if (nearRoot <= tmin || nearRoot >= tmax) {
        const float edge = nearRoot <= tmin ? tmin : tmax;
        if (!(crossing_alpha(AA, BB, CC, density, edge) >= required)) return false;
        depth = edge;
        rate = 0.0f;
        return true;
    }
    const float r = -0.5f * (tBefore - threshold) * (2.0f * AA * nearRoot + BB);
    depth = nearRoot;
    rate = (disc == 0.0f || !isfinite_f(r) || !(r > 0.0f)) ? 0.0f : r;
    return true;
}

// One composited hit into the geometric channels.  rec: the particle's render
// record; row: its packed [N,32] row (quaternion, intrinsic scale).
__device__ __forceinline__ void geo_hit(PixelGeo& g, const Ray& ray, const Record& rec, const float* __restrict__ row,
                                        float hitT, float w, float tBefore, float tAfter) {
    const V3 grdu = binv_times(rec.b, rec.c, rec.d, ray.d);
    const float len = __fsqrt_rn(fdot3(grdu, grdu));
    const V3 grd = v3(grdu.x / len, grdu.y / len, grdu.z / len);
    // B^-T grd; B^-1 rows: r0 = (b.x b.y b.z), r1 = (b.w c.x c.y), r2 = (c.z c.w d.x)
    const V3 nu = v3(__fmaf_rn(rec.c.z, grd.z, __fmaf_rn(rec.b.w, grd.y, rec.b.x * grd.x)),
                     __fmaf_rn(rec.c.w, grd.z, __fmaf_rn(rec.c.x, grd.y, rec.b.y * grd.x)),
                     __fmaf_rn(rec.d.x, grd.z, __fmaf_rn(rec.c.y, grd.y, rec.b.z * grd.x)));
    const float inv = -1.0f / __fsqrt_rn(fdot3(nu, nu));
    g.n[0] = __fmaf_rn(w, inv * nu.x, g.n[0]);
    g.n[1] = __fmaf_rn(w, inv * nu.y, g.n[1]);
    g.n[2] = __fmaf_rn(w, inv * nu.z, g.n[2]);
    g.sumWD2 = __fmaf_rn(w * hitT, hitT, g.sumWD2);
    const float dd = hitT * g.dscale;
    const bool active = dd > kParticleMinSensorZ;
    const float invD = active ? 1.0f / dd : 1.0f / kParticleMinSensorZ;
    const float invD2 = active ? 1.0f / ((hitT * hitT) * (g.dscale * g.dscale))
                               : 1.0f / (kParticleMinSensorZ * kParticleMinSensorZ);
    g.sumInvD = __fmaf_rn(w, invD, g.sumInvD);
    g.sumInvD2 = __fmaf_rn(w, invD2, g.sumInvD2);
    g.sumExt = __fmaf_rn(w, extent_sigma(__ldg(reinterpret_cast<const float4*>(row + 4)),
                                         __ldg(reinterpret_cast<const float4*>(row + 8)), ray.d), g.sumExt);
    const float oAcc = 1.0f - tAfter;
#pragma unroll
    for (int i = 0; i < kQuantiles; ++i)
        if (g.q[i] == 0.0f && oAcc >= quantile_threshold(i)) g.q[i] = hitT;
    if (w > g.tauMaxW) {
        g.tauMaxW = w;
        g.tauMaxD = hitT;
    }
    if (g.exactDepth == 0.0f && tBefore > 0.5f && tAfter <= 0.5f) {
        const V3 gro = binv_times(rec.b, rec.c, rec.d, v3(ray.o.x - rec.a.x, ray.o.y - rec.a.y, ray.o.z - rec.a.z));
        float depth = hitT, rate = 0.0f;
        if (!exact_crossing(fdot3(grdu, grdu), 2.0f * fdot3(gro, grdu), fdot3(gro, gro), rec.a.w, tBefore, ray.tmin,
                            ray.tmax, depth, rate)) {
            depth = hitT;
            rate = 0.0f;
        }
        g.exactDepth = depth;
        g.exactRate = rate;
    }
}

__device__ __forceinline__ void geo_store(const GeoOut& o, size_t pix, const PixelGeo& g, bool valid) {
    if (o.normal != nullptr) {
        o.normal[3 * pix] = valid ? g.n[0] : 0.0f;
        o.normal[3 * pix + 1] = valid ? g.n[1] : 0.0f;
        o.normal[3 * pix + 2] = valid ? g.n[2] : 0.0f;
    }
    if (o.depthVar != nullptr) o.depthVar[pix] = valid ? g.sumWD2 : 0.0f;
    if (o.extent != nullptr) o.extent[pix] = valid ? g.sumExt : 0.0f;
    if (o.invD != nullptr) o.invD[pix] = valid ? g.sumInvD : 0.0f;
    if (o.invD2 != nullptr) o.invD2[pix] = valid ? g.sumInvD2 : 0.0f;
    if (o.quant != nullptr) {
        float* q = o.quant + size_t(kQuantStride) * pix;
#pragma unroll
        for (int i = 0; i < kQuantiles; ++i) q[i] = valid ? g.q[i] : 0.0f;
        q[kQuantiles] = valid ? g.tauMaxD : 0.0f;
        q[kQuantiles + 1] = valid ? g.exactDepth : 0.0f;
        q[kQuantiles + 2] = valid ? g.exactRate : 0.0f;
    }
}

__device__ __forceinline__ uint32_t id_at(const RenderArgs& a, const Batch& b, uint32_t sp) {
    const uint32_t j = sp - b.base;
    if (j < b.cnt) return b.ids[j];
    return __ldg(a.sortedIds + sp);
}

// The per-pixel rings follow `offset` bytes of staging.
__device__ __forceinline__ float2* ring_ta(unsigned char* smem, size_t offset) {
    return reinterpret_cast<float2*>(smem + offset);
}
template <int K>
__device__ __forceinline__ uint32_t* ring_id(unsigned char* smem, size_t offset) {
    return reinterpret_cast<uint32_t*>(smem + offset + sizeof(float2) * K * kTileThreads);
}

// Forward shared memory: two staging buffers of kFwdBatch records, ids and
// support radii, then the rings.
constexpr size_t kFwdStagingBytes = (sizeof(Staged) + 2 * sizeof(uint32_t)) * kFwdBatch * kFwdBuffers;
__host__ __device__ constexpr size_t fwd_smem_bytes(int K) {
    return kFwdStagingBytes + size_t(K > 0 ? K : 1) * kTileThreads * (sizeof(float2) + sizeof(uint32_t));
}

// Blocks per SM the forward is built for: four (64 registers a thread) when
// its shared memory allows them (K <= 16) and it carries no geometric
// channels, which would spill at 64 registers; else two.
__host__ __device__ constexpr int fwd_min_blocks(int K, bool geo) {
    return (!geo && fwd_smem_bytes(K) <= 55u * 1024u) ? 4 : 2;
}

template <int K, bool kGeo>
__global__ __launch_bounds__(kTileThreads, fwd_min_blocks(K, kGeo)) void k_render_fwd(RenderArgs a, float* __restrict__ rgba,
                                                                                 float* __restrict__ hitDistance,
                                                                                 float* __restrict__ hitCount) {
    constexpr int KR = K > 0 ? K : 1;
    extern __shared__ __align__(16) unsigned char smem[];
    // staging buffer b: sRec[b * kFwdBatch + j], sIdB[b * kFwdBatch + j], sBound[b * kFwdBatch + j]
    Staged* sRec = reinterpret_cast<Staged*>(smem);
    uint32_t* sIdB = reinterpret_cast<uint32_t*>(smem + sizeof(Staged) * kFwdBatch * kFwdBuffers);
    float* sBound = reinterpret_cast<float*>(sIdB + kFwdBatch * kFwdBuffers);
    const bool retained = a.mask[blockIdx.x] != 0u;
    const TileSetup ts = tile_setup(a, retained, int(blockIdx.x));
    PixelFwd s{1.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0u, ts.ray.valid};
    RingKBuffer<KR> kb;
    kb.init(ring_ta(smem, kFwdStagingBytes), ring_id<KR>(smem, kFwdStagingBytes), threadIdx.x);
    Batch bt{sRec, sIdB, 0u, 0u};
    uint32_t nlog = 0, candidates = 0;
    PixelGeo geo;
    if constexpr (kGeo) {
        const bool pinhole = a.f.cam.model == GF_CAMERA_OPENCV_PINHOLE;
        geo_init(geo, (pinhole && ts.inImage && retained) ? a.rayD[3 * ts.pix + 2] : 1.0f);
    }
    // one composited hit into the geometric channels (T before and after it)
    auto geoHit = [&](uint32_t id, float ht, float ha, float tBefore) {
        if constexpr (kGeo) {
            const Record rec = load_record(a.records, id);
            geo_hit(geo, ts.ray, rec, a.geo.particles + 32 * size_t(id), ht, ha * tBefore, tBefore, s.T);
        }
    };
    if (retained) {
        const uint2 range = a.ranges[ts.tile];
        candidates = range.y - range.x;
        // composites one staged batch: `cnt` candidates from sorted position `base`
        auto runBatch = [&](const Staged* cur, const uint32_t* ids, uint32_t base, int cnt) {
            bt.rec = cur;
            bt.ids = ids;
            bt.base = base;
            bt.cnt = uint32_t(cnt);
            const int words = (cnt + 31) >> 5;
#pragma unroll 1
            for (int k = 0; k < words && __any_sync(0xffffffffu, s.alive); ++k) {
                uint32_t m = warp_mask(ts, cur, cnt, k);
                while (m != 0u && s.alive) {
                    const int j = k * 32 + __ffs(m) - 1;
                    m &= m - 1u;
                    float alpha, ht;
                    if (hit_staged<true>(ts, cur[j], alpha, ht)) {
                        if constexpr (K == 0) {
                            log_composite(a.log, uint32_t(ts.tile), nlog, base + uint32_t(j) - range.x);
                            const float tBefore = s.T;
                            composite_fwd(s, ht, alpha, cur[j].d);
                            geoHit(bt.ids[j], ht, alpha, tBefore);
                        } else {
                            if (kb.full()) {
                                float t0, a0;
                                uint32_t s0;
                                kb.pop_front(t0, a0, s0);
                                log_composite(a.log, uint32_t(ts.tile), nlog, s0 - range.x);
                                const float tBefore = s.T;
                                composite_fwd(s, t0, a0, color_at(a, bt, s0));
                                if constexpr (kGeo) geoHit(id_at(a, bt, s0), t0, a0, tBefore);
                            }
                            kb.insert(ht, alpha, base + uint32_t(j));
                        }
                    }
                }
            }
        };
        if constexpr (fwd_min_blocks(K, kGeo) == 2) {
            // Two-block kernels (K > 16 or the geometric channels) stage
            // both buffers' room as one batch of 64, synchronously: at 16
            // warps per SM the asynchronous double buffer was slower (K = 32:
            // 17.24 ms per 2560^2 inference frame against 16.64 ms).
            constexpr int kBatch64 = kFwdBatch * kFwdBuffers;
            for (uint32_t base = range.x; base < range.y; base += kBatch64) {
                if (__syncthreads_and(!s.alive)) break;
                const uint32_t sIdx = base + threadIdx.x;
                if (threadIdx.x < kBatch64 && sIdx < range.y) {
                    sIdB[threadIdx.x] = __ldg(a.sortedIds + sIdx);
                    stage<true>(a, ts, sIdx, sRec[threadIdx.x]);
                }
                __syncthreads();
                runBatch(sRec, sIdB, base, int(min(uint32_t(kBatch64), range.y - base)));
            }
        } else {
            // The first warp stages: candidate base + lane of each batch.  It
            // holds the id of the batch after the one in flight in a register.
            const bool stager = threadIdx.x < kFwdBatch;
            uint32_t nextId = 0u;
            if (stager) {
                const uint32_t i0 = range.x + threadIdx.x;
                if (i0 < range.y) {
                    const uint32_t id = __ldg(a.sortedIds + i0);
                    sIdB[threadIdx.x] = id;
                    fetch_async(a, id, sRec[threadIdx.x], sBound[threadIdx.x]);
                }
                cp_async_commit();
                const uint32_t i1 = i0 + kFwdBatch;
                if (i1 < range.y) nextId = __ldg(a.sortedIds + i1);
            }
            int buf = 0;
            for (uint32_t base = range.x; base < range.y; base += kFwdBatch, buf ^= 1) {
                Staged* cur = sRec + buf * kFwdBatch;
                if (stager) {
                    // this batch's copies have landed: add the derived fields
                    cp_async_wait_all();
                    if (base + threadIdx.x < range.y) derive(ts, cur[threadIdx.x], sBound[buf * kFwdBatch + threadIdx.x]);
                }
                // publishes the batch; every warp is done with the other buffer
                if (__syncthreads_and(!s.alive)) break;
                if (stager) {
                    const int nb = buf ^ 1;
                    const uint32_t i1 = base + kFwdBatch + threadIdx.x;
                    if (i1 < range.y) {
                        sIdB[nb * kFwdBatch + threadIdx.x] = nextId;
                        fetch_async(a, nextId, sRec[nb * kFwdBatch + threadIdx.x], sBound[nb * kFwdBatch + threadIdx.x]);
                    }
                    cp_async_commit();
                    const uint32_t i2 = i1 + kFwdBatch;
                    nextId = i2 < range.y ? __ldg(a.sortedIds + i2) : 0u;
                }
                runBatch(cur, sIdB + buf * kFwdBatch, base, int(min(uint32_t(kFwdBatch), range.y - base)));
            }
            if (stager) cp_async_wait_all();  // no copy outlives the block
        }
        if constexpr (K > 0) {
            for (int i = 0; s.alive && i < kb.n; ++i) {
                float ht, ha;
                uint32_t sp;
                kb.entry(i, ht, ha, sp);
                log_composite(a.log, uint32_t(ts.tile), nlog, sp - range.x);
                const float tBefore = s.T;
                composite_fwd(s, ht, ha, color_at(a, bt, sp));
                if constexpr (kGeo) geoHit(id_at(a, bt, sp), ht, ha, tBefore);
            }
        }
    }
    if (a.log.ids != nullptr) log_finish(a.log, uint32_t(ts.tile), nlog, candidates);
    if (!ts.inImage) return;
    float4 out = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float hd = 1e06f, hc = 0.0f;
    if (ts.ray.valid) {
        out = make_float4(s.r, s.g, s.b, 1.0f - s.T);
        hd = s.hitT;
        hc = float(s.hitN);
    }
    reinterpret_cast<float4*>(rgba)[ts.pix] = out;
    hitDistance[ts.pix] = hd;
    if (hitCount != nullptr) hitCount[ts.pix] = hc;
    if constexpr (kGeo) geo_store(a.geo, ts.pix, geo, ts.ray.valid);
}

// ------------------------------------------------------------------ backward
struct PixelBwd {
    float T, depth;
    float r, g, b;
    float featB[3], featG[3];
    float TB, TG, hitTB, hitTG;
    bool alive;
};

// Geometric channels in the backward: running sums (re-accumulated exactly as
// the forward accumulated them), the forward's final values and the output
// gradients (rayPayloadBackward.cuh:110-150).
struct PixelGeoBwd {
    float n[3], wd2;                          // running (the channels whose residuals reach alpha)
    float nB[3], wd2B;                        // forward outputs
    float nG[3], wd2G, extG, invDG, invD2G;   // output gradients
    float dscale;
    float crossG, crossT;                     // -(dL/dt*) / (dO/dt at t*) and the crossing depth t* (0: none)
};

__device__ __forceinline__ void geo_bwd_init(PixelGeoBwd& g, const GeoBwd& a, size_t pix, float dscale) {
    const auto val = [&](const float* p, size_t i) { return p != nullptr ? p[i] : 0.0f; };
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        g.n[k] = 0.0f;
        g.nB[k] = val(a.normal, 3 * pix + k);
        g.nG[k] = a.normal != nullptr ? val(a.gradNormal, 3 * pix + k) : 0.0f;
    }
    g.wd2 = 0.0f;
    g.wd2B = val(a.depthVar, pix);
    g.wd2G = a.depthVar != nullptr ? val(a.gradDepthVar, pix) : 0.0f;
    g.extG = val(a.gradExtent, pix);
    g.invDG = val(a.gradInvD, pix);
    g.invD2G = val(a.gradInvD2, pix);
    g.dscale = dscale;
    // the crossing depth's gradient scale (rayPayloadBackward.cuh:122-128)
    g.crossG = 0.0f;
    g.crossT = 0.0f;
    if (a.quant != nullptr && a.gradQuant != nullptr) {
        const float t = a.quant[size_t(kQuantStride) * pix + kQuantiles + 1];
        const float rate = a.quant[size_t(kQuantStride) * pix + kQuantiles + 2];
        const float dLdt = a.gradQuant[size_t(kQuantStride) * pix + kQuantiles + 1];
        if (fabsf(rate) > 1e-8f && t > 0.0f) {
            g.crossG = -dLdt / rate;
            g.crossT = t;
        }
    }
}

// d/dv of v / |v| applied to the output gradient go (safe_normalize_bw,
// mathUtils.cuh:411-421): go / |v| - v (v . go) / |v|^3; zero for v = 0.
__device__ __forceinline__ V3 normalize_vjp(V3 v, V3 go) {
    const float l = v.x * v.x + v.y * v.y + v.z * v.z;
    if (!(l > 0.0f)) return v3(0.0f, 0.0f, 0.0f);
    const float il = 1.0f / __fsqrt_rn(l);
    const float il3 = il * il * il;
    return v3(il * go.x - il3 * (go.x * (v.x * v.x) + go.y * (v.y * v.x) + go.z * (v.z * v.x)),
              il * go.y - il3 * (go.x * (v.x * v.y) + go.y * (v.y * v.y) + go.z * (v.z * v.y)),
              il * go.z - il3 * (go.x * (v.x * v.z) + go.y * (v.y * v.z) + go.z * (v.z * v.z)));
}

// Gradient with respect to the quaternion (w, x, y, z) of y = M(q) p, where
// M's rows are those of rotate_transpose, for dL/dy = go.
__device__ __forceinline__ float4 rotate_transpose_vjp(float4 q, V3 p, V3 go) {
    const float r = q.x, x = q.y, y = q.z, z = q.w;
    const float G00 = go.x * p.x, G01 = go.x * p.y, G02 = go.x * p.z;
    const float G10 = go.y * p.x, G11 = go.y * p.y, G12 = go.y * p.z;
    const float G20 = go.z * p.x, G21 = go.z * p.y, G22 = go.z * p.z;
    const float dr = 2.0f * (z * G01 - y * G02 - z * G10 + x * G12 + y * G20 - x * G21);
    const float dx = 2.0f * (y * G01 + z * G02 + y * G10 + r * G12 + z * G20 - r * G21) - 4.0f * x * (G11 + G22);
    const float dy = 2.0f * (x * G01 - r * G02 + x * G10 + z * G12 + r * G20 + z * G21) - 4.0f * y * (G00 + G22);
    const float dz = 2.0f * (r * G01 + x * G02 - r * G10 + y * G12 + x * G20 + y * G21) - 4.0f * z * (G00 + G11);
    return make_float4(dr, dx, dy, dz);
}

// Gradient of one composited hit (reference processHitBwd,
// gaussianParticles.cuh:736-1155, geometric channels inactive).  The hit is
// evaluated here with the forward hit test's exact arithmetic
// (hit_with_origin: the same closest point, response and alpha, so the same
// tau and alpha the forward composited) and back-propagated in the same
// pass.  The walking state (T, depth, colour) advances with the forward's
// exact arithmetic; quotients that only scale gradients use fast
// reciprocals.  Returns false (state unchanged) when the candidate is not a
// hit, which a composited entry always is.
template <bool kGeo = false>
__device__ __forceinline__ bool hit_vjp(PixelBwd& s, const Ray& ray, const Record& q, float4 g[4],
                                        PixelGeoBwd* geo = nullptr, const float* row = nullptr,
                                        float4* gShape = nullptr) {
    const V3 gp = v3(ray.o.x - q.a.x, ray.o.y - q.a.y, ray.o.z - q.a.z);
    const V3 gro = binv_times(q.b, q.c, q.d, gp);
    const V3 grdu = binv_times(q.b, q.c, q.d, ray.d);
    const float denom = fdot3(grdu, grdu);
    // callers test valid rays only, and make_ray's valid (tmax > tmin, tmin =
    // max(., 0)) already means a finite tmin below tmax
    if (!(denom > 0.0f && isfinite_f(denom))) return false;
    const float num = fdot3(gro, grdu);
    const float tauLine = -num / denom;
    const float tau = fminf(fmaxf(tauLine, ray.tmin), ray.tmax);
    const V3 p = v3(__fmaf_rn(tau, grdu.x, gro.x), __fmaf_rn(tau, grdu.y, gro.y), __fmaf_rn(tau, grdu.z, gro.z));
    const float grayDist = fdot3(p, p);
    if (grayDist > kResponseCutoff2) return false;
    const float gres = gf_expf(-0.5f * grayDist);
    const float density = q.a.w;
    const float galphaU = gres * density;
    const float galpha = fminf(kMaxAlpha, galphaU);
    if (!(gres > kMinKernelResponse && galpha > kAlphaThreshold && tau >= ray.tmin && tau <= ray.tmax)) return false;
    const bool interior = tau > ray.tmin && tau < ray.tmax;
    const float gdist = tau;
    const float weight = galpha * s.T;
    const float nextT = (1.0f - galpha) * s.T;
    s.depth = s.depth + gdist * weight;
    const bool tail = nextT <= kMinTransmittance;
    const float invNext = tail ? 0.0f : __fdividef(1.0f, nextT);
    // From here on the values only scale gradients (compared with tolerances,
    // not bit for bit): products and sums are fused where they pair up.
    const float residualHitT = fmaxf((s.hitTB - s.depth) * invNext, 0.0f);
    const float galphaRayHitGrd = (gdist - residualHitT) * s.T * s.hitTG;
    const float residualTrm = galpha < 0.999999f ? s.TB * __fdividef(1.0f, 1.0f - galpha) : s.T;
    const float cr = fmaxf(q.d.y, 0.0f), cg = fmaxf(q.d.z, 0.0f), cb = fmaxf(q.d.w, 0.0f);
    s.r = __fmaf_rn(cr, weight, s.r);
    s.g = __fmaf_rn(cg, weight, s.g);
    s.b = __fmaf_rn(cb, weight, s.b);
    const float rr = fmaxf((s.featB[0] - s.r) * invNext, 0.0f);
    const float rg = fmaxf((s.featB[1] - s.g) * invNext, 0.0f);
    const float rb = fmaxf((s.featB[2] - s.b) * invNext, 0.0f);
    float comp = __fmaf_rn(residualTrm, -s.TG, galphaRayHitGrd);
    const float colourGrad = __fmaf_rn(cb - rb, s.featG[2], __fmaf_rn(cg - rg, s.featG[1], (cr - rr) * s.featG[0]));
    comp = __fmaf_rn(s.T, colourGrad, comp);
    float tauGrad = weight * s.hitTG;
    // Geometric channels (gaussianParticles.cuh:786-1062): the depth moment
    // and the normal sum reach alpha through their residuals; the depth moment
    // and the inverse-depth moments reach tau; the normal reaches B^-1 and the
    // ray's canonical direction; the extent reaches the intrinsic rotation and
    // scale only.
    V3 grduGeo = v3(0.0f, 0.0f, 0.0f);
    float gBinvN[9];
    if constexpr (kGeo) {
        PixelGeoBwd& G = *geo;
        const float gsq = gdist * gdist;
        G.wd2 = __fmaf_rn(weight * gdist, gdist, G.wd2);
        const float residualWD2 = fmaxf((G.wd2B - G.wd2) * invNext, 0.0f);
        comp += (gsq - residualWD2) * s.T * G.wd2G;
        tauGrad += 2.0f * gdist * weight * G.wd2G;
        // inverse-depth moments (detached from alpha)
        const float dd = gdist * G.dscale;
        const bool active = dd > kParticleMinSensorZ;
        if (active) {
            tauGrad += (-weight / (G.dscale * gdist * gdist)) * G.invDG;
            tauGrad += (-2.0f * weight / ((G.dscale * G.dscale) * gdist * gdist * gdist)) * G.invD2G;
        }
        // normal n = -normalize(B^-T normalize(grdu))
        const float len = __fsqrt_rn(denom);
        const V3 grd = v3(grdu.x / len, grdu.y / len, grdu.z / len);
        const V3 nu = v3(__fmaf_rn(q.c.z, grd.z, __fmaf_rn(q.b.w, grd.y, q.b.x * grd.x)),
                         __fmaf_rn(q.c.w, grd.z, __fmaf_rn(q.c.x, grd.y, q.b.y * grd.x)),
                         __fmaf_rn(q.d.x, grd.z, __fmaf_rn(q.c.y, grd.y, q.b.z * grd.x)));
        const float inv = -1.0f / __fsqrt_rn(fdot3(nu, nu));
        const V3 n = v3(inv * nu.x, inv * nu.y, inv * nu.z);
        G.n[0] = __fmaf_rn(weight, n.x, G.n[0]);
        G.n[1] = __fmaf_rn(weight, n.y, G.n[1]);
        G.n[2] = __fmaf_rn(weight, n.z, G.n[2]);
        const V3 resN = tail ? v3(0.0f, 0.0f, 0.0f)
                             : v3((G.nB[0] - G.n[0]) * invNext, (G.nB[1] - G.n[1]) * invNext,
                                  (G.nB[2] - G.n[2]) * invNext);
        comp += s.T * ((n.x - resN.x) * G.nG[0] + (n.y - resN.y) * G.nG[1] + (n.z - resN.z) * G.nG[2]);
        const V3 nuGrd = normalize_vjp(nu, v3(-weight * G.nG[0], -weight * G.nG[1], -weight * G.nG[2]));
        // nu_j = sum_i B^-1[i][j] grd_i: d/dB^-1[i][j] = grd_i nuGrd_j; d/dgrd = B^-1 nuGrd
        const float gd[3] = {grd.x, grd.y, grd.z};
        const float ng[3] = {nuGrd.x, nuGrd.y, nuGrd.z};
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) gBinvN[3 * i + j] = gd[i] * ng[j];
        const V3 grdGrd = binv_times(q.b, q.c, q.d, nuGrd);
        grduGeo = normalize_vjp(grdu, grdGrd);
        // extent sigma = |s * (R^T d)|
        const float4 quat = __ldg(reinterpret_cast<const float4*>(row + 4));
        const float4 sc = __ldg(reinterpret_cast<const float4*>(row + 8));
        const V3 rd = rotate_transpose(quat, ray.d);
        const V3 sd = v3(sc.x * rd.x, sc.y * rd.y, sc.z * rd.z);
        const float sigma = __fsqrt_rn(fdot3(sd, sd) + 1e-18f);
        const float nG = (weight * G.extG) / sigma;
        const V3 rdGrd = v3(nG * (sc.x * sc.x * rd.x), nG * (sc.y * sc.y * rd.y), nG * (sc.z * sc.z * rd.z));
        gShape[0] = rotate_transpose_vjp(quat, ray.d, rdGrd);
        gShape[1] = make_float4(nG * (sc.x * rd.x * rd.x), nG * (sc.y * rd.y * rd.y), nG * (sc.z * rd.z * rd.z), 0.0f);
    }
    // The exact 0.5-crossing depth t* by the implicit function theorem
    // (gaussianParticles.cuh:934-986): F = T_before (1 - alpha_k(t)) - 1/2 in
    // the crossing Gaussian k, so dL/dtheta = g dO/dtheta at t*, g = -(dL/dt*)
    // / Odot*.  Hits before the crossing add g * 0.5 / (1 - alpha_i) to their
    // alpha gradient; the crossing hit differentiates its alpha at t* (its
    // canonical point gro + t* grdu, with its own cap mask); later hits add
    // nothing.
    float crossDensity = 0.0f;
    V3 groCross = v3(0.0f, 0.0f, 0.0f), grduCross = v3(0.0f, 0.0f, 0.0f);
    if constexpr (kGeo) {
        const PixelGeoBwd& G = *geo;
        if (G.crossG != 0.0f && s.T > 0.5f) {
            if (nextT > 0.5f) {
                comp += G.crossG * fminf(0.5f / fmaxf(1.0f - galpha, 1.0f - kMaxAlpha), 1.0f);
            } else {
                const float ts = G.crossT;
                const float AA = fdot3(grdu, grdu), BB = 2.0f * fdot3(gro, grdu), CC = fdot3(gro, gro);
                const float gd = fmaxf(AA * ts * ts + BB * ts + CC, 0.0f);
                const float gr = gf_expf(-0.5f * gd);
                const float aU = gr * density;
                const float aC = fminf(kMaxAlpha, aU);
                const float dLda = G.crossG * fminf(0.5f / fmaxf(1.0f - aC, 1.0f - kMaxAlpha), 1.0f);
                const float capC = aU < kMaxAlpha ? 1.0f : 0.0f;
                crossDensity = capC * dLda * gr;
                const float dgd = capC * dLda * density * (-0.5f * gr);
                grduCross = v3(dgd * 2.0f * (ts * ts * grdu.x + ts * gro.x), dgd * 2.0f * (ts * ts * grdu.y + ts * gro.y),
                               dgd * 2.0f * (ts * ts * grdu.z + ts * gro.z));
                groCross = v3(dgd * 2.0f * (ts * grdu.x + gro.x), dgd * 2.0f * (ts * grdu.y + gro.y),
                              dgd * 2.0f * (ts * grdu.z + gro.z));
            }
        }
    }
    const float gU = (galphaU < kMaxAlpha ? 1.0f : 0.0f) * comp;
    const float gDensity = gres * gU + crossDensity;
    const float gresGrd = density * gU;
    const float grayDistGrd = -0.5f * gres * gresGrd;
    // Closest-point VJP (reference gutHalfRayResponse.cuh:39-62).
    const float pg = 2.0f * grayDistGrd;
    V3 groGrd = v3(pg * p.x, pg * p.y, pg * p.z);
    V3 grduGrd = v3(tau * groGrd.x, tau * groGrd.y, tau * groGrd.z);
    const float totalTauGrad = __fmaf_rn(groGrd.z, grdu.z, __fmaf_rn(groGrd.y, grdu.y, __fmaf_rn(groGrd.x, grdu.x, tauGrad)));
    if (interior) {
        const float invDen = __fdividef(1.0f, denom);
        // tau = -num / denom: dtau/dgro = -grdu / denom, dtau/dgrdu = -gro / denom + 2 num grdu / denom^2
        const float a = -totalTauGrad * invDen;
        const float b = (2.0f * num) * (invDen * invDen) * totalTauGrad;
        groGrd = v3(__fmaf_rn(a, grdu.x, groGrd.x), __fmaf_rn(a, grdu.y, groGrd.y), __fmaf_rn(a, grdu.z, groGrd.z));
        grduGrd = v3(__fmaf_rn(b, grdu.x, __fmaf_rn(a, gro.x, grduGrd.x)),
                     __fmaf_rn(b, grdu.y, __fmaf_rn(a, gro.y, grduGrd.y)),
                     __fmaf_rn(b, grdu.z, __fmaf_rn(a, gro.z, grduGrd.z)));
    }
    if constexpr (kGeo) {
        groGrd = v3(groGrd.x + groCross.x, groGrd.y + groCross.y, groGrd.z + groCross.z);
        grduGrd = v3(grduGrd.x + grduCross.x, grduGrd.y + grduCross.y, grduGrd.z + grduCross.z);
    }
    // Binv rows: r0 = (b.x b.y b.z), r1 = (b.w c.x c.y), r2 = (c.z c.w d.x).
    const float gpx = -__fmaf_rn(groGrd.z, q.c.z, __fmaf_rn(groGrd.y, q.b.w, groGrd.x * q.b.x));
    const float gpy = -__fmaf_rn(groGrd.z, q.c.w, __fmaf_rn(groGrd.y, q.c.x, groGrd.x * q.b.y));
    const float gpz = -__fmaf_rn(groGrd.z, q.d.x, __fmaf_rn(groGrd.y, q.c.y, groGrd.x * q.b.z));
    const float m00 = __fmaf_rn(grduGrd.x, ray.d.x, groGrd.x * gp.x), m01 = __fmaf_rn(grduGrd.x, ray.d.y, groGrd.x * gp.y),
                m02 = __fmaf_rn(grduGrd.x, ray.d.z, groGrd.x * gp.z);
    const float m10 = __fmaf_rn(grduGrd.y, ray.d.x, groGrd.y * gp.x), m11 = __fmaf_rn(grduGrd.y, ray.d.y, groGrd.y * gp.y),
                m12 = __fmaf_rn(grduGrd.y, ray.d.z, groGrd.y * gp.z);
    const float m20 = __fmaf_rn(grduGrd.z, ray.d.x, groGrd.z * gp.x), m21 = __fmaf_rn(grduGrd.z, ray.d.y, groGrd.z * gp.y),
                m22 = __fmaf_rn(grduGrd.z, ray.d.z, groGrd.z * gp.z);
    g[0] = make_float4(gpx, gpy, gpz, gDensity);
    g[1] = make_float4(m00, m01, m02, m10);
    g[2] = make_float4(m11, m12, m20, m21);
    g[3] = make_float4(m22, s.featG[0] * weight, s.featG[1] * weight, s.featG[2] * weight);
    if constexpr (kGeo) {
        // the normal's B^-1 term and its canonical-direction term through grdu = B^-1 d
        g[1].x += gBinvN[0] + grduGeo.x * ray.d.x;
        g[1].y += gBinvN[1] + grduGeo.x * ray.d.y;
        g[1].z += gBinvN[2] + grduGeo.x * ray.d.z;
        g[1].w += gBinvN[3] + grduGeo.y * ray.d.x;
        g[2].x += gBinvN[4] + grduGeo.y * ray.d.y;
        g[2].y += gBinvN[5] + grduGeo.y * ray.d.z;
        g[2].z += gBinvN[6] + grduGeo.z * ray.d.x;
        g[2].w += gBinvN[7] + grduGeo.z * ray.d.y;
        g[3].x += gBinvN[8] + grduGeo.z * ray.d.z;
    }
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

// Lane offsets of the gradient merge tree: horizontal pairs, then vertical
// pairs (lane = 8 y + x over the warp's 8x4 pixel block).  On the bench view a
// third level (horizontal pairs of those) made the backward 4% slower and five
// levels 13% slower: they cost more shuffles than they save atomics.
constexpr int kMergeLevels = 2;
__host__ __device__ constexpr int merge_offset(int level) { return level == 0 ? 1 : 8; }

// Warp-aggregated accumulation of one gradient per lane: when every active
// lane of the warp holds the same particle the 16 components are reduced
// with shuffles and written by one lane; otherwise lanes holding the same
// particle are summed along a merge tree of neighbouring pixels, and each
// remaining lane adds its own (vector red.global.add of 4 floats).
// Neighbouring pixels composite the same particle in the same step often (44%
// of the hits on the 1M-Gaussian bench view are in such a horizontal pair),
// and same-address atomics of one instruction serialise in L2.
__device__ __forceinline__ void accumulate_grad(float4* __restrict__ gradRecords, bool have, uint32_t idx,
                                                float4 g[4]) {
    const uint32_t hm = __ballot_sync(0xffffffffu, have);
    if (hm == 0u) return;
    const int lane = threadIdx.x & 31;
    const int leader = __ffs(hm) - 1;
    const uint32_t leaderIdx = __shfl_sync(0xffffffffu, idx, leader);
    const bool uniform = __all_sync(0xffffffffu, !have || idx == leaderIdx);
    if (uniform && __popc(hm) > 1) {
        // Reduce-scatter over the warp: at each level the lane pair (lane,
        // lane ^ o) splits the components it still holds, each keeping one
        // half and adding its partner's copy of that half (16 + 8 + 4 + 2
        // shuffles), then the last pair adds its one component; lane 2c
        // ends with component c of the warp's sum and the 16 lanes add their
        // components with one instruction.
        float v[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[4 * k] = have ? g[k].x : 0.0f;
            v[4 * k + 1] = have ? g[k].y : 0.0f;
            v[4 * k + 2] = have ? g[k].z : 0.0f;
            v[4 * k + 3] = have ? g[k].w : 0.0f;
        }
#pragma unroll
        for (int half = 8, o = 16; half >= 1; half >>= 1, o >>= 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < half; ++i) {
                const float keep = upper ? v[i + half] : v[i];
                const float send = upper ? v[i] : v[i + half];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        const float total = v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
        if ((lane & 1) == 0) atomicAdd(reinterpret_cast<float*>(gradRecords + 4 * size_t(leaderIdx)) + (lane >> 1), total);
    } else {
        // Merge tree over the 8x4 pixel block: at each level (horizontal pairs,
        // vertical pairs, then pairs of those) two lanes that own sums for the
        // same particle add them in the lane with the offset bit clear.
        float4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = g[k];
        bool own = have;
#pragma unroll
        for (int level = 0; level < kMergeLevels; ++level) {
            const int o = merge_offset(level);
            const uint32_t otherIdx = __shfl_xor_sync(0xffffffffu, idx, o);
            const bool otherOwn = __shfl_xor_sync(0xffffffffu, own ? 1 : 0, o) != 0;
            const bool merge = own && otherOwn && otherIdx == idx;
            if (!__any_sync(0xffffffffu, merge)) continue;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 w = make_float4(__shfl_xor_sync(0xffffffffu, v[k].x, o),
                                             __shfl_xor_sync(0xffffffffu, v[k].y, o),
                                             __shfl_xor_sync(0xffffffffu, v[k].z, o),
                                             __shfl_xor_sync(0xffffffffu, v[k].w, o));
                if (merge) v[k] = add4(v[k], w);
            }
            if (merge && (lane & o)) own = false;
        }
        if (own) {
            float4* dst = gradRecords + 4 * size_t(idx);
#pragma unroll
            for (int k = 0; k < 4; ++k) atomicAdd(dst + k, v[k]);
        }
    }
}

// The densification statistic of one composited hit per lane
// (gutKBufferRenderer.cuh:283-296): the absolute values of the hit's position
// gradient `gp` (screen mode: of the two rows of the particle's map times it),
// added to the particle's sums; a warp whose lanes all hold one particle adds
// its warp sums once.  Sums of absolute values are additive, so the warp sum
// gives the same statistic as per-lane additions.  The composite-log backward
// is instantiated with kAbs = false for backwards without the statistic, so
// their inner loop carries none of it.
template <bool kAbs = true>
__device__ __forceinline__ void accumulate_abs_grad(float* __restrict__ absGrad, int mode, bool have, uint32_t idx,
                                                    float4 gp) {
    if constexpr (!kAbs) return;
    if (absGrad == nullptr) return;  // kernel-uniform
    float v0 = 0.0f, v1 = 0.0f, v2 = 0.0f;
    if (have) {
        if (mode == GF_ABS_GRAD_SCREEN) {
            const float* row = absGrad + 8 * size_t(idx);
            v0 = fabsf(row[0] * gp.x + row[1] * gp.y + row[2] * gp.z);
            v1 = fabsf(row[3] * gp.x + row[4] * gp.y + row[5] * gp.z);
        } else {
            v0 = fabsf(gp.x);
            v1 = fabsf(gp.y);
            v2 = fabsf(gp.z);
        }
    }
    const uint32_t hm = __ballot_sync(0xffffffffu, have);
    if (hm == 0u) return;
    const int leader = __ffs(hm) - 1;
    const uint32_t leaderIdx = __shfl_sync(0xffffffffu, idx, leader);
    if (__all_sync(0xffffffffu, !have || idx == leaderIdx)) {
        v0 = warp_sum(v0);
        v1 = warp_sum(v1);
        v2 = warp_sum(v2);
        if ((threadIdx.x & 31) != leader) return;
    } else if (!have) {
        return;
    }
    if (mode == GF_ABS_GRAD_SCREEN) {
        atomicAdd(absGrad + 8 * size_t(idx) + 6, v0);
        atomicAdd(absGrad + 8 * size_t(idx) + 7, v1);
    } else {
        atomicAdd(absGrad + 3 * size_t(idx), v0);
        atomicAdd(absGrad + 3 * size_t(idx) + 1, v1);
        atomicAdd(absGrad + 3 * size_t(idx) + 2, v2);
    }
}

// Backward replay: the identical traversal and k-buffer, each composited hit
// back-propagated from the final pixel values.  Loops are warp-uniform so
// the gradient reduction can use full-warp shuffles.
template <int K, bool kGeo>
__device__ __forceinline__ void replay_tile(const RenderBwdArgs& a, unsigned char* smem, int tile) {
    constexpr int KR = K > 0 ? K : 1;
    Staged* sRec = reinterpret_cast<Staged*>(smem);
    uint32_t* sId = reinterpret_cast<uint32_t*>(smem + sizeof(Staged) * kBatch);
    if (a.r.mask[tile] == 0u) return;  // block-uniform
    const TileSetup ts = tile_setup(a.r, true, tile);
    const Ray& ray = ts.ray;
    PixelBwd s;
    s.T = 1.0f;
    s.depth = 0.0f;
    s.r = s.g = s.b = 0.0f;
    s.alive = ray.valid;
    if (ray.valid) {
        const float4 fo = reinterpret_cast<const float4*>(a.rgba)[ts.pix];
        const float4 go = reinterpret_cast<const float4*>(a.gradRgba)[ts.pix];
        s.featB[0] = fo.x; s.featB[1] = fo.y; s.featB[2] = fo.z;
        s.featG[0] = go.x; s.featG[1] = go.y; s.featG[2] = go.z;
        s.TB = 1.0f - fo.w;
        s.TG = -1.0f * go.w;
        s.hitTB = a.hitDistance[ts.pix];
        s.hitTG = a.gradHitDistance[ts.pix];
    }
    PixelGeoBwd geo;
    if constexpr (kGeo) {
        const bool pinhole = a.r.f.cam.model == GF_CAMERA_OPENCV_PINHOLE;
        geo_bwd_init(geo, a.geo, ray.valid ? ts.pix : 0, (pinhole && ray.valid) ? a.r.rayD[3 * ts.pix + 2] : 1.0f);
    }
    auto vjp = [&](const Record& q, uint32_t cid, float4* g) -> bool {
        if constexpr (kGeo) {
            float4 gs[2] = {};
            const bool h = hit_vjp<true>(s, ray, q, g, &geo, a.geo.particles + 32 * size_t(cid), gs);
            if (h) {
                atomicAdd(a.geo.gradShape + 2 * size_t(cid), gs[0]);
                atomicAdd(a.geo.gradShape + 2 * size_t(cid) + 1, gs[1]);
            }
            return h;
        } else {
            return hit_vjp(s, ray, q, g);
        }
    };
    RingKBuffer<KR> kb;
    constexpr size_t kRingOffset = (sizeof(Staged) + sizeof(uint32_t)) * kBatch;
    kb.init(ring_ta(smem, kRingOffset), ring_id<KR>(smem, kRingOffset), threadIdx.x);
    Batch bt{sRec, sId, 0u, 0u};
    const uint2 range = a.r.ranges[ts.tile];
    for (uint32_t base = range.x; base < range.y; base += kBatch) {
        if (__syncthreads_and(!s.alive)) break;
        const uint32_t sIdx = base + threadIdx.x;
        if (sIdx < range.y) {
            sId[threadIdx.x] = __ldg(a.r.sortedIds + sIdx);
            stage(a.r, ts, sIdx, sRec[threadIdx.x]);
        }
        __syncthreads();
        const int cnt = min(uint32_t(kBatch), range.y - base);
        bt.base = base;
        bt.cnt = uint32_t(cnt);
        const int words = (cnt + 31) >> 5;
        bool warpAlive = __any_sync(0xffffffffu, s.alive);
#pragma unroll 1
        for (int k = 0; k < words && warpAlive; ++k) {
            uint32_t m = warp_mask(ts, sRec, cnt, k);
            while (m != 0u) {
                warpAlive = __any_sync(0xffffffffu, s.alive);
                if (!warpAlive) break;
                const int j = k * 32 + __ffs(m) - 1;
                m &= m - 1u;
                bool have = false;
                uint32_t cid = kInvalidParticle;
                float4 g[4] = {};
                if (s.alive) {
                    float alpha, ht;
                    if (hit_staged(ts, sRec[j], alpha, ht)) {
                        if constexpr (K == 0) {
                            const Record q = record_at(a.r, bt, base + uint32_t(j), cid);
                            have = vjp(q, cid, g);
                        } else {
                            if (kb.full()) {
                                float t0, a0;
                                uint32_t s0;
                                kb.pop_front(t0, a0, s0);
                                const Record q = record_at(a.r, bt, s0, cid);
                                have = vjp(q, cid, g);
                            }
                            kb.insert(ht, alpha, base + uint32_t(j));
                        }
                        if (s.T < kMinTransmittance) s.alive = false;
                    }
                }
                accumulate_abs_grad(a.absGrad, a.absMode, have, cid, g[0]);
                accumulate_grad(a.gradRecords, have, cid, g);
            }
        }
    }
    if constexpr (K > 0) {
        for (int i = 0; i < K; ++i) {
            if (!__any_sync(0xffffffffu, s.alive && i < kb.n)) break;
            bool have = false;
            uint32_t cid = kInvalidParticle;
            float4 g[4] = {};
            if (s.alive && i < kb.n) {
                float ht, ha;
                uint32_t sp;
                kb.entry(i, ht, ha, sp);
                const Record q = record_at(a.r, bt, sp, cid);
                have = vjp(q, cid, g);
                if (s.T < kMinTransmittance) s.alive = false;
            }
            accumulate_abs_grad(a.absGrad, a.absMode, have, cid, g[0]);
            accumulate_grad(a.gradRecords, have, cid, g);
        }
    }
}

// Backward replay kernel: one block per tile, or, when the forward kept a
// composite log, a resident grid that walks the list of tiles whose log
// overflowed (usually empty).
template <int K, bool kGeo>
__global__ __launch_bounds__(kTileThreads, 3) void k_render_bwd(RenderBwdArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    if (a.r.log.ids == nullptr) {
        replay_tile<K, kGeo>(a, smem, int(blockIdx.x));
        return;
    }
    const uint32_t count = *a.r.log.overflowCount;
    for (uint32_t w = blockIdx.x; w < count; w += gridDim.x) {
        replay_tile<K, kGeo>(a, smem, int(a.r.log.overflowList[w]));
        __syncthreads();  // the next tile restages the shared batch
    }
}

// Backward from the composite log.  Each pixel re-evaluates only the hits the
// forward composited, in the logged order, with the forward's arithmetic
// (the canonical origin B^-1 (o - mu) of a central tile equals the per-pixel
// one bit for bit), and back-propagates them exactly as the replay does.
// The render records of the tile's first kBwdSlots candidates (read by every
// pixel that composites them) are staged in shared memory, one array per
// float4 of the record so that lanes reading different candidates spread
// over the banks; later candidates are read from global memory.  The next log
// entry is loaded one step ahead.  Gradients go to the particles' records
// with vector atomics (warp-reduced when every lane holds the same
// particle): neighbouring pixels often composite the same particle in the
// same step, and shared-memory atomics on one address serialise.  Tiles whose
// log overflowed are left to k_render_bwd.  The loop runs to the warp's
// longest log so that the gradient reduction can use full-warp shuffles.
constexpr int kBwdSlots = 512;

__host__ __device__ constexpr size_t bwd_log_smem_bytes() {
    return size_t(kBwdSlots) * (4 * sizeof(float4) + sizeof(uint32_t));
}

#ifndef GF_BWD_LOG_MIN_BLOCKS
#define GF_BWD_LOG_MIN_BLOCKS 3
#endif
template <bool kGeo, bool kAbs>
__global__ __launch_bounds__(kTileThreads, GF_BWD_LOG_MIN_BLOCKS) void k_render_bwd_log(RenderBwdArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    float4* sRec = reinterpret_cast<float4*>(smem);                                      // [4][kBwdSlots]
    uint32_t* sIds = reinterpret_cast<uint32_t*>(smem + 4 * sizeof(float4) * kBwdSlots);  // [kBwdSlots]
    const uint32_t tile = blockIdx.x;
    if (a.r.mask[tile] == 0u) return;                    // block-uniform
    const CompositeLog& lg = a.r.log;
    if (lg.overflow[tile] != 0u) return;                 // block-uniform
    const uint2 range = a.r.ranges[tile];
    const uint32_t staged = min(range.y - range.x, uint32_t(kBwdSlots));
    for (uint32_t j = threadIdx.x; j < staged; j += kTileThreads) {
        const uint32_t id = __ldg(a.r.sortedIds + range.x + j);
        sIds[j] = id;
        const Record q = load_record(a.r.records, id);
        sRec[j] = q.a;
        sRec[kBwdSlots + j] = q.b;
        sRec[2 * kBwdSlots + j] = q.c;
        sRec[3 * kBwdSlots + j] = q.d;
    }
    __syncthreads();
    const FrameArgs& f = a.r.f;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int px = int(tile % uint32_t(f.gx)) * kTile + (warp & 1) * 8 + (lane & 7);
    const int py = int(tile / uint32_t(f.gx)) * kTile + (warp >> 1) * 4 + (lane >> 3);
    const bool inImage = px < f.W && py < f.H;
    const size_t pix = size_t(px) + size_t(f.W) * size_t(py);
    Ray ray;
    ray.valid = false;
    ray.o = v3(0.0f, 0.0f, 0.0f);
    ray.d = v3(0.0f, 0.0f, 1.0f);
    ray.tmin = 0.0f;
    ray.tmax = 0.0f;
    if (inImage) {
        ray = make_ray(f.pose, v3(a.r.rayO[3 * pix], a.r.rayO[3 * pix + 1], a.r.rayO[3 * pix + 2]),
                       v3(a.r.rayD[3 * pix], a.r.rayD[3 * pix + 1], a.r.rayD[3 * pix + 2]));
    }
    PixelBwd s;
    s.T = 1.0f;
    s.depth = 0.0f;
    s.r = s.g = s.b = 0.0f;
    s.alive = ray.valid;
    uint32_t n = 0;
    if (ray.valid) {
        const float4 fo = reinterpret_cast<const float4*>(a.rgba)[pix];
        const float4 go = reinterpret_cast<const float4*>(a.gradRgba)[pix];
        s.featB[0] = fo.x; s.featB[1] = fo.y; s.featB[2] = fo.z;
        s.featG[0] = go.x; s.featG[1] = go.y; s.featG[2] = go.z;
        s.TB = 1.0f - fo.w;
        s.TG = -1.0f * go.w;
        s.hitTB = a.hitDistance[pix];
        s.hitTG = a.gradHitDistance[pix];
        n = lg.count[size_t(tile) * kTileThreads + threadIdx.x];
    }
    PixelGeoBwd geo;
    if constexpr (kGeo) {
        const bool pinhole = f.cam.model == GF_CAMERA_OPENCV_PINHOLE;
        geo_bwd_init(geo, a.geo, ray.valid ? pix : 0, (pinhole && ray.valid) ? a.r.rayD[3 * pix + 2] : 1.0f);
    }
    uint32_t warpN = n;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) warpN = max(warpN, __shfl_xor_sync(0xffffffffu, warpN, o));
    const uint16_t* entries = lg.ids + size_t(tile) * kTileThreads + threadIdx.x;
    const size_t stride = size_t(lg.tiles) * kTileThreads;
    uint32_t next = n > 0 ? __ldg(entries) : 0u;
#pragma unroll 1
    for (uint32_t i = 0; i < warpN; ++i) {
        const bool active = i < n && s.alive;
        const uint32_t local = next;
        if (i + 1 < n) next = __ldg(entries + (i + 1) * stride);
        bool have = false;
        uint32_t cid = kInvalidParticle;
        float4 g[4] = {};
        if (active) {
            Record q;
            if (local < staged) {
                cid = sIds[local];
                q.a = sRec[local];
                q.b = sRec[kBwdSlots + local];
                q.c = sRec[2 * kBwdSlots + local];
                q.d = sRec[3 * kBwdSlots + local];
            } else {
                cid = __ldg(a.r.sortedIds + range.x + local);
                q = load_record(a.r.records, cid);
            }
            if constexpr (kGeo) {
                float4 gs[2] = {};
                have = hit_vjp<true>(s, ray, q, g, &geo, a.geo.particles + 32 * size_t(cid), gs);
                if (have) {
                    atomicAdd(a.geo.gradShape + 2 * size_t(cid), gs[0]);
                    atomicAdd(a.geo.gradShape + 2 * size_t(cid) + 1, gs[1]);
                }
            } else {
                have = hit_vjp(s, ray, q, g);
            }
            if (s.T < kMinTransmittance) s.alive = false;
        }
        accumulate_abs_grad<kAbs>(a.absGrad, a.absMode, have, cid, g[0]);
        accumulate_grad(a.gradRecords, have, cid, g);
    }
}

}  // namespace gf
