// SOF's hierarchical compositor on sm_100a: per-pixel HEAD4 <- per-2x2 MID8
// <- per-4x4 TAIL64 (reference sofMid8Hierarchy.inl:161-598, the training
// renderer's default, render.splat.hierarchical_sort with
// sof_mid8_hierarchy).
//
// One CTA per 16x16 tile.  The tile's sorted candidates stream in chunks of
// 32 into the 16 TAIL windows (one per 4x4 pixel group, up to 64 entries),
// each ordered by (representative depth, position in the tile list): the
// maximum-response depth of the particle along the group's representative
// ray, the mean of the central 2x2 in-raster world rays (all of them when
// none).  A TAIL holding more than 32 entries emits its 16 nearest, twice per
// chunk; an emission reaches the four MID windows (one per 2x2 group, up to 8
// entries, keyed the same way with the 2x2 mean ray) under it in batches of
// 4; a MID holding more than 4 emits its 4 nearest, and every pixel of the
// group feeds them through its own HEAD, a k-buffer of 4 by exact hit
// distance (the flat renderer's ring).  At the end the TAILs drain in two
// emissions of up to 16, then the MIDs, then the HEADs.
//
// Layout: 16 threads per TAIL group rank its retained and new entries by
// counting (retained entries are sorted, so a retained entry's rank is its
// index plus the new entries below it), 4 threads per MID group the same way;
// windows live in shared memory.  The cascade is the same for every pixel of
// a group, so the pixels' state only decides which fed candidates they
// composite: when every pixel of the tile is done the tile stops, which does
// not change any output.  Forward and the backward replay of tiles whose
// composite log overflowed share the cascade (the replay's per-feed work is
// a gradient, accumulated with warp-wide shuffles, so every feed loop is
// warp-uniform).
#pragma once

#include "gf_render.cuh"

namespace gf {

constexpr int kSofTails = 16;     // 4x4 groups of a tile
constexpr int kSofMids = 64;      // 2x2 groups
constexpr int kSofTailCap = 64;
constexpr int kSofTailKeep = 32;  // a TAIL emits while it holds more than this
constexpr int kSofTailEmit = 16;
constexpr int kSofMidCap = 8;
constexpr int kSofMidEmit = 4;
constexpr int kSofHead = 4;
constexpr int kSofChunk = 32;

struct SofSmem {
    float tailKey[kSofTails][kSofTailCap];
    uint32_t tailPos[kSofTails][kSofTailCap];
    float midKey[kSofMids][kSofMidCap];
    uint32_t midPos[kSofMids][kSofMidCap];
    float mergeKey[kSofTails * kSofTailCap];
    uint32_t mergePos[kSofTails * kSofTailCap];
    float newKey[kSofTails][kSofChunk];
    uint32_t newPos[kSofTails][kSofChunk];
    uint32_t tailEmit[kSofTails][kSofTailEmit];
    uint32_t midEmit[kSofMids][kSofMidEmit];
    float4 tailRay[kSofTails][2];  // origin, direction
    float4 midRay[kSofMids][2];
    float4 pixO[kTileThreads];     // world ray origin per local pixel (row-major), w = in raster
    float4 pixD[kTileThreads];
    int tailCount[kSofTails];
    int tailEmitCount[kSofTails];
    int midCount[kSofMids];
    int midEmitCount[kSofMids];
    int emitted;
};

__host__ __device__ constexpr size_t sof_ring_offset() { return (sizeof(SofSmem) + 15) / 16 * 16; }
__host__ __device__ constexpr size_t sof_smem_bytes() {
    return sof_ring_offset() + size_t(kSofHead) * kTileThreads * (sizeof(float2) + sizeof(uint32_t));
}

__device__ __forceinline__ bool sof_less(float ka, uint32_t pa, float kb, uint32_t pb) {
    return ka < kb || (ka == kb && pa < pb);
}

// Mean of the listed rays: origin sum x (1 / count), direction d / sqrt(|d|^2)
// of the summed directions ((0, 0, 1) when degenerate).
__device__ __forceinline__ void sof_mean_ray(const SofSmem& sm, const int* idx, int count, float4 out[2]) {
    V3 o = v3(0.0f, 0.0f, 0.0f), d = v3(0.0f, 0.0f, 0.0f);
    for (int k = 0; k < count; ++k) {
        const float4 po = sm.pixO[idx[k]], pd = sm.pixD[idx[k]];
        o = v3(o.x + po.x, o.y + po.y, o.z + po.z);
        d = v3(d.x + pd.x, d.y + pd.y, d.z + pd.z);
    }
    const float inv = count > 0 ? 1.0f / float(count) : 0.0f;
    out[0] = count > 0 ? make_float4(o.x * inv, o.y * inv, o.z * inv, 0.0f) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float n2 = fdot3(d, d);
    if (!(n2 > 0.0f) || !isfinite_f(n2)) {
        out[1] = make_float4(0.0f, 0.0f, 1.0f, 0.0f);
    } else {
        const float inorm = 1.0f / sqrtf(n2);
        out[1] = make_float4(d.x * inorm, d.y * inorm, d.z * inorm, 0.0f);
    }
}

// Maximum-response depth along a representative ray (sofMid8Hierarchy.inl:95-129).
__device__ __forceinline__ float sof_depth(const Record& q, const float4 ray[2]) {
    const V3 co = binv_times(q.b, q.c, q.d, v3(ray[0].x - q.a.x, ray[0].y - q.a.y, ray[0].z - q.a.z));
    const V3 cd = binv_times(q.b, q.c, q.d, v3(ray[1].x, ray[1].y, ray[1].z));
    const float den = fdot3(cd, cd);
    const V3 delta = v3(q.a.x - ray[0].x, q.a.y - ray[0].y, q.a.z - ray[0].z);
    const float radial = sqrtf(fdot3(delta, delta));
    if (!(den > 0.0f) || !isfinite_f(den)) return radial;
    const float depth = -fdot3(co, cd) / den;
    return isfinite_f(depth) ? fmaxf(0.0f, depth) : radial;
}

// The cascade of one tile.  `feed(m, slot)` is called by every thread once
// per MID emission slot (slot < 4, warp-uniform: each thread tests whether
// its 2x2 group emitted that slot); `done()` (block-uniform after a barrier)
// lets the tile stop early.  Returns after the MID drain; the caller drains
// the HEADs.
template <typename Feed, typename Done>
__device__ __forceinline__ void sof_cascade(const RenderArgs& a, SofSmem& sm, const TileSetup& ts, uint2 range,
                                            Feed&& feed, Done&& done) {
    const int tid = threadIdx.x;
    const int lx = ts.px - (ts.tile % a.f.gx) * kTile, ly = ts.py - (ts.tile / a.f.gx) * kTile;
    const int local = ly * kTile + lx;
    sm.pixO[local] = make_float4(ts.ray.o.x, ts.ray.o.y, ts.ray.o.z, ts.inImage ? 1.0f : 0.0f);
    sm.pixD[local] = make_float4(ts.ray.d.x, ts.ray.d.y, ts.ray.d.z, 0.0f);
    if (tid < kSofTails) {
        sm.tailCount[tid] = 0;
        sm.tailEmitCount[tid] = 0;
    }
    if (tid < kSofMids) {
        sm.midCount[tid] = 0;
        sm.midEmitCount[tid] = 0;
    }
    __syncthreads();
    if (tid < kSofTails) {
        const int bx = (tid & 3) * 4, by = (tid >> 2) * 4;
        int idx[16];
        int n = 0;
        for (int oy = 1; oy <= 2; ++oy)
            for (int ox = 1; ox <= 2; ++ox)
                if (sm.pixO[(by + oy) * kTile + bx + ox].w != 0.0f) idx[n++] = (by + oy) * kTile + bx + ox;
        if (n == 0)
            for (int oy = 0; oy < 4; ++oy)
                for (int ox = 0; ox < 4; ++ox)
                    if (sm.pixO[(by + oy) * kTile + bx + ox].w != 0.0f) idx[n++] = (by + oy) * kTile + bx + ox;
        sof_mean_ray(sm, idx, n, sm.tailRay[tid]);
    } else if (tid < kSofTails + kSofMids) {
        const int m = tid - kSofTails;
        const int bx = (m & 7) * 2, by = (m >> 3) * 2;
        int idx[4];
        int n = 0;
        for (int oy = 0; oy < 2; ++oy)
            for (int ox = 0; ox < 2; ++ox)
                if (sm.pixO[(by + oy) * kTile + bx + ox].w != 0.0f) idx[n++] = (by + oy) * kTile + bx + ox;
        sof_mean_ray(sm, idx, n, sm.midRay[m]);
    }
    __syncthreads();
    const int myMid = (ly >> 1) * 8 + (lx >> 1);

    // MID windows of the current TAIL emissions, in batches of 4, each
    // batch's MID emissions fed to the pixels.
    auto route = [&]() {
        const int m = tid >> 2, lane = tid & 3;
        const int parent = ((m >> 3) >> 1) * 4 + ((m & 7) >> 1);
        for (int batch = 0; batch < 4; ++batch) {
            const int retained = sm.midCount[m];
            const int fresh = min(4, max(0, sm.tailEmitCount[parent] - 4 * batch));
            float nk = 0.0f;
            uint32_t np = 0u;
            if (lane < fresh) {
                np = sm.tailEmit[parent][4 * batch + lane];
                nk = sof_depth(load_record(a.records, __ldg(a.sortedIds + np)), sm.midRay[m]);
                sm.mergeKey[m * kSofMidCap + 4 + lane] = nk;  // new entries staged above the merge slots' use
                sm.mergePos[m * kSofMidCap + 4 + lane] = np;
            }
            __syncthreads();
            float rk = 0.0f;
            uint32_t rp = 0u;
            int rRank = 0, nRank = 0;
            if (lane < retained) {
                rk = sm.midKey[m][lane];
                rp = sm.midPos[m][lane];
                rRank = lane;
                for (int j = 0; j < fresh; ++j)
                    rRank += sof_less(sm.mergeKey[m * kSofMidCap + 4 + j], sm.mergePos[m * kSofMidCap + 4 + j], rk, rp);
            }
            if (lane < fresh) {
                for (int j = 0; j < retained; ++j) nRank += sof_less(sm.midKey[m][j], sm.midPos[m][j], nk, np);
                for (int j = 0; j < fresh; ++j)
                    nRank += sof_less(sm.mergeKey[m * kSofMidCap + 4 + j], sm.mergePos[m * kSofMidCap + 4 + j], nk, np);
            }
            __syncthreads();
            if (lane < retained) {
                sm.midKey[m][rRank] = rk;  // ranks are distinct: writes of one group never collide
                sm.midPos[m][rRank] = rp;
            }
            if (lane < fresh) {
                sm.midKey[m][nRank] = nk;
                sm.midPos[m][nRank] = np;
            }
            __syncthreads();
            const int merged = retained + fresh;
            const int emit = merged > kSofMidEmit ? kSofMidEmit : 0;
            uint32_t moveP = 0u;
            float moveK = 0.0f;
            if (emit > 0) sm.midEmit[m][lane] = sm.midPos[m][lane];
            if (emit > 0 && lane + 4 < merged) {
                moveK = sm.midKey[m][lane + 4];
                moveP = sm.midPos[m][lane + 4];
            }
            __syncthreads();
            if (emit > 0 && lane + 4 < merged) {
                sm.midKey[m][lane] = moveK;
                sm.midPos[m][lane] = moveP;
            }
            if (lane == 0) {
                sm.midCount[m] = merged - emit;
                sm.midEmitCount[m] = emit;
            }
            __syncthreads();
            for (int slot = 0; slot < kSofMidEmit; ++slot) feed(myMid, slot);
            __syncthreads();
        }
    };
    // Every TAIL with more than `keep` entries (drain: any) emits up to 16;
    // the emissions are routed when any TAIL emitted.
    auto emit_tails = [&](bool drain) {
        const int g = tid >> 4, lane = tid & 15;
        const int count = sm.tailCount[g];
        const int emit = drain ? min(kSofTailEmit, count) : (count > kSofTailKeep ? kSofTailEmit : 0);
        if (lane < emit) sm.tailEmit[g][lane] = sm.tailPos[g][lane];
        float k[3];
        uint32_t p[3];
#pragma unroll
        for (int r = 0; r < 3; ++r) {
            const int src = emit + lane + 16 * r;
            if (emit > 0 && src < count) {
                k[r] = sm.tailKey[g][src];
                p[r] = sm.tailPos[g][src];
            }
        }
        if (tid == 0) sm.emitted = 0;
        __syncthreads();
#pragma unroll
        for (int r = 0; r < 3; ++r) {
            const int src = emit + lane + 16 * r;
            if (emit > 0 && src < count) {
                sm.tailKey[g][lane + 16 * r] = k[r];
                sm.tailPos[g][lane + 16 * r] = p[r];
            }
        }
        if (lane == 0) {
            sm.tailCount[g] = count - emit;
            sm.tailEmitCount[g] = emit;
            if (emit > 0) atomicOr(&sm.emitted, 1);
        }
        __syncthreads();
        if (sm.emitted) route();  // block-uniform
    };

    bool stopped = false;
    for (uint32_t chunk = range.x; chunk < range.y; chunk += kSofChunk) {
        if (done()) {
            stopped = true;
            break;
        }
        // ingest 32 candidates into every TAIL
        const int g = tid >> 4, lane = tid & 15;
        const int fresh = int(min(uint32_t(kSofChunk), range.y - chunk));
        const int retained = sm.tailCount[g];
        for (int h = 0; h < 2; ++h) {
            const int j = lane + 16 * h;
            if (j < fresh) {
                const uint32_t pos = chunk + uint32_t(j);
                sm.newKey[g][j] = sof_depth(load_record(a.records, __ldg(a.sortedIds + pos)), sm.tailRay[g]);
                sm.newPos[g][j] = pos;
            }
        }
        __syncthreads();
        float rk[2], nk[2];
        uint32_t rp[2], np[2];
        int rRank[2], nRank[2];
        for (int h = 0; h < 2; ++h) {
            const int i = lane + 16 * h;
            rRank[h] = nRank[h] = 0;
            if (i < retained) {
                rk[h] = sm.tailKey[g][i];
                rp[h] = sm.tailPos[g][i];
                rRank[h] = i;
                for (int j = 0; j < fresh; ++j) rRank[h] += sof_less(sm.newKey[g][j], sm.newPos[g][j], rk[h], rp[h]);
            }
            if (i < fresh) {
                nk[h] = sm.newKey[g][i];
                np[h] = sm.newPos[g][i];
                // retained entries are sorted: binary search for the count below
                int lo = 0, hi = retained;
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if (sof_less(sm.tailKey[g][mid], sm.tailPos[g][mid], nk[h], np[h])) lo = mid + 1;
                    else hi = mid;
                }
                nRank[h] = lo;
                for (int j = 0; j < fresh; ++j) nRank[h] += sof_less(sm.newKey[g][j], sm.newPos[g][j], nk[h], np[h]);
            }
        }
        __syncthreads();
        for (int h = 0; h < 2; ++h) {
            const int i = lane + 16 * h;
            if (i < retained) {
                sm.tailKey[g][rRank[h]] = rk[h];
                sm.tailPos[g][rRank[h]] = rp[h];
            }
            if (i < fresh) {
                sm.tailKey[g][nRank[h]] = nk[h];
                sm.tailPos[g][nRank[h]] = np[h];
            }
        }
        __syncthreads();
        if (lane == 0) sm.tailCount[g] = retained + fresh;
        __syncthreads();
        emit_tails(false);
        emit_tails(false);
    }
    if (stopped) return;
    emit_tails(true);
    emit_tails(true);
    // MID drain: every remaining entry of the pixel's 2x2 group, in order
    for (int slot = 0; slot < kSofMidEmit; ++slot) {
        if (tid < kSofMids) {
            sm.midEmitCount[tid] = sm.midCount[tid];
            if (slot < sm.midCount[tid]) sm.midEmit[tid][slot] = sm.midPos[tid][slot];
        }
    }
    __syncthreads();
    for (int slot = 0; slot < kSofMidEmit; ++slot) feed(myMid, slot);
    __syncthreads();
}

// Forward of a tile with the SOF hierarchy (composite log as the flat forward).
template <bool kGeo>
__global__ __launch_bounds__(kTileThreads) void k_render_fwd_sof(RenderArgs a, float* __restrict__ rgba,
                                                                 float* __restrict__ hitDistance,
                                                                 float* __restrict__ hitCount) {
    extern __shared__ __align__(16) unsigned char smem[];
    SofSmem& sm = *reinterpret_cast<SofSmem*>(smem);
    const bool retained = a.mask[blockIdx.x] != 0u;
    const TileSetup ts = tile_setup(a, retained, int(blockIdx.x));
    PixelFwd s{1.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0u, ts.ray.valid};
    RingKBuffer<kSofHead> kb;
    kb.init(reinterpret_cast<float2*>(smem + sof_ring_offset()),
            reinterpret_cast<uint32_t*>(smem + sof_ring_offset() + sizeof(float2) * kSofHead * kTileThreads),
            threadIdx.x);
    uint32_t nlog = 0;
    PixelGeo geo;
    if constexpr (kGeo) {
        const bool pinhole = a.f.cam.model == GF_CAMERA_OPENCV_PINHOLE;
        geo_init(geo, (pinhole && ts.inImage && retained) ? a.rayD[3 * ts.pix + 2] : 1.0f);
    }
    const uint2 range = retained ? a.ranges[ts.tile] : make_uint2(0u, 0u);
    // one composited hit (sorted position sp)
    auto composite = [&](float ht, float ha, uint32_t sp) {
        const uint32_t id = __ldg(a.sortedIds + sp);
        log_composite(a.log, uint32_t(ts.tile), nlog, sp - range.x);
        const float tBefore = s.T;
        composite_fwd(s, ht, ha, __ldg(a.records + 4 * size_t(id) + 3));
        if constexpr (kGeo) {
            const Record rec = load_record(a.records, id);
            geo_hit(geo, ts.ray, rec, a.geo.particles + 32 * size_t(id), ht, ha * tBefore, tBefore, s.T);
        }
    };
    if (retained) {
        SofSmem& S = sm;
        auto feed = [&](int m, int slot) {
            if (!(s.alive && slot < S.midEmitCount[m])) return;
            const uint32_t sp = S.midEmit[m][slot];
            const Record q = load_record(a.records, __ldg(a.sortedIds + sp));
            const V3 gro = binv_times(q.b, q.c, q.d, v3(ts.ray.o.x - q.a.x, ts.ray.o.y - q.a.y, ts.ray.o.z - q.a.z));
            float alpha, ht;
            if (!hit_with_origin(ts.ray, gro, q.b, q.c, q.d, q.a.w, alpha, ht)) return;
            if (kb.full()) {
                float t0, a0;
                uint32_t s0;
                kb.pop_front(t0, a0, s0);
                composite(t0, a0, s0);
            }
            kb.insert(ht, alpha, sp);
        };
        auto done = [&]() { return __syncthreads_and(!s.alive) != 0; };
        sof_cascade(a, sm, ts, range, feed, done);
        for (int i = 0; s.alive && i < kb.n; ++i) {
            float ht, ha;
            uint32_t sp;
            kb.entry(i, ht, ha, sp);
            composite(ht, ha, sp);
        }
    }
    if (a.log.ids != nullptr) log_finish(a.log, uint32_t(ts.tile), nlog, range.y - range.x);
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

// Backward replay of one tile with the SOF hierarchy: the same cascade and
// HEAD, each composited hit back-propagated from the final pixel values
// (the replay of tiles whose composite log overflowed, or of every tile
// without a log).
template <bool kGeo>
__device__ __forceinline__ void replay_tile_sof(const RenderBwdArgs& a, unsigned char* smem, int tile) {
    SofSmem& sm = *reinterpret_cast<SofSmem*>(smem);
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
    auto vjp = [&](uint32_t sp, uint32_t& cid, float4* g) -> bool {
        cid = __ldg(a.r.sortedIds + sp);
        const Record q = load_record(a.r.records, cid);
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
    RingKBuffer<kSofHead> kb;
    kb.init(reinterpret_cast<float2*>(smem + sof_ring_offset()),
            reinterpret_cast<uint32_t*>(smem + sof_ring_offset() + sizeof(float2) * kSofHead * kTileThreads),
            threadIdx.x);
    const uint2 range = a.r.ranges[ts.tile];
    auto feed = [&](int m, int slot) {  // every thread, in step: the gradient merge is warp-wide
        bool have = false;
        uint32_t cid = kInvalidParticle;
        float4 g[4] = {};
        if (s.alive && slot < sm.midEmitCount[m]) {
            const uint32_t sp = sm.midEmit[m][slot];
            const Record q = load_record(a.r.records, __ldg(a.r.sortedIds + sp));
            const V3 gro = binv_times(q.b, q.c, q.d, v3(ray.o.x - q.a.x, ray.o.y - q.a.y, ray.o.z - q.a.z));
            float alpha, ht;
            if (hit_with_origin(ray, gro, q.b, q.c, q.d, q.a.w, alpha, ht)) {
                if (kb.full()) {
                    float t0, a0;
                    uint32_t s0;
                    kb.pop_front(t0, a0, s0);
                    have = vjp(s0, cid, g);
                }
                kb.insert(ht, alpha, sp);
                if (s.T < kMinTransmittance) s.alive = false;
            }
        }
        accumulate_abs_grad(a.absGrad, a.absMode, have, cid, g[0]);
        accumulate_grad(a.gradRecords, have, cid, g);
    };
    auto done = [&]() { return __syncthreads_and(!s.alive) != 0; };
    sof_cascade(a.r, sm, ts, range, feed, done);
    for (int i = 0; i < kSofHead; ++i) {
        if (!__any_sync(0xffffffffu, s.alive && i < kb.n)) break;
        bool have = false;
        uint32_t cid = kInvalidParticle;
        float4 g[4] = {};
        if (s.alive && i < kb.n) {
            float ht, ha;
            uint32_t sp;
            kb.entry(i, ht, ha, sp);
            have = vjp(sp, cid, g);
            if (s.T < kMinTransmittance) s.alive = false;
        }
        accumulate_abs_grad(a.absGrad, a.absMode, have, cid, g[0]);
        accumulate_grad(a.gradRecords, have, cid, g);
    }
}

// Backward replay kernel of the SOF hierarchy: one block per tile, or, when
// the forward kept a composite log, a resident grid over the overflowed tiles.
template <bool kGeo>
__global__ __launch_bounds__(kTileThreads) void k_render_bwd_sof(RenderBwdArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    if (a.r.log.ids == nullptr) {
        replay_tile_sof<kGeo>(a, smem, int(blockIdx.x));
        return;
    }
    const uint32_t count = *a.r.log.overflowCount;
    for (uint32_t w = blockIdx.x; w < count; w += gridDim.x) {
        replay_tile_sof<kGeo>(a, smem, int(a.r.log.overflowList[w]));
        __syncthreads();  // the next tile reuses the shared windows
    }
}

}  // namespace gf
