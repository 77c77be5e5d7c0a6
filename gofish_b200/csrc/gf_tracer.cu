// Host orchestration and C ABI of the B200 fisheye tracer.
//
// One gf_tracer owns the device buffers of one renderer instance (the
// reference's GutRenderForwardContext, gutRenderer.cu:229-671): projected
// particle state, render records, tile counts and offsets, the (tile|depth)
// keys and particle ids with their sort ping-pong buffers, per-tile ranges
// and the backward gradient records.  Buffers grow geometrically and are
// stream-ordered (cudaMallocAsync), so steady-state frames allocate nothing.
//
// Host synchronization: none in the steady state.  The number of tile
// intersections is known only on the device after the count scan; the keys
// and ids are sized by a speculative capacity (1.5x the largest count of the
// earlier forwards) and every kernel after the scan reads the count from
// device memory.  A device-side plan records the count and whether it
// exceeded the capacity; the host reads the plans of finished forwards
// without waiting (at most kMaxInFlight forwards are left unread), and
// reports an overflowed forward -- which emitted, sorted and composited
// nothing -- as GF_ERR_CAPACITY from the next call, with the capacity grown.
// The first forward, a forward whose particle count or raster differs from
// the last one read, and every forward of a tracer configured with
// GF_CAPACITY_EXACT read the count after the scan with one synchronization
// (the reference synchronizes about eight times, gutRenderer.cu:843-1599).
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <deque>
#include <map>
#include <string>
#include <vector>

#include "../../include/gofish_b200.h"
#include "gf_host.cuh"
#include "gf_render.cuh"
#include "gf_render_sof.cuh"
#include "gf_sof_opacity.cuh"
#include "gf_tracer_kernels.cuh"

namespace {

// Sine of a cap half-angle bound of the cone_big window: the half-angle lies
// in [0, pi/2], where the sine is increasing, so the window is tested on the
// caps' sines (1 for bounds of pi/2 and above).
float cap_sine(float angle) {
    if (!(angle < 1.5707963267948966f)) return 1.0f;
    return static_cast<float>(std::sin(static_cast<double>(angle > 0.0f ? angle : 0.0f)));
}
thread_local std::string g_lastError;
}  // namespace

// Records an error for gf_last_error() from every translation unit of the library.
int gf_record_error(int code, const char* message) {
    g_lastError = message;
    return code;
}

namespace {

struct TileMask {
    DeviceBuffer buf;
    uint32_t ty = 0, tx = 0;
};

bool valid_k(int k) { return k == 0 || k == 4 || k == 8 || k == 12 || k == 16 || k == 24 || k == 32; }

// Forwards whose intersection plan the host has not read yet, at most (the
// next forward waits for the oldest beyond this), and the pinned plan slots.
constexpr size_t kMaxInFlight = 8;
// Tiles of the fallback walks kept for the emit pass (16 MB); walks beyond it are repeated.
constexpr uint32_t kFallbackCacheTiles = 1u << 22;
constexpr int kPlanSlots = 16;

struct InFlight {
    cudaEvent_t done;   // recorded after the plan's copy to hostPlans[slot]
    int slot;
    uint64_t capacity;  // keys reserved for the forward
    uint32_t N, T;
};

}  // namespace

struct gf_tracer {
    gf_tracer_config cfg{};
    int device = -1;
    std::map<std::string, TileMask> masks;

    // Forward context.
    DeviceBuffer proj, records, bounds, counts, offsets, scanTiles, total, tileRays, ranges;
    DeviceBuffer keys[2], ids[2], hist;
    DeviceBuffer gradRecords;
    DeviceBuffer gradShape;  // extent gradient: quaternion, intrinsic scale [N,2] float4 (enable_normals)
    DeviceBuffer coneA, coneS, caps, bigList, bigCount;  // cone-fallback admission
    DeviceBuffer tileCache, cacheStart;                    // the fallback walks' tile lists
    DeviceBuffer wideList;                                // projected particles with a large tile box
    DeviceBuffer logIds, logCount, logOverflow, logList;  // composite log of the last training forward
    int residentBlocks = 0;                               // SMs x 3: the replay grid when a log exists
    gf::CompositeLog frameLog{};
    bool frameGeo = false;                                // the last forward wrote the geometric channels
    bool frameSof = false;                                // the last forward wrote the SOF opacity field
    DeviceBuffer gradIntrinsic;                           // SOF opacity field gradient [N,4] float4
    uint64_t* hostTotal = nullptr;  // [0] intersections, [1] fallback list size, [2] log overflow tiles (low 32 bits)
    uint32_t fallbackParticles = 0;
    // Intersection plans (speculative key capacity).
    DeviceBuffer plan;                    // gf::FramePlan of the current forward
    gf::FramePlan* hostPlans = nullptr;   // pinned [kPlanSlots]
    std::deque<InFlight> inflight;
    int nextSlot = 0;
    uint64_t maxIntersections = 0;        // largest count read so far
    uint64_t forwardsRead = 0, intersectionsRead = 0, fallbackRead = 0;  // sums over the plans read
    uint64_t hostWaitUs = 0;  // time blocked in synchronizations and plan waits
    uint32_t lastN = 0, lastT = 0;        // sizes of the last forward read
    bool haveHistory = false;
    std::string overflowMessage;          // an overflowed forward, reported by the next call
    std::vector<cudaEvent_t> planEventPool;
    cudaEvent_t logCopied = nullptr;  // recorded after the copy of the last forward's log overflow count
    bool logCounted = false;
    int finalBuf = 0;
    bool haveForward = false;
    gf::FrameArgs frame{};
    const uint8_t* frameMask = nullptr;
    const float* frameRayO = nullptr;
    const float* frameRayD = nullptr;
    uint64_t numIntersections = 0;
    uint32_t launches = 0;
    uint64_t totalLaunches = 0;

    // Per-stage event timing (enabled by gf_tracer_enable_timing).
    bool timing = false;
    struct StageEvent {
        int stage;
        cudaEvent_t start, end;
    };
    std::vector<StageEvent> pending;
    std::vector<cudaEvent_t> eventPool;
};

namespace {

cudaEvent_t take_event(gf_tracer* t) {
    if (!t->eventPool.empty()) {
        cudaEvent_t e = t->eventPool.back();
        t->eventPool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    return e;
}

// Brackets one stage with events when timing is enabled.
struct StageTimer {
    gf_tracer* t;
    int stage;
    cudaStream_t stream;
    cudaEvent_t start = nullptr;
    StageTimer(gf_tracer* t_, int stage_, cudaStream_t s) : t(t_), stage(stage_), stream(s) {
        if (t->timing) {
            start = take_event(t);
            if (start != nullptr) cudaEventRecord(start, stream);
        }
    }
    ~StageTimer() {
        if (start == nullptr) return;
        cudaEvent_t end = take_event(t);
        if (end == nullptr) return;
        cudaEventRecord(end, stream);
        t->pending.push_back({stage, start, end});
    }
};

int bind_device(gf_tracer* t) {
    int dev = -1;
    GF_CUDA(cudaGetDevice(&dev));
    if (t->device < 0) {
        t->device = dev;
        GF_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&t->hostTotal), 3 * sizeof(uint64_t), cudaHostAllocDefault));
        GF_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&t->hostPlans), kPlanSlots * sizeof(gf::FramePlan),
                              cudaHostAllocDefault));
    } else if (t->device != dev) {
        return fail(GF_ERR_STATE, "tracer bound to device %d, called on device %d", t->device, dev);
    }
    return GF_OK;
}

// Reads the plans of finished forwards in order, waiting only while more
// than `keep` forwards remain unread.  The last plan read gives the
// intersection count, the fallback list size and the history of the
// speculative capacity; an overflowed plan leaves a message for the next call.
int harvest(gf_tracer* t, size_t keep) {
    while (!t->inflight.empty()) {
        const InFlight f = t->inflight.front();
        if (t->inflight.size() > keep) {
            const auto w0 = std::chrono::steady_clock::now();
            GF_CUDA(cudaEventSynchronize(f.done));
            t->hostWaitUs += uint64_t(std::chrono::duration_cast<std::chrono::microseconds>(
                std::chrono::steady_clock::now() - w0).count());
        } else {
            const cudaError_t q = cudaEventQuery(f.done);
            if (q == cudaErrorNotReady) break;
            if (q != cudaSuccess) return fail(GF_ERR_CUDA, "cudaEventQuery failed: %s", cudaGetErrorString(q));
        }
        const gf::FramePlan& p = t->hostPlans[f.slot];
        t->maxIntersections = std::max<uint64_t>(t->maxIntersections, p.intersections);
        t->forwardsRead += 1;
        t->intersectionsRead += p.intersections;
        t->fallbackRead += p.fallback;
        t->numIntersections = p.count;
        t->fallbackParticles = p.fallback;
        t->lastN = f.N;
        t->lastT = f.T;
        t->haveHistory = true;
        if (p.overflow != 0u) {
            char msg[256];
            snprintf(msg, sizeof(msg),
                     "a forward produced %llu tile intersections, more than the %llu its keys were reserved for; "
                     "it rendered nothing. The capacity has grown: render that frame again",
                     static_cast<unsigned long long>(p.intersections), static_cast<unsigned long long>(f.capacity));
            t->overflowMessage = msg;
        }
        t->planEventPool.push_back(f.done);
        t->inflight.pop_front();
    }
    return GF_OK;
}

// GF_ERR_CAPACITY for a forward found overflowed since the last call.
int report_overflow(gf_tracer* t) {
    if (t->overflowMessage.empty()) return GF_OK;
    const std::string m = t->overflowMessage;
    t->overflowMessage.clear();
    return fail(GF_ERR_CAPACITY, "%s", m.c_str());
}

int validate_inputs(const gf_tracer* t, const gf_trace_inputs* in, const TileMask** maskOut) {
    if (in == nullptr) return fail(GF_ERR_BAD_INPUT, "inputs is NULL");
    const gf_camera& cam = in->camera;
    if (cam.width <= 0 || cam.height <= 0) return fail(GF_ERR_BAD_INPUT, "camera resolution must be positive");
    if (cam.model != GF_CAMERA_OPENCV_FISHEYE && cam.model != GF_CAMERA_OPENCV_PINHOLE)
        return fail(GF_ERR_BAD_INPUT, "only OPENCV_FISHEYE and PINHOLE cameras are supported");
    if (cam.shutter != GF_SHUTTER_GLOBAL)
        return fail(GF_ERR_BAD_INPUT, "unconditional support union requires global shutter");
    for (int k = 0; k < 7; ++k) {
        if (in->pose_start[k] != in->pose_end[k])
            return fail(GF_ERR_BAD_INPUT, "conservative opacity bound requires exact global-shutter poses");
    }
    if (in->sh_coeffs != 1 && in->sh_coeffs != 4 && in->sh_coeffs != 9 && in->sh_coeffs != 16)
        return fail(GF_ERR_BAD_INPUT, "sh_coeffs must be 1, 4, 9 or 16 (got %u)", in->sh_coeffs);
    if (in->sh_degree < 0 || in->sh_degree > 3) return fail(GF_ERR_BAD_INPUT, "sh_degree must be in [0,3]");
    if (in->num_particles > 0 && (in->particles == nullptr || in->features == nullptr))
        return fail(GF_ERR_BAD_INPUT, "particle buffers are NULL");
    if (in->ray_origin == nullptr || in->ray_direction == nullptr) return fail(GF_ERR_BAD_INPUT, "ray buffers are NULL");
    if ((reinterpret_cast<uintptr_t>(in->particles) & 15u) != 0u)
        return fail(GF_ERR_BAD_INPUT, "particle rows must be 16-byte aligned");
    if (in->tile_token == nullptr) return fail(GF_ERR_BAD_INPUT, "tile token is NULL");
    const auto it = t->masks.find(in->tile_token);
    if (it == t->masks.end()) return fail(GF_ERR_NOT_REGISTERED, "physical tile token is not registered on this tracer");
    const uint32_t gx = uint32_t((cam.width + 15) / 16), gy = uint32_t((cam.height + 15) / 16);
    if (it->second.tx != gx || it->second.ty != gy)
        return fail(GF_ERR_BAD_INPUT, "physical tile token does not match current raster");
    *maskOut = &it->second;
    return GF_OK;
}

template <typename In, typename Out>
int exclusive_scan(gf_tracer* t, const In* in, uint64_t n, Out* out, Out* grandTotal, cudaStream_t stream) {
    return scan_exclusive<In, Out>(t->scanTiles, t->launches, in, n, out, grandTotal, stream);
}

int radix_sort(gf_tracer* t, uint32_t n, int endBit, cudaStream_t stream, const uint32_t* nDev) {
    return sort_pairs(t->hist, t->scanTiles, t->launches, t->keys, t->ids, n, 0, endBit, &t->finalBuf, stream, nDev);
}

template <int K, bool kGeo>
void launch_render_fwd_geo(const gf::RenderArgs& a, uint32_t tiles, float* rgba, float* hd, float* hc,
                           cudaStream_t stream) {
    const size_t smem = gf::fwd_smem_bytes(K);
    cudaFuncSetAttribute(gf::k_render_fwd<K, kGeo>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    cudaFuncSetAttribute(gf::k_render_fwd<K, kGeo>, cudaFuncAttributePreferredSharedMemoryCarveout,
                         int(cudaSharedmemCarveoutMaxShared));
    gf::k_render_fwd<K, kGeo><<<tiles, gf::kTileThreads, smem, stream>>>(a, rgba, hd, hc);
}

template <int K>
void launch_render_fwd(const gf::RenderArgs& a, uint32_t tiles, float* rgba, float* hd, float* hc,
                       cudaStream_t stream) {
    if (a.geo.particles != nullptr) launch_render_fwd_geo<K, true>(a, tiles, rgba, hd, hc, stream);
    else launch_render_fwd_geo<K, false>(a, tiles, rgba, hd, hc, stream);
}

template <int K, bool kGeo>
void launch_render_bwd_geo(const gf::RenderBwdArgs& a, uint32_t tiles, cudaStream_t stream) {
    const size_t smem = gf::render_smem_bytes(K);
    cudaFuncSetAttribute(gf::k_render_bwd<K, kGeo>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    gf::k_render_bwd<K, kGeo><<<tiles, gf::kTileThreads, smem, stream>>>(a);
}

template <int K>
void launch_render_bwd(const gf::RenderBwdArgs& a, uint32_t tiles, cudaStream_t stream) {
    if (a.geo.gradShape != nullptr) launch_render_bwd_geo<K, true>(a, tiles, stream);
    else launch_render_bwd_geo<K, false>(a, tiles, stream);
}

template <bool kGeo, bool kAbs>
void launch_render_bwd_log_abs(const gf::RenderBwdArgs& a, uint32_t tiles, cudaStream_t stream) {
    const size_t smem = gf::bwd_log_smem_bytes();
    cudaFuncSetAttribute(gf::k_render_bwd_log<kGeo, kAbs>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    gf::k_render_bwd_log<kGeo, kAbs><<<tiles, gf::kTileThreads, smem, stream>>>(a);
}

template <bool kGeo>
void launch_render_bwd_log(const gf::RenderBwdArgs& a, uint32_t tiles, cudaStream_t stream) {
    if (a.absGrad != nullptr) launch_render_bwd_log_abs<kGeo, true>(a, tiles, stream);
    else launch_render_bwd_log_abs<kGeo, false>(a, tiles, stream);
}

// Blocks of the replay grid that walks the overflowed tiles: 3 per SM.
uint32_t resident_blocks() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 148u * 3u;
    return uint32_t(sms) * 3u;
}

int dispatch_fwd(int K, const gf::RenderArgs& a, uint32_t tiles, float* rgba, float* hd, float* hc,
                 cudaStream_t s) {
    switch (K) {
        case 0: launch_render_fwd<0>(a, tiles, rgba, hd, hc, s); break;
        case 4: launch_render_fwd<4>(a, tiles, rgba, hd, hc, s); break;
        case 8: launch_render_fwd<8>(a, tiles, rgba, hd, hc, s); break;
        case 12: launch_render_fwd<12>(a, tiles, rgba, hd, hc, s); break;
        case 16: launch_render_fwd<16>(a, tiles, rgba, hd, hc, s); break;
        case 24: launch_render_fwd<24>(a, tiles, rgba, hd, hc, s); break;
        case 32: launch_render_fwd<32>(a, tiles, rgba, hd, hc, s); break;
        default: return fail(GF_ERR_BAD_INPUT, "unsupported k-buffer size %d", K);
    }
    return GF_OK;
}

int dispatch_bwd(int K, const gf::RenderBwdArgs& a, uint32_t tiles, cudaStream_t s) {
    switch (K) {
        case 0: launch_render_bwd<0>(a, tiles, s); break;
        case 4: launch_render_bwd<4>(a, tiles, s); break;
        case 8: launch_render_bwd<8>(a, tiles, s); break;
        case 12: launch_render_bwd<12>(a, tiles, s); break;
        case 16: launch_render_bwd<16>(a, tiles, s); break;
        case 24: launch_render_bwd<24>(a, tiles, s); break;
        case 32: launch_render_bwd<32>(a, tiles, s); break;
        default: return fail(GF_ERR_BAD_INPUT, "unsupported k-buffer size %d", K);
    }
    return GF_OK;
}

// Composite log capacity: entries per pixel (256 covers the deepest pixels of
// the 1M-Gaussian 200 deg view with the 0.3 px^2 footprint; a tile with a
// deeper pixel is replayed through the k-buffer, at several times the cost of
// the log backward), bounded so that the log stays within 8 GiB.
constexpr uint32_t kLogCapacity = 256;
constexpr size_t kLogBudgetBytes = size_t(8) << 30;

// Projection, binning, sort and forward composite; a training forward
// (logComposites) also records the composite log for the backward.
int forward(gf_tracer* t, const gf_trace_inputs* in, float* rgba, float* hd, float* hc, float* vis,
            bool logComposites, const gf_trace_outputs* geoOut, cudaStream_t stream) {
    if (int e = bind_device(t)) return e;
    const TileMask* mask = nullptr;
    if (int e = validate_inputs(t, in, &mask)) return e;
    if (rgba == nullptr || hd == nullptr) return fail(GF_ERR_BAD_INPUT, "output buffers are NULL");
    // read what has finished; at most kMaxInFlight - 1 earlier forwards stay unread
    if (int e = harvest(t, kMaxInFlight - 1)) return e;
    if (int e = report_overflow(t)) return e;
    t->launches = 0;
    t->haveForward = false;

    gf::FrameArgs& f = t->frame;
    f.cam = in->camera;
    prepare_pose(in->pose_start, f.pose);
    f.W = in->camera.width;
    f.H = in->camera.height;
    f.gx = (f.W + gf::kTile - 1) / gf::kTile;
    f.gy = (f.H + gf::kTile - 1) / gf::kTile;
    f.N = in->num_particles;
    f.shDegree = in->sh_degree;
    f.shCoeffs = in->sh_coeffs;
    f.keyMode = t->cfg.sort_key;
    f.utPartialScale2 = t->cfg.partial_ut_scale > 0.0f ? t->cfg.partial_ut_scale * t->cfg.partial_ut_scale : 0.0f;
    const uint32_t T = uint32_t(f.gx * f.gy);
    const uint32_t N = f.N;

    if (int e = t->proj.ensure(sizeof(float4) * 2 * size_t(N) + 16, stream)) return e;
    if (int e = t->records.ensure(sizeof(float4) * 4 * size_t(N) + 16, stream)) return e;
    if (int e = t->counts.ensure(sizeof(uint32_t) * size_t(N) + 16, stream)) return e;
    if (int e = t->bounds.ensure(sizeof(float) * size_t(N) + 16, stream)) return e;
    if (int e = t->offsets.ensure(sizeof(uint64_t) * size_t(N) + 16, stream)) return e;
    if (int e = t->total.ensure(sizeof(uint64_t) * 2, stream)) return e;
    if (int e = t->tileRays.ensure(sizeof(float4) * 2 * size_t(T), stream)) return e;
    if (int e = t->ranges.ensure(sizeof(uint2) * size_t(T), stream)) return e;

    gf::FallbackArgs fa{};
    fa.complete = t->cfg.complete_admission != 0 ? 1 : 0;
    fa.enabled = (t->cfg.admission_fallback == GF_FALLBACK_CONE || t->cfg.admission_fallback == GF_FALLBACK_CONE_BIG ||
                  fa.complete)
                     ? 1
                     : 0;
    fa.coneBig = t->cfg.admission_fallback == GF_FALLBACK_CONE_BIG ? 1 : 0;
    fa.sinMin = cap_sine(t->cfg.fallback_min_angle);
    fa.sinMax = cap_sine(t->cfg.fallback_max_angle);
    if (int e = t->caps.ensure(sizeof(float4) * 2 * size_t(N) + 16, stream)) return e;
    if (int e = t->bigList.ensure(sizeof(uint32_t) * size_t(N) + 16, stream)) return e;
    if (int e = t->bigCount.ensure(sizeof(uint32_t) * 5, stream)) return e;
    if (int e = t->cacheStart.ensure(sizeof(uint32_t) * size_t(N) + 16, stream)) return e;
    if (int e = t->tileCache.ensure(sizeof(uint32_t) * size_t(kFallbackCacheTiles), stream)) return e;
    if (int e = t->wideList.ensure(sizeof(uint32_t) * size_t(N) + 16, stream)) return e;
    fa.caps = t->caps.as<float4>();
    fa.big = t->bigList.as<uint32_t>();
    fa.bigCount = t->bigCount.as<uint32_t>();
    fa.wide = t->wideList.as<uint32_t>();
    fa.wideCount = t->bigCount.as<uint32_t>() + 1;
    fa.bigCursor = t->bigCount.as<uint32_t>() + 2;
    fa.cacheCursor = t->bigCount.as<uint32_t>() + 4;
    fa.cacheStart = t->cacheStart.as<uint32_t>();
    fa.tileCache = t->tileCache.as<uint32_t>();
    fa.cacheCapacity = kFallbackCacheTiles;
    {
        StageTimer st(t, GF_STAGE_TILE_RAYS, stream);
        if (f.keyMode == GF_KEY_PER_TILE_DEPTH) {
            gf::k_tile_rays<<<(T + 127) / 128, 128, 0, stream>>>(f, in->ray_origin, in->ray_direction,
                                                                  t->tileRays.as<float4>());
            t->launches += 1;
            GF_LAUNCH_CHECK();
        }
        if (fa.enabled) {
            // tile ray-cone quadtree, leaves (tiles) up to one root
            gf::fb::TileTree& tr = fa.tree;
            tr.n = 0;
            uint32_t nodes = 0;
            int gx = f.gx, gy = f.gy;
            // the warp descent packs (level << 24 | node)
            if (T >= (1u << 24)) return fail(GF_ERR_BAD_INPUT, "raster too large for the tile cone tree");
            while (true) {
                if (tr.n >= gf::fb::kMaxLevels) return fail(GF_ERR_BAD_INPUT, "raster too large for the tile cone tree");
                tr.gx[tr.n] = gx;
                tr.gy[tr.n] = gy;
                tr.offset[tr.n] = nodes;
                nodes += uint32_t(gx * gy);
                ++tr.n;
                if (gx == 1 && gy == 1) break;
                gx = (gx + gf::fb::kFan - 1) / gf::fb::kFan;
                gy = (gy + gf::fb::kFan - 1) / gf::fb::kFan;
            }
            tr.optical[0] = f.pose.Rinv[2];
            tr.optical[1] = f.pose.Rinv[5];
            tr.optical[2] = f.pose.Rinv[8];
            tr.second = nodes;     // the leaves' second cones follow the levels,
            tr.sums = nodes + T;   // then one ray sum per node
            if (int e = t->coneA.ensure(sizeof(float4) * (2 * size_t(nodes) + T), stream)) return e;
            if (int e = t->coneS.ensure(sizeof(float) * (size_t(nodes) + T), stream)) return e;
            float4* A = t->coneA.as<float4>();
            float* S = t->coneS.as<float>();
            tr.A = A;
            tr.S = S;
            // one warp per tile, four tiles per block
            gf::fb::k_tile_cones<<<(T + 3) / 4, 128, 0, stream>>>(f, mask->buf.as<uint8_t>(), in->ray_direction, A,
                                                                  S, tr.second, tr.sums);
            t->launches += 1;
            GF_LAUNCH_CHECK();
            int span = 1;  // leaves per node side at level l
            for (int l = 1; l < tr.n; ++l) {
                const int pn = tr.gx[l] * tr.gy[l];
                span *= gf::fb::kFan;
                const int threads = gf::fb::cone_level_threads(std::min(span, f.gx) * std::min(span, f.gy));
                gf::fb::k_tile_cone_level<<<pn, threads, 0, stream>>>(tr, l, A, S);
                t->launches += 1;
                GF_LAUNCH_CHECK();
            }
        }
    }
    if (N > 0) {
        StageTimer st(t, GF_STAGE_PROJECT, stream);
        // fallback and wide lists, and the fallback kernels' cursors
        GF_CUDA(cudaMemsetAsync(fa.bigCount, 0, 5 * sizeof(uint32_t), stream));
        gf::k_project<<<(N + 255) / 256, 256, 0, stream>>>(f, in->particles, in->features, mask->buf.as<uint8_t>(),
                                                          t->proj.as<float4>(), t->records.as<float4>(),
                                                          t->counts.as<uint32_t>(), reinterpret_cast<uint32_t*>(vis),
                                                          t->bounds.as<float>(), fa);
        t->launches += 1;
        GF_LAUNCH_CHECK();
        if (fa.enabled) {
            gf::k_fallback_big<false><<<148 * 8, 256, 0, stream>>>(
                f, fa, mask->buf.as<uint8_t>(), t->records.as<float4>(), t->tileRays.as<float4>(),
                t->counts.as<uint32_t>(), reinterpret_cast<uint32_t*>(vis), nullptr, nullptr, nullptr);
            t->launches += 1;
            GF_LAUNCH_CHECK();
        }
        gf::k_wide<false><<<148 * 8, 256, 0, stream>>>(f, fa, mask->buf.as<uint8_t>(), t->proj.as<float4>(),
                                                      t->records.as<float4>(), t->tileRays.as<float4>(),
                                                      t->counts.as<uint32_t>(), reinterpret_cast<uint32_t*>(vis),
                                                      nullptr, nullptr, nullptr);
        t->launches += 1;
        GF_LAUNCH_CHECK();
    }
    {
        StageTimer st(t, GF_STAGE_SCAN, stream);
        if (int e = exclusive_scan<uint32_t, uint64_t>(t, t->counts.as<uint32_t>(), N, t->offsets.as<uint64_t>(),
                                                        t->total.as<uint64_t>(), stream))
            return e;
    }
    // Key capacity: speculative (no synchronization) when the history covers
    // this particle count and raster, else the exact count read back now.
    constexpr uint64_t kMaxKeys = 0xffffffffull - gf::kSortTile;
    const bool speculative = t->cfg.intersection_capacity == GF_CAPACITY_SPECULATIVE && t->haveHistory &&
                             N == t->lastN && T == t->lastT;
    uint64_t capacity = 0;
    if (speculative) {
        capacity = std::min<uint64_t>(kMaxKeys, std::max<uint64_t>(t->maxIntersections + t->maxIntersections / 2,
                                                                   uint64_t(1) << 16));
    } else {
        GF_CUDA(cudaMemcpyAsync(t->hostTotal, t->total.ptr, sizeof(uint64_t), cudaMemcpyDeviceToHost, stream));
        t->hostTotal[1] = 0;
        if (fa.enabled && N > 0)
            GF_CUDA(cudaMemcpyAsync(t->hostTotal + 1, fa.bigCount, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream));
        const auto w0 = std::chrono::steady_clock::now();
        GF_CUDA(cudaStreamSynchronize(stream));
        t->hostWaitUs += uint64_t(std::chrono::duration_cast<std::chrono::microseconds>(
            std::chrono::steady_clock::now() - w0).count());
        if (int e = harvest(t, 0)) return e;  // earlier forwards on this stream are complete
        if (int e = report_overflow(t)) return e;
        const uint64_t I = *t->hostTotal;
        if (I > kMaxKeys)
            return fail(GF_ERR_CAPACITY, "%llu tile intersections exceed the 32-bit index range",
                        static_cast<unsigned long long>(I));
        capacity = I;
        t->maxIntersections = std::max<uint64_t>(t->maxIntersections, I);
        t->numIntersections = I;
        t->fallbackParticles = uint32_t(t->hostTotal[1]);
        t->lastN = N;
        t->lastT = T;
        t->haveHistory = true;
    }
    for (int b = 0; b < 2; ++b) {
        if (int e = t->keys[b].ensure(sizeof(uint64_t) * (capacity + 1), stream)) return e;
        if (int e = t->ids[b].ensure(sizeof(uint32_t) * (capacity + 1), stream)) return e;
    }
    if (int e = t->plan.ensure(sizeof(gf::FramePlan), stream)) return e;
    gf::FramePlan* plan = t->plan.as<gf::FramePlan>();
    gf::k_plan_intersections<<<1, 32, 0, stream>>>(t->total.as<uint64_t>(), fa.enabled && N > 0 ? fa.bigCount : nullptr,
                                                   capacity, plan);
    t->launches += 1;
    GF_LAUNCH_CHECK();
    fa.overflow = &plan->overflow;
    const uint32_t* count = &plan->count;
    if (capacity > 0 && N > 0) {
        StageTimer st(t, GF_STAGE_EMIT, stream);
        gf::k_emit<<<(N + 255) / 256, 256, 0, stream>>>(f, t->proj.as<float4>(), t->records.as<float4>(),
                                                        mask->buf.as<uint8_t>(), t->tileRays.as<float4>(),
                                                        t->offsets.as<uint64_t>(), t->counts.as<uint32_t>(),
                                                        t->keys[0].as<uint64_t>(), t->ids[0].as<uint32_t>(), fa);
        t->launches += 1;
        GF_LAUNCH_CHECK();
        if (fa.enabled) {
            gf::k_fallback_big<true><<<148 * 8, 256, 0, stream>>>(
                f, fa, mask->buf.as<uint8_t>(), t->records.as<float4>(), t->tileRays.as<float4>(),
                t->counts.as<uint32_t>(), nullptr, t->offsets.as<uint64_t>(), t->keys[0].as<uint64_t>(),
                t->ids[0].as<uint32_t>());
            t->launches += 1;
            GF_LAUNCH_CHECK();
        }
        gf::k_wide<true><<<148 * 8, 256, 0, stream>>>(f, fa, mask->buf.as<uint8_t>(), t->proj.as<float4>(),
                                                     t->records.as<float4>(), t->tileRays.as<float4>(),
                                                     t->counts.as<uint32_t>(), nullptr, t->offsets.as<uint64_t>(),
                                                     t->keys[0].as<uint64_t>(), t->ids[0].as<uint32_t>());
        t->launches += 1;
        GF_LAUNCH_CHECK();
    }
    const int endBit = 32 + int(bit_length(T));
    {
        StageTimer st(t, GF_STAGE_SORT, stream);
        if (int e = radix_sort(t, uint32_t(capacity), endBit, stream, count)) return e;
    }
    {
        StageTimer st(t, GF_STAGE_RANGES, stream);
        GF_CUDA(cudaMemsetAsync(t->ranges.ptr, 0, sizeof(uint2) * T, stream));
        if (capacity > 0) {
            gf::k_tile_ranges<<<uint32_t((capacity + 255) / 256), 256, 0, stream>>>(
                t->keys[t->finalBuf].as<uint64_t>(), uint32_t(capacity), t->ranges.as<uint2>(), count);
            t->launches += 1;
            GF_LAUNCH_CHECK();
        }
    }
    // the plan goes to a pinned slot, read by a later call without waiting
    {
        const int slot = t->nextSlot;
        t->nextSlot = (t->nextSlot + 1) % kPlanSlots;
        GF_CUDA(cudaMemcpyAsync(t->hostPlans + slot, plan, sizeof(gf::FramePlan), cudaMemcpyDeviceToHost, stream));
        cudaEvent_t done = nullptr;
        if (!t->planEventPool.empty()) {
            done = t->planEventPool.back();
            t->planEventPool.pop_back();
        } else {
            GF_CUDA(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
        }
        GF_CUDA(cudaEventRecord(done, stream));
        t->inflight.push_back(InFlight{done, slot, capacity, N, T});
    }
    gf::RenderArgs a;
    a.f = f;
    a.mask = mask->buf.as<uint8_t>();
    a.ranges = t->ranges.as<uint2>();
    a.sortedIds = t->ids[t->finalBuf].as<uint32_t>();
    a.records = t->records.as<float4>();
    a.bounds = t->bounds.as<float>();
    a.rayO = in->ray_origin;
    a.rayD = in->ray_direction;
    a.log = gf::CompositeLog{};
    if (logComposites && T > 0 && t->cfg.composite_log_capacity >= 0) {
        const size_t perEntry = size_t(T) * gf::kTileThreads * sizeof(uint16_t);
        const size_t want = t->cfg.composite_log_capacity > 0 ? size_t(t->cfg.composite_log_capacity) : kLogCapacity;
        const uint32_t cap = uint32_t(std::min<size_t>(want, std::max<size_t>(1, kLogBudgetBytes / perEntry)));
        if (int e = t->logIds.ensure(perEntry * cap, stream)) return e;
        if (int e = t->logCount.ensure(size_t(T) * gf::kTileThreads * sizeof(uint32_t), stream)) return e;
        if (int e = t->logOverflow.ensure(sizeof(uint32_t) * size_t(T), stream)) return e;
        if (int e = t->logList.ensure(sizeof(uint32_t) * (size_t(T) + 1), stream)) return e;
        a.log.ids = t->logIds.as<uint16_t>();
        a.log.count = t->logCount.as<uint32_t>();
        a.log.overflow = t->logOverflow.as<uint32_t>();
        a.log.overflowCount = t->logList.as<uint32_t>();
        a.log.overflowList = t->logList.as<uint32_t>() + 1;
        GF_CUDA(cudaMemsetAsync(a.log.overflowCount, 0, sizeof(uint32_t), stream));
        a.log.capacity = cap;
        a.log.tiles = T;
    }
    t->frameLog = a.log;
    a.geo = gf::GeoOut{};
    if (geoOut != nullptr) {
        a.geo.normal = geoOut->normal;
        a.geo.depthVar = geoOut->depth_var;
        a.geo.quant = geoOut->quant;
        a.geo.extent = geoOut->extent;
        a.geo.invD = geoOut->inv_depth;
        a.geo.invD2 = geoOut->inv_depth2;
        a.geo.particles = in->particles;
    }
    t->frameGeo = geoOut != nullptr;
    {
        StageTimer st(t, GF_STAGE_RENDER_FWD, stream);
        if (t->cfg.compositor == GF_COMPOSITOR_SOF) {
            const int smem = int(gf::sof_smem_bytes());
            if (a.geo.particles != nullptr) {
                GF_CUDA(cudaFuncSetAttribute(gf::k_render_fwd_sof<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem));
                gf::k_render_fwd_sof<true><<<T, gf::kTileThreads, smem, stream>>>(a, rgba, hd, hc);
            } else {
                GF_CUDA(cudaFuncSetAttribute(gf::k_render_fwd_sof<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem));
                gf::k_render_fwd_sof<false><<<T, gf::kTileThreads, smem, stream>>>(a, rgba, hd, hc);
            }
        } else if (int e = dispatch_fwd(t->cfg.k_buffer_size, a, T, rgba, hd, hc, stream)) {
            return e;
        }
    }
    t->launches += 1;
    GF_LAUNCH_CHECK();
    t->frameSof = false;
    if (in->sof_opacity_active != 0) {
        if (geoOut == nullptr || geoOut->quant == nullptr || geoOut->opacity_field == nullptr)
            return fail(GF_ERR_BAD_INPUT, "the SOF opacity field needs enable_normals (its exact crossing depth)");
        gf::SofOpacityArgs so{};
        so.f = f;
        so.mask = a.mask;
        so.ranges = a.ranges;
        so.sortedIds = a.sortedIds;
        so.particles = in->particles;
        so.rayO = in->ray_origin;
        so.rayD = in->ray_direction;
        so.quant = geoOut->quant;
        so.opacity = geoOut->opacity_field;
        gf::k_sof_opacity<false><<<T, gf::kTileThreads, 0, stream>>>(so);
        t->launches += 1;
        GF_LAUNCH_CHECK();
        t->frameSof = true;
    }
    // the overflow count for gf_tracer_stats, read without a synchronization here
    t->logCounted = false;
    if (a.log.ids != nullptr) {
        if (t->logCopied == nullptr) GF_CUDA(cudaEventCreateWithFlags(&t->logCopied, cudaEventDisableTiming));
        t->hostTotal[2] = 0;
        GF_CUDA(cudaMemcpyAsync(t->hostTotal + 2, a.log.overflowCount, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream));
        GF_CUDA(cudaEventRecord(t->logCopied, stream));
        t->logCounted = true;
    }
    t->frameMask = a.mask;
    t->frameRayO = in->ray_origin;
    t->frameRayD = in->ray_direction;
    t->haveForward = true;
    t->totalLaunches += t->launches;
    return GF_OK;
}

}  // namespace

extern "C" {

int gf_abi_version(void) { return GF_ABI_VERSION; }

const char* gf_last_error(void) { return g_lastError.c_str(); }

gf_tracer* gf_tracer_create(const gf_tracer_config* config) {
    if (config == nullptr) {
        fail(GF_ERR_BAD_INPUT, "config is NULL");
        return nullptr;
    }
    if (!valid_k(config->k_buffer_size)) {
        fail(GF_ERR_BAD_INPUT, "k_buffer_size must be one of 0, 4, 8, 12, 16, 24, 32 (got %d)",
             config->k_buffer_size);
        return nullptr;
    }
    if (config->sort_key != GF_KEY_PER_TILE_DEPTH && config->sort_key != GF_KEY_GLOBAL_DEPTH) {
        fail(GF_ERR_BAD_INPUT, "unknown sort key %d", config->sort_key);
        return nullptr;
    }
    if (config->admission_fallback != GF_FALLBACK_NONE && config->admission_fallback != GF_FALLBACK_CONE &&
        config->admission_fallback != GF_FALLBACK_CONE_BIG) {
        fail(GF_ERR_BAD_INPUT, "unknown admission fallback %d", config->admission_fallback);
        return nullptr;
    }
    if (config->admission_fallback == GF_FALLBACK_CONE_BIG &&
        !(std::isfinite(config->fallback_min_angle) && std::isfinite(config->fallback_max_angle) &&
          config->fallback_min_angle >= 0.0f && config->fallback_min_angle <= config->fallback_max_angle)) {
        fail(GF_ERR_BAD_INPUT, "cone_big needs finite fallback angles with 0 <= min <= max (got %g, %g)",
             double(config->fallback_min_angle), double(config->fallback_max_angle));
        return nullptr;
    }
    if (!(std::isfinite(config->partial_ut_scale) && config->partial_ut_scale >= 0.0f)) {
        fail(GF_ERR_BAD_INPUT, "partial_ut_scale must be finite and >= 0 (got %g)", double(config->partial_ut_scale));
        return nullptr;
    }
    if (config->compositor != GF_COMPOSITOR_KBUFFER && config->compositor != GF_COMPOSITOR_SOF) {
        fail(GF_ERR_BAD_INPUT, "unknown compositor %d", config->compositor);
        return nullptr;
    }
    if (config->intersection_capacity != GF_CAPACITY_SPECULATIVE &&
        config->intersection_capacity != GF_CAPACITY_EXACT) {
        fail(GF_ERR_BAD_INPUT, "unknown intersection capacity mode %d", config->intersection_capacity);
        return nullptr;
    }
    gf_tracer* t = new gf_tracer();
    t->cfg = *config;
    return t;
}

void gf_tracer_destroy(gf_tracer* t) {
    if (t == nullptr) return;
    if (t->device >= 0) {
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(t->device);
        cudaDeviceSynchronize();
        for (DeviceBuffer* b : {&t->coneA, &t->coneS, &t->caps, &t->bigList, &t->bigCount, &t->wideList,
                                &t->tileCache, &t->cacheStart})
            b->release();
        for (DeviceBuffer* b : {&t->logIds, &t->logCount, &t->logOverflow, &t->logList}) b->release();
        DeviceBuffer* bufs[] = {&t->proj,    &t->records, &t->bounds, &t->counts, &t->offsets, &t->scanTiles, &t->total,
                                &t->tileRays, &t->ranges,  &t->keys[0], &t->keys[1], &t->ids[0],   &t->ids[1],
                                &t->hist,    &t->gradRecords, &t->gradShape, &t->gradIntrinsic};
        for (DeviceBuffer* b : bufs) b->release();
        for (auto& kv : t->masks) kv.second.buf.release();
        for (auto& ev : t->pending) {
            cudaEventDestroy(ev.start);
            cudaEventDestroy(ev.end);
        }
        for (cudaEvent_t e : t->eventPool) cudaEventDestroy(e);
        for (const InFlight& f : t->inflight) cudaEventDestroy(f.done);
        for (cudaEvent_t e : t->planEventPool) cudaEventDestroy(e);
        t->plan.release();
        if (t->hostPlans != nullptr) cudaFreeHost(t->hostPlans);
        if (t->logCopied != nullptr) cudaEventDestroy(t->logCopied);
        if (t->hostTotal != nullptr) cudaFreeHost(t->hostTotal);
        if (prev >= 0) cudaSetDevice(prev);
    }
    delete t;
}

int gf_tracer_register_tile_mask(gf_tracer* t, const uint8_t* mask, uint32_t tiles_y, uint32_t tiles_x,
                                 const char* token, void* stream) {
    if (t == nullptr || mask == nullptr || token == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL argument");
    if (tiles_y == 0 || tiles_x == 0) return fail(GF_ERR_BAD_INPUT, "empty tile mask");
    if (int e = bind_device(t)) return e;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    TileMask& m = t->masks[token];
    const size_t bytes = size_t(tiles_y) * tiles_x;
    if (int e = m.buf.ensure(bytes, s)) return e;
    GF_CUDA(cudaMemcpyAsync(m.buf.ptr, mask, bytes, cudaMemcpyDeviceToDevice, s));
    m.ty = tiles_y;
    m.tx = tiles_x;
    return GF_OK;
}

int gf_tracer_trace(gf_tracer* t, const gf_trace_inputs* in, const gf_trace_outputs* out, void* stream) {
    if (t == nullptr || out == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL argument");
    return forward(t, in, out->rgba, out->hit_distance, t->cfg.enable_hit_counts ? out->hit_count : nullptr,
                   out->visibility, true, t->cfg.enable_normals ? out : nullptr, static_cast<cudaStream_t>(stream));
}

int gf_tracer_trace_inference(gf_tracer* t, const gf_trace_inputs* in, float* rgba, float* hit_distance,
                              void* stream) {
    if (t == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL argument");
    return forward(t, in, rgba, hit_distance, nullptr, nullptr, false, nullptr, static_cast<cudaStream_t>(stream));
}

int gf_tracer_trace_bwd(gf_tracer* t, const gf_trace_inputs* in, const gf_trace_grads* g, void* stream) {
    if (t == nullptr || in == nullptr || g == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL argument");
    if (!t->haveForward) return fail(GF_ERR_STATE, "trace_bwd requires a preceding trace");
    if (int e = bind_device(t)) return e;
    if (int e = harvest(t, kMaxInFlight)) return e;  // without waiting
    if (int e = report_overflow(t)) return e;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    gf::FrameArgs& f = t->frame;
    if (in->num_particles != f.N || in->camera.width != f.W || in->camera.height != f.H ||
        in->sh_coeffs != f.shCoeffs || in->ray_origin != t->frameRayO || in->ray_direction != t->frameRayD)
        return fail(GF_ERR_STATE, "trace_bwd inputs differ from the preceding trace");
    if (g->rgba == nullptr || g->hit_distance == nullptr || g->grad_rgba == nullptr || g->grad_hit_distance == nullptr ||
        g->grad_particles == nullptr || g->grad_features == nullptr)
        return fail(GF_ERR_BAD_INPUT, "backward buffers are NULL");
    t->launches = 0;
    const uint32_t N = f.N;
    const uint32_t T = uint32_t(f.gx * f.gy);
    if (int e = t->gradRecords.ensure(sizeof(float4) * 4 * size_t(N) + 16, s)) return e;
    GF_CUDA(cudaMemsetAsync(t->gradRecords.ptr, 0, sizeof(float4) * 4 * size_t(N), s));
    gf::RenderBwdArgs a;
    a.r.f = f;
    a.r.mask = t->frameMask;
    a.r.ranges = t->ranges.as<uint2>();
    a.r.sortedIds = t->ids[t->finalBuf].as<uint32_t>();
    a.r.records = t->records.as<float4>();
    a.r.bounds = t->bounds.as<float>();
    a.r.rayO = t->frameRayO;
    a.r.rayD = t->frameRayD;
    a.r.log = t->frameLog;
    a.rgba = g->rgba;
    a.hitDistance = g->hit_distance;
    a.gradRgba = g->grad_rgba;
    a.gradHitDistance = g->grad_hit_distance;
    a.gradRecords = t->gradRecords.as<float4>();
    a.absGrad = g->position_abs_grad;
    a.absMode = g->position_abs_grad_mode;
    if (a.absGrad != nullptr && a.absMode != GF_ABS_GRAD_SCREEN && a.absMode != GF_ABS_GRAD_WORLD)
        return fail(GF_ERR_BAD_INPUT, "unknown position_abs_grad_mode %d", int(a.absMode));
    a.geo = gf::GeoBwd{};
    if (t->cfg.enable_normals && t->frameGeo) {
        a.geo.normal = g->normal;
        a.geo.gradNormal = g->grad_normal;
        a.geo.depthVar = g->depth_var;
        a.geo.gradDepthVar = g->grad_depth_var;
        a.geo.extent = g->extent;
        a.geo.gradExtent = g->grad_extent;
        a.geo.invD = g->inv_depth;
        a.geo.gradInvD = g->grad_inv_depth;
        a.geo.invD2 = g->inv_depth2;
        a.geo.gradInvD2 = g->grad_inv_depth2;
        a.geo.particles = in->particles;
        if (g->grad_quant != nullptr) {
            if (g->quant == nullptr) return fail(GF_ERR_BAD_INPUT, "a quantile-channel gradient needs the forward quant");
            a.geo.quant = g->quant;
            a.geo.gradQuant = g->grad_quant;
        }
        if (int e = t->gradShape.ensure(sizeof(float4) * 2 * size_t(N) + 16, s)) return e;
        GF_CUDA(cudaMemsetAsync(t->gradShape.ptr, 0, sizeof(float4) * 2 * size_t(N), s));
        a.geo.gradShape = t->gradShape.as<float4>();
    }
    {
        StageTimer st(t, GF_STAGE_RENDER_BWD, s);
        if (a.r.log.ids != nullptr) {
            // tiles with a complete log, then the replay of the tiles whose log overflowed
            if (a.geo.gradShape != nullptr) launch_render_bwd_log<true>(a, T, s);
            else launch_render_bwd_log<false>(a, T, s);
            t->launches += 1;
            GF_LAUNCH_CHECK();
        }
        if (t->residentBlocks == 0) t->residentBlocks = int(resident_blocks());
        const uint32_t grid = a.r.log.ids != nullptr ? std::min<uint32_t>(T, uint32_t(t->residentBlocks)) : T;
        if (t->cfg.compositor == GF_COMPOSITOR_SOF) {
            const int smem = int(gf::sof_smem_bytes());
            if (a.geo.gradShape != nullptr) {
                GF_CUDA(cudaFuncSetAttribute(gf::k_render_bwd_sof<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem));
                gf::k_render_bwd_sof<true><<<grid, gf::kTileThreads, smem, s>>>(a);
            } else {
                GF_CUDA(cudaFuncSetAttribute(gf::k_render_bwd_sof<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem));
                gf::k_render_bwd_sof<false><<<grid, gf::kTileThreads, smem, s>>>(a);
            }
        } else if (int e = dispatch_bwd(t->cfg.k_buffer_size, a, grid, s)) {
            return e;
        }
    }
    t->launches += 1;
    GF_LAUNCH_CHECK();
    float4* gradIntrinsic = nullptr;
    if (g->grad_opacity_field != nullptr) {
        if (!t->frameSof || g->opacity_field == nullptr || g->quant == nullptr)
            return fail(GF_ERR_STATE, "an opacity-field gradient needs a forward with the SOF opacity field");
        if (int e = t->gradIntrinsic.ensure(sizeof(float4) * 4 * size_t(N) + 16, s)) return e;
        GF_CUDA(cudaMemsetAsync(t->gradIntrinsic.ptr, 0, sizeof(float4) * 4 * size_t(N), s));
        gradIntrinsic = t->gradIntrinsic.as<float4>();
        gf::SofOpacityArgs so{};
        so.f = f;
        so.mask = t->frameMask;
        so.ranges = t->ranges.as<uint2>();
        so.sortedIds = t->ids[t->finalBuf].as<uint32_t>();
        so.particles = in->particles;
        so.rayO = t->frameRayO;
        so.rayD = t->frameRayD;
        so.quant = g->quant;
        so.opacityIn = g->opacity_field;
        so.gradOpacity = g->grad_opacity_field;
        so.gradIntrinsic = gradIntrinsic;
        gf::k_sof_opacity<true><<<T, gf::kTileThreads, 0, s>>>(so);
        t->launches += 1;
        GF_LAUNCH_CHECK();
    }
    if (N > 0) {
        StageTimer st(t, GF_STAGE_PROJECT_BWD, s);
        gf::k_project_bwd<<<(N + gf::kProjectBwdThreads - 1) / gf::kProjectBwdThreads, gf::kProjectBwdThreads,
                             gf::project_bwd_smem_bytes(f.shCoeffs), s>>>(
            f, in->particles, in->features, t->counts.as<uint32_t>(), t->gradRecords.as<float4>(), a.geo.gradShape,
            gradIntrinsic, g->grad_particles, g->grad_features);
        t->launches += 1;
        GF_LAUNCH_CHECK();
    }
    t->totalLaunches += t->launches;
    return GF_OK;
}

int gf_tracer_enable_timing(gf_tracer* t, int enable) {
    if (t == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL argument");
    t->timing = enable != 0;
    if (t->timing) {
        // Events for a few hundred traces, created now so that creating them
        // (a driver call of several microseconds each) adds no host time to
        // the timed calls; collect_times returns them to the pool.
        constexpr size_t kPoolEvents = 4096;
        while (t->eventPool.size() + 2 * t->pending.size() < kPoolEvents) {
            cudaEvent_t e = nullptr;
            GF_CUDA(cudaEventCreate(&e));
            t->eventPool.push_back(e);
        }
        t->pending.reserve(kPoolEvents / 2);
    }
    return GF_OK;
}

int gf_tracer_collect_times(gf_tracer* t, float* ms, uint32_t* launches) {
    if (t == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL argument");
    float acc[GF_NUM_STAGES] = {};
    uint32_t cnt[GF_NUM_STAGES] = {};
    for (auto& ev : t->pending) {
        GF_CUDA(cudaEventSynchronize(ev.end));
        float v = 0.0f;
        GF_CUDA(cudaEventElapsedTime(&v, ev.start, ev.end));
        acc[ev.stage] += v;
        cnt[ev.stage] += 1;
        t->eventPool.push_back(ev.start);
        t->eventPool.push_back(ev.end);
    }
    t->pending.clear();
    for (int i = 0; i < GF_NUM_STAGES; ++i) {
        if (ms != nullptr) ms[i] = acc[i];
        if (launches != nullptr) launches[i] = cnt[i];
    }
    return GF_OK;
}

int gf_tracer_stats(const gf_tracer* tc, gf_trace_stats* st) {
    if (tc == nullptr || st == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL argument");
    gf_tracer* t = const_cast<gf_tracer*>(tc);  // reading the plans of finished forwards updates the counts
    if (t->device >= 0) {
        if (int e = harvest(t, 0)) return e;
        if (int e = report_overflow(t)) return e;
    }
    st->num_intersections = t->numIntersections;
    st->num_tiles = uint32_t(t->frame.gx * t->frame.gy);
    st->num_particles = t->frame.N;
    st->kernel_launches = t->launches;
    st->fallback_particles = t->fallbackParticles;
    st->total_kernel_launches = t->totalLaunches;
    st->total_forwards = t->forwardsRead;
    st->total_intersections = t->intersectionsRead;
    st->total_fallback_particles = t->fallbackRead;
    st->total_host_wait_us = t->hostWaitUs;
    return GF_OK;
}

int gf_tracer_log_overflow_tiles(const gf_tracer* t, uint32_t* tiles) {
    if (t == nullptr || tiles == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL argument");
    *tiles = 0;
    if (t->logCounted) {
        GF_CUDA(cudaEventSynchronize(t->logCopied));
        *tiles = uint32_t(t->hostTotal[2]);
    }
    return GF_OK;
}

int gf_tracer_copy_intermediates(const gf_tracer* t, float* projected, float* radiance, uint32_t* counts,
                                 uint64_t* sorted_keys, uint32_t* sorted_ids, uint64_t capacity, uint32_t* ranges,
                                 void* stream) {
    if (t == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL argument");
    if (!t->haveForward) return fail(GF_ERR_STATE, "no forward pass to copy");
    if (int e = harvest(const_cast<gf_tracer*>(t), 0)) return e;  // the last forward's count
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t N = t->frame.N;
    const size_t T = size_t(t->frame.gx) * t->frame.gy;
    if (projected != nullptr && N > 0)
        GF_CUDA(cudaMemcpyAsync(projected, t->proj.ptr, sizeof(float4) * 2 * N, cudaMemcpyDeviceToDevice, s));
    if (radiance != nullptr && N > 0)
        GF_CUDA(cudaMemcpy2DAsync(radiance, 3 * sizeof(float), static_cast<const char*>(t->records.ptr) + 52,
                                  sizeof(float4) * 4, 3 * sizeof(float), N, cudaMemcpyDeviceToDevice, s));
    if (counts != nullptr && N > 0)
        GF_CUDA(cudaMemcpyAsync(counts, t->counts.ptr, sizeof(uint32_t) * N, cudaMemcpyDeviceToDevice, s));
    const uint64_t I = t->numIntersections;
    if ((sorted_keys != nullptr || sorted_ids != nullptr) && capacity < I)
        return fail(GF_ERR_CAPACITY, "capacity %llu < %llu intersections", static_cast<unsigned long long>(capacity),
                    static_cast<unsigned long long>(I));
    if (sorted_keys != nullptr && I > 0)
        GF_CUDA(cudaMemcpyAsync(sorted_keys, t->keys[t->finalBuf].ptr, sizeof(uint64_t) * I, cudaMemcpyDeviceToDevice, s));
    if (sorted_ids != nullptr && I > 0)
        GF_CUDA(cudaMemcpyAsync(sorted_ids, t->ids[t->finalBuf].ptr, sizeof(uint32_t) * I, cudaMemcpyDeviceToDevice, s));
    if (ranges != nullptr)
        GF_CUDA(cudaMemcpyAsync(ranges, t->ranges.ptr, sizeof(uint2) * T, cudaMemcpyDeviceToDevice, s));
    return GF_OK;
}

}  // extern "C"
