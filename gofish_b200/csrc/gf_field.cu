// Host orchestration and C ABI of the mesh opacity field and its bisection
// table (reference gofish/mesh/native/include/3dgut/kernels/cuda/common/
// opacityFieldBinding.inl).
//
// A gf_field holds at most one context at a time, as the reference's
// SplatRaster does (opacityFieldBinding.inl:206-207): a field context
// (begin / integrate camera* / finish / release) or a bisection table
// (begin / stage camera* / seal / round 0..7 [/ reset / round 0..7]* /
// release).  The context copies its Gaussians, query points and staged
// camera rays and owns them until release.  Every call must come from the
// device and the stream the context was begun on.
//
// Host synchronization: one per camera pass (the number of candidate pairs
// sizes the sort), one in finish and one per bisection round (the reference
// also synchronizes once per round, opacityFieldBinding.inl:507-515).
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/gofish_b200.h"
#include "gf_host.cuh"
#include "gf_field_kernels.cuh"

namespace {

struct StagedCamera {
    gf_camera cam{};
    gf::Pose pose{};
    DeviceBuffer rayO, mask;
    bool masked = false;
};

// One camera pass's view of a camera: where its rays and mask live.
struct CameraView {
    gf_camera cam;
    gf::Pose pose;
    const float* rayO;
    const uint8_t* mask;
};

}  // namespace

struct gf_field {
    int device = -1;
    bool live = false;
    int64_t token = 0;
    int64_t nextToken = 1;
    cudaStream_t stream = nullptr;
    bool finished = false;
    bool table = false, sealed = false;
    uint32_t round = 0;
    uint32_t cameras = 0;
    uint32_t N = 0, Q = 0;

    DeviceBuffer posd, binv, points, minimum, observed, active, exact, err;
    DeviceBuffer pixKey, info, sorted, hist, pointStart, coneA, coneB, cellBlocks, blockStart;
    DeviceBuffer cull, hit, counts, offsets, totals, keys[2], ids[2], sortHist, scanTiles, cellRanges;
    DeviceBuffer bigList, bigCount;  // Gaussians binned by warps (over the per-thread traversal budget)
    std::vector<StagedCamera> staged;
    uint64_t* host = nullptr;  // pinned: pairs, blocks | valid points, error flag
    uint32_t launches = 0;
    gf_field_stats stats{};
    DeviceBuffer counters;  // u64 [4]: candidates staged, exact hit tests, hits, warp candidate iterations

    // Per-stage event timing (gf_field_enable_timing).
    bool timing = false;
    struct StageEvent {
        int stage;
        uint32_t launches;
        cudaEvent_t start, end;
    };
    std::vector<StageEvent> pending;
    std::vector<cudaEvent_t> eventPool;
};

namespace {

constexpr uint32_t kMaxRaster = 32768;
constexpr uint32_t kBigBlocks = 148 * 8;  // warp-cooperative binning grid (8 warps per block)

#define GF_TRY(...)                           \
    do {                                      \
        if (int e_ = (__VA_ARGS__)) return e_; \
    } while (0)

int require_device(gf_field* f) {
    int dev = -1;
    GF_CUDA(cudaGetDevice(&dev));
    if (f->device < 0) {
        f->device = dev;
        GF_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&f->host), 4 * sizeof(uint64_t), cudaHostAllocDefault));
        return GF_OK;
    }
    if (f->device != dev)
        return fail(GF_ERR_STATE, "opacity field: expected cuda:%d, current cuda:%d", f->device, dev);
    return GF_OK;
}

int require_context(gf_field* f, int64_t token, cudaStream_t stream, const char* operation) {
    if (f == nullptr) return fail(GF_ERR_BAD_INPUT, "field is NULL");
    if (!f->live || f->token != token) return fail(GF_ERR_STATE, "missing or stale opacity-field context");
    GF_TRY(require_device(f));
    if (stream != f->stream)
        return fail(GF_ERR_STATE, "%s: the opacity field must run on the stream it was created on", operation);
    return GF_OK;
}

cudaEvent_t take_event(gf_field* f) {
    if (!f->eventPool.empty()) {
        cudaEvent_t e = f->eventPool.back();
        f->eventPool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    return e;
}

// Brackets one stage with events (when timing is on) and attributes the
// kernels launched inside it.
struct StageTimer {
    gf_field* f;
    int stage;
    cudaStream_t stream;
    uint32_t launches0;
    cudaEvent_t start = nullptr;
    StageTimer(gf_field* f_, int stage_, cudaStream_t s) : f(f_), stage(stage_), stream(s), launches0(f_->launches) {
        if (f->timing) {
            start = take_event(f);
            if (start != nullptr) cudaEventRecord(start, stream);
        }
    }
    ~StageTimer() {
        if (start == nullptr) return;
        cudaEvent_t end = take_event(f);
        if (end == nullptr) return;
        cudaEventRecord(end, stream);
        f->pending.push_back({stage, f->launches - launches0, start, end});
    }
};

bool finite7(const float* p) {
    for (int k = 0; k < 7; ++k)
        if (!std::isfinite(p[k])) return false;
    return true;
}

int validate_camera(const gf_field_camera* c) {
    if (c == nullptr) return fail(GF_ERR_BAD_INPUT, "camera is NULL");
    const gf_camera& cam = c->camera;
    if (c->ray_origin == nullptr) return fail(GF_ERR_BAD_INPUT, "ray origin is NULL");
    if (cam.width <= 0 || cam.height <= 0) return fail(GF_ERR_BAD_INPUT, "rays must be nonempty [1,H,W,3]");
    if (uint32_t(cam.width) > kMaxRaster || uint32_t(cam.height) > kMaxRaster)
        return fail(GF_ERR_BAD_INPUT, "camera raster is too large (at most %u per side)", kMaxRaster);
    if (cam.model != GF_CAMERA_OPENCV_FISHEYE && cam.model != GF_CAMERA_OPENCV_PINHOLE)
        return fail(GF_ERR_BAD_INPUT, "only OPENCV_FISHEYE and PINHOLE cameras are supported");
    if (cam.shutter != GF_SHUTTER_GLOBAL)
        return fail(GF_ERR_BAD_INPUT, "the opacity field supports global-shutter cameras only");
    if (!finite7(c->pose_start) || !finite7(c->pose_end) || std::memcmp(c->pose_start, c->pose_end, 7 * sizeof(float)))
        return fail(GF_ERR_BAD_INPUT, "global-shutter camera poses must be finite and identical");
    return GF_OK;
}

// Level grids of the cone quadtree for a raster.
int make_levels(uint32_t W, uint32_t H, gf::field::Levels& L, uint32_t& totalNodes) {
    uint32_t gx = (W + gf::field::kCell - 1) / gf::field::kCell, gy = (H + gf::field::kCell - 1) / gf::field::kCell;
    L.n = 0;
    totalNodes = 0;
    while (true) {
        if (L.n >= gf::field::kMaxLevels) return fail(GF_ERR_BAD_INPUT, "camera raster is too large for the cell tree");
        L.gx[L.n] = gx;
        L.gy[L.n] = gy;
        L.offset[L.n] = totalNodes;
        totalNodes += gx * gy;
        ++L.n;
        if (gx * gy == 1u) break;
        gx = (gx + gf::field::kFan - 1) / gf::field::kFan;
        gy = (gy + gf::field::kFan - 1) / gf::field::kFan;
    }
    return GF_OK;
}

// One camera pass over the current points: field mode (round == false)
// updates the camera-min field, round mode classifies the active points.
int run_camera(gf_field* f, const CameraView& v, bool round, const float* points, cudaStream_t s) {
    using namespace gf::field;
    const uint32_t W = uint32_t(v.cam.width), H = uint32_t(v.cam.height);
    Levels L{};
    uint32_t totalNodes = 0;
    GF_TRY(make_levels(W, H, L, totalNodes));
    const uint32_t cells = L.gx[0] * L.gy[0];
    const uint32_t pixKeys = cells * kCellPixels;
    const uint32_t Q = f->Q, N = f->N;

    GF_TRY(f->pixKey.ensure(sizeof(uint32_t) * Q, s));
    GF_TRY(f->info.ensure(sizeof(float4) * Q, s));
    GF_TRY(f->sorted.ensure(sizeof(uint32_t) * Q, s));
    GF_TRY(f->hist.ensure(sizeof(uint32_t) * pixKeys, s));
    GF_TRY(f->pointStart.ensure(sizeof(uint32_t) * (size_t(pixKeys) + 1), s));
    GF_TRY(f->coneA.ensure(sizeof(float4) * totalNodes, s));
    GF_TRY(f->coneB.ensure(sizeof(float4) * totalNodes, s));
    GF_TRY(f->cellBlocks.ensure(sizeof(uint32_t) * cells, s));
    GF_TRY(f->blockStart.ensure(sizeof(uint32_t) * (size_t(cells) + 1), s));
    GF_TRY(f->cull.ensure(sizeof(float4) * N, s));
    GF_TRY(f->hit.ensure(sizeof(float4) * 4 * size_t(N), s));
    GF_TRY(f->counts.ensure(sizeof(uint32_t) * N, s));
    GF_TRY(f->offsets.ensure(sizeof(uint64_t) * N, s));
    GF_TRY(f->totals.ensure(sizeof(uint64_t) * 2, s));
    GF_TRY(f->cellRanges.ensure(sizeof(uint2) * cells, s));
    GF_TRY(f->bigList.ensure(sizeof(uint32_t) * N, s));
    GF_TRY(f->bigCount.ensure(sizeof(uint32_t), s));

    CameraArgs a{};
    a.cam = v.cam;
    a.pose = v.pose;
    a.rayO = v.rayO;
    a.mask = v.mask;
    a.W = W;
    a.H = H;
    a.gx = L.gx[0];
    a.gy = L.gy[0];
    L.A = f->coneA.as<float4>();
    L.B = f->coneB.as<float4>();

    uint32_t* hist = f->hist.as<uint32_t>();
    uint32_t* pointStart = f->pointStart.as<uint32_t>();
    const uint32_t qBlocks = (Q + 255) / 256;
    {
        StageTimer st(f, GF_FIELD_STAGE_POINTS, s);
        GF_CUDA(cudaMemsetAsync(hist, 0, sizeof(uint32_t) * pixKeys, s));
        k_field_points<<<qBlocks, 256, 0, s>>>(a, points, Q, round ? f->active.as<uint8_t>() : nullptr,
                                               f->pixKey.as<uint32_t>(), f->info.as<float4>(), hist,
                                               f->err.as<uint32_t>());
        f->launches += 1;
        GF_LAUNCH_CHECK();
        GF_TRY(scan_exclusive<uint32_t, uint32_t>(f->scanTiles, f->launches, hist, pixKeys, pointStart,
                                                  pointStart + pixKeys, s));
        k_field_scatter<<<qBlocks, 256, 0, s>>>(f->pixKey.as<uint32_t>(), Q, pointStart, hist,
                                                f->sorted.as<uint32_t>());
        f->launches += 1;
        GF_LAUNCH_CHECK();
    }
    {
        StageTimer st(f, GF_FIELD_STAGE_CONES, s);
        k_cell_cones<<<(cells * 32 + 255) / 256, 256, 0, s>>>(pointStart, f->sorted.as<uint32_t>(), f->info.as<float4>(),
                                                             cells, f->coneA.as<float4>(), f->coneB.as<float4>());
        f->launches += 1;
        GF_LAUNCH_CHECK();
        for (int l = 1; l < L.n; ++l) {
            const uint32_t nodes = L.gx[l] * L.gy[l];
            k_cone_reduce<<<(nodes + 255) / 256, 256, 0, s>>>(
                f->coneA.as<float4>() + L.offset[l - 1], f->coneB.as<float4>() + L.offset[l - 1], L.gx[l - 1], L.gy[l - 1],
                f->coneA.as<float4>() + L.offset[l], f->coneB.as<float4>() + L.offset[l], L.gx[l], L.gy[l]);
            f->launches += 1;
            GF_LAUNCH_CHECK();
        }
        k_cell_blocks<<<(cells + 255) / 256, 256, 0, s>>>(pointStart, cells, f->cellBlocks.as<uint32_t>());
        f->launches += 1;
        GF_LAUNCH_CHECK();
        uint32_t* totals32 = reinterpret_cast<uint32_t*>(f->totals.as<uint64_t>() + 1);
        GF_TRY(scan_exclusive<uint32_t, uint32_t>(f->scanTiles, f->launches, f->cellBlocks.as<uint32_t>(), cells,
                                                  f->blockStart.as<uint32_t>(), totals32, s));
    }
    {
        StageTimer st(f, GF_FIELD_STAGE_CANDIDATES, s);
        ParticleArgs p{f->posd.as<float4>(), f->binv.as<float4>(), N};
        GF_CUDA(cudaMemsetAsync(f->bigCount.ptr, 0, sizeof(uint32_t), s));
        k_field_particles<<<(N + 255) / 256, 256, 0, s>>>(a, p, L, f->cull.as<float4>(), f->hit.as<float4>(),
                                                          f->counts.as<uint32_t>(), f->bigList.as<uint32_t>(),
                                                          f->bigCount.as<uint32_t>());
        k_field_big<false><<<kBigBlocks, 256, 0, s>>>(L, f->bigList.as<uint32_t>(), f->bigCount.as<uint32_t>(),
                                                      f->cull.as<float4>(), f->hit.as<float4>(),
                                                      f->counts.as<uint32_t>(), nullptr, nullptr, nullptr);
        f->launches += 2;
        GF_LAUNCH_CHECK();
        GF_TRY(scan_exclusive<uint32_t, uint64_t>(f->scanTiles, f->launches, f->counts.as<uint32_t>(), N,
                                                  f->offsets.as<uint64_t>(), f->totals.as<uint64_t>(), s));
    }
    GF_CUDA(cudaMemcpyAsync(f->host, f->totals.ptr, 2 * sizeof(uint64_t), cudaMemcpyDeviceToHost, s));
    GF_CUDA(cudaMemcpyAsync(reinterpret_cast<uint32_t*>(f->host + 2), pointStart + pixKeys, sizeof(uint32_t),
                            cudaMemcpyDeviceToHost, s));
    GF_CUDA(cudaStreamSynchronize(s));
    const uint64_t pairs = f->host[0];
    const uint32_t blocks = reinterpret_cast<const uint32_t*>(f->host + 1)[0];
    const uint32_t validPoints = reinterpret_cast<const uint32_t*>(f->host + 2)[0];
    if (pairs > 0xffffffffull - gf::kSortTile)
        return fail(GF_ERR_CAPACITY, "%llu candidate pairs exceed the 32-bit index range",
                    static_cast<unsigned long long>(pairs));
    for (int b = 0; b < 2; ++b) {
        GF_TRY(f->keys[b].ensure(sizeof(uint64_t) * (pairs + 1), s));
        GF_TRY(f->ids[b].ensure(sizeof(uint32_t) * (pairs + 1), s));
    }
    int finalBuf = 0;
    {
        StageTimer st(f, GF_FIELD_STAGE_SORT, s);
        if (pairs > 0) {
            k_field_emit<<<(N + 255) / 256, 256, 0, s>>>(L, N, f->cull.as<float4>(), f->hit.as<float4>(),
                                                         f->counts.as<uint32_t>(), f->offsets.as<uint64_t>(),
                                                         f->keys[0].as<uint64_t>(), f->ids[0].as<uint32_t>());
            k_field_big<true><<<kBigBlocks, 256, 0, s>>>(L, f->bigList.as<uint32_t>(), f->bigCount.as<uint32_t>(),
                                                         f->cull.as<float4>(), f->hit.as<float4>(),
                                                         f->counts.as<uint32_t>(), f->offsets.as<uint64_t>(),
                                                         f->keys[0].as<uint64_t>(), f->ids[0].as<uint32_t>());
            f->launches += 2;
            GF_LAUNCH_CHECK();
        }
        GF_TRY(sort_pairs(f->sortHist, f->scanTiles, f->launches, f->keys, f->ids, uint32_t(pairs), 32,
                          32 + int(bit_length(cells)), &finalBuf, s));
        GF_CUDA(cudaMemsetAsync(f->cellRanges.ptr, 0, sizeof(uint2) * cells, s));
        if (pairs > 0) {
            k_cell_ranges<<<uint32_t((pairs + 255) / 256), 256, 0, s>>>(f->keys[finalBuf].as<uint64_t>(), uint32_t(pairs),
                                                                        f->cellRanges.as<uint2>());
            f->launches += 1;
            GF_LAUNCH_CHECK();
        }
    }
    if (blocks > 0) {
        StageTimer st(f, GF_FIELD_STAGE_INTEGRATE, s);
        IntegrateArgs ia{};
        ia.blockStart = f->blockStart.as<uint32_t>();
        ia.cells = cells;
        ia.pointStart = pointStart;
        ia.sorted = f->sorted.as<uint32_t>();
        ia.pixKey = f->pixKey.as<uint32_t>();
        ia.info = f->info.as<float4>();
        ia.cellRanges = f->cellRanges.as<uint2>();
        ia.candIds = f->ids[finalBuf].as<uint32_t>();
        ia.cull = f->cull.as<float4>();
        ia.hit = f->hit.as<float4>();
        ia.minimum = f->minimum.as<float>();
        ia.observed = f->observed.as<uint8_t>();
        ia.active = f->active.as<uint8_t>();
        ia.exact = f->exact.as<uint8_t>();
        ia.counters = f->counters.as<unsigned long long>();
        if (round) k_field_integrate<true><<<blocks, kBlock, 0, s>>>(ia);
        else k_field_integrate<false><<<blocks, kBlock, 0, s>>>(ia);
        f->launches += 1;
        GF_LAUNCH_CHECK();
    }
    f->stats.evaluations += validPoints;
    f->stats.pairs += pairs;
    f->stats.cameras += 1;
    f->stats.kernel_launches += f->launches;
    f->launches = 0;
    return GF_OK;
}

int begin_context(gf_field* f, const float* particles, const float* sigmaMax, uint32_t N, const float* points,
                  uint32_t Q, int64_t* token, cudaStream_t s, bool table) {
    if (f == nullptr || token == nullptr) return fail(GF_ERR_BAD_INPUT, "field or token is NULL");
    if (f->live) return fail(GF_ERR_STATE, "cannot begin a second opacity field while one is active");
    GF_TRY(require_device(f));
    if (Q == 0 || Q > 0x7fffffffu) return fail(GF_ERR_BAD_INPUT, "query points must be nonempty float32 [Q,3]");
    if (N == 0) return fail(GF_ERR_BAD_INPUT, "particle density must be float32 [N,32]");
    if (particles == nullptr || sigmaMax == nullptr || points == nullptr)
        return fail(GF_ERR_BAD_INPUT, "particle, sigma_max and point buffers must not be NULL");
    GF_TRY(f->posd.ensure(sizeof(float4) * N, s));
    GF_TRY(f->binv.ensure(sizeof(float4) * 3 * size_t(N), s));
    GF_TRY(f->points.ensure(sizeof(float) * 3 * size_t(Q), s));
    GF_TRY(f->minimum.ensure(sizeof(float) * Q, s));
    GF_TRY(f->observed.ensure(Q, s));
    GF_TRY(f->active.ensure(Q, s));
    GF_TRY(f->exact.ensure(Q, s));
    GF_TRY(f->err.ensure(sizeof(uint32_t), s));
    if (f->counters.ptr == nullptr) {
        GF_TRY(f->counters.ensure(4 * sizeof(unsigned long long), s));
        GF_CUDA(cudaMemsetAsync(f->counters.ptr, 0, 4 * sizeof(unsigned long long), s));
    }
    gf::field::k_field_pack<<<(N + 255) / 256, 256, 0, s>>>(particles, N, f->posd.as<float4>(), f->binv.as<float4>());
    f->stats.kernel_launches += 1;
    GF_LAUNCH_CHECK();
    GF_CUDA(cudaMemcpyAsync(f->points.ptr, points, sizeof(float) * 3 * size_t(Q), cudaMemcpyDeviceToDevice, s));
    GF_CUDA(cudaMemsetAsync(f->observed.ptr, 0, Q, s));
    GF_CUDA(cudaMemsetAsync(f->err.ptr, 0, sizeof(uint32_t), s));
    f->N = N;
    f->Q = Q;
    f->stream = s;
    f->live = true;
    f->finished = false;
    f->table = table;
    f->sealed = false;
    f->round = 0;
    f->cameras = 0;
    f->staged.clear();
    f->token = f->nextToken++;
    *token = f->token;
    return GF_OK;
}

int check_error_flag(gf_field* f, cudaStream_t s) {
    GF_CUDA(cudaMemcpyAsync(f->host + 3, f->err.ptr, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    GF_CUDA(cudaStreamSynchronize(s));
    if (reinterpret_cast<const uint32_t*>(f->host + 3)[0] != 0u)
        return fail(GF_ERR_BAD_INPUT, "the opacity field requires one camera center per view");
    return GF_OK;
}

void end_context(gf_field* f) {
    f->live = false;
    f->staged.clear();
}

}  // namespace

extern "C" {

gf_field* gf_field_create(void) { return new (std::nothrow) gf_field(); }

void gf_field_destroy(gf_field* f) {
    if (f == nullptr) return;
    if (f->device >= 0) {
        int prior = -1;
        cudaGetDevice(&prior);
        cudaSetDevice(f->device);
        cudaDeviceSynchronize();
        DeviceBuffer* bufs[] = {&f->posd,      &f->binv,       &f->points,     &f->minimum, &f->observed,
                                &f->active,    &f->exact,      &f->err,        &f->pixKey,  &f->info,
                                &f->sorted,    &f->hist,       &f->pointStart, &f->coneA,   &f->coneB,
                                &f->cellBlocks, &f->blockStart, &f->cull,      &f->hit,     &f->counts,
                                &f->offsets,   &f->totals,     &f->keys[0],    &f->keys[1], &f->ids[0],
                                &f->ids[1],    &f->sortHist,   &f->scanTiles,  &f->cellRanges};
        for (DeviceBuffer* b : bufs) b->release();
        f->counters.release();
        f->bigList.release();
        f->bigCount.release();
        for (auto& e : f->pending) {
            cudaEventDestroy(e.start);
            cudaEventDestroy(e.end);
        }
        for (cudaEvent_t e : f->eventPool) cudaEventDestroy(e);
        for (StagedCamera& c : f->staged) {
            c.rayO.release();
            c.mask.release();
        }
        if (f->host != nullptr) cudaFreeHost(f->host);
        if (prior >= 0) cudaSetDevice(prior);
    }
    delete f;
}

int gf_field_begin(gf_field* f, const float* particles, const float* sigma_max, uint32_t num_particles,
                   const float* points, uint32_t num_points, int64_t* token, void* stream) {
    return begin_context(f, particles, sigma_max, num_particles, points, num_points, token,
                         static_cast<cudaStream_t>(stream), false);
}

int gf_field_integrate_camera(gf_field* f, int64_t token, const gf_field_camera* camera, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GF_TRY(require_context(f, token, s, "integrate opacity-field camera"));
    if (f->table) return fail(GF_ERR_STATE, "camera integration rejected a bisection table");
    if (f->finished) return fail(GF_ERR_STATE, "cannot integrate a camera after finish");
    GF_TRY(validate_camera(camera));
    CameraView v{};
    v.cam = camera->camera;
    prepare_pose(camera->pose_start, v.pose);
    v.rayO = camera->ray_origin;
    v.mask = camera->pixel_mask;
    GF_TRY(run_camera(f, v, false, f->points.as<float>(), s));
    ++f->cameras;
    return GF_OK;
}

int gf_field_finish(gf_field* f, int64_t token, float* opacity, uint8_t* observed, uint8_t* above, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GF_TRY(require_context(f, token, s, "finish opacity field"));
    if (f->table) return fail(GF_ERR_STATE, "finish rejected a bisection table");
    if (f->finished) return fail(GF_ERR_STATE, "the opacity field was already finished");
    if (f->cameras == 0) return fail(GF_ERR_STATE, "the opacity field has no camera");
    if (opacity == nullptr || observed == nullptr || above == nullptr)
        return fail(GF_ERR_BAD_INPUT, "output buffers must not be NULL");
    {
        StageTimer st(f, GF_FIELD_STAGE_FINISH, s);
        gf::field::k_field_finish<<<(f->Q + 255) / 256, 256, 0, s>>>(
            f->minimum.as<float>(), f->observed.as<uint8_t>(), f->Q, opacity, observed, above);
        f->launches += 1;
        GF_LAUNCH_CHECK();
    }
    f->stats.kernel_launches += f->launches;
    f->launches = 0;
    GF_TRY(check_error_flag(f, s));
    f->finished = true;
    return GF_OK;
}

int gf_field_release(gf_field* f, int64_t token, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GF_TRY(require_context(f, token, s, "release opacity field"));
    if (f->table) return fail(GF_ERR_STATE, "release rejected a bisection table");
    if (!f->finished) return fail(GF_ERR_STATE, "cannot release an opacity field before finish");
    GF_CUDA(cudaStreamSynchronize(s));
    end_context(f);
    return GF_OK;
}

int gf_field_begin_table(gf_field* f, const float* particles, const float* sigma_max, uint32_t num_particles,
                         const float* probe_points, uint32_t num_points, int64_t* token, void* stream) {
    return begin_context(f, particles, sigma_max, num_particles, probe_points, num_points, token,
                         static_cast<cudaStream_t>(stream), true);
}

int gf_field_stage_camera(gf_field* f, int64_t token, const gf_field_camera* camera, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GF_TRY(require_context(f, token, s, "stage bisection camera"));
    if (!f->table) return fail(GF_ERR_STATE, "stage requires a bisection table");
    if (f->sealed) return fail(GF_ERR_STATE, "cannot append to a sealed bisection table");
    GF_TRY(validate_camera(camera));
    f->staged.emplace_back();
    StagedCamera& c = f->staged.back();
    c.cam = camera->camera;
    prepare_pose(camera->pose_start, c.pose);
    const size_t pixels = size_t(c.cam.width) * size_t(c.cam.height);
    int e = c.rayO.ensure(sizeof(float) * 3 * pixels, s);
    if (e == GF_OK) {
        const cudaError_t ce = cudaMemcpyAsync(c.rayO.ptr, camera->ray_origin, sizeof(float) * 3 * pixels,
                                               cudaMemcpyDeviceToDevice, s);
        if (ce != cudaSuccess) e = fail(GF_ERR_CUDA, "ray origin copy failed: %s", cudaGetErrorString(ce));
    }
    if (e == GF_OK && camera->pixel_mask != nullptr) {
        c.masked = true;
        e = c.mask.ensure(pixels, s);
        if (e == GF_OK) {
            const cudaError_t ce = cudaMemcpyAsync(c.mask.ptr, camera->pixel_mask, pixels, cudaMemcpyDeviceToDevice, s);
            if (ce != cudaSuccess) e = fail(GF_ERR_CUDA, "mask copy failed: %s", cudaGetErrorString(ce));
        }
    }
    if (e != GF_OK) {
        c.rayO.release();
        c.mask.release();
        f->staged.pop_back();
        return e;
    }
    ++f->cameras;
    return GF_OK;
}

int gf_field_seal_table(gf_field* f, int64_t token, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GF_TRY(require_context(f, token, s, "seal bisection table"));
    if (!f->table) return fail(GF_ERR_STATE, "seal requires a bisection table");
    if (f->sealed || f->staged.empty() || f->cameras != f->staged.size())
        return fail(GF_ERR_STATE, "bisection table camera population differs");
    GF_CUDA(cudaStreamSynchronize(s));
    f->sealed = true;
    f->finished = false;
    f->round = 0;
    return GF_OK;
}

int gf_field_evaluate_round(gf_field* f, int64_t token, const float* points, uint32_t num_points, uint32_t round,
                            uint8_t* above, uint8_t* observed, uint8_t* exact, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GF_TRY(require_context(f, token, s, "evaluate bisection round"));
    if (!f->table) return fail(GF_ERR_STATE, "round requires a bisection table");
    if (!f->sealed || f->finished || round != f->round || round >= 8u)
        return fail(GF_ERR_STATE, "bisection rounds must run in order [0,8)");
    if (points == nullptr || num_points != f->Q)
        return fail(GF_ERR_BAD_INPUT, "round query shape differs from the table capacity");
    if (above == nullptr || observed == nullptr || exact == nullptr)
        return fail(GF_ERR_BAD_INPUT, "output buffers must not be NULL");
    GF_CUDA(cudaMemsetAsync(f->active.ptr, 1, f->Q, s));
    GF_CUDA(cudaMemsetAsync(f->observed.ptr, 0, f->Q, s));
    GF_CUDA(cudaMemsetAsync(f->exact.ptr, 0, f->Q, s));
    GF_CUDA(cudaMemsetAsync(f->err.ptr, 0, sizeof(uint32_t), s));
    for (StagedCamera& c : f->staged) {
        CameraView v{c.cam, c.pose, c.rayO.as<float>(), c.masked ? c.mask.as<uint8_t>() : nullptr};
        GF_TRY(run_camera(f, v, true, points, s));
    }
    {
        StageTimer st(f, GF_FIELD_STAGE_FINISH, s);
        gf::field::k_round_finalize<<<(f->Q + 255) / 256, 256, 0, s>>>(
            f->active.as<uint8_t>(), f->observed.as<uint8_t>(), f->exact.as<uint8_t>(), f->Q, above, observed, exact);
        f->launches += 1;
        GF_LAUNCH_CHECK();
    }
    f->stats.kernel_launches += f->launches;
    f->launches = 0;
    GF_TRY(check_error_flag(f, s));
    ++f->round;
    if (f->round == 8u) f->finished = true;
    return GF_OK;
}

int gf_field_reset_batch(gf_field* f, int64_t token, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GF_TRY(require_context(f, token, s, "reset bisection batch"));
    if (!f->table) return fail(GF_ERR_STATE, "reset requires a bisection table");
    if (!f->sealed || !f->finished || f->round != 8u)
        return fail(GF_ERR_STATE, "a query batch can be reset only after all eight rounds");
    f->round = 0;
    f->finished = false;
    return GF_OK;
}

int gf_field_release_table(gf_field* f, int64_t token, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GF_TRY(require_context(f, token, s, "release bisection table"));
    if (!f->table) return fail(GF_ERR_STATE, "release requires a bisection table");
    if (!f->sealed || !f->finished || f->round != 8u)
        return fail(GF_ERR_STATE, "the bisection table can be released only after all eight rounds");
    GF_CUDA(cudaStreamSynchronize(s));
    for (StagedCamera& c : f->staged) {
        c.rayO.release();
        c.mask.release();
    }
    end_context(f);
    return GF_OK;
}

int gf_field_get_stats(gf_field* f, gf_field_stats* stats) {
    if (f == nullptr || stats == nullptr) return fail(GF_ERR_BAD_INPUT, "field or stats is NULL");
    *stats = f->stats;
    if (f->counters.ptr != nullptr) {
        unsigned long long c[4] = {0, 0, 0, 0};
        GF_CUDA(cudaMemcpy(c, f->counters.ptr, sizeof(c), cudaMemcpyDeviceToHost));
        stats->candidate_loads = c[0];
        stats->hit_tests = c[1];
        stats->hits = c[2];
        stats->warp_iterations = c[3];
    }
    return GF_OK;
}

int gf_field_enable_timing(gf_field* f, int enable) {
    if (f == nullptr) return fail(GF_ERR_BAD_INPUT, "field is NULL");
    f->timing = enable != 0;
    return GF_OK;
}

int gf_field_collect_times(gf_field* f, float* ms, uint32_t* launches) {
    if (f == nullptr) return fail(GF_ERR_BAD_INPUT, "field is NULL");
    float acc[GF_FIELD_STAGES] = {0};
    uint32_t cnt[GF_FIELD_STAGES] = {0};
    int status = GF_OK;
    for (auto& e : f->pending) {
        float t = 0.0f;
        if (status == GF_OK) {
            cudaError_t ce = cudaEventSynchronize(e.end);
            if (ce == cudaSuccess) ce = cudaEventElapsedTime(&t, e.start, e.end);
            if (ce != cudaSuccess) status = fail(GF_ERR_CUDA, "stage timing failed: %s", cudaGetErrorString(ce));
        }
        if (e.stage >= 0 && e.stage < GF_FIELD_STAGES) {
            acc[e.stage] += t;
            cnt[e.stage] += e.launches;
        }
        f->eventPool.push_back(e.start);
        f->eventPool.push_back(e.end);
    }
    f->pending.clear();
    for (int i = 0; i < GF_FIELD_STAGES; ++i) {
        if (ms != nullptr) ms[i] = acc[i];
        if (launches != nullptr) launches[i] = cnt[i];
    }
    return status;
}

}  // extern "C"
