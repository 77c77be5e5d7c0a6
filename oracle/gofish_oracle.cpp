// CPU oracle for the GOFish fisheye tracer hot path -- TEST INFRASTRUCTURE.
//
// This file is a scalar C++ restatement of the reference renderer's equations
// (tuallen/GOFish, threedgut_tracer/...).  It is used only by tests/, by
// __graft_entry__.smoke() and by bench.py's CPU baseline leg, always as the
// checker or the timed CPU baseline, never as the product path.
//
// Parity pinning: the reference CUDA extension cannot be built or run here
// as a whole (its tiny-cuda-nn submodule is empty and slangc is absent), and
// the reference has no tests or golden vectors for this path.  Its
// header-only per-hit device code (gaussianParticles.cuh processHitFwd,
// processHitBwd, particleExactDepthCrossingRaw, radianceFromSpH) is compiled
// for the host from the reference checkout (oracle/ref_device, `make ref`),
// and tests/test_hit_golden.py checks this file's hit test, compositing,
// training channels, backward and SH radiance against its outputs
// (tests/golden/hit_golden.npz).  The projection, admission, binning, sort
// and k-buffer order are pinned by analytic known-answer tests in
// tests/test_oracle_kat.py (on-axis Gaussian, equidistant projection
// identities, ...), and the backward passes also by the finite-difference
// gradient checks of tests/test_oracle_gradcheck.py.
//
// Floating-point contract (shared with the sm_100a kernels): IEEE single
// precision, no implicit contraction (-ffp-contract=off), fmaf only where
// written, transcendental functions from gf_elementary.h.
//
// Each function cites the reference file:line it restates.

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include <atomic>
#include <cstdlib>
#include <thread>

#include "../gofish_b200/csrc/gf_elementary.h"

using gf::fmaf_rn;

namespace {

// threedgut_tracer/configs/render/3dgut.yaml + include/3dgut/threedgut.cuh:41-68
constexpr float kAlphaThreshold = 0.00392156862745098f;   // particle_kernel_min_alpha
constexpr float kMinKernelResponse = 0.0113f;             // particle_kernel_min_response
constexpr float kMaxAlpha = 0.99f;                         // particle_kernel_max_alpha
constexpr float kMinTransmittance = 0.0001f;               // min_transmittance
constexpr float kCovarianceDilation = 0.3f;                // threedgut.cuh:58
constexpr float kParticleMinSensorZ = 0.2f;                // sensorConstants.cuh:12
constexpr float kMaxDepthValue = 3.4028235e+38f;           // threedgut.cuh:64
constexpr float kUtDelta = 1.7320508075688772f;            // sqrt(alpha^2 (D + kappa)), setup_3dgut.py:178
constexpr float kUtImageMargin = 0.1f;                     // ut_in_image_margin_factor
constexpr float kUtWeightI = 1.0f / 6.0f;                  // gutProjector.cuh:433 1/(2(D+lambda)), lambda = 0
constexpr float kUtWeight0 = 2.0f;                         // gutProjector.cuh:502 lambda/(D+lambda) + (1-a^2+b)
constexpr float kAabbHalfExtent = 1e06f;                   // splatRaster.cpp:345
constexpr int kTile = 16;                                  // gutRendererParameters.h:21-22
constexpr uint32_t kInvalidParticle = 0xffffffffu;

struct float2_ { float x, y; };
struct float3_ { float x, y, z; };

inline float3_ f3(float x, float y, float z) { return {x, y, z}; }
inline float3_ add(float3_ a, float3_ b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
inline float3_ sub(float3_ a, float3_ b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
inline float3_ scale(float s, float3_ a) { return {s * a.x, s * a.y, s * a.z}; }
inline float dot(float3_ a, float3_ b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
// M (row-major 3x3) times v, each row summed left to right.
inline float3_ matvec(const float* m, float3_ v) {
    return {m[0] * v.x + m[1] * v.y + m[2] * v.z,
            m[3] * v.x + m[4] * v.y + m[5] * v.z,
            m[6] * v.x + m[7] * v.y + m[8] * v.z};
}
// Fused dot product used by the ray-particle hit test: fma(a.z,b.z,fma(a.y,b.y,a.x*b.x)).
inline float fdot(float3_ a, float3_ b) { return fmaf_rn(a.z, b.z, fmaf_rn(a.y, b.y, a.x * b.x)); }
inline float3_ fmatvec(const float* m, float3_ v) {
    return {fdot(f3(m[0], m[1], m[2]), v), fdot(f3(m[3], m[4], m[5]), v), fdot(f3(m[6], m[7], m[8]), v)};
}

// Saturating float -> int conversion toward zero (NaN -> 0), the semantics of
// the GPU's cvt.rzi.s32.f32 that the reference's static_cast<int> compiles to.
inline int f2i_sat(float f) {
    if (f != f) return 0;
    if (f >= 2147483648.0f) return 2147483647;
    if (f <= -2147483648.0f) return (-2147483647 - 1);
    return int(f);
}
inline float saturate(float x) {  // __saturatef: clamp to [0,1], NaN -> 0
    if (!(x > 0.0f)) return 0.0f;
    return x < 1.0f ? x : 1.0f;
}


// Worker count: ORACLE_THREADS, else every host core.
int worker_count() {
    const char* env = std::getenv("ORACLE_THREADS");
    if (env != nullptr && std::atoi(env) > 0) return std::atoi(env);
    const unsigned n = std::thread::hardware_concurrency();
    return n == 0 ? 1 : int(n);
}

// Dynamic parallel loop over [begin, end) in chunks; fn(i, worker).
template <typename Fn>
void parallel_for(int begin, int end, int chunk, Fn&& fn) {
    const int workers = worker_count();
    std::atomic<int> next(begin);
    auto body = [&](int worker) {
        for (;;) {
            const int b = next.fetch_add(chunk);
            if (b >= end) break;
            const int e = std::min(end, b + chunk);
            for (int i = b; i < e; ++i) fn(i, worker);
        }
    };
    if (workers <= 1 || end - begin <= chunk) {
        body(0);
        return;
    }
    std::vector<std::thread> pool;
    for (int w = 1; w < workers; ++w) pool.emplace_back(body, w);
    body(0);
    for (auto& t : pool) t.join();
}
// Complete admission (oracle_set_complete_admission): every particle of
// density >= 1/255 is admitted by the conservative cone test of its support
// sphere, none by its projected footprint.
bool g_completeAdmission = false;
// Densification statistic of oracle_render_backward(_geo) (oracle_set_abs_grad):
// map [N,6] (screen mode) or NULL, sums [N,2] / [N,3], mode 1 screen, 2 world, 0 off.
const float* g_absMap = nullptr;
float* g_absOut = nullptr;
int g_absMode = 0;

// Adds |M g| (screen) or |g| (world) of one hit's position gradient g to the
// worker's partial sums (gutKBufferRenderer.cuh:54-60,283-296).
inline void abs_grad_hit(std::vector<float>& partial, int N, uint32_t idx, float gx, float gy, float gz) {
    if (g_absMode == 0) return;
    const int width = g_absMode == 1 ? 2 : 3;
    if (partial.empty()) partial.assign(size_t(N) * width, 0.0f);
    float* o = partial.data() + size_t(idx) * width;
    if (g_absMode == 1) {
        const float* row = g_absMap + size_t(idx) * 6;
        o[0] += std::fabs(row[0] * gx + row[1] * gy + row[2] * gz);
        o[1] += std::fabs(row[3] * gx + row[4] * gy + row[5] * gz);
    } else {
        o[0] += std::fabs(gx);
        o[1] += std::fabs(gy);
        o[2] += std::fabs(gz);
    }
}

void abs_grad_reduce(const std::vector<std::vector<float>>& partial, int N) {
    if (g_absMode == 0) return;
    const size_t count = size_t(N) * (g_absMode == 1 ? 2 : 3);
    for (const auto& p : partial)
        if (!p.empty())
            for (size_t i = 0; i < count; ++i) g_absOut[i] += p[i];
}
// Partial UT covariance scale (oracle_set_admission_variants; 0 = off) and
// the cone_big fallback window on the caps' sines.
float g_partialUtScale2 = 0.0f;
bool g_coneBig = false;
float g_coneSinMin = 0.0f, g_coneSinMax = 1.0f;

// Optional explicit tile list of the render entry points (oracle_set_tile_list):
// when one is set they visit its tiles instead of the range [tileBegin, tileEnd).
const int* g_tileList = nullptr;
int g_tileListCount = 0;

template <typename Fn>
void parallel_tiles(int tileBegin, int tileEnd, Fn&& fn) {
    if (g_tileList == nullptr) {
        parallel_for(tileBegin, tileEnd, 1, fn);
        return;
    }
    parallel_for(0, g_tileListCount, 1, [&](int i, int worker) { fn(g_tileList[i], worker); });
}
}  // namespace

extern "C" {

// Selects (1) or clears (0) complete admission for oracle_project / oracle_bin.
void oracle_set_complete_admission(int complete) { g_completeAdmission = complete != 0; }

// Arms (mode 1: screen, map [N,6]; mode 2: world) or clears (0) the
// densification statistic of oracle_render_backward(_geo): each composited
// hit adds |M g| or |g| of its position gradient g to out ([N,2] / [N,3]).
void oracle_set_abs_grad(const float* map, float* out, int mode) {
    g_absMap = map;
    g_absOut = out;
    g_absMode = (out != nullptr && (mode == 2 || (mode == 1 && map != nullptr))) ? mode : 0;
}

// Partial UT (partialScale2 = scale^2 > 0, 0 = off) and the cone_big window
// (coneBig != 0; the caps' sine bounds) of oracle_project / oracle_bin.
void oracle_set_admission_variants(float partialScale2, int coneBig, float sinMin, float sinMax) {
    g_partialUtScale2 = partialScale2;
    g_coneBig = coneBig != 0;
    g_coneSinMin = sinMin;
    g_coneSinMax = sinMax;
}

// Sets (tiles != NULL) or clears the tile list of the render entry points;
// the caller keeps the list alive until it is cleared.
void oracle_set_tile_list(const int* tiles, int count) {
    g_tileList = tiles;
    g_tileListCount = tiles != nullptr ? count : 0;
}

// Camera model parameters: threedgut_tracer/include/3dgut/sensors/cameraModels.h
// (OpenCVPinholeProjectionParameters / OpenCVFisheyeProjectionParameters).
struct OracleCamera {
    int32_t model;   // 0 = OpenCV pinhole, 1 = OpenCV fisheye (Kannala-Brandt)
    int32_t width;
    int32_t height;
    int32_t pad0;
    float principal[2];
    float focal[2];
    float radial[6];
    float tangential[2];
    float thin_prism[4];
    float max_angle;
    float pad1;
};

// Prepared global-shutter pose: world->sensor rotation R (row-major) and
// translation t, its inverse rotation Rinv = R^T and the sensor centre c.
struct OraclePose {
    float R[9];
    float t[3];
    float Rinv[9];
    float c[3];
};

// Prepare an OraclePose from the reference's 7-float world->sensor pose
// [tx, ty, tz, qx, qy, qz, qw] (tracer.py:466-474, sensors.h:44-73).  Done in
// double and rounded once, so the product and the oracle see the same floats.
void oracle_prepare_pose(const float* pose7, OraclePose* out) {
    const double tx = pose7[0], ty = pose7[1], tz = pose7[2];
    const double x = pose7[3], y = pose7[4], z = pose7[5], w = pose7[6];
    double R[9];
    R[0] = 1.0 - 2.0 * (y * y + z * z);
    R[1] = 2.0 * (x * y - w * z);
    R[2] = 2.0 * (x * z + w * y);
    R[3] = 2.0 * (x * y + w * z);
    R[4] = 1.0 - 2.0 * (x * x + z * z);
    R[5] = 2.0 * (y * z - w * x);
    R[6] = 2.0 * (x * z - w * y);
    R[7] = 2.0 * (y * z + w * x);
    R[8] = 1.0 - 2.0 * (x * x + y * y);
    for (int i = 0; i < 9; ++i) out->R[i] = float(R[i]);
    out->t[0] = float(tx);
    out->t[1] = float(ty);
    out->t[2] = float(tz);
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c) out->Rinv[3 * r + c] = out->R[3 * c + r];
    // c = -R^T t
    for (int r = 0; r < 3; ++r) {
        const double v = -(R[0 * 3 + r] * tx + R[1 * 3 + r] * ty + R[2 * 3 + r] * tz);
        out->c[r] = float(v);
    }
}

}  // extern "C"

namespace {

// cameraProjections.cuh:26-37
float stable_norm2(float x, float y) {
    const float ax = gf::abs_f(x), ay = gf::abs_f(y);
    const float mn = gf::min_f(ax, ay), mx = gf::max_f(ax, ay);
    if (mx <= 0.0f) return 0.0f;
    const float r = mn / mx;
    return mx * sqrtf(1.0f + r * r);
}

// cameraProjections.cuh:86-122 (OpenCV pinhole), requireRasterBounds = false.
bool project_pinhole(const OracleCamera& cam, float3_ p, float2_& out) {
    if (p.z <= 0.0f) {
        out = {0.0f, 0.0f};
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
    const float ux = icD * u + dx, uy = icD * v + dy;
    const bool validRadial = icD > 0.8f && icD < 1.2f;
    if (validRadial) {
        out = {ux * cam.focal[0] + cam.principal[0], uy * cam.focal[1] + cam.principal[1]};
    } else {
        const float clip = float(std::hypot(double(cam.width), double(cam.height)));
        const float s = clip / sqrtf(r2);
        out = {s * u + cam.principal[0], s * v + cam.principal[1]};
    }
    return validRadial && gf::isfinite_f(out.x) && gf::isfinite_f(out.y);
}

// cameraProjections.cuh:124-152 (OpenCV fisheye / Kannala-Brandt), requireRasterBounds = false.
bool project_fisheye(const OracleCamera& cam, float3_ p, float2_& out) {
    float rho = stable_norm2(p.x, p.y);
    if (rho <= 0.0f) rho = FLT_EPSILON;
    const float thetaFull = gf::gf_atan2f(rho, p.z);
    const float theta = gf::min_f(thetaFull, cam.max_angle);
    const float theta2 = theta * theta;
    // evalPolyHorner<4>(k, theta2): y = k4; y = x*y + k3; ...
    float poly = cam.radial[3];
    poly = theta2 * poly + cam.radial[2];
    poly = theta2 * poly + cam.radial[1];
    poly = theta2 * poly + cam.radial[0];
    const float delta = (theta * (poly * theta2 + 1.0f)) / rho;
    out = {cam.focal[0] * p.x * delta + cam.principal[0], cam.focal[1] * p.y * delta + cam.principal[1]};
    return theta < cam.max_angle && gf::isfinite_f(out.x) && gf::isfinite_f(out.y);
}

// cameraProjections.cuh:228-240, global shutter: R * p + t, then project.
bool project_world(const OracleCamera& cam, const OraclePose& pose, float3_ pw, float2_& out) {
    const float3_ ps = add(matvec(pose.R, pw), f3(pose.t[0], pose.t[1], pose.t[2]));
    if (cam.model == 1) return project_fisheye(cam, ps, out);
    return project_pinhole(cam, ps, out);
}

}  // namespace

extern "C" {

// The UT projection alone (unscented_projection) of n packed rows:
// out[n*6] = centre u, v, covariance xx, xy, yy, valid (0 or 1).
int oracle_ut_project(const OracleCamera* cam, const OraclePose* pose, int n, const float* particles, float* out);

// Composite order of the k-buffer (KBuffer, fed as traverse() feeds it) for
// hits i = 0..n-1 with distances hitT[i]: order[n] of hit indices.
int oracle_kbuffer_order(int K, int n, const float* hitT, uint32_t* order);

// Sensor-space point projection of the camera (pinhole or fisheye, without
// raster bounds, as the UT uses it): uv[n*2], valid[n].
int oracle_project_points(const OracleCamera* cam, int n, const float* pts, float* uv, uint8_t* valid) {
    for (int i = 0; i < n; ++i) {
        const float3_ p = f3(pts[3 * i], pts[3 * i + 1], pts[3 * i + 2]);
        float2_ o{0.0f, 0.0f};
        const bool ok = cam->model == 1 ? project_fisheye(*cam, p, o) : project_pinhole(*cam, p, o);
        uv[2 * i] = o.x;
        uv[2 * i + 1] = o.y;
        valid[i] = ok ? 1u : 0u;
    }
    return 0;
}

}  // extern "C"

namespace {

// Packed particle row accessors, tracer.py:171-179 / inference.py:43-47.
struct Particle {
    float3_ pos;
    float density;
    float quat[4];  // intrinsic rotation (w, x, y, z), slots 4-7
    float scale[3]; // intrinsic scale, slots 8-10
    float B[9];     // factor, row-major (slots 12-20)
    float Binv[9];  // inverse factor, row-major (slots 21-29)
};
inline Particle load_particle(const float* row) {
    Particle p;
    p.pos = f3(row[0], row[1], row[2]);
    p.density = row[3];
    for (int i = 0; i < 4; ++i) p.quat[i] = row[4 + i];
    for (int i = 0; i < 3; ++i) p.scale[i] = row[8 + i];
    for (int i = 0; i < 9; ++i) p.B[i] = row[12 + i];
    for (int i = 0; i < 9; ++i) p.Binv[i] = row[21 + i];
    return p;
}

struct Projection {
    float2_ center;
    float conic[3];
    float opacity;
    float2_ extent;
    bool valid;
};

// gutProjector.cuh:359-518, unscentedParticleProjection; with
// g_partialUtScale2 > 0 the partial UT of :470-499 (each invalid sigma point
// replaced by the reflection of its mirror about the projected mean when the
// mean and one point per axis project; mean re-accumulated over points 1..6
// in order; covariance scaled).
bool unscented_projection(const OracleCamera& cam, const OraclePose& pose, const Particle& P,
                          float2_& center, float cov[3]) {
    if (P.density < kAlphaThreshold) return false;  // :375-378
    const bool fisheye = cam.model == 1;
    if (fisheye) {
        // :389-398 cameraNativeRadialNearAdmitted (cameraNativeRayAdmission.cuh:29-35)
        const float3_ ray = sub(P.pos, f3(pose.c[0], pose.c[1], pose.c[2]));
        const float r2 = dot(ray, ray);
        const float near2 = kParticleMinSensorZ * kParticleMinSensorZ;
        if (!(gf::isfinite_f(r2) && r2 >= near2)) return false;
    } else {
        // :399-405 pinhole near plane (z row of the world->sensor matrix)
        const float z = P.pos.x * pose.R[6] + P.pos.y * pose.R[7] + P.pos.z * pose.R[8] + pose.t[2];
        if (z < kParticleMinSensorZ) return false;
    }
    float2_ s[7];
    bool ok[7];
    int numValid = 0;
    const bool c0 = project_world(cam, pose, P.pos, s[0]);  // :413-420
    if (fisheye && !c0) return false;                         // :421-428
    if (c0) numValid++;
    center = {s[0].x * 0.0f, s[0].y * 0.0f};                 // lambda / (D + lambda) = 0
    for (int i = 0; i < 3; ++i) {                             // :434-462
        const float3_ col = f3(P.B[0 * 3 + i], P.B[1 * 3 + i], P.B[2 * 3 + i]);
        const float3_ delta = scale(kUtDelta, col);
        ok[i + 1] = project_world(cam, pose, add(P.pos, delta), s[i + 1]);
        if (ok[i + 1]) numValid++;
        center.x = center.x + kUtWeightI * s[i + 1].x;
        center.y = center.y + kUtWeightI * s[i + 1].y;
        ok[i + 4] = project_world(cam, pose, sub(P.pos, delta), s[i + 4]);
        if (ok[i + 4]) numValid++;
        center.x = center.x + kUtWeightI * s[i + 4].x;
        center.y = center.y + kUtWeightI * s[i + 4].y;
    }
    float covScale = 1.0f;
    if (numValid != 7) {  // :466-499
        if (!(g_partialUtScale2 > 0.0f) || !c0) return false;
        for (int i = 0; i < 3; ++i)
            if (!ok[i + 1] && !ok[i + 4]) return false;  // both points of an axis invalid: no footprint
        for (int i = 0; i < 3; ++i) {
            if (!ok[i + 1]) s[i + 1] = {2.0f * s[0].x - s[i + 4].x, 2.0f * s[0].y - s[i + 4].y};
            if (!ok[i + 4]) s[i + 4] = {2.0f * s[0].x - s[i + 1].x, 2.0f * s[0].y - s[i + 1].y};
        }
        center = {s[0].x * 0.0f, s[0].y * 0.0f};
        for (int k = 1; k < 7; ++k) {
            center.x = center.x + kUtWeightI * s[k].x;
            center.y = center.y + kUtWeightI * s[k].y;
        }
        covScale = g_partialUtScale2;
    }
    {
        const float cx = s[0].x - center.x, cy = s[0].y - center.y;  // :501-506
        cov[0] = kUtWeight0 * (cx * cx);
        cov[1] = kUtWeight0 * (cx * cy);
        cov[2] = kUtWeight0 * (cy * cy);
    }
    for (int i = 0; i < 6; ++i) {  // :507-513
        const float cx = s[i + 1].x - center.x, cy = s[i + 1].y - center.y;
        cov[0] = cov[0] + kUtWeightI * (cx * cx);
        cov[1] = cov[1] + kUtWeightI * (cx * cy);
        cov[2] = cov[2] + kUtWeightI * (cy * cy);
    }
    if (covScale != 1.0f) {  // :514
        cov[0] = cov[0] * covScale;
        cov[1] = cov[1] * covScale;
        cov[2] = cov[2] * covScale;
    }
    return true;
}

// gutProjector.cuh:249-288 computeProjectedExtentConicOpacity.
bool conic_extent(const float cov[3], float opacity, Projection& out) {
    const float dx = cov[0] + kCovarianceDilation, dy = cov[1], dz = cov[2] + kCovarianceDilation;
    const float det = dx * dz - dy * dy;
    if (det == 0.0f) return false;
    out.conic[0] = dz / det;
    out.conic[1] = -dy / det;
    out.conic[2] = dx / det;
    out.opacity = opacity;
    if (opacity < kAlphaThreshold) return false;
    const float maxPower = gf::gf_logf(opacity / kAlphaThreshold);
    const float extentFactor = gf::min_f(3.33f, sqrtf(2.0f * maxPower));
    const float mid = 0.5f * (dx + dz);
    const float lambda = mid + sqrtf(gf::max_f(0.01f, mid * mid - det));
    const float radius = extentFactor * sqrtf(lambda);
    out.extent = {gf::min_f(extentFactor * sqrtf(dx), radius), gf::min_f(extentFactor * sqrtf(dz), radius)};
    return radius > 0.0f;
}

// gutProjector.cuh:85-96 computeTileSpaceBBox.
void tile_bbox(int gx, int gy, float2_ c, float2_ e, int& x0, int& y0, int& x1, int& y1) {
    auto clampg = [](int v, int g) { return std::min(g, std::max(0, v)); };
    x0 = clampg(f2i_sat(floorf(((c.x - 0.5f) - e.x) / 16.0f)), gx);
    y0 = clampg(f2i_sat(floorf(((c.y - 0.5f) - e.y) / 16.0f)), gy);
    x1 = clampg(f2i_sat(ceilf(((c.x - 0.5f) + e.x) / 16.0f)), gx);
    y1 = clampg(f2i_sat(ceilf(((c.y - 0.5f) + e.y) / 16.0f)), gy);
}

// gutProjector.cuh:217-246 tileMinParticlePowerResponse.
float tile_min_power(int tx, int ty, const float conic[3], float2_ m) {
    const float tminx = 16.0f * float(tx), tminy = 16.0f * float(ty);
    const float tmaxx = 16.0f + tminx, tmaxy = 16.0f + tminy;
    const float ox = tminx - m.x, oy = tminy - m.y;
    const float lax = ox > 0.0f ? 1.0f : 0.0f, lay = oy > 0.0f ? 1.0f : 0.0f;
    const float nirx = lax + (m.x > tmaxx ? 1.0f : 0.0f);
    const float niry = lay + (m.y > tmaxy ? 1.0f : 0.0f);
    if ((nirx + niry) > 0.0f) {
        const float px = lax != 0.0f ? tminx : tmaxx;
        const float py = lay != 0.0f ? tminy : tmaxy;
        const float dxy_x = gf::copysign_f(16.0f, ox), dxy_y = gf::copysign_f(16.0f, oy);
        const float diffx = m.x - px, diffy = m.y - py;
        const float rcpx = 1.0f / (256.0f * conic[0]);
        const float rcpy = 1.0f / (256.0f * conic[2]);
        const float tx_ = niry * saturate((dxy_x * conic[0] * diffx + dxy_x * conic[1] * diffy) * rcpx);
        const float ty_ = nirx * saturate((dxy_y * conic[1] * diffx + dxy_y * conic[2] * diffy) * rcpy);
        const float mx = m.x - (px + tx_ * dxy_x), my = m.y - (py + ty_ * dxy_y);
        return 0.5f * (conic[0] * mx * mx + conic[2] * my * my) + conic[1] * mx * my;
    }
    return 0.0f;
}

inline bool fast_ut_valid(const Projection& p) {  // gutProjector.cuh:181-184
    return p.extent.x > 1e-06f && p.opacity >= kAlphaThreshold;
}

// gutProjector.cuh:186-210 fastAdmittedTiles (scale s = 1), y-major visit order.
template <typename Visit>
uint32_t admitted_tiles(int gx, int gy, const uint8_t* mask, const Projection& p, Visit&& visit) {
    if (!fast_ut_valid(p)) return 0u;
    int x0, y0, x1, y1;
    tile_bbox(gx, gy, p.center, p.extent, x0, y0, x1, y1);
    const float maxPower = gf::gf_logf(p.opacity / kAlphaThreshold) * 1.0f;
    uint32_t n = 0;
    for (int y = y0; y < y1; ++y) {
        for (int x = x0; x < x1; ++x) {
            if (mask[y * gx + x] == 0u) continue;
            if (!(tile_min_power(x, y, p.conic, p.center) < maxPower)) continue;
            visit(x, y);
            ++n;
        }
    }
    return n;
}

// Cone fallback admission for particles without a valid projection
// (gutProjector.cuh:100-183 fastFallbackTiles; fast_admission_fallback =
// "cone").  Tile ray cones over a 4x4 quadtree up to one root; a tile is
// admitted when its cone and every ancestor's meet the particle's cap (the
// bounding sphere seen from the camera); a sphere holding the camera admits
// every retained tile.  Same arithmetic, in the same order, as the sm_100a
// kernels (cos/sin forms only: +, -, *, /, sqrt and gf_logf).
namespace fallback {

constexpr float kEps = 1e-6f;
constexpr int kFan = 4;

struct Node {
    float ax, ay, az, c;  // axis, cos phi (> 1.5: empty)
    float s;              // sin phi
};

struct Tree {
    std::vector<int> gx, gy;
    std::vector<std::vector<Node>> level;
    std::vector<Node> second;                // the leaves' second cones
    std::vector<std::vector<float3_>> sums;  // per node: sum of its unit pixel rays
    float3_ optical;                         // the camera's optical axis in world coordinates (not normalised)
};

inline float3_ matvec_plain(const float* m, float3_ v) { return matvec(m, v); }

// Unit world direction of pixel (x, y); false for a zero or non-finite ray.
inline bool pixel_dir(const OraclePose& pose, const float* rayD, int W, int x, int y, float3_& u) {
    const size_t p = size_t(x) + size_t(W) * size_t(y);
    const float3_ d = f3(rayD[3 * p], rayD[3 * p + 1], rayD[3 * p + 2]);
    const float n2 = dot(d, d);
    if (!(n2 > 0.0f) || !gf::isfinite_f(n2)) return false;
    const float3_ w = matvec_plain(pose.Rinv, d);
    const float wn = sqrtf(dot(w, w));
    u = f3(w.x / wn, w.y / wn, w.z / wn);
    return true;
}

// Sum of the unit rays of rows y0..y1 for which keep(u) holds, each row summed
// left to right and the non-empty row sums added in row order.
template <typename Keep>
float3_ row_sums(const OraclePose& pose, const float* rayD, int W, int x0, int y0, int x1, int y1, Keep&& keep,
                 int& all) {
    float3_ sum = f3(0.0f, 0.0f, 0.0f);
    all = 0;
    for (int y = y0; y < y1; ++y) {
        float3_ rs = f3(0.0f, 0.0f, 0.0f);
        int rc = 0;
        for (int x = x0; x < x1; ++x) {
            float3_ u;
            if (!pixel_dir(pose, rayD, W, x, y, u) || !keep(u)) continue;
            rs = add(rs, u);
            ++rc;
        }
        if (rc > 0) sum = add(sum, rs);
        all += rc;
    }
    return sum;
}

inline Node cone_from(float3_ a, float mn) {
    const float cphi = gf::max_f(-1.0f, mn - kEps);
    return Node{a.x, a.y, a.z, cphi, sqrtf(gf::max_f(0.0f, 1.0f - cphi * cphi))};
}

// The two cones of one tile: its unit pixel rays split by the nearer of the
// two mutually farthest rays (far1 = first ray farthest from the mean ray in
// row-major order, far2 = first ray farthest from far1; ties to far1); cone k
// = normalised sum of its rays, cos phi = smallest cosine to that axis less
// kEps.  A tile mixing rim rays with the forward rays of pixels outside the
// image circle gets two narrow cones instead of one wide one.
void leaf_cones(const OraclePose& pose, const float* rayD, int W, int x0, int y0, int x1, int y1, Node& c0,
                Node& c1, float3_& sum) {
    const Node empty{0.0f, 0.0f, 1.0f, 2.0f, 0.0f};
    c0 = c1 = empty;
    int all = 0;
    sum = row_sums(pose, rayD, W, x0, y0, x1, y1, [](float3_) { return true; }, all);
    if (all == 0) return;
    const float sn = sqrtf(dot(sum, sum));
    if (!(sn > 0.0f) || !gf::isfinite_f(sn)) {
        c0 = Node{0.0f, 0.0f, 1.0f, -1.0f, 0.0f};
        return;
    }
    const float3_ mean = f3(sum.x / sn, sum.y / sn, sum.z / sn);
    float3_ far1 = mean, far2 = mean;
    for (int pass = 0; pass < 2; ++pass) {
        const float3_ ref = pass == 0 ? mean : far1;
        float best = 2.0f;
        float3_ bu = ref;
        for (int y = y0; y < y1; ++y)
            for (int x = x0; x < x1; ++x) {
                float3_ u;
                if (!pixel_dir(pose, rayD, W, x, y, u)) continue;
                const float c = dot(ref, u);
                if (c < best) {
                    best = c;
                    bu = u;
                }
            }
        if (pass == 0) far1 = bu;
        else far2 = bu;
    }
    auto first = [&](float3_ u) { return dot(far1, u) >= dot(far2, u); };
    int all0 = 0, all1 = 0;
    const float3_ t0 = row_sums(pose, rayD, W, x0, y0, x1, y1, first, all0);
    const float3_ t1 = row_sums(pose, rayD, W, x0, y0, x1, y1, [&](float3_ u) { return !first(u); }, all1);
    const float l0 = sqrtf(dot(t0, t0)), l1 = sqrtf(dot(t1, t1));
    const bool ok0 = l0 > 0.0f && gf::isfinite_f(l0), ok1 = l1 > 0.0f && gf::isfinite_f(l1);
    const float3_ a0 = ok0 ? f3(t0.x / l0, t0.y / l0, t0.z / l0) : mean;
    const float3_ a1 = ok1 ? f3(t1.x / l1, t1.y / l1, t1.z / l1) : mean;
    float m0 = 1.0f, m1 = 1.0f;
    for (int y = y0; y < y1; ++y)
        for (int x = x0; x < x1; ++x) {
            float3_ u;
            if (!pixel_dir(pose, rayD, W, x, y, u)) continue;
            if (first(u)) m0 = gf::min_f(m0, dot(a0, u));
            else m1 = gf::min_f(m1, dot(a1, u));
        }
    if (ok0) c0 = cone_from(a0, m0);
    else if (all0 > 0) c0 = Node{a0.x, a0.y, a0.z, -1.0f, 0.0f};
    if (ok1) c1 = cone_from(a1, m1);
    else if (all1 > 0) c1 = Node{a1.x, a1.y, a1.z, -1.0f, 0.0f};
}

// cos(angle(axis, a) + phi_a) of one non-empty cone into the running minimum;
// false once the sum reaches past pi.
inline bool bound_cone(float3_ a, const Node& c, float& cphi) {
    if (c.c > 1.5f) return true;
    const float3_ ca = f3(c.ax, c.ay, c.az);
    const float3_ cr = f3(a.y * ca.z - a.z * ca.y, a.z * ca.x - a.x * ca.z, a.x * ca.y - a.y * ca.x);
    const float sang = sqrtf(dot(cr, cr));
    const float cang = dot(a, ca);
    if (sang * c.c + cang * c.s < 0.0f) return false;
    cphi = gf::min_f(cphi, cang * c.c - sang * c.s);
    return true;
}

// Parent cone at level l: ray sum = the sum of the 4x4 children's ray sums in
// row-major order; empty when every child is.  Two axes are bounded: the
// normalised ray sum (the mean direction of the pixel rays under the node)
// and the camera's optical axis.  For each, cos phi = the smallest, over the
// non-empty cones of the leaves under the node, of cos(angle(axis, a) +
// phi_a) = (axis . a) cos phi_a - |axis x a| sin phi_a, or the whole sphere
// once a cone reaches past pi.  The node keeps the axis with the larger
// cos phi (the mean on ties), less kEps; a node whose both bounds cover the
// sphere gets (cos -1, sin 0).
Node parent_cone(const Tree& t, int l, int px, int py, float3_& sum) {
    const std::vector<Node>& ch = t.level[size_t(l) - 1];
    const std::vector<float3_>& cs = t.sums[size_t(l) - 1];
    const int gx = t.gx[size_t(l) - 1], gy = t.gy[size_t(l) - 1];
    sum = f3(0.0f, 0.0f, 0.0f);
    bool any = false;
    for (int j = 0; j < kFan; ++j)
        for (int i = 0; i < kFan; ++i) {
            const int cx = px * kFan + i, cy = py * kFan + j;
            if (cx >= gx || cy >= gy) continue;
            const size_t k = size_t(cy) * gx + cx;
            sum = add(sum, cs[k]);
            if (ch[k].c <= 1.5f || (l == 1 && t.second[k].c <= 1.5f)) any = true;
        }
    const float sn = sqrtf(dot(sum, sum));
    const bool meanOk = sn > 0.0f && gf::isfinite_f(sn);
    const float3_ am = meanOk ? f3(sum.x / sn, sum.y / sn, sum.z / sn) : f3(0.0f, 0.0f, 1.0f);
    if (!any) return Node{am.x, am.y, am.z, 2.0f, 0.0f};
    const float on = sqrtf(dot(t.optical, t.optical));
    const bool optOk = on > 0.0f && gf::isfinite_f(on);
    const float3_ ao = optOk ? f3(t.optical.x / on, t.optical.y / on, t.optical.z / on) : f3(0.0f, 0.0f, 1.0f);
    int span = 1;
    for (int k = 0; k < l; ++k) span *= kFan;
    const int gx0 = t.gx[0], gy0 = t.gy[0];
    const int x0 = px * span, y0 = py * span, x1 = std::min(gx0, x0 + span), y1 = std::min(gy0, y0 + span);
    float mm = 1.0f, mo = 1.0f;
    bool fm = !meanOk, fo = !optOk;
    for (int y = y0; y < y1; ++y)
        for (int x = x0; x < x1; ++x) {
            const size_t k = size_t(y) * gx0 + x;
            if (!bound_cone(am, t.level[0][k], mm) || !bound_cone(am, t.second[k], mm)) fm = true;
            if (!bound_cone(ao, t.level[0][k], mo) || !bound_cone(ao, t.second[k], mo)) fo = true;
        }
    const float vm = fm ? -2.0f : mm, vo = fo ? -2.0f : mo;
    const bool useOptical = vo > vm;
    const float3_ a = useOptical ? ao : am;
    const float best = useOptical ? vo : vm;
    if (best < -1.5f) return Node{a.x, a.y, a.z, -1.0f, 0.0f};
    const float cphi = gf::max_f(-1.0f, best - kEps);
    return Node{a.x, a.y, a.z, cphi, sqrtf(gf::max_f(0.0f, 1.0f - cphi * cphi))};
}

Tree build(const OracleCamera& cam, const OraclePose& pose, const uint8_t* mask, const float* rayD) {
    Tree t;
    t.optical = f3(pose.Rinv[2], pose.Rinv[5], pose.Rinv[8]);
    const int W = cam.width, H = cam.height;
    int gx = (W + kTile - 1) / kTile, gy = (H + kTile - 1) / kTile;
    const Node empty{0.0f, 0.0f, 1.0f, 2.0f, 0.0f};
    std::vector<Node> leaves(size_t(gx) * gy, empty);
    std::vector<float3_> leafSums(size_t(gx) * gy, f3(0.0f, 0.0f, 0.0f));
    t.second.assign(size_t(gx) * gy, empty);
    for (int tile = 0; tile < gx * gy; ++tile) {
        if (mask[tile] == 0u) continue;
        const int tx = tile % gx, ty = tile / gx;
        const int x0 = tx * kTile, y0 = ty * kTile;
        leaf_cones(pose, rayD, W, x0, y0, std::min(W, x0 + kTile), std::min(H, y0 + kTile), leaves[tile],
                   t.second[tile], leafSums[tile]);
    }
    t.sums.push_back(std::move(leafSums));
    t.gx.push_back(gx);
    t.gy.push_back(gy);
    t.level.push_back(std::move(leaves));
    while (!(gx == 1 && gy == 1)) {
        const int pgx = (gx + kFan - 1) / kFan, pgy = (gy + kFan - 1) / kFan;
        std::vector<Node> par(size_t(pgx) * pgy);
        t.gx.push_back(pgx);
        t.gy.push_back(pgy);
        const int l = int(t.gx.size()) - 1;
        std::vector<float3_> parSums(size_t(pgx) * pgy);
        for (int node = 0; node < pgx * pgy; ++node)
            par[node] = parent_cone(t, l, node % pgx, node / pgx, parSums[node]);
        gx = pgx;
        gy = pgy;
        t.level.push_back(std::move(par));
        t.sums.push_back(std::move(parSums));
    }
    return t;
}

struct Cap {
    float ux, uy, uz, cosA, sinA;
    int mode;  // 0 none, 1 cone, 2 every retained tile
};

Cap cap_of(const Particle& P, const OraclePose& pose) {
    Cap c{0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0};
    const float* B = P.B;
    const float m00 = B[0] * B[0] + B[1] * B[1] + B[2] * B[2];
    const float m01 = B[0] * B[3] + B[1] * B[4] + B[2] * B[5];
    const float m02 = B[0] * B[6] + B[1] * B[7] + B[2] * B[8];
    const float m11 = B[3] * B[3] + B[4] * B[4] + B[5] * B[5];
    const float m12 = B[3] * B[6] + B[4] * B[7] + B[5] * B[8];
    const float m22 = B[6] * B[6] + B[7] * B[7] + B[8] * B[8];
    const float g0 = m00 + gf::abs_f(m01) + gf::abs_f(m02);
    const float g1 = gf::abs_f(m01) + m11 + gf::abs_f(m12);
    const float g2 = gf::abs_f(m02) + gf::abs_f(m12) + m22;
    const float lam = gf::max_f(g0, gf::max_f(g1, g2));
    const float rho = gf::min_f(kMaxAlpha, P.density);
    const float canonical =
        gf::min_f(2.994f, sqrtf(gf::max_f(0.0f, 2.0f * gf::gf_logf(rho / kAlphaThreshold))));
    const float r = canonical * sqrtf(lam) * 1.001f;
    const float3_ v = sub(P.pos, f3(pose.c[0], pose.c[1], pose.c[2]));
    const float D = sqrtf(dot(v, v));
    if (!(gf::isfinite_f(r) && gf::isfinite_f(D)) || !(r > 0.0f)) return c;
    if (D <= r) {
        c.mode = 2;
        return c;
    }
    c.ux = v.x / D;
    c.uy = v.y / D;
    c.uz = v.z / D;
    c.sinA = gf::min_f(1.0f, (r / D) * 1.0001f);
    c.cosA = sqrtf(gf::max_f(0.0f, 1.0f - c.sinA * c.sinA));
    c.mode = 1;
    return c;
}

// The cap the fallback admits by: cap_of, except that "cone_big"
// (gutProjector.cuh:145-154) admits no sphere holding the camera and no cap
// whose half-angle (its sine here) lies outside the window; complete
// admission ignores the window.
Cap admitted_cap(const Particle& P, const OraclePose& pose) {
    Cap c = cap_of(P, pose);
    if (g_coneBig && !g_completeAdmission &&
        (c.mode == 2 || (c.mode == 1 && (c.sinA < g_coneSinMin || c.sinA > g_coneSinMax))))
        c.mode = 0;
    return c;
}

// Cone (axis, phi) meets cap (u, alpha) iff angle(axis, u) <= phi + alpha:
// always once phi + alpha passes pi (sin(phi + alpha) < 0), else
// axis . u >= cos phi cos alpha - sin phi sin alpha.
inline bool pass(const Node& n, const Cap& c) {
    if (n.c > 1.5f) return false;
    if (n.s * c.cosA + n.c * c.sinA < 0.0f) return true;
    const float d = n.ax * c.ux + n.ay * c.uy + n.az * c.uz;
    return d >= n.c * c.cosA - n.s * c.sinA - kEps;
}

// Visits the admitted tiles of one cap in tile order.
template <typename Visit>
uint32_t tiles(const Tree& t, const uint8_t* mask, const Cap& c, Visit&& visit) {
    uint32_t n = 0;
    if (c.mode == 0) return 0;
    const int gx = t.gx[0], gy = t.gy[0];
    for (int tile = 0; tile < gx * gy; ++tile) {
        if (c.mode == 2) {
            if (mask[tile] == 0u) continue;
        } else {
            int x = tile % gx, y = tile / gx;
            bool ok = true;
            for (size_t l = 0; l < t.level.size() && ok; ++l) {
                const size_t k = size_t(y) * t.gx[l] + x;
                ok = pass(t.level[l][k], c) || (l == 0 && pass(t.second[k], c));
                x /= kFan;
                y /= kFan;
            }
            if (!ok) continue;
        }
        visit(tile % gx, tile / gx);
        ++n;
    }
    return n;
}

}  // namespace fallback

// SH radiance, gaussianParticles.cuh:181-219 / sphericalHarmonics.slang decode.
constexpr float SH_C0 = 0.28209479177387814f;
constexpr float SH_C1 = 0.4886025119029199f;
constexpr float SH_C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f, -1.0925484305920792f,
                            0.5462742152960396f};
constexpr float SH_C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f, 0.3731763325901154f,
                            -0.4570457994644658f, 1.445305721320277f, -0.5900435899266435f};

void sh_basis(int deg, float3_ d, float b[16]) {
    for (int i = 0; i < 16; ++i) b[i] = 0.0f;
    b[0] = SH_C0;
    if (deg > 0) {
        const float x = d.x, y = d.y, z = d.z;
        b[1] = -SH_C1 * y;
        b[2] = SH_C1 * z;
        b[3] = -SH_C1 * x;
        if (deg > 1) {
            const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
            b[4] = SH_C2[0] * xy;
            b[5] = SH_C2[1] * yz;
            b[6] = SH_C2[2] * (2.0f * zz - xx - yy);
            b[7] = SH_C2[3] * xz;
            b[8] = SH_C2[4] * (xx - yy);
            if (deg > 2) {
                b[9] = SH_C3[0] * y * (3.0f * xx - yy);
                b[10] = SH_C3[1] * xy * z;
                b[11] = SH_C3[2] * y * (4.0f * zz - xx - yy);
                b[12] = SH_C3[3] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
                b[13] = SH_C3[4] * x * (4.0f * zz - xx - yy);
                b[14] = SH_C3[5] * z * (xx - yy);
                b[15] = SH_C3[6] * x * (xx - 3.0f * yy);
            }
        }
    }
}

// d(basis_k)/d(dir) for k < 16, as three rows (x, y, z).
void sh_basis_grad(int deg, float3_ d, float gx[16], float gy[16], float gz[16]) {
    for (int i = 0; i < 16; ++i) gx[i] = gy[i] = gz[i] = 0.0f;
    if (deg < 1) return;
    const float x = d.x, y = d.y, z = d.z;
    gy[1] = -SH_C1;
    gz[2] = SH_C1;
    gx[3] = -SH_C1;
    if (deg < 2) return;
    gx[4] = SH_C2[0] * y; gy[4] = SH_C2[0] * x;
    gy[5] = SH_C2[1] * z; gz[5] = SH_C2[1] * y;
    gx[6] = SH_C2[2] * (-2.0f * x); gy[6] = SH_C2[2] * (-2.0f * y); gz[6] = SH_C2[2] * (4.0f * z);
    gx[7] = SH_C2[3] * z; gz[7] = SH_C2[3] * x;
    gx[8] = SH_C2[4] * (2.0f * x); gy[8] = SH_C2[4] * (-2.0f * y);
    if (deg < 3) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    gx[9] = SH_C3[0] * (6.0f * x * y); gy[9] = SH_C3[0] * (3.0f * xx - 3.0f * yy);
    gx[10] = SH_C3[1] * (y * z); gy[10] = SH_C3[1] * (x * z); gz[10] = SH_C3[1] * (x * y);
    gx[11] = SH_C3[2] * (-2.0f * x * y); gy[11] = SH_C3[2] * (4.0f * zz - xx - 3.0f * yy); gz[11] = SH_C3[2] * (8.0f * y * z);
    gx[12] = SH_C3[3] * (-6.0f * x * z); gy[12] = SH_C3[3] * (-6.0f * y * z); gz[12] = SH_C3[3] * (6.0f * zz - 3.0f * xx - 3.0f * yy);
    gx[13] = SH_C3[4] * (4.0f * zz - 3.0f * xx - yy); gy[13] = SH_C3[4] * (-2.0f * x * y); gz[13] = SH_C3[4] * (8.0f * x * z);
    gx[14] = SH_C3[5] * (2.0f * x * z); gy[14] = SH_C3[5] * (-2.0f * y * z); gz[14] = SH_C3[5] * (xx - yy);
    gx[15] = SH_C3[6] * (3.0f * xx - 3.0f * yy); gy[15] = SH_C3[6] * (-6.0f * x * y);
}

// Incident direction of the SH evaluation: (mu - camera) / |mu - camera|
// (gutProjector.cuh:239-245, :551).
float3_ incident_direction(const float3_& mu, const OraclePose& pose, float& dist) {
    const float3_ v = sub(mu, f3(pose.c[0], pose.c[1], pose.c[2]));
    dist = sqrtf(dot(v, v));
    return {v.x / dist, v.y / dist, v.z / dist};
}

// ------------------------------------------------------------------ render
struct Ray {
    float3_ o, d;
    float tmin, tmax;
    bool valid;
    int local = 0;  // pixel index within its 16x16 tile (row-major), for the SOF feed
};

// bounding_box.h:89-133 ray_intersect against the +-1e6 box; rayPayload.cuh:113-162.
Ray make_ray(const OraclePose& pose, const float* ro, const float* rd) {
    Ray r;
    const float3_ os = f3(ro[0], ro[1], ro[2]);
    const float3_ ds = f3(rd[0], rd[1], rd[2]);
    r.o = add(matvec(pose.Rinv, os), f3(pose.c[0], pose.c[1], pose.c[2]));
    r.d = matvec(pose.Rinv, ds);
    const float lo = -kAabbHalfExtent, hi = kAabbHalfExtent;
    float tmin = (lo - r.o.x) / r.d.x, tmax = (hi - r.o.x) / r.d.x;
    if (tmin > tmax) std::swap(tmin, tmax);
    float tymin = (lo - r.o.y) / r.d.y, tymax = (hi - r.o.y) / r.d.y;
    if (tymin > tymax) std::swap(tymin, tymax);
    if (tmin > tymax || tymin > tmax) {
        tmin = FLT_MAX;
        tmax = FLT_MAX;
    } else {
        if (tymin > tmin) tmin = tymin;
        if (tymax < tmax) tmax = tymax;
        float tzmin = (lo - r.o.z) / r.d.z, tzmax = (hi - r.o.z) / r.d.z;
        if (tzmin > tzmax) std::swap(tzmin, tzmax);
        if (tmin > tzmax || tzmin > tmax) {
            tmin = FLT_MAX;
            tmax = FLT_MAX;
        } else {
            if (tzmin > tmin) tmin = tzmin;
            if (tzmax < tmax) tmax = tzmax;
        }
    }
    r.tmin = gf::max_f(tmin, 0.0f);
    r.tmax = tmax;
    r.valid = r.tmax > r.tmin;
    return r;
}

struct HalfRay {
    float3_ gro, grdu, p;
    float denom, num, tauLine, tau;
    bool interior, valid;
};

// gaussianParticles.slang:293-325 hitInterval == gutHalfRayResponse.cuh:17-37
// (fused dot products, see the file header).
HalfRay half_ray(const Ray& r, const Particle& P) {
    HalfRay h;
    const float3_ gposc = sub(r.o, P.pos);
    h.gro = fmatvec(P.Binv, gposc);
    h.grdu = fmatvec(P.Binv, r.d);
    h.denom = fdot(h.grdu, h.grdu);
    h.valid = h.denom > 0.0f && gf::isfinite_f(h.denom) && gf::isfinite_f(r.tmin) && r.tmax > r.tmin;
    if (!h.valid) {
        h.num = 0.0f;
        h.tauLine = 0.0f;
        h.tau = 0.0f;
        h.p = h.gro;
        h.interior = false;
        return h;
    }
    h.num = fdot(h.gro, h.grdu);
    h.tauLine = -h.num / h.denom;
    h.tau = gf::min_f(gf::max_f(h.tauLine, r.tmin), r.tmax);
    h.interior = h.tauLine > r.tmin && h.tauLine < r.tmax;
    h.p = f3(fmaf_rn(h.tau, h.grdu.x, h.gro.x), fmaf_rn(h.tau, h.grdu.y, h.gro.y), fmaf_rn(h.tau, h.grdu.z, h.gro.z));
    return h;
}

struct Hit {
    uint32_t idx;
    float hitT;
    float alpha;
};

// gaussianParticles.slang:309-338 hit acceptance; returns response.
bool hit_test(const Ray& r, const Particle& P, float& alpha, float& hitT, float& resp, HalfRay& h) {
    h = half_ray(r, P);
    if (!h.valid) return false;
    const float g = fdot(h.p, h.p);
    resp = gf::gf_expf(-0.5f * g);
    alpha = gf::min_f(kMaxAlpha, resp * P.density);
    hitT = h.tau;
    return resp > kMinKernelResponse && alpha > kAlphaThreshold;
}

struct PixelState {
    float T;
    float rgb[3];
    float hitT;
    uint32_t hitN;
    bool alive;
};

// Front-to-back composite of one hit (gutKBufferRenderer.cuh:307-416).
void composite(PixelState& s, const Hit& h, const float* rgb) {
    const float w = h.alpha * s.T;
    s.hitT = s.hitT + h.hitT * w;
    s.T = s.T * (1.0f - h.alpha);
    if (w > 0.0f) {
        const float* c = rgb + 3 * size_t(h.idx);
        for (int k = 0; k < 3; ++k) s.rgb[k] = fmaf_rn(gf::max_f(c[k], 0.0f), w, s.rgb[k]);
        s.hitN++;
    }
    if (s.T < kMinTransmittance) s.alive = false;
}

// HitParticleKBufferT (gutKBufferRenderer.cuh:120-166).
struct KBuffer {
    int K;
    uint32_t n;
    Hit e[64];
    void init(int k) {
        K = k;
        n = 0;
        for (int i = 0; i < k; ++i) e[i] = {kInvalidParticle, -1.0f, 0.0f};
    }
    bool full() const { return K == 0 || n == uint32_t(K); }
    void insert(Hit h) {
        if (K == 0) return;
        if (full()) {
            e[0].hitT = -1.0f;
        } else {
            n++;
        }
        for (int i = K - 1; i >= 0; --i) {
            if (h.hitT > e[i].hitT) std::swap(e[i], h);
        }
    }
};

uint64_t next_scene_serial() {
    static std::atomic<uint64_t> counter{0};
    return counter.fetch_add(1) + 1;
}

struct Scene {
    const OracleCamera* cam;
    const OraclePose* pose;
    int N;
    const float* particles;
    const float* rgb;
    const float* rayO;
    const float* rayD;
    const uint8_t* mask;
    const uint32_t* ranges;
    const uint32_t* sortedIds;
    int K;  // k-buffer size; kSofHierarchy: SOF's HEAD4 / MID8 / TAIL64 hierarchy
    // Distinct for every Scene built in this process: the per-thread SOF feed
    // cache is keyed on it, not on the Scene's address, which a later call's
    // Scene may reuse (the calling thread keeps its cache between calls).
    uint64_t serial = next_scene_serial();
};

// ------------------------------------------------------------------ SOF hierarchy
// The SOF compositor (sofMid8Hierarchy.inl:161-598, gutRenderer training
// default): per 4x4 pixel group a TAIL window of up to 64 candidates, per 2x2
// group a MID window of up to 8, per pixel a HEAD k-buffer of 4 by exact hit
// distance.  TAIL and MID order candidates by (representative depth, position
// in the tile's sorted list), the representative depth being the
// maximum-response depth of the particle along the group's representative
// ray (mean of the group's in-raster world rays: the central 2x2 pixels of a
// 4x4 group, else all of them; the four pixels of a 2x2 group).  The tile's
// candidates stream in chunks of 32 into every TAIL; a TAIL holding more than
// 32 emits its 16 nearest (twice per chunk); an emission reaches the four MID
// windows under it in batches of 4; a MID holding more than 4 emits its 4
// nearest, which every pixel of the 2x2 group feeds through its HEAD.  At the
// end the TAILs drain in two emissions of up to 16, then the MIDs and the
// HEADs.  The cascade does not depend on the pixels' state, so it is
// computed once per tile as each pixel's feed sequence (sorted positions).
constexpr int kSofHierarchy = -1;
constexpr int kSofHead = 4;

struct SofItem {
    float key;
    uint32_t pos;  // position in the tile's sorted list (unique: the tie-break)
};
inline bool sof_less(const SofItem& a, const SofItem& b) { return a.key < b.key || (a.key == b.key && a.pos < b.pos); }

// Merge of two windows by rank counting: item order is (key, position), and
// each item's place is the number of items below it (as the GPU writes by rank).
std::vector<SofItem> sof_merge(const std::vector<SofItem>& a, const std::vector<SofItem>& b) {
    std::vector<SofItem> all(a);
    all.insert(all.end(), b.begin(), b.end());
    std::vector<SofItem> out(all.size());
    for (size_t i = 0; i < all.size(); ++i) {
        size_t rank = 0;
        for (size_t j = 0; j < all.size(); ++j) rank += sof_less(all[j], all[i]) ? 1 : 0;
        out[rank] = all[i];
    }
    return out;
}

struct SofRay {
    float3_ o, d;
};

// Mean of the listed world rays: origin sum x (1 / count), direction
// d / sqrt(|d|^2) of the summed directions ((0,0,1) when degenerate).
SofRay sof_mean_ray(const std::vector<const Ray*>& rays) {
    float3_ o = f3(0.0f, 0.0f, 0.0f), d = f3(0.0f, 0.0f, 0.0f);
    for (const Ray* r : rays) {
        o = add(o, r->o);
        d = add(d, r->d);
    }
    SofRay out;
    const float inv = rays.empty() ? 0.0f : 1.0f / float(rays.size());
    out.o = rays.empty() ? f3(0.0f, 0.0f, 0.0f) : f3(o.x * inv, o.y * inv, o.z * inv);
    const float n2 = fdot(d, d);
    if (!(n2 > 0.0f) || !gf::isfinite_f(n2)) {
        out.d = f3(0.0f, 0.0f, 1.0f);
    } else {
        const float inorm = 1.0f / sqrtf(n2);
        out.d = f3(d.x * inorm, d.y * inorm, d.z * inorm);
    }
    return out;
}

// Maximum-response depth of a particle along a representative ray
// (sofMid8Hierarchy.inl:95-129): max(0, -(B^-1 (o - mu)) . (B^-1 d) / |B^-1 d|^2),
// the radial distance |mu - o| when that is not defined.
float sof_depth(const Particle& P, const SofRay& r) {
    const float3_ co = fmatvec(P.Binv, sub(r.o, P.pos));
    const float3_ cd = fmatvec(P.Binv, r.d);
    const float den = fdot(cd, cd);
    const float3_ delta = sub(P.pos, r.o);
    const float radial = sqrtf(fdot(delta, delta));
    if (!(den > 0.0f) || !gf::isfinite_f(den)) return radial;
    const float depth = -fdot(co, cd) / den;
    return gf::isfinite_f(depth) ? gf::max_f(0.0f, depth) : radial;
}

// Feed sequences (sorted positions) of the 256 pixels of a tile.
std::vector<std::vector<uint32_t>> sof_feeds(const Scene& sc, uint32_t tile) {
    const int W = sc.cam->width, H = sc.cam->height;
    const int gx = (W + kTile - 1) / kTile;
    const int tx = int(tile) % gx, ty = int(tile) / gx;
    std::vector<Ray> rays(256);
    std::vector<bool> inb(256, false);
    for (int ly = 0; ly < 16; ++ly)
        for (int lx = 0; lx < 16; ++lx) {
            const int px = tx * kTile + lx, py = ty * kTile + ly;
            if (px < W && py < H) {
                const size_t pix = size_t(px) + size_t(W) * py;
                rays[size_t(ly * 16 + lx)] = make_ray(*sc.pose, sc.rayO + 3 * pix, sc.rayD + 3 * pix);
                inb[size_t(ly * 16 + lx)] = true;
            }
        }
    SofRay tailRay[16], midRay[64];
    for (int g = 0; g < 16; ++g) {
        const int bx = (g & 3) * 4, by = (g >> 2) * 4;
        std::vector<const Ray*> sel;
        for (int oy = 1; oy <= 2; ++oy)
            for (int ox = 1; ox <= 2; ++ox)
                if (inb[size_t((by + oy) * 16 + bx + ox)]) sel.push_back(&rays[size_t((by + oy) * 16 + bx + ox)]);
        if (sel.empty())
            for (int oy = 0; oy < 4; ++oy)
                for (int ox = 0; ox < 4; ++ox)
                    if (inb[size_t((by + oy) * 16 + bx + ox)]) sel.push_back(&rays[size_t((by + oy) * 16 + bx + ox)]);
        tailRay[g] = sof_mean_ray(sel);
    }
    for (int m = 0; m < 64; ++m) {
        const int bx = (m & 7) * 2, by = (m >> 3) * 2;
        std::vector<const Ray*> sel;
        for (int oy = 0; oy < 2; ++oy)
            for (int ox = 0; ox < 2; ++ox)
                if (inb[size_t((by + oy) * 16 + bx + ox)]) sel.push_back(&rays[size_t((by + oy) * 16 + bx + ox)]);
        midRay[m] = sof_mean_ray(sel);
    }
    std::vector<std::vector<uint32_t>> feeds(256);
    std::vector<SofItem> tail[16], mid[64];
    auto key_of = [&](uint32_t pos, const SofRay& r) {
        const Particle P = load_particle(sc.particles + 32 * size_t(sc.sortedIds[pos]));
        return SofItem{sof_depth(P, r), pos};
    };
    // MID windows of one tail emission per tail group, in batches of four
    auto route = [&](std::vector<SofItem> (&emitted)[16]) {
        for (int batch = 0; batch < 4; ++batch) {
            for (int m = 0; m < 64; ++m) {
                const int parent = ((m >> 3) >> 1) * 4 + ((m & 7) >> 1);
                std::vector<SofItem> fresh;
                for (int k = 4 * batch; k < 4 * batch + 4 && k < int(emitted[parent].size()); ++k)
                    fresh.push_back(key_of(emitted[parent][size_t(k)].pos, midRay[m]));
                mid[m] = sof_merge(mid[m], fresh);
                if (mid[m].size() > 4) {
                    const int bx = (m & 7) * 2, by = (m >> 3) * 2;
                    for (int i = 0; i < 4; ++i)
                        for (int oy = 0; oy < 2; ++oy)
                            for (int ox = 0; ox < 2; ++ox) feeds[size_t((by + oy) * 16 + bx + ox)].push_back(mid[m][size_t(i)].pos);
                    mid[m].erase(mid[m].begin(), mid[m].begin() + 4);
                }
            }
        }
    };
    auto emit_tails = [&](bool drain) {
        std::vector<SofItem> emitted[16];
        for (int g = 0; g < 16; ++g) {
            const size_t count = drain ? std::min<size_t>(16, tail[g].size()) : (tail[g].size() > 32 ? 16 : 0);
            emitted[g].assign(tail[g].begin(), tail[g].begin() + long(count));
            tail[g].erase(tail[g].begin(), tail[g].begin() + long(count));
        }
        route(emitted);
    };
    const uint32_t b = sc.ranges[2 * tile], e = sc.ranges[2 * tile + 1];
    for (uint32_t chunk = b; chunk < e; chunk += 32) {
        const uint32_t stop = std::min(chunk + 32u, e);
        for (int g = 0; g < 16; ++g) {
            std::vector<SofItem> fresh;
            for (uint32_t pos = chunk; pos < stop; ++pos) fresh.push_back(key_of(pos, tailRay[g]));
            tail[g] = sof_merge(tail[g], fresh);
        }
        emit_tails(false);
        emit_tails(false);
    }
    emit_tails(true);
    emit_tails(true);
    for (int m = 0; m < 64; ++m) {
        const int bx = (m & 7) * 2, by = (m >> 3) * 2;
        for (const SofItem& it : mid[m])
            for (int oy = 0; oy < 2; ++oy)
                for (int ox = 0; ox < 2; ++ox) feeds[size_t((by + oy) * 16 + bx + ox)].push_back(it.pos);
        mid[m].clear();
    }
    return feeds;
}

// The feed sequence of one pixel, computed once per tile and worker thread.
const std::vector<uint32_t>& sof_pixel_feed(const Scene& sc, uint32_t tile, const Ray& ray) {
    thread_local uint64_t cachedScene = 0;
    thread_local uint32_t cachedTile = 0xffffffffu;
    thread_local std::vector<std::vector<uint32_t>> cached;
    if (cachedScene != sc.serial || cachedTile != tile) {
        cached = sof_feeds(sc, tile);
        cachedScene = sc.serial;
        cachedTile = tile;
    }
    return cached[size_t(ray.local)];
}

// Walk one pixel's tile list in the order of gutKBufferRenderer.cuh:614-700,
// calling `hitFn(Hit, state)` for each composited hit; with the SOF
// hierarchy, walk its feed sequence through a HEAD of 4.
template <typename HitFn>
void traverse(const Scene& sc, uint32_t tile, const Ray& ray, bool& alive, HitFn&& hitFn) {
    if (sc.K == kSofHierarchy) {
        const std::vector<uint32_t>& feed = sof_pixel_feed(sc, tile, ray);
        KBuffer kb;
        kb.init(kSofHead);
        for (size_t f = 0; f < feed.size() && alive; ++f) {
            const uint32_t idx = sc.sortedIds[feed[f]];
            const Particle P = load_particle(sc.particles + 32 * size_t(idx));
            Hit h;
            h.idx = idx;
            float resp;
            HalfRay hr;
            if (hit_test(ray, P, h.alpha, h.hitT, resp, hr) && h.hitT >= ray.tmin && h.hitT <= ray.tmax) {
                if (kb.full()) hitFn(kb.e[0]);
                kb.insert(h);
            }
        }
        for (uint32_t i = 0; alive && i < kb.n; ++i) hitFn(kb.e[kSofHead - kb.n + i]);
        return;
    }
    const uint32_t b = sc.ranges[2 * tile], e = sc.ranges[2 * tile + 1];
    KBuffer kb;
    kb.init(sc.K);
    for (uint32_t s = b; s < e && alive; ++s) {
        const uint32_t idx = sc.sortedIds[s];
        if (idx == kInvalidParticle) break;
        const Particle P = load_particle(sc.particles + 32 * size_t(idx));
        Hit h;
        h.idx = idx;
        float resp;
        HalfRay hr;
        if (hit_test(ray, P, h.alpha, h.hitT, resp, hr) && h.hitT >= ray.tmin && h.hitT <= ray.tmax) {
            if (kb.full()) hitFn(sc.K == 0 ? h : kb.e[0]);
            kb.insert(h);
        }
    }
    if (sc.K > 0) {
        for (uint32_t i = 0; alive && i < kb.n; ++i) hitFn(kb.e[sc.K - kb.n + i]);
    }
}

// ------------------------------------------------------------------ geometric channels
// The training channels of processHitParticle (gutKBufferRenderer.cuh:330-392)
// and finalizeRay (rayPayload.cuh:242-322), per composited hit, w = alpha T_before:
// normal += w n with n = -normalize(B^-T normalize(B^-1 d))
// (gaussianParticles.slang:254-265); depth var += (w t) t; extent += w
// |s * (R^T d)| of the intrinsic rotation and scale (gaussianParticles.cuh:131-141,
// quaternionWXYZToMatrix :55-75); inverse depth moments with the 0.2 near clip
// (sensorConstants.cuh:28-42); the first depth where 1 - T_after reaches each
// opacity threshold; the largest-weight depth; the exact 0.5 crossing
// (finiteIntervalExactCrossing.cuh:42-109).
constexpr int kQuantiles = 7;
constexpr float kQuantileThresholds[kQuantiles] = {0.05f, 0.10f, 0.15f, 0.20f, 0.30f, 0.40f, 0.50f};

struct GeoState {
    float n[3];
    float sumWD2, sumExt, sumInvD, sumInvD2;
    float q[kQuantiles];
    float tauMaxW, tauMaxD, exactDepth, exactRate;
    float dscale;
};

inline float3_ rotate_transpose(const float* q, float3_ d) {
    const float r = q[0], x = q[1], y = q[2], z = q[3];
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z, rx = r * x, ry = r * y,
                rz = r * z;
    const float3_ r0 = f3(1.0f - 2.0f * (yy + zz), 2.0f * (xy + rz), 2.0f * (xz - ry));
    const float3_ r1 = f3(2.0f * (xy - rz), 1.0f - 2.0f * (xx + zz), 2.0f * (yz + rx));
    const float3_ r2 = f3(2.0f * (xz + ry), 2.0f * (yz - rx), 1.0f - 2.0f * (xx + yy));
    return f3(fdot(r0, d), fdot(r1, d), fdot(r2, d));
}

inline float extent_sigma(const Particle& P, float3_ d) {
    const float3_ rd = rotate_transpose(P.quat, d);
    const float3_ sd = f3(P.scale[0] * rd.x, P.scale[1] * rd.y, P.scale[2] * rd.z);
    return std::sqrt(fdot(sd, sd) + 1e-18f);
}

inline float crossing_alpha(float AA, float BB, float CC, float density, float t) {
    const float qd = gf::max_f(fmaf_rn(fmaf_rn(AA, t, BB), t, CC), 0.0f);
    return gf::min_f(kMaxAlpha, density * gf::gf_expf(-0.5f * qd));
}

inline bool exact_crossing(float AA, float BB, float CC, float density, float tBefore, float tmin, float tmax,
                           float& depth, float& rate) {
    const float threshold = 0.5f;
    if (!(gf::isfinite_f(AA) && gf::isfinite_f(BB) && gf::isfinite_f(CC) && gf::isfinite_f(density) &&
          gf::isfinite_f(tBefore) && gf::isfinite_f(tmin) && gf::isfinite_f(tmax)))
        return false;
    if (!(AA > 0.0f) || !(density > 0.0f) || !(tmax > tmin) || !(tBefore > threshold) || !(tBefore <= 1.0f))
        return false;
    const float tLine = -BB / (2.0f * AA);
    const float tPeak = gf::min_f(gf::max_f(tLine, tmin), tmax);
    const float peakAlpha = crossing_alpha(AA, BB, CC, density, tPeak);
    const float required = 1.0f - threshold / tBefore;
    if (!(required > 0.0f) || !(required < kMaxAlpha) || !(peakAlpha >= required)) return false;
    const float level = required / density;
    if (!(level > 0.0f) || !(level <= 1.0f) || !gf::isfinite_f(level)) return false;
    const float con = CC + 2.0f * gf::gf_logf(level);
    const float disc = BB * BB - (4.0f * AA) * con;
    if (!(disc >= 0.0f) || !gf::isfinite_f(disc)) return false;
    const float nearRoot = (-BB - std::sqrt(disc)) / (2.0f * AA);
    if (!gf::isfinite_f(nearRoot)) return false;
    if (nearRoot <= tmin || nearRoot >= tmax) {
        const float edge = nearRoot <= tmin ? tmin : tmax;
        if (!(crossing_alpha(AA, BB, CC, density, edge) >= required)) return false;
        depth = edge;
        rate = 0.0f;
        return true;
    }
    const float r = -0.5f * (tBefore - threshold) * (2.0f * AA * nearRoot + BB);
    depth = nearRoot;
    rate = (disc == 0.0f || !gf::isfinite_f(r) || !(r > 0.0f)) ? 0.0f : r;
    return true;
}

// d/dv of v/|v| applied to the output gradient go (safe_normalize_bw,
// mathUtils.cuh:411-421): go/|v| - v (v . go)/|v|^3; zero for v = 0.
inline float3_ normalize_vjp(float3_ v, float3_ go) {
    const float l = v.x * v.x + v.y * v.y + v.z * v.z;
    if (!(l > 0.0f)) return f3(0.0f, 0.0f, 0.0f);
    const float il = 1.0f / std::sqrt(l);
    const float il3 = il * il * il;
    return f3(il * go.x - il3 * (go.x * (v.x * v.x) + go.y * (v.y * v.x) + go.z * (v.z * v.x)),
              il * go.y - il3 * (go.x * (v.x * v.y) + go.y * (v.y * v.y) + go.z * (v.z * v.y)),
              il * go.z - il3 * (go.x * (v.x * v.z) + go.y * (v.y * v.z) + go.z * (v.z * v.z)));
}

// d/dq (w, x, y, z) of y = M(q) p (the rows of rotate_transpose) for dL/dy = go.
inline void rotate_transpose_vjp(const float* q, float3_ p, float3_ go, float* out) {
    const float r = q[0], x = q[1], y = q[2], z = q[3];
    const float G00 = go.x * p.x, G01 = go.x * p.y, G02 = go.x * p.z;
    const float G10 = go.y * p.x, G11 = go.y * p.y, G12 = go.y * p.z;
    const float G20 = go.z * p.x, G21 = go.z * p.y, G22 = go.z * p.z;
    out[0] = 2.0f * (z * G01 - y * G02 - z * G10 + x * G12 + y * G20 - x * G21);
    out[1] = 2.0f * (y * G01 + z * G02 + y * G10 + r * G12 + z * G20 - r * G21) - 4.0f * x * (G11 + G22);
    out[2] = 2.0f * (x * G01 - r * G02 + x * G10 + z * G12 + r * G20 + z * G21) - 4.0f * y * (G00 + G22);
    out[3] = 2.0f * (r * G01 + x * G02 - r * G10 + y * G12 + x * G20 + y * G21) - 4.0f * z * (G00 + G11);
}

void geo_hit(GeoState& g, const Ray& ray, const Particle& P, float hitT, float w, float tBefore, float tAfter) {
    const float3_ grdu = fmatvec(P.Binv, ray.d);
    const float len = std::sqrt(fdot(grdu, grdu));
    const float3_ grd = f3(grdu.x / len, grdu.y / len, grdu.z / len);
    const float* M = P.Binv;  // B^-T grd
    const float3_ nu = f3(fmaf_rn(M[6], grd.z, fmaf_rn(M[3], grd.y, M[0] * grd.x)),
                          fmaf_rn(M[7], grd.z, fmaf_rn(M[4], grd.y, M[1] * grd.x)),
                          fmaf_rn(M[8], grd.z, fmaf_rn(M[5], grd.y, M[2] * grd.x)));
    const float inv = -1.0f / std::sqrt(fdot(nu, nu));
    g.n[0] = fmaf_rn(w, inv * nu.x, g.n[0]);
    g.n[1] = fmaf_rn(w, inv * nu.y, g.n[1]);
    g.n[2] = fmaf_rn(w, inv * nu.z, g.n[2]);
    g.sumWD2 = fmaf_rn(w * hitT, hitT, g.sumWD2);
    const float dd = hitT * g.dscale;
    const bool active = dd > kParticleMinSensorZ;
    const float invD = active ? 1.0f / dd : 1.0f / kParticleMinSensorZ;
    const float invD2 = active ? 1.0f / ((hitT * hitT) * (g.dscale * g.dscale))
                               : 1.0f / (kParticleMinSensorZ * kParticleMinSensorZ);
    g.sumInvD = fmaf_rn(w, invD, g.sumInvD);
    g.sumInvD2 = fmaf_rn(w, invD2, g.sumInvD2);
    g.sumExt = fmaf_rn(w, extent_sigma(P, ray.d), g.sumExt);
    const float oAcc = 1.0f - tAfter;
    for (int i = 0; i < kQuantiles; ++i)
        if (g.q[i] == 0.0f && oAcc >= kQuantileThresholds[i]) g.q[i] = hitT;
    if (w > g.tauMaxW) {
        g.tauMaxW = w;
        g.tauMaxD = hitT;
    }
    if (g.exactDepth == 0.0f && tBefore > 0.5f && tAfter <= 0.5f) {
        const float3_ gro = fmatvec(P.Binv, sub(ray.o, P.pos));
        float depth = hitT, rate = 0.0f;
        if (!exact_crossing(fdot(grdu, grdu), 2.0f * fdot(gro, grdu), fdot(gro, gro), P.density, tBefore, ray.tmin,
                            ray.tmax, depth, rate)) {
            depth = hitT;
            rate = 0.0f;
        }
        g.exactDepth = depth;
        g.exactRate = rate;
    }
}

}  // namespace

extern "C" {

// Per-particle projected state, gutProjector.cuh:653-286 (projectOnTiles, fast UT
// admission).  proj[N*8] = center.xy, conic.xyz, opacity, extent.xy (zero when
// the projection is invalid); rgb[N*3] precomputed radiance; counts[N].
int oracle_project(const OracleCamera* cam, const OraclePose* pose, int N, const float* particles,
                   const float* sh, int shCoeffs, int shDegree, const uint8_t* mask, const float* rayD,
                   float* proj, float* rgb, uint32_t* counts) {
    const int gx = (cam->width + kTile - 1) / kTile, gy = (cam->height + kTile - 1) / kTile;
    fallback::Tree tree;
    if (rayD != nullptr) tree = fallback::build(*cam, *pose, mask, rayD);
    parallel_for(0, N, 1024, [&](int i, int) {
        const Particle P = load_particle(particles + 32 * size_t(i));
        float2_ center{0.0f, 0.0f};
        float cov[3] = {0.0f, 0.0f, 0.0f};
        Projection pr{};
        bool valid = unscented_projection(*cam, *pose, P, center, cov);
        if (valid) {
            pr.center = center;
            valid = conic_extent(cov, P.density, pr);
        }
        if (!valid) pr = Projection{};
        pr.valid = valid;
        float* o = proj + 8 * size_t(i);
        o[0] = pr.center.x; o[1] = pr.center.y;
        o[2] = pr.conic[0]; o[3] = pr.conic[1]; o[4] = pr.conic[2];
        o[5] = pr.opacity;
        o[6] = pr.extent.x; o[7] = pr.extent.y;
        // SH radiance at the incident direction (gutProjector.cuh:239-245).
        float dist;
        const float3_ dir = incident_direction(P.pos, *pose, dist);
        float basis[16];
        sh_basis(shDegree, dir, basis);
        const float* c = sh + size_t(i) * 3 * shCoeffs;
        const int nb = shDegree >= 3 ? 16 : (shDegree == 2 ? 9 : (shDegree == 1 ? 4 : 1));
        for (int ch = 0; ch < 3; ++ch) {
            float acc = basis[0] * c[ch];
            for (int k = 1; k < nb && k < shCoeffs; ++k) acc = fmaf_rn(basis[k], c[3 * k + ch], acc);
            const float v = acc + 0.5f;
            rgb[3 * size_t(i) + ch] = gf::max_f(v, 0.0f);
        }
        counts[i] = g_completeAdmission ? 0u : admitted_tiles(gx, gy, mask, pr, [](int, int) {});
        if (rayD != nullptr && (g_completeAdmission || !fast_ut_valid(pr)) && P.density >= kAlphaThreshold)
            counts[i] = fallback::tiles(tree, mask, fallback::admitted_cap(P, *pose), [](int, int) {});
    });
    return 0;
}

// Per-tile central rays for the per-tile depth key (gutProjector.cuh:364-417):
// tileRays[T*8] = world origin.xyz, flag, world direction.xyz, pad.  flag = 1
// when the direction is usable, 0 when the key must use the radial fallback.
int oracle_tile_rays(const OracleCamera* cam, const OraclePose* pose, const float* rayO, const float* rayD,
                     float* tileRays) {
    const int W = cam->width, H = cam->height;
    const int gx = (W + kTile - 1) / kTile, gy = (H + kTile - 1) / kTile;
    for (int ty = 0; ty < gy; ++ty) {
        for (int tx = 0; tx < gx; ++tx) {
            const int xb = tx * kTile, yb = ty * kTile;
            const int xe = std::min(W - 1, (tx + 1) * kTile - 1), ye = std::min(H - 1, (ty + 1) * kTile - 1);
            const int xlo = (xb + xe) / 2, xhi = (xb + xe + 1) / 2, ylo = (yb + ye) / 2, yhi = (yb + ye + 1) / 2;
            const size_t p[4] = {size_t(xlo) + size_t(W) * ylo, size_t(xhi) + size_t(W) * ylo,
                                 size_t(xlo) + size_t(W) * yhi, size_t(xhi) + size_t(W) * yhi};
            float3_ so = f3(0, 0, 0), sd = f3(0, 0, 0);
            for (int k = 0; k < 4; ++k) {
                so = add(so, f3(rayO[3 * p[k]], rayO[3 * p[k] + 1], rayO[3 * p[k] + 2]));
                sd = add(sd, f3(rayD[3 * p[k]], rayD[3 * p[k] + 1], rayD[3 * p[k] + 2]));
            }
            so = scale(0.25f, so);
            sd = scale(0.25f, sd);
            const float3_ wo = add(matvec(pose->Rinv, so), f3(pose->c[0], pose->c[1], pose->c[2]));
            float* out = tileRays + 8 * size_t(ty * gx + tx);
            out[0] = wo.x; out[1] = wo.y; out[2] = wo.z;
            out[3] = 0.0f;
            out[4] = out[5] = out[6] = out[7] = 0.0f;
            const float n2 = dot(sd, sd);
            if (!(n2 > 0.0f) || !gf::isfinite_f(n2)) continue;
            sd = scale(1.0f / sqrtf(n2), sd);
            float3_ wd = matvec(pose->Rinv, sd);
            const float m2 = dot(wd, wd);
            if (!(m2 > 0.0f) || !gf::isfinite_f(m2)) continue;
            wd = scale(1.0f / sqrtf(m2), wd);
            out[3] = 1.0f;
            out[4] = wd.x; out[5] = wd.y; out[6] = wd.z;
        }
    }
    return 0;
}

}  // extern "C"

namespace {

// sofDepthFallback.cuh:13-17
inline float finite_nonneg(float v, float fallbackMax) {
    if (gf::isfinite_f(v) && v >= 0.0f) return v;
    return (gf::isfinite_f(fallbackMax) && fallbackMax >= 0.0f) ? fallbackMax : 0.0f;
}

// Sort key depth of one (particle, tile), gutProjector.cuh:354-417 and
// sofMaximumResponseDepth.cuh:19-45.  keyMode 0 = per-tile maximum-response
// depth (training/exact key), 1 = global camera radial distance (real-time key).
uint32_t depth_key(int keyMode, const Particle& P, const OraclePose& pose, const float* tileRay) {
    const float3_ cam = f3(pose.c[0], pose.c[1], pose.c[2]);
    const float3_ v = sub(P.pos, cam);
    const float camRadial = finite_nonneg(sqrtf(dot(v, v)), kMaxDepthValue);
    if (keyMode == 1) return gf::f2u(camRadial);
    const float3_ wo = f3(tileRay[0], tileRay[1], tileRay[2]);
    const float3_ u = sub(P.pos, wo);
    const float tileRadial = finite_nonneg(sqrtf(dot(u, u)), camRadial);
    if (tileRay[3] == 0.0f) return gf::f2u(finite_nonneg(tileRadial, camRadial));
    const float3_ wd = f3(tileRay[4], tileRay[5], tileRay[6]);
    const float3_ lo = sub(wo, P.pos);
    const float3_ co = matvec(P.Binv, lo);
    const float3_ cd = matvec(P.Binv, wd);
    const float den = dot(cd, cd);
    if (!(den > 0.0f) || !gf::isfinite_f(den)) return gf::f2u(finite_nonneg(tileRadial, 0.0f));
    const float t = -dot(co, cd) / den;
    if (!gf::isfinite_f(t)) return gf::f2u(finite_nonneg(tileRadial, 0.0f));
    return gf::f2u(gf::max_f(0.0f, t));
}

}  // namespace

extern "C" {

// Emit (tile << 32 | depth) keys and particle ids in particle order, then a
// stable sort and the per-tile ranges (gutProjector.cuh:947-1113 expand,
// gutRenderer.cu:114-144 computeSortedTileRangeIndices, :1527-1539 CUB
// stable radix sort).  Returns the number of intersections, or -1 when
// `capacity` is too small (keys/ids are then untouched).
int64_t oracle_bin(const OracleCamera* cam, const OraclePose* pose, int N, const float* particles,
                   const float* proj, const uint32_t* counts, const uint8_t* mask, const float* tileRays,
                   const float* rayD, int keyMode, uint64_t* keys, uint32_t* ids, int64_t capacity,
                   uint32_t* ranges) {
    const int gx = (cam->width + kTile - 1) / kTile, gy = (cam->height + kTile - 1) / kTile;
    fallback::Tree tree;
    if (rayD != nullptr) tree = fallback::build(*cam, *pose, mask, rayD);
    std::vector<uint64_t> offsets(static_cast<size_t>(N) + 1, 0);
    for (int i = 0; i < N; ++i) offsets[i + 1] = offsets[i] + counts[i];
    const int64_t total = int64_t(offsets[N]);
    if (total > capacity) return -1;
    parallel_for(0, N, 1024, [&](int i, int) {
        const Particle P = load_particle(particles + 32 * size_t(i));
        const float* o = proj + 8 * size_t(i);
        Projection pr{};
        pr.center = {o[0], o[1]};
        pr.conic[0] = o[2]; pr.conic[1] = o[3]; pr.conic[2] = o[4];
        pr.opacity = o[5];
        pr.extent = {o[6], o[7]};
        uint64_t k = offsets[i];
        const uint64_t end = offsets[i + 1];
        auto emit = [&](int x, int y) {
            if (k < end) {
                const uint32_t tile = uint32_t(y * gx + x);
                keys[k] = (uint64_t(tile) << 32) | depth_key(keyMode, P, *pose, tileRays + 8 * size_t(tile));
                ids[k] = uint32_t(i);
            }
            ++k;
        };
        if (!g_completeAdmission) admitted_tiles(gx, gy, mask, pr, emit);
        if (rayD != nullptr && (g_completeAdmission || !fast_ut_valid(pr)) && P.density >= kAlphaThreshold)
            fallback::tiles(tree, mask, fallback::admitted_cap(P, *pose), emit);
    });
    // Stable sort of (key, id) pairs by key.
    std::vector<uint64_t> order(static_cast<size_t>(total));
    for (int64_t i = 0; i < total; ++i) order[i] = uint64_t(i);
    std::stable_sort(order.begin(), order.end(), [&](uint64_t a, uint64_t b) { return keys[a] < keys[b]; });
    std::vector<uint64_t> k2(static_cast<size_t>(total));
    std::vector<uint32_t> i2(static_cast<size_t>(total));
    for (int64_t i = 0; i < total; ++i) {
        k2[i] = keys[order[i]];
        i2[i] = ids[order[i]];
    }
    std::memcpy(keys, k2.data(), sizeof(uint64_t) * size_t(total));
    std::memcpy(ids, i2.data(), sizeof(uint32_t) * size_t(total));
    const int T = gx * gy;
    std::memset(ranges, 0, sizeof(uint32_t) * 2 * size_t(T));
    for (int64_t i = 0; i < total; ++i) {
        const uint32_t tile = uint32_t(keys[i] >> 32);
        if (i == 0 || uint32_t(keys[i - 1] >> 32) != tile) ranges[2 * tile] = uint32_t(i);
        if (i == total - 1 || uint32_t(keys[i + 1] >> 32) != tile) ranges[2 * tile + 1] = uint32_t(i + 1);
    }
    return total;
}

// Per-pixel forward composite over tiles [tileBegin, tileEnd) (render kernel,
// gutRenderer.cuh:217-265; finalizeRay, rayPayload.cuh:242-322).  Outputs keep
// their initial values (rgba 0, hitT 1e6, count 0) outside retained tiles
// and for invalid rays; the caller initializes them.
int oracle_render_forward(const OracleCamera* cam, const OraclePose* pose, int N, const float* particles,
                          const float* rgb, const float* rayO, const float* rayD, const uint8_t* mask,
                          const uint32_t* ranges, const uint32_t* sortedIds, int K, int tileBegin, int tileEnd,
                          float* rgba, float* hitT, float* hitCount) {
    const int W = cam->width, H = cam->height;
    const int gx = (W + kTile - 1) / kTile;
    Scene sc{cam, pose, N, particles, rgb, rayO, rayD, mask, ranges, sortedIds, K};
    parallel_tiles(tileBegin, tileEnd, [&](int tile, int) {
        if (mask[tile] == 0u) return;
        const int tx = tile % gx, ty = tile / gx;
        for (int py = ty * kTile; py < std::min(H, (ty + 1) * kTile); ++py) {
            for (int px = tx * kTile; px < std::min(W, (tx + 1) * kTile); ++px) {
                const size_t pix = size_t(px) + size_t(W) * py;
                Ray ray = make_ray(*pose, rayO + 3 * pix, rayD + 3 * pix);
                ray.local = (py - ty * kTile) * kTile + (px - tx * kTile);
                if (!ray.valid) continue;
                PixelState s{1.0f, {0.0f, 0.0f, 0.0f}, 0.0f, 0u, true};
                traverse(sc, uint32_t(tile), ray, s.alive, [&](const Hit& h) { composite(s, h, rgb); });
                rgba[4 * pix + 0] = s.rgb[0];
                rgba[4 * pix + 1] = s.rgb[1];
                rgba[4 * pix + 2] = s.rgb[2];
                rgba[4 * pix + 3] = 1.0f - s.T;
                hitT[pix] = s.hitT;
                hitCount[pix] = float(s.hitN);
            }
        }
    });
    return 0;
}

// The forward of oracle_render_forward with the geometric training channels
// (enable_normals): normal[P*3], depthVar[P], quant[P*10], extent[P],
// invD[P], invD2[P]; pinhole selects the sensor ray's z as the distortion
// depth scale (rayPayload.cuh:129-136), a fisheye uses 1.
int oracle_render_forward_geo(const OracleCamera* cam, const OraclePose* pose, int N, const float* particles,
                              const float* rgb, const float* rayO, const float* rayD, const uint8_t* mask,
                              const uint32_t* ranges, const uint32_t* sortedIds, int K, int tileBegin, int tileEnd,
                              int pinhole, float* rgba, float* hitT, float* hitCount, float* normal, float* depthVar,
                              float* quant, float* extent, float* invD, float* invD2) {
    const int W = cam->width, H = cam->height;
    const int gx = (W + kTile - 1) / kTile;
    Scene sc{cam, pose, N, particles, rgb, rayO, rayD, mask, ranges, sortedIds, K};
    parallel_tiles(tileBegin, tileEnd, [&](int tile, int) {
        if (mask[tile] == 0u) return;
        const int tx = tile % gx, ty = tile / gx;
        for (int py = ty * kTile; py < std::min(H, (ty + 1) * kTile); ++py) {
            for (int px = tx * kTile; px < std::min(W, (tx + 1) * kTile); ++px) {
                const size_t pix = size_t(px) + size_t(W) * py;
                Ray ray = make_ray(*pose, rayO + 3 * pix, rayD + 3 * pix);
                ray.local = (py - ty * kTile) * kTile + (px - tx * kTile);
                if (!ray.valid) continue;
                PixelState s{1.0f, {0.0f, 0.0f, 0.0f}, 0.0f, 0u, true};
                GeoState g{};
                g.dscale = pinhole ? rayD[3 * pix + 2] : 1.0f;
                traverse(sc, uint32_t(tile), ray, s.alive, [&](const Hit& h) {
                    const float tBefore = s.T;
                    composite(s, h, rgb);
                    const Particle P = load_particle(particles + 32 * size_t(h.idx));
                    geo_hit(g, ray, P, h.hitT, h.alpha * tBefore, tBefore, s.T);
                });
                rgba[4 * pix + 0] = s.rgb[0];
                rgba[4 * pix + 1] = s.rgb[1];
                rgba[4 * pix + 2] = s.rgb[2];
                rgba[4 * pix + 3] = 1.0f - s.T;
                hitT[pix] = s.hitT;
                hitCount[pix] = float(s.hitN);
                for (int k = 0; k < 3; ++k) normal[3 * pix + k] = g.n[k];
                depthVar[pix] = g.sumWD2;
                extent[pix] = g.sumExt;
                invD[pix] = g.sumInvD;
                invD2[pix] = g.sumInvD2;
                float* q = quant + 10 * pix;
                for (int k = 0; k < kQuantiles; ++k) q[k] = g.q[k];
                q[kQuantiles] = g.tauMaxD;
                q[kQuantiles + 1] = g.exactDepth;
                q[kQuantiles + 2] = g.exactRate;
            }
        }
    });
    return 0;
}

// Per-pixel backward replay (renderBackward, gutRenderer.cuh:555-626;
// processHitBwd, gaussianParticles.cuh:736-1155, with the geometric channels
// inactive).  Accumulates into gradRecord[N*16]: position.xyz, density,
// inverse factor (row-major, 9), rgb.xyz.  Each worker accumulates into its
// own buffer; the buffers are summed in worker order.
int oracle_render_backward(const OracleCamera* cam, const OraclePose* pose, int N, const float* particles,
                           const float* rgb, const float* rayO, const float* rayD, const uint8_t* mask,
                           const uint32_t* ranges, const uint32_t* sortedIds, int K, int tileBegin, int tileEnd,
                           const float* rgba, const float* hitT, const float* gradRgba, const float* gradHitT,
                           float* gradRecord) {
    const int W = cam->width, H = cam->height;
    const int gx = (W + kTile - 1) / kTile;
    Scene sc{cam, pose, N, particles, rgb, rayO, rayD, mask, ranges, sortedIds, K};
    const int nthreads = worker_count();
    std::vector<std::vector<float>> partial(static_cast<size_t>(nthreads));
    std::vector<std::vector<float>> absPartial(static_cast<size_t>(nthreads));
    {
        parallel_tiles(tileBegin, tileEnd, [&](int tile, int tid) {
            std::vector<float>& acc = partial[size_t(tid)];
            if (acc.empty()) acc.assign(size_t(N) * 16, 0.0f);
            if (mask[tile] == 0u) return;
            const int tx = tile % gx, ty = tile / gx;
            for (int py = ty * kTile; py < std::min(H, (ty + 1) * kTile); ++py) {
                for (int px = tx * kTile; px < std::min(W, (tx + 1) * kTile); ++px) {
                    const size_t pix = size_t(px) + size_t(W) * py;
                    Ray ray = make_ray(*pose, rayO + 3 * pix, rayD + 3 * pix);
                    ray.local = (py - ty * kTile) * kTile + (px - tx * kTile);
                    if (!ray.valid) continue;
                    // initializeBackwardRay, rayPayloadBackward.cuh:59-120
                    const float featB[3] = {rgba[4 * pix], rgba[4 * pix + 1], rgba[4 * pix + 2]};
                    const float featG[3] = {gradRgba[4 * pix], gradRgba[4 * pix + 1], gradRgba[4 * pix + 2]};
                    const float TB = 1.0f - rgba[4 * pix + 3];
                    const float TG = -1.0f * gradRgba[4 * pix + 3];
                    const float hitTB = hitT[pix];
                    const float hitTG = gradHitT[pix];
                    float T = 1.0f, depth = 0.0f;
                    float radiance[3] = {0.0f, 0.0f, 0.0f};
                    bool alive = true;
                    traverse(sc, uint32_t(tile), ray, alive, [&](const Hit& hh) {
                        const Particle P = load_particle(particles + 32 * size_t(hh.idx));
                        const HalfRay h = half_ray(ray, P);
                        if (h.valid) {
                            const float grayDist = fdot(h.p, h.p);
                            const float gres = gf::gf_expf(-0.5f * grayDist);
                            const float galphaU = gres * P.density;
                            const float galpha = gf::min_f(kMaxAlpha, galphaU);
                            if (gres > kMinKernelResponse && galpha > kAlphaThreshold) {
                                const float gdist = h.tau;
                                const float weight = galpha * T;
                                const float nextT = (1.0f - galpha) * T;
                                depth = depth + gdist * weight;
                                const float residualHitT =
                                    gf::max_f(nextT <= kMinTransmittance ? 0.0f : (hitTB - depth) / nextT, 0.0f);
                                const float galphaRayHitGrd = (gdist - residualHitT) * T * hitTG;
                                const float residualTrm = galpha < 0.999999f ? TB / (1.0f - galpha) : T;
                                const float galphaRayDnsGrd = residualTrm * -TG;
                                const float* c = rgb + 3 * size_t(hh.idx);
                                float col[3], resid[3];
                                for (int k = 0; k < 3; ++k) {
                                    col[k] = gf::max_f(c[k], 0.0f);
                                    radiance[k] = fmaf_rn(col[k], weight, radiance[k]);
                                }
                                for (int k = 0; k < 3; ++k) {
                                    resid[k] = gf::max_f(
                                        nextT <= kMinTransmittance ? 0.0f : (featB[k] - radiance[k]) / nextT, 0.0f);
                                }
                                float comp = galphaRayHitGrd + galphaRayDnsGrd;
                                for (int k = 0; k < 3; ++k) comp += T * (col[k] - resid[k]) * featG[k];
                                const float gU = (galphaU < kMaxAlpha ? 1.0f : 0.0f) * comp;
                                float* g = acc.data() + 16 * size_t(hh.idx);
                                g[3] += gres * gU;
                                const float gresGrd = P.density * gU;
                                const float grayDistGrd = -0.5f * gres * gresGrd;
                                const float tauGrad = weight * hitTG;
                                // gutHalfRayResponse.cuh:39-62
                                const float3_ pointGrad = scale(2.0f * grayDistGrd, h.p);
                                float3_ groGrd = pointGrad;
                                float3_ grduGrd = scale(h.tau, pointGrad);
                                const float totalTauGrad = tauGrad + dot(pointGrad, h.grdu);
                                if (h.interior) {
                                    const float3_ tauOriginGrad = scale(-1.0f / h.denom, h.grdu);
                                    const float3_ tauDirectionGrad =
                                        add(scale(-1.0f / h.denom, h.gro),
                                            scale((2.0f * h.num) / (h.denom * h.denom), h.grdu));
                                    groGrd = add(groGrd, scale(totalTauGrad, tauOriginGrad));
                                    grduGrd = add(grduGrd, scale(totalTauGrad, tauDirectionGrad));
                                }
                                // position: -(Binv^T groGrd); Binv rows: += groGrd[i] gposc + grduGrd[i] d
                                const float* M = P.Binv;
                                const float px = -(groGrd.x * M[0] + groGrd.y * M[3] + groGrd.z * M[6]);
                                const float py = -(groGrd.x * M[1] + groGrd.y * M[4] + groGrd.z * M[7]);
                                const float pz = -(groGrd.x * M[2] + groGrd.y * M[5] + groGrd.z * M[8]);
                                g[0] += px;
                                g[1] += py;
                                g[2] += pz;
                                abs_grad_hit(absPartial[size_t(tid)], N, hh.idx, px, py, pz);
                                const float3_ gposc = sub(ray.o, P.pos);
                                const float gr[3] = {groGrd.x, groGrd.y, groGrd.z};
                                const float gd[3] = {grduGrd.x, grduGrd.y, grduGrd.z};
                                for (int r = 0; r < 3; ++r) {
                                    g[4 + 3 * r + 0] += gr[r] * gposc.x + gd[r] * ray.d.x;
                                    g[4 + 3 * r + 1] += gr[r] * gposc.y + gd[r] * ray.d.y;
                                    g[4 + 3 * r + 2] += gr[r] * gposc.z + gd[r] * ray.d.z;
                                }
                                for (int k = 0; k < 3; ++k) g[13 + k] += featG[k] * weight;
                                T = nextT;
                            }
                        }
                        if (T < kMinTransmittance) alive = false;
                    });
                }
            }
        });
    }
    std::memset(gradRecord, 0, sizeof(float) * size_t(N) * 16);
    for (int t = 0; t < nthreads; ++t) {
        if (partial[size_t(t)].empty()) continue;
        const float* a = partial[size_t(t)].data();
        for (size_t i = 0; i < size_t(N) * 16; ++i) gradRecord[i] += a[i];
    }
    abs_grad_reduce(absPartial, N);
    return 0;
}

// The backward of oracle_render_backward with the geometric training
// channels (gaussianParticles.cuh:786-1062): each channel pointer pair (value,
// gradient) may be NULL.  The depth moment and the normal sum reach alpha
// through their residuals, the depth moment and the inverse-depth moments
// reach the closest-point parameter tau, the normal reaches B^-1 and the
// canonical direction, and the extent reaches the intrinsic quaternion and
// scale only, accumulated into gradShape[N*8] (quaternion w,x,y,z | scale xyz, 0).
int oracle_render_backward_geo(const OracleCamera* cam, const OraclePose* pose, int N, const float* particles,
                               const float* rgb, const float* rayO, const float* rayD, const uint8_t* mask,
                               const uint32_t* ranges, const uint32_t* sortedIds, int K, int tileBegin, int tileEnd,
                               int pinhole, const float* rgba, const float* hitT, const float* gradRgba,
                               const float* gradHitT, const float* normal, const float* gradNormal,
                               const float* depthVar, const float* gradDepthVar, const float* gradExtent,
                               const float* gradInvD, const float* gradInvD2, const float* quant,
                               const float* gradQuant, float* gradRecord, float* gradShape) {
    const int W = cam->width, H = cam->height;
    const int gx = (W + kTile - 1) / kTile;
    Scene sc{cam, pose, N, particles, rgb, rayO, rayD, mask, ranges, sortedIds, K};
    const int nthreads = worker_count();
    std::vector<std::vector<float>> partial(static_cast<size_t>(nthreads)), partialShape(static_cast<size_t>(nthreads));
    std::vector<std::vector<float>> absPartial(static_cast<size_t>(nthreads));
    const auto val = [](const float* p, size_t i) { return p != nullptr ? p[i] : 0.0f; };
    parallel_tiles(tileBegin, tileEnd, [&](int tile, int tid) {
        std::vector<float>& acc = partial[size_t(tid)];
        std::vector<float>& accS = partialShape[size_t(tid)];
        if (acc.empty()) acc.assign(size_t(N) * 16, 0.0f);
        if (accS.empty()) accS.assign(size_t(N) * 8, 0.0f);
        if (mask[tile] == 0u) return;
        const int tx = tile % gx, ty = tile / gx;
        for (int py = ty * kTile; py < std::min(H, (ty + 1) * kTile); ++py) {
            for (int px = tx * kTile; px < std::min(W, (tx + 1) * kTile); ++px) {
                const size_t pix = size_t(px) + size_t(W) * py;
                Ray ray = make_ray(*pose, rayO + 3 * pix, rayD + 3 * pix);
                ray.local = (py - ty * kTile) * kTile + (px - tx * kTile);
                if (!ray.valid) continue;
                const float featB[3] = {rgba[4 * pix], rgba[4 * pix + 1], rgba[4 * pix + 2]};
                const float featG[3] = {gradRgba[4 * pix], gradRgba[4 * pix + 1], gradRgba[4 * pix + 2]};
                const float TB = 1.0f - rgba[4 * pix + 3];
                const float TG = -1.0f * gradRgba[4 * pix + 3];
                const float hitTB = hitT[pix];
                const float hitTG = gradHitT[pix];
                float nB[3], nG[3];
                for (int k = 0; k < 3; ++k) {
                    nB[k] = val(normal, 3 * pix + k);
                    nG[k] = normal != nullptr ? val(gradNormal, 3 * pix + k) : 0.0f;
                }
                const float wd2B = val(depthVar, pix);
                const float wd2G = depthVar != nullptr ? val(gradDepthVar, pix) : 0.0f;
                const float extG = val(gradExtent, pix), invDG = val(gradInvD, pix), invD2G = val(gradInvD2, pix);
                const float dscale = pinhole ? rayD[3 * pix + 2] : 1.0f;
                // exact 0.5-crossing depth t* and its gradient scale g = -(dL/dt*) / Odot*
                // (rayPayloadBackward.cuh:122-128)
                float crossG = 0.0f, crossT = 0.0f;
                if (quant != nullptr && gradQuant != nullptr) {
                    const float t = quant[10 * pix + 8], rate = quant[10 * pix + 9], dLdt = gradQuant[10 * pix + 8];
                    if (std::fabs(rate) > 1e-8f && t > 0.0f) {
                        crossG = -dLdt / rate;
                        crossT = t;
                    }
                }
                float T = 1.0f, depth = 0.0f, wd2 = 0.0f;
                float nRun[3] = {0.0f, 0.0f, 0.0f};
                float radiance[3] = {0.0f, 0.0f, 0.0f};
                bool alive = true;
                traverse(sc, uint32_t(tile), ray, alive, [&](const Hit& hh) {
                    const Particle P = load_particle(particles + 32 * size_t(hh.idx));
                    const HalfRay h = half_ray(ray, P);
                    if (h.valid) {
                        const float grayDist = fdot(h.p, h.p);
                        const float gres = gf::gf_expf(-0.5f * grayDist);
                        const float galphaU = gres * P.density;
                        const float galpha = gf::min_f(kMaxAlpha, galphaU);
                        if (gres > kMinKernelResponse && galpha > kAlphaThreshold) {
                            const float gdist = h.tau;
                            const float weight = galpha * T;
                            const float nextT = (1.0f - galpha) * T;
                            const bool tail = nextT <= kMinTransmittance;
                            depth = depth + gdist * weight;
                            const float residualHitT = gf::max_f(tail ? 0.0f : (hitTB - depth) / nextT, 0.0f);
                            const float galphaRayHitGrd = (gdist - residualHitT) * T * hitTG;
                            const float residualTrm = galpha < 0.999999f ? TB / (1.0f - galpha) : T;
                            const float galphaRayDnsGrd = residualTrm * -TG;
                            const float* c = rgb + 3 * size_t(hh.idx);
                            float col[3], resid[3];
                            for (int k = 0; k < 3; ++k) {
                                col[k] = gf::max_f(c[k], 0.0f);
                                radiance[k] = fmaf_rn(col[k], weight, radiance[k]);
                            }
                            for (int k = 0; k < 3; ++k)
                                resid[k] = gf::max_f(tail ? 0.0f : (featB[k] - radiance[k]) / nextT, 0.0f);
                            float comp = galphaRayHitGrd + galphaRayDnsGrd;
                            for (int k = 0; k < 3; ++k) comp += T * (col[k] - resid[k]) * featG[k];
                            float tauGrad = weight * hitTG;
                            // depth moment
                            const float gsq = gdist * gdist;
                            wd2 = fmaf_rn(weight * gdist, gdist, wd2);
                            const float residualWD2 = gf::max_f(tail ? 0.0f : (wd2B - wd2) / nextT, 0.0f);
                            comp += (gsq - residualWD2) * T * wd2G;
                            tauGrad += 2.0f * gdist * weight * wd2G;
                            // inverse-depth moments
                            const float dd = gdist * dscale;
                            if (dd > kParticleMinSensorZ) {
                                tauGrad += (-weight / (dscale * gdist * gdist)) * invDG;
                                tauGrad += (-2.0f * weight / ((dscale * dscale) * gdist * gdist * gdist)) * invD2G;
                            }
                            // normal
                            const float len = std::sqrt(h.denom);
                            const float3_ grd = f3(h.grdu.x / len, h.grdu.y / len, h.grdu.z / len);
                            const float* M = P.Binv;
                            const float3_ nu = f3(fmaf_rn(M[6], grd.z, fmaf_rn(M[3], grd.y, M[0] * grd.x)),
                                                  fmaf_rn(M[7], grd.z, fmaf_rn(M[4], grd.y, M[1] * grd.x)),
                                                  fmaf_rn(M[8], grd.z, fmaf_rn(M[5], grd.y, M[2] * grd.x)));
                            const float inv = -1.0f / std::sqrt(fdot(nu, nu));
                            const float n[3] = {inv * nu.x, inv * nu.y, inv * nu.z};
                            for (int k = 0; k < 3; ++k) nRun[k] = fmaf_rn(weight, n[k], nRun[k]);
                            float resN[3];
                            for (int k = 0; k < 3; ++k) resN[k] = tail ? 0.0f : (nB[k] - nRun[k]) / nextT;
                            comp += T * ((n[0] - resN[0]) * nG[0] + (n[1] - resN[1]) * nG[1] + (n[2] - resN[2]) * nG[2]);
                            const float3_ nuGrd = normalize_vjp(nu, f3(-weight * nG[0], -weight * nG[1], -weight * nG[2]));
                            const float gdv[3] = {grd.x, grd.y, grd.z};
                            const float ngv[3] = {nuGrd.x, nuGrd.y, nuGrd.z};
                            float gBinvN[9];
                            for (int i = 0; i < 3; ++i)
                                for (int j = 0; j < 3; ++j) gBinvN[3 * i + j] = gdv[i] * ngv[j];
                            const float3_ grdGrd = fmatvec(M, nuGrd);
                            const float3_ grduGeo = normalize_vjp(h.grdu, grdGrd);
                            // extent
                            const float3_ rd = rotate_transpose(P.quat, ray.d);
                            const float3_ sd = f3(P.scale[0] * rd.x, P.scale[1] * rd.y, P.scale[2] * rd.z);
                            const float sigma = std::sqrt(fdot(sd, sd) + 1e-18f);
                            const float nGe = (weight * extG) / sigma;
                            const float3_ rdGrd = f3(nGe * (P.scale[0] * P.scale[0] * rd.x),
                                                     nGe * (P.scale[1] * P.scale[1] * rd.y),
                                                     nGe * (P.scale[2] * P.scale[2] * rd.z));
                            float gq[4];
                            rotate_transpose_vjp(P.quat, ray.d, rdGrd, gq);
                            float* gs = accS.data() + 8 * size_t(hh.idx);
                            for (int k = 0; k < 4; ++k) gs[k] += gq[k];
                            gs[4] += nGe * (P.scale[0] * rd.x * rd.x);
                            gs[5] += nGe * (P.scale[1] * rd.y * rd.y);
                            gs[6] += nGe * (P.scale[2] * rd.z * rd.z);
                            // the crossing depth by the implicit function theorem
                            // (gaussianParticles.cuh:934-986): earlier hits through their
                            // peak alpha, the crossing hit through its alpha at t*
                            float crossDensity = 0.0f;
                            float3_ groCross = f3(0.0f, 0.0f, 0.0f), grduCross = f3(0.0f, 0.0f, 0.0f);
                            if (crossG != 0.0f && T > 0.5f) {
                                if (nextT > 0.5f) {
                                    comp += crossG * gf::min_f(0.5f / gf::max_f(1.0f - galpha, 1.0f - kMaxAlpha), 1.0f);
                                } else {
                                    const float ts = crossT;
                                    const float AA = fdot(h.grdu, h.grdu), BB = 2.0f * fdot(h.gro, h.grdu),
                                                CC = fdot(h.gro, h.gro);
                                    const float gdc = gf::max_f(AA * ts * ts + BB * ts + CC, 0.0f);
                                    const float grc = gf::gf_expf(-0.5f * gdc);
                                    const float aU = grc * P.density;
                                    const float aC = gf::min_f(kMaxAlpha, aU);
                                    const float dLda =
                                        crossG * gf::min_f(0.5f / gf::max_f(1.0f - aC, 1.0f - kMaxAlpha), 1.0f);
                                    const float capC = aU < kMaxAlpha ? 1.0f : 0.0f;
                                    crossDensity = capC * dLda * grc;
                                    const float dgd = capC * dLda * P.density * (-0.5f * grc);
                                    grduCross = f3(dgd * 2.0f * (ts * ts * h.grdu.x + ts * h.gro.x),
                                                   dgd * 2.0f * (ts * ts * h.grdu.y + ts * h.gro.y),
                                                   dgd * 2.0f * (ts * ts * h.grdu.z + ts * h.gro.z));
                                    groCross = f3(dgd * 2.0f * (ts * h.grdu.x + h.gro.x),
                                                  dgd * 2.0f * (ts * h.grdu.y + h.gro.y),
                                                  dgd * 2.0f * (ts * h.grdu.z + h.gro.z));
                                }
                            }
                            // alpha, response, closest point
                            const float gU = (galphaU < kMaxAlpha ? 1.0f : 0.0f) * comp;
                            float* g = acc.data() + 16 * size_t(hh.idx);
                            g[3] += gres * gU + crossDensity;
                            const float gresGrd = P.density * gU;
                            const float grayDistGrd = -0.5f * gres * gresGrd;
                            const float3_ pointGrad = scale(2.0f * grayDistGrd, h.p);
                            float3_ groGrd = pointGrad;
                            float3_ grduGrd = scale(h.tau, pointGrad);
                            const float totalTauGrad = tauGrad + dot(pointGrad, h.grdu);
                            if (h.interior) {
                                const float3_ tauOriginGrad = scale(-1.0f / h.denom, h.grdu);
                                const float3_ tauDirectionGrad =
                                    add(scale(-1.0f / h.denom, h.gro), scale((2.0f * h.num) / (h.denom * h.denom), h.grdu));
                                groGrd = add(groGrd, scale(totalTauGrad, tauOriginGrad));
                                grduGrd = add(grduGrd, scale(totalTauGrad, tauDirectionGrad));
                            }
                            groGrd = add(groGrd, groCross);
                            grduGrd = add(grduGrd, grduCross);
                            const float px = -(groGrd.x * M[0] + groGrd.y * M[3] + groGrd.z * M[6]);
                            const float py = -(groGrd.x * M[1] + groGrd.y * M[4] + groGrd.z * M[7]);
                            const float pz = -(groGrd.x * M[2] + groGrd.y * M[5] + groGrd.z * M[8]);
                            g[0] += px;
                            g[1] += py;
                            g[2] += pz;
                            abs_grad_hit(absPartial[size_t(tid)], N, hh.idx, px, py, pz);
                            const float3_ gposc = sub(ray.o, P.pos);
                            const float gr[3] = {groGrd.x, groGrd.y, groGrd.z};
                            const float gd[3] = {grduGrd.x, grduGrd.y, grduGrd.z};
                            const float gn[3] = {grduGeo.x, grduGeo.y, grduGeo.z};
                            for (int r = 0; r < 3; ++r) {
                                g[4 + 3 * r + 0] += gr[r] * gposc.x + gd[r] * ray.d.x + (gBinvN[3 * r + 0] + gn[r] * ray.d.x);
                                g[4 + 3 * r + 1] += gr[r] * gposc.y + gd[r] * ray.d.y + (gBinvN[3 * r + 1] + gn[r] * ray.d.y);
                                g[4 + 3 * r + 2] += gr[r] * gposc.z + gd[r] * ray.d.z + (gBinvN[3 * r + 2] + gn[r] * ray.d.z);
                            }
                            for (int k = 0; k < 3; ++k) g[13 + k] += featG[k] * weight;
                            T = nextT;
                        }
                    }
                    if (T < kMinTransmittance) alive = false;
                });
            }
        }
    });
    std::memset(gradRecord, 0, sizeof(float) * size_t(N) * 16);
    std::memset(gradShape, 0, sizeof(float) * size_t(N) * 8);
    for (int t = 0; t < nthreads; ++t) {
        if (!partial[size_t(t)].empty()) {
            const float* a = partial[size_t(t)].data();
            for (size_t i = 0; i < size_t(N) * 16; ++i) gradRecord[i] += a[i];
        }
        if (!partialShape[size_t(t)].empty()) {
            const float* a = partialShape[size_t(t)].data();
            for (size_t i = 0; i < size_t(N) * 8; ++i) gradShape[i] += a[i];
        }
    }
    abs_grad_reduce(absPartial, N);
    return 0;
}

// Projection backward (projectBackward, gutRenderer.cuh:643 ->
// gutProjector.cuh:1171-1222; radianceFromSpHBwd, gaussianParticles.cuh:234-310;
// incidentDirectionFromBuffer VJP): turns the per-particle record gradient into
// the reference's [N,32] density gradient and [N, 3*shCoeffs] SH gradient.
int oracle_project_backward(const OraclePose* pose, int N, const float* particles, const float* sh, int shCoeffs,
                            int shDegree, const uint32_t* counts, const float* gradRecord, float* gradParticles,
                            float* gradSh) {
    std::memset(gradParticles, 0, sizeof(float) * size_t(N) * 32);
    std::memset(gradSh, 0, sizeof(float) * size_t(N) * 3 * shCoeffs);
    parallel_for(0, N, 4096, [&](int i, int) {
        const float* g = gradRecord + 16 * size_t(i);
        float* gp = gradParticles + 32 * size_t(i);
        gp[0] = g[0]; gp[1] = g[1]; gp[2] = g[2];
        gp[3] = g[3];
        for (int k = 0; k < 9; ++k) gp[21 + k] = g[4 + k];
        if (counts[i] == 0u) return;
        const Particle P = load_particle(particles + 32 * size_t(i));
        float dist;
        const float3_ dir = incident_direction(P.pos, *pose, dist);
        float basis[16], bx[16], by[16], bz[16];
        sh_basis(shDegree, dir, basis);
        sh_basis_grad(shDegree, dir, bx, by, bz);
        const int nb = shDegree >= 3 ? 16 : (shDegree == 2 ? 9 : (shDegree == 1 ? 4 : 1));
        const float* c = sh + size_t(i) * 3 * shCoeffs;
        float* gs = gradSh + size_t(i) * 3 * shCoeffs;
        float3_ dirGrad = f3(0, 0, 0);
        for (int ch = 0; ch < 3; ++ch) {
            float acc = basis[0] * c[ch];
            for (int k = 1; k < nb && k < shCoeffs; ++k) acc = fmaf_rn(basis[k], c[3 * k + ch], acc);
            const float masked = (acc + 0.5f) > 0.0f ? g[13 + ch] : 0.0f;
            for (int k = 0; k < nb && k < shCoeffs; ++k) gs[3 * k + ch] = basis[k] * masked;
            for (int k = 1; k < nb && k < shCoeffs; ++k) {
                dirGrad.x += bx[k] * c[3 * k + ch] * masked;
                dirGrad.y += by[k] * c[3 * k + ch] * masked;
                dirGrad.z += bz[k] * c[3 * k + ch] * masked;
            }
        }
        // d(v/|v|)/dv^T g = (g - n (n.g)) / |v|
        const float ndg = dot(dir, dirGrad);
        gp[0] += (dirGrad.x - dir.x * ndg) / dist;
        gp[1] += (dirGrad.y - dir.y * ndg) / dist;
        gp[2] += (dirGrad.z - dir.z * ndg) / dist;
    });
    return 0;
}

// ------------------------------------------------------------------ SOF opacity field
// gutRenderer.cuh:297-430 with gaussianParticles.cuh:496-588: the opacity of
// the intrinsic Gaussians (slots 4-11: rotation, physical scale, peak
// opacity) replayed over every candidate of the tile, in list order, on
// [tmin, min(rho*, tmax)] (rho*: the exact 0.5-crossing depth of the
// quantile channel; the whole ray without one).
namespace sofop {

struct Intrinsic {
    float3_ mu;
    float rho;
    float3_ r0, r1, r2;  // rows of R^T
    float is[3];         // 1 / s
};

Intrinsic intrinsic(const float* row) {
    Intrinsic g;
    g.mu = f3(row[0], row[1], row[2]);
    g.rho = row[11];
    const float r = row[4], x = row[5], y = row[6], z = row[7];
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z, rx = r * x, ry = r * y,
                rz = r * z;
    g.r0 = f3(1.0f - 2.0f * (yy + zz), 2.0f * (xy + rz), 2.0f * (xz - ry));
    g.r1 = f3(2.0f * (xy - rz), 1.0f - 2.0f * (xx + zz), 2.0f * (yz + rx));
    g.r2 = f3(2.0f * (xz + ry), 2.0f * (yz - rx), 1.0f - 2.0f * (xx + yy));
    for (int k = 0; k < 3; ++k) g.is[k] = 1.0f / row[8 + k];
    return g;
}

float3_ local(const Intrinsic& g, float3_ v) {
    return f3(fdot(g.r0, v) * g.is[0], fdot(g.r1, v) * g.is[1], fdot(g.r2, v) * g.is[2]);
}

struct Sample {
    bool accepted = false;
    float alpha = 0.0f, response = 0.0f, depth = 0.0f;
    float3_ p{};
};

Sample sample(const Intrinsic& g, const Ray& ray, float tmin, float tmax) {
    Sample s;
    if (!(tmax >= tmin)) return s;
    const float3_ gro = local(g, sub(ray.o, g.mu));
    const float3_ grdu = local(g, ray.d);
    float tau;
    if (tmax == tmin) {
        tau = tmin;
    } else {
        const float denom = fdot(grdu, grdu);
        if (!(denom > 0.0f && gf::isfinite_f(denom) && gf::isfinite_f(tmin))) return s;
        const float tauLine = -fdot(gro, grdu) / denom;
        tau = gf::min_f(gf::max_f(tauLine, tmin), tmax);
    }
    s.depth = tau;
    s.p = f3(fmaf_rn(tau, grdu.x, gro.x), fmaf_rn(tau, grdu.y, gro.y), fmaf_rn(tau, grdu.z, gro.z));
    const float arg = gf::max_f(fdot(s.p, s.p), 0.0f);
    s.response = gf::gf_expf(-0.5f * arg);
    s.alpha = gf::min_f(kMaxAlpha, s.response * g.rho);
    s.accepted = s.response > kMinKernelResponse && s.alpha > kAlphaThreshold;
    return s;
}

float replay_end(const float* quant, size_t pix, const Ray& ray) {
    const float rho = quant[10 * pix + 8];
    return (rho > 0.0f && gf::isfinite_f(rho)) ? gf::min_f(rho, ray.tmax) : ray.tmax;
}

}  // namespace sofop

// opacity[P] (zero for invalid rays and pixels of dropped tiles).
int oracle_sof_opacity_forward(const OracleCamera* cam, const OraclePose* pose, const float* particles,
                               const float* rayO, const float* rayD, const uint8_t* mask, const uint32_t* ranges,
                               const uint32_t* sortedIds, const float* quant, float* opacity) {
    const int W = cam->width, H = cam->height;
    const int gx = (W + kTile - 1) / kTile, gy = (H + kTile - 1) / kTile;
    parallel_for(0, gx * gy, 1, [&](int tile, int) {
        if (mask[tile] == 0u) return;
        const int tx = tile % gx, ty = tile / gx;
        for (int py = ty * kTile; py < std::min(H, (ty + 1) * kTile); ++py)
            for (int px = tx * kTile; px < std::min(W, (tx + 1) * kTile); ++px) {
                const size_t pix = size_t(px) + size_t(W) * py;
                const Ray ray = make_ray(*pose, rayO + 3 * pix, rayD + 3 * pix);
                if (!ray.valid) continue;
                const float end = sofop::replay_end(quant, pix, ray);
                if (!(end >= ray.tmin)) {
                    opacity[pix] = 0.0f;
                    continue;
                }
                float product = 1.0f;
                for (uint32_t s = ranges[2 * tile]; s < ranges[2 * tile + 1]; ++s) {
                    const sofop::Sample smp =
                        sofop::sample(sofop::intrinsic(particles + 32 * size_t(sortedIds[s])), ray, ray.tmin, end);
                    if (smp.accepted) product = product * (1.0f - smp.alpha);
                }
                opacity[pix] = 1.0f - product;
            }
    });
    return 0;
}

// Gradient of the opacity field: grad[N*16] = position xyz, intrinsic
// density | quaternion w x y z | scale xyz, 0 | 0 (accumulated in double).
int oracle_sof_opacity_backward(const OracleCamera* cam, const OraclePose* pose, int N, const float* particles,
                                const float* rayO, const float* rayD, const uint8_t* mask, const uint32_t* ranges,
                                const uint32_t* sortedIds, const float* quant, const float* opacity,
                                const float* gradOpacity, float* grad) {
    const int W = cam->width, H = cam->height;
    const int gx = (W + kTile - 1) / kTile, gy = (H + kTile - 1) / kTile;
    std::vector<std::vector<double>> partial(static_cast<size_t>(worker_count()));
    parallel_for(0, gx * gy, 1, [&](int tile, int worker) {
        std::vector<double>& acc = partial[size_t(worker)];
        if (acc.empty()) acc.assign(size_t(N) * 16, 0.0);
        if (mask[tile] == 0u) return;
        const int tx = tile % gx, ty = tile / gx;
        for (int py = ty * kTile; py < std::min(H, (ty + 1) * kTile); ++py)
            for (int px = tx * kTile; px < std::min(W, (tx + 1) * kTile); ++px) {
                const size_t pix = size_t(px) + size_t(W) * py;
                const Ray ray = make_ray(*pose, rayO + 3 * pix, rayD + 3 * pix);
                if (!ray.valid) continue;
                const float end = sofop::replay_end(quant, pix, ray);
                const float upstream = gradOpacity[pix];
                if (!(end >= ray.tmin) || upstream == 0.0f) continue;
                const float full = gf::min_f(gf::max_f(1.0f - opacity[pix], 0.0f), 1.0f);
                for (uint32_t s = ranges[2 * tile]; s < ranges[2 * tile + 1]; ++s) {
                    const uint32_t idx = sortedIds[s];
                    const float* row = particles + 32 * size_t(idx);
                    const sofop::Intrinsic g = sofop::intrinsic(row);
                    const sofop::Sample smp = sofop::sample(g, ray, ray.tmin, end);
                    if (!smp.accepted) continue;
                    const float exclusive =
                        gf::min_f(gf::max_f(full / gf::max_f(1.0f - smp.alpha, 1.0f - kMaxAlpha), 0.0f), 1.0f);
                    const float dAlpha = upstream * exclusive;
                    const float cap = smp.response * g.rho < kMaxAlpha ? 1.0f : 0.0f;
                    const float gDensity = cap * dAlpha * smp.response;
                    const float dArg = cap * dAlpha * g.rho * (-0.5f * smp.response);
                    const float lpg[3] = {2.0f * dArg * smp.p.x, 2.0f * dArg * smp.p.y, 2.0f * dArg * smp.p.z};
                    const float rpg[3] = {g.is[0] * lpg[0], g.is[1] * lpg[1], g.is[2] * lpg[2]};
                    const float3_ w = f3(fmaf_rn(smp.depth, ray.d.x, ray.o.x) - g.mu.x,
                                         fmaf_rn(smp.depth, ray.d.y, ray.o.y) - g.mu.y,
                                         fmaf_rn(smp.depth, ray.d.z, ray.o.z) - g.mu.z);
                    const float rot[3] = {fdot(g.r0, w), fdot(g.r1, w), fdot(g.r2, w)};
                    double* a = acc.data() + 16 * size_t(idx);
                    a[0] += -(double(g.r0.x) * rpg[0] + double(g.r1.x) * rpg[1] + double(g.r2.x) * rpg[2]);
                    a[1] += -(double(g.r0.y) * rpg[0] + double(g.r1.y) * rpg[1] + double(g.r2.y) * rpg[2]);
                    a[2] += -(double(g.r0.z) * rpg[0] + double(g.r1.z) * rpg[1] + double(g.r2.z) * rpg[2]);
                    a[3] += gDensity;
                    float gq[4];
                    rotate_transpose_vjp(row + 4, w, f3(rpg[0], rpg[1], rpg[2]), gq);
                    for (int k = 0; k < 4; ++k) a[4 + k] += gq[k];
                    for (int k = 0; k < 3; ++k) a[8 + k] += -double(rot[k]) * g.is[k] * g.is[k] * lpg[k];
                }
            }
    });
    for (size_t i = 0; i < size_t(N) * 16; ++i) {
        double v = 0.0;
        for (const auto& part : partial)
            if (!part.empty()) v += part[i];
        grad[i] = float(v);
    }
    return 0;
}

// Completeness of a binning: for every valid ray of a retained tile, the
// particles whose hit test passes on that ray (by brute force over all N)
// but that are not in the tile's candidate list.  Returns their number; the
// first misses go to missPixel / missParticle (up to maxMisses).
int64_t oracle_admission_misses(const OracleCamera* cam, const OraclePose* pose, int N, const float* particles,
                                const float* rayO, const float* rayD, const uint8_t* mask, const uint32_t* ranges,
                                const uint32_t* sortedIds, int64_t maxMisses, int64_t* missPixel,
                                uint32_t* missParticle) {
    const int W = cam->width, H = cam->height;
    const int gx = (W + kTile - 1) / kTile, gy = (H + kTile - 1) / kTile;
    std::atomic<int64_t> misses(0);
    parallel_for(0, gx * gy, 1, [&](int tile, int) {
        if (mask[tile] == 0u) return;
        std::vector<uint8_t> listed(size_t(N), 0u);
        for (uint32_t s = ranges[2 * tile]; s < ranges[2 * tile + 1]; ++s) listed[sortedIds[s]] = 1u;
        const int tx = tile % gx, ty = tile / gx;
        for (int py = ty * kTile; py < std::min(H, (ty + 1) * kTile); ++py)
            for (int px = tx * kTile; px < std::min(W, (tx + 1) * kTile); ++px) {
                const size_t pix = size_t(px) + size_t(W) * py;
                const Ray ray = make_ray(*pose, rayO + 3 * pix, rayD + 3 * pix);
                if (!ray.valid) continue;
                for (int i = 0; i < N; ++i) {
                    if (listed[size_t(i)]) continue;
                    const Particle P = load_particle(particles + 32 * size_t(i));
                    float alpha, hitT, resp;
                    HalfRay hr;
                    if (hit_test(ray, P, alpha, hitT, resp, hr) && hitT >= ray.tmin && hitT <= ray.tmax) {
                        const int64_t k = misses.fetch_add(1);
                        if (k < maxMisses) {
                            missPixel[k] = int64_t(pix);
                            missParticle[k] = uint32_t(i);
                        }
                    }
                }
            }
    });
    return misses.load();
}

// The SOF hierarchy's feed sequences of one tile: for local pixel p,
// feed[offset[p] .. offset[p+1]) are the sorted positions fed to its HEAD in
// order (offset has 257 entries).  Returns the total, or -1 when it exceeds
// capacity.
int64_t oracle_sof_feeds(const OracleCamera* cam, const OraclePose* pose, int N, const float* particles,
                         const float* rayO, const float* rayD, const uint32_t* ranges, const uint32_t* sortedIds,
                         int tile, uint32_t* offset, uint32_t* feed, int64_t capacity) {
    Scene sc{cam, pose, N, particles, nullptr, rayO, rayD, nullptr, ranges, sortedIds, kSofHierarchy};
    const auto feeds = sof_feeds(sc, uint32_t(tile));
    int64_t total = 0;
    for (int p = 0; p < 256; ++p) {
        offset[p] = uint32_t(total);
        total += int64_t(feeds[size_t(p)].size());
    }
    offset[256] = uint32_t(total);
    if (total > capacity) return -1;
    int64_t k = 0;
    for (int p = 0; p < 256; ++p)
        for (const uint32_t v : feeds[size_t(p)]) feed[k++] = v;
    return total;
}

// Visibility of gutRenderer.cu:204-209: 1 (as an int bit pattern) when the
// particle has at least one admitted tile.
int oracle_visibility(int N, const uint32_t* counts, uint32_t* visibility) {
    for (int i = 0; i < N; ++i) visibility[i] = counts[i] ? 1u : 0u;
    return 0;
}

int oracle_num_threads(void) { return worker_count(); }

// ------------------------------------------------------------------ mesh opacity field
// One camera of the matched camera-min opacity field (gofish/mesh/field.py:4-11;
// opacityField.cuh:699-745 preprocessPoints, :775-829 integratePoints,
// :172-185 fixed8ResponseAlphaUpdate).  The reference's candidate admission
// is complete (native UT union certified support cap), so its product equals
// the product over every particle whose hit test passes on the segment
// [0, t_query], in ascending particle id; this restatement evaluates exactly
// that by brute force.  For each query point: opacity[q] = 1 - prod(1 - alpha)
// and observed[q] = 1 when the point projects into the raster, onto an
// unmasked pixel, at a positive finite range; otherwise observed[q] = 0.
int oracle_field_camera(const OracleCamera* cam, const OraclePose* pose, int N, const float* particles,
                        const float* rayO, const uint8_t* pixelMask, int Q, const float* points, float* opacity,
                        uint8_t* observed) {
    const int W = cam->width, H = cam->height;
    parallel_for(0, Q, 256, [&](int q, int) {
        opacity[q] = 0.0f;
        observed[q] = 0u;
        const float3_ x = f3(points[3 * size_t(q)], points[3 * size_t(q) + 1], points[3 * size_t(q) + 2]);
        float2_ pr;
        if (!project_world(*cam, *pose, x, pr)) return;
        // requireRasterBounds with zero tolerance (cameraProjections.cuh:69-73)
        if (!(pr.x >= 0.0f && pr.y >= 0.0f && pr.x < float(W) && pr.y < float(H))) return;
        const int px = int(floorf(pr.x)), py = int(floorf(pr.y));
        if (px < 0 || py < 0 || px >= W || py >= H) return;
        const size_t pix = size_t(px) + size_t(W) * size_t(py);
        if (pixelMask != nullptr && pixelMask[pix] == 0u) return;
        const float3_ os = f3(rayO[3 * pix], rayO[3 * pix + 1], rayO[3 * pix + 2]);
        const float3_ o = add(matvec(pose->Rinv, os), f3(pose->c[0], pose->c[1], pose->c[2]));
        const float3_ delta = sub(x, o);
        const float range = sqrtf(dot(delta, delta));
        if (!(range > 0.0f) || !gf::isfinite_f(range)) return;
        Ray ray;
        ray.o = o;
        ray.d = f3(delta.x / range, delta.y / range, delta.z / range);
        ray.tmin = 0.0f;
        ray.tmax = range;
        ray.valid = true;
        float T = 1.0f;
        for (int i = 0; i < N; ++i) {
            const Particle P = load_particle(particles + 32 * size_t(i));
            float alpha, hitT, resp;
            HalfRay h;
            if (hit_test(ray, P, alpha, hitT, resp, h)) T = T * (1.0f - alpha);
        }
        opacity[q] = 1.0f - T;
        observed[q] = 1u;
    });
    return 0;
}

// The same field with a conservative spatial index, for point counts the
// brute force cannot reach (millions of points over millions of particles).
// A particle can pass the hit test on a segment only if the segment comes
// within R of its mean: with M = B^-1 (the stored float inverse factor) the
// world point w of the clamped closest point satisfies w - mu = M^-1 p, and
// the hit needs |p| < 3 (response above 0.0113 needs |p|^2 < 8.97) for the
// float p, which differs from the exact one by at most 8u |M|_F (|o - mu| +
// tmax) (u = 2^-24); so R = (3 + 8u |M|_F 2D) |M^-1|_F (1 + 1e-3) with D
// bounding |o - mu| and tmax over the scene, |M^-1|_F from the double-precision
// inverse of M.  Particles with density <= 1/255 never pass and are left out.
// A bounding volume hierarchy over the spheres (median splits, leaves of at
// most 4) yields every particle whose sphere meets the segment; they are
// tested in ascending id, exactly as the brute force multiplies them, and the
// walk stops once 1 - T rounds to 1 (later factors only shrink T, and the
// rounding of 1 - T is monotone, so the result is the full product's).
namespace fieldbvh {

struct Node {
    double lo[3], hi[3];
    int32_t left, right;  // children, or -1 for a leaf
    int32_t begin, end;   // leaf: prims[begin, end)
};

struct Index {
    std::vector<Node> nodes;
    std::vector<int32_t> prims;        // particle ids, permuted by the build
    std::vector<double> centre, radius;  // [N*3], [N] (radius < 0: never hit)
    const float* particles = nullptr;
    int n = 0;
};

double inverse_frobenius(const float* Mf) {
    double M[9];
    for (int i = 0; i < 9; ++i) M[i] = double(Mf[i]);
    const double c00 = M[4] * M[8] - M[5] * M[7], c01 = M[5] * M[6] - M[3] * M[8], c02 = M[3] * M[7] - M[4] * M[6];
    const double det = M[0] * c00 + M[1] * c01 + M[2] * c02;
    if (!(std::fabs(det) > 0.0) || !std::isfinite(det)) return INFINITY;
    const double inv[9] = {c00, M[2] * M[7] - M[1] * M[8], M[1] * M[5] - M[2] * M[4],
                           c01, M[0] * M[8] - M[2] * M[6], M[2] * M[3] - M[0] * M[5],
                           c02, M[1] * M[6] - M[0] * M[7], M[0] * M[4] - M[1] * M[3]};
    double f = 0.0;
    for (int i = 0; i < 9; ++i) f += (inv[i] / det) * (inv[i] / det);
    return std::sqrt(f);
}

int build_node(Index& ix, int begin, int end) {
    Node nd;
    for (int a = 0; a < 3; ++a) {
        nd.lo[a] = INFINITY;
        nd.hi[a] = -INFINITY;
    }
    double clo[3] = {INFINITY, INFINITY, INFINITY}, chi[3] = {-INFINITY, -INFINITY, -INFINITY};
    for (int k = begin; k < end; ++k) {
        const int i = ix.prims[size_t(k)];
        for (int a = 0; a < 3; ++a) {
            const double c = ix.centre[3 * size_t(i) + a], r = ix.radius[size_t(i)];
            nd.lo[a] = std::min(nd.lo[a], c - r);
            nd.hi[a] = std::max(nd.hi[a], c + r);
            clo[a] = std::min(clo[a], c);
            chi[a] = std::max(chi[a], c);
        }
    }
    const int id = int(ix.nodes.size());
    ix.nodes.push_back(nd);
    if (end - begin <= 4) {
        ix.nodes[size_t(id)].left = ix.nodes[size_t(id)].right = -1;
        ix.nodes[size_t(id)].begin = begin;
        ix.nodes[size_t(id)].end = end;
        return id;
    }
    int axis = 0;
    for (int a = 1; a < 3; ++a)
        if (chi[a] - clo[a] > chi[axis] - clo[axis]) axis = a;
    const int mid = begin + (end - begin) / 2;
    std::nth_element(ix.prims.begin() + begin, ix.prims.begin() + mid, ix.prims.begin() + end, [&](int32_t x, int32_t y) {
        const double cx = ix.centre[3 * size_t(x) + axis], cy = ix.centre[3 * size_t(y) + axis];
        return cx < cy || (cx == cy && x < y);
    });
    const int l = build_node(ix, begin, mid);
    const int r = build_node(ix, mid, end);
    ix.nodes[size_t(id)].left = l;
    ix.nodes[size_t(id)].right = r;
    ix.nodes[size_t(id)].begin = ix.nodes[size_t(id)].end = 0;
    return id;
}

// Segment a + t (b - a), t in [0, 1], against an axis-aligned box (slabs, in double).
bool segment_meets_box(const double a[3], const double b[3], const double lo[3], const double hi[3]) {
    double t0 = 0.0, t1 = 1.0;
    for (int k = 0; k < 3; ++k) {
        const double d = b[k] - a[k];
        if (d == 0.0) {
            if (a[k] < lo[k] || a[k] > hi[k]) return false;
            continue;
        }
        double ta = (lo[k] - a[k]) / d, tb = (hi[k] - a[k]) / d;
        if (ta > tb) std::swap(ta, tb);
        t0 = std::max(t0, ta);
        t1 = std::min(t1, tb);
        if (t0 > t1) return false;
    }
    return true;
}

bool segment_meets_sphere(const double a[3], const double b[3], const double c[3], double r) {
    double ab[3], ac[3];
    double ab2 = 0.0, t = 0.0;
    for (int k = 0; k < 3; ++k) {
        ab[k] = b[k] - a[k];
        ac[k] = c[k] - a[k];
        ab2 += ab[k] * ab[k];
        t += ac[k] * ab[k];
    }
    t = ab2 > 0.0 ? std::min(1.0, std::max(0.0, t / ab2)) : 0.0;
    double d2 = 0.0;
    for (int k = 0; k < 3; ++k) {
        const double e = a[k] + t * ab[k] - c[k];
        d2 += e * e;
    }
    return d2 <= r * r;
}

}  // namespace fieldbvh

// Builds the index of oracle_field_camera_indexed over N particles (rows are
// borrowed: keep them alive and unchanged until oracle_field_index_free).
// sceneBound bounds every |camera origin - mean| and every segment length.
void* oracle_field_index_build(int N, const float* particles, double sceneBound) {
    auto* ix = new fieldbvh::Index();
    ix->n = N;
    ix->particles = particles;
    ix->centre.resize(3 * size_t(N));
    ix->radius.resize(size_t(N));
    const double u = std::ldexp(1.0, -24);
    for (int i = 0; i < N; ++i) {
        const Particle P = load_particle(particles + 32 * size_t(i));
        ix->centre[3 * size_t(i)] = P.pos.x;
        ix->centre[3 * size_t(i) + 1] = P.pos.y;
        ix->centre[3 * size_t(i) + 2] = P.pos.z;
        double mf = 0.0;
        for (int k = 0; k < 9; ++k) mf += double(P.Binv[k]) * double(P.Binv[k]);
        const double inv = fieldbvh::inverse_frobenius(P.Binv);
        double r = (3.0 + 8.0 * u * std::sqrt(mf) * 2.0 * sceneBound) * inv * (1.0 + 1e-3);
        if (!(P.density > kAlphaThreshold) || !std::isfinite(r)) r = -1.0;
        ix->radius[size_t(i)] = r;
        if (r >= 0.0) ix->prims.push_back(i);
    }
    if (!ix->prims.empty()) fieldbvh::build_node(*ix, 0, int(ix->prims.size()));
    return ix;
}

void oracle_field_index_free(void* handle) { delete static_cast<fieldbvh::Index*>(handle); }

// oracle_field_camera over the particles of an index (see above); identical
// results, with particles whose sphere misses the segment skipped.
int oracle_field_camera_indexed(void* handle, const OracleCamera* cam, const OraclePose* pose, const float* rayO,
                                const uint8_t* pixelMask, int Q, const float* points, float* opacity,
                                uint8_t* observed) {
    const auto& ix = *static_cast<const fieldbvh::Index*>(handle);
    const int W = cam->width, H = cam->height;
    parallel_for(0, Q, 64, [&](int q, int) {
        opacity[q] = 0.0f;
        observed[q] = 0u;
        const float3_ x = f3(points[3 * size_t(q)], points[3 * size_t(q) + 1], points[3 * size_t(q) + 2]);
        float2_ pr;
        if (!project_world(*cam, *pose, x, pr)) return;
        if (!(pr.x >= 0.0f && pr.y >= 0.0f && pr.x < float(W) && pr.y < float(H))) return;
        const int px = int(floorf(pr.x)), py = int(floorf(pr.y));
        if (px < 0 || py < 0 || px >= W || py >= H) return;
        const size_t pix = size_t(px) + size_t(W) * size_t(py);
        if (pixelMask != nullptr && pixelMask[pix] == 0u) return;
        const float3_ os = f3(rayO[3 * pix], rayO[3 * pix + 1], rayO[3 * pix + 2]);
        const float3_ o = add(matvec(pose->Rinv, os), f3(pose->c[0], pose->c[1], pose->c[2]));
        const float3_ delta = sub(x, o);
        const float range = sqrtf(dot(delta, delta));
        if (!(range > 0.0f) || !gf::isfinite_f(range)) return;
        Ray ray;
        ray.o = o;
        ray.d = f3(delta.x / range, delta.y / range, delta.z / range);
        ray.tmin = 0.0f;
        ray.tmax = range;
        ray.valid = true;
        // the segment from o to o + range d (in double, the float ray's own end)
        const double a[3] = {o.x, o.y, o.z};
        const double b[3] = {double(o.x) + double(range) * double(ray.d.x),
                             double(o.y) + double(range) * double(ray.d.y),
                             double(o.z) + double(range) * double(ray.d.z)};
        std::vector<int32_t> cand;
        if (!ix.nodes.empty()) {
            int32_t stack[128];
            int top = 0;
            stack[top++] = 0;
            while (top > 0) {
                const fieldbvh::Node& nd = ix.nodes[size_t(stack[--top])];
                if (!fieldbvh::segment_meets_box(a, b, nd.lo, nd.hi)) continue;
                if (nd.left < 0) {
                    for (int k = nd.begin; k < nd.end; ++k) {
                        const int32_t i = ix.prims[size_t(k)];
                        if (fieldbvh::segment_meets_sphere(a, b, &ix.centre[3 * size_t(i)], ix.radius[size_t(i)]))
                            cand.push_back(i);
                    }
                } else {
                    stack[top++] = nd.left;
                    stack[top++] = nd.right;
                }
            }
        }
        std::sort(cand.begin(), cand.end());
        float T = 1.0f;
        for (const int32_t i : cand) {
            const Particle P = load_particle(ix.particles + 32 * size_t(i));
            float alpha, hitT, resp;
            HalfRay h;
            if (hit_test(ray, P, alpha, hitT, resp, h)) T = T * (1.0f - alpha);
            if (1.0f - T == 1.0f) break;
        }
        opacity[q] = 1.0f - T;
        observed[q] = 1u;
    });
    return 0;
}

// ------------------------------------------------------------------ physical-mip 3-D filter
// Finest pixel sampling rate of a point over the training frames
// (threedgrut/physical_mip_csrc/fused_refresh_cuda.cu:40-219,
// camera_local_validity.cuh; physical_mip.py:226-245).  Double precision,
// no contraction; atan2 and hypot from gf_elementary.h.
namespace mip {

constexpr double kCenterEps = 1.0e-12;  // fused_refresh_cuda.cu:22
constexpr double kNear = 0.2;           // camera_local_validity.cuh:15
constexpr int kParams = 12;

struct Projection {
    double u = 0.0, v = 0.0;
    double J[6] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0};  // d(u,v)/d(camera xyz), row-major 2x3
    bool ok = false;
};

// SIMPLE_PINHOLE / PINHOLE (model 0, 1): fused_refresh_cuda.cu:90-103.
Projection pinhole(const double* P, double x, double y, double z) {
    Projection o;
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

// SIMPLE_RADIAL / RADIAL / OPENCV / FULL_OPENCV (3..6): fused_refresh_cuda.cu:104-150.
Projection radial(int model, const double* P, double x, double y, double z) {
    Projection o;
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

// OPENCV_FISHEYE (2): fused_refresh_cuda.cu:151-183.
Projection fisheye(const double* P, double x, double y, double z, double dist, double rho, double theta) {
    Projection o;
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
    for (int k = 0; k < 3; ++k) {
        o.J[k] = fx * (dq * c * dth[k] - q * s * dph[k]);
        o.J[3 + k] = fy * (dq * s * dth[k] + q * c * dph[k]);
    }
    if (rho <= kCenterEps && z > 0.0) {
        o.u = cx;
        o.v = cy;
        for (int k = 0; k < 6; ++k) o.J[k] = 0.0;
        o.J[0] = fx / dist;
        o.J[4] = fy / dist;
    }
    o.ok = (rho > kCenterEps || z > 0.0) && dq > 0.0;
    return o;
}

}  // namespace mip

int oracle_mip_best_rate(const double* positions, int64_t N, const double* rotations, const double* centers,
                         const int32_t* frameCamera, const int32_t* frameIndex, const int64_t* frameRank,
                         int64_t F, const int32_t* cameraModel, const int32_t* cameraWidth,
                         const int32_t* cameraHeight, const double* cameraParams, const double* cameraMaxAngle,
                         const int32_t* rowLo, const int32_t* rowHi, int64_t rowStride, double* best,
                         int32_t* owner, uint8_t* observed, double* direction) {
    parallel_for(0, int(N), 64, [&](int i, int) {
        const double px = positions[3 * size_t(i)], py = positions[3 * size_t(i) + 1],
                     pz = positions[3 * size_t(i) + 2];
        double bestRate = 0.0, bx = 0.0, by = 0.0, bz = 0.0;
        int64_t bestRank = INT64_MAX;
        int32_t bestFrame = -1;
        for (int64_t f = 0; f < F; ++f) {
            const int cam = frameCamera[f];
            const int model = cameraModel[cam];
            const double* R = rotations + 9 * f;  // camera-to-world, row-major
            const double dx = px - centers[3 * f], dy = py - centers[3 * f + 1], dz = pz - centers[3 * f + 2];
            // camera coordinates: R^T (p - c)
            const double x = dx * R[0] + dy * R[3] + dz * R[6];
            const double y = dx * R[1] + dy * R[4] + dz * R[7];
            const double z = dx * R[2] + dy * R[5] + dz * R[8];
            const double dist = sqrt(x * x + y * y + z * z);
            const double rho = gf::gf_hypotd(x, y);
            const double theta = gf::gf_atan2d(rho, z);
            const double* P = cameraParams + mip::kParams * cam;
            mip::Projection pr;
            if (model == 0 || model == 1) pr = mip::pinhole(P, x, y, z);
            else if (model >= 3 && model <= 6) pr = mip::radial(model, P, x, y, z);
            else if (model == 2) pr = mip::fisheye(P, x, y, z, dist, rho, theta);
            else continue;
            const double local = model == 2 ? dist : z;
            bool ok = local > mip::kNear && pr.ok;
            for (int k = 0; k < 6; ++k) ok = ok && std::isfinite(pr.J[k]);
            ok = ok && std::isfinite(pr.u) && std::isfinite(pr.v);
            ok = ok && pr.u >= 0.0 && pr.u < cameraWidth[cam] && pr.v >= 0.0 && pr.v < cameraHeight[cam];
            if (cameraMaxAngle[cam] >= 0.0) ok = ok && theta < cameraMaxAngle[cam];
            if (ok) {
                const int64_t ix = int64_t(floor(pr.u)), iy = int64_t(floor(pr.v));
                ok = iy >= 0 && iy < cameraHeight[cam] && ix >= rowLo[cam * rowStride + iy] &&
                     ix < rowHi[cam * rowStride + iy];
            }
            if (!ok) continue;
            // world Jacobian rows J R^T
            double w0[3], w1[3];
            for (int k = 0; k < 3; ++k) {
                w0[k] = pr.J[0] * R[3 * k] + pr.J[1] * R[3 * k + 1] + pr.J[2] * R[3 * k + 2];
                w1[k] = pr.J[3] * R[3 * k] + pr.J[4] * R[3 * k + 1] + pr.J[5] * R[3 * k + 2];
            }
            const double a = w0[0] * w0[0] + w0[1] * w0[1] + w0[2] * w0[2];
            const double b = w0[0] * w1[0] + w0[1] * w1[1] + w0[2] * w1[2];
            const double c = w1[0] * w1[0] + w1[1] * w1[1] + w1[2] * w1[2];
            const double lmax = 0.5 * (a + c + gf::gf_hypotd(a - c, 2.0 * b));
            const double lmin = (a * c - b * b) / lmax;
            if (!std::isfinite(lmax) || !std::isfinite(lmin) || !(lmax > 0.0) || !(lmin > 0.0)) continue;
            const double rate = sqrt(lmin);
            const int64_t rank = frameRank[f];
            if (rate > bestRate || (rate == bestRate && rank < bestRank)) {
                bestRate = rate;
                bestRank = rank;
                bestFrame = frameIndex[f];
                bx = dx;
                by = dy;
                bz = dz;
            }
        }
        best[i] = bestRate;
        owner[i] = bestFrame;
        observed[i] = bestFrame >= 0 ? 1u : 0u;
        if (bestFrame >= 0) {
            const double n = sqrt(bx * bx + by * by + bz * bz);
            direction[3 * size_t(i)] = bx / n;
            direction[3 * size_t(i) + 1] = by / n;
            direction[3 * size_t(i) + 2] = bz / n;
        } else {
            direction[3 * size_t(i)] = direction[3 * size_t(i) + 1] = direction[3 * size_t(i) + 2] = 0.0;
        }
    });
    return 0;
}

// Exported scalar elementary functions, for the accuracy tests.
float oracle_expf(float x) { return gf::gf_expf(x); }
float oracle_logf(float x) { return gf::gf_logf(x); }
float oracle_atan2f(float y, float x) { return gf::gf_atan2f(y, x); }
double oracle_atan2d(double y, double x) { return gf::gf_atan2d(y, x); }

}  // extern "C"

extern "C" int oracle_kbuffer_order(int K, int n, const float* hitT, uint32_t* order) {
    if (K <= 0 || K > 64) return -1;
    KBuffer kb;
    kb.init(K);
    int at = 0;
    for (int i = 0; i < n; ++i) {
        const Hit h{uint32_t(i), hitT[i], 0.5f};
        if (kb.full()) order[at++] = kb.e[0].idx;
        kb.insert(h);
    }
    for (uint32_t i = 0; i < kb.n; ++i) order[at++] = kb.e[K - kb.n + i].idx;
    return 0;
}

extern "C" int oracle_ut_project(const OracleCamera* cam, const OraclePose* pose, int n, const float* particles,
                                 float* out) {
    for (int i = 0; i < n; ++i) {
        const Particle P = load_particle(particles + 32 * size_t(i));
        float2_ center{0.0f, 0.0f};
        float cov[3] = {0.0f, 0.0f, 0.0f};
        const bool valid = unscented_projection(*cam, *pose, P, center, cov);
        float* o = out + 6 * size_t(i);
        o[0] = center.x;
        o[1] = center.y;
        o[2] = cov[0];
        o[3] = cov[1];
        o[4] = cov[2];
        o[5] = valid ? 1.0f : 0.0f;
    }
    return 0;
}
