// Kernels of the mesh opacity field (reference gofish/mesh/native/include/
// 3dgut/kernels/cuda/common/opacityField.cuh and bisectionTableImpl.inl).
//
// Per camera, the work is organised around the query points rather than the
// camera's pixel footprint:
//   1. k_field_points    project each point, keep it if it lands on an
//                        unmasked pixel at a positive range, and key it by
//                        (8x8-pixel cell, pixel within the cell);
//   2. a counting sort   groups the points by that key, so that 32
//                        consecutive points (one warp) lie in one or two
//                        pixels;
//   3. k_cell_cones      bound each cell's point directions by a cone
//                        (axis, half angle) and its largest range, and
//                        k_cone_reduce builds a 4x4-fan-out quadtree of cones;
//   4. k_field_particles give each Gaussian a support sphere (radius from
//                        B^-1) seen from the camera centre as a cap, and
//                        count the cells whose cone meets the cap;
//   5. k_field_emit      writes (cell << 32 | id) keys in id order; a stable
//                        sort over the cell bits keeps ids ascending per cell;
//   6. k_field_integrate one block per 256 points of a cell: stage the cell's
//                        candidates in shared memory, cull them per warp
//                        against the warp's own direction cone, then run the
//                        exact hit test per point in ascending id and
//                        multiply T by (1 - alpha).
// Culling only skips Gaussians whose support cannot reach the segment, so
// each point multiplies exactly the alphas of the reference's complete
// admission, in the same order, with the same arithmetic as the oracle.
#pragma once

#include "gf_device.cuh"

namespace gf {
namespace field {

constexpr int kCellShift = 3;  // 8 x 8-pixel cells
constexpr int kCell = 1 << kCellShift;
constexpr int kCellPixels = kCell * kCell;
constexpr int kFan = 4;  // quadtree fan-out per axis
constexpr int kMaxLevels = 8;  // cells up to the single root cone
constexpr int kStack = 112;    // traversal stack (test-before-push: at most 15 per level + 16)
constexpr int kVisitBudget = 256;  // node tests one thread may spend on a Gaussian
constexpr int kBlock = 256;  // points per integration block and candidates per batch
constexpr uint32_t kNoKey = 0xffffffffu;
constexpr float kCapAll = -2.0f;       // cos(theta) marker: the support sphere holds the camera centre
constexpr float kCosMargin = 1e-6f;    // slack on every cosine comparison
constexpr float kAngleMargin = 2e-6f;  // slack on every cone half angle (radians)
constexpr float kWideCone = 1.5f;      // cones at least this wide (radians) meet every cap
constexpr float kPiF = 3.14159265358979f;

struct CameraArgs {
    gf_camera cam;
    Pose pose;
    const float* rayO;    // [H*W*3], sensor frame
    const uint8_t* mask;  // [H*W] or null
    uint32_t W, H;        // raster
    uint32_t gx, gy;      // cell grid
};

// Camera centre in the world from pixel 0's ray origin, with the arithmetic
// that turns every pixel's origin into the world (make_ray).
__device__ __forceinline__ V3 camera_centre(const CameraArgs& a, V3& os0) {
    os0 = v3(a.rayO[0], a.rayO[1], a.rayO[2]);
    return mat3(a.pose.Rinv, os0) + v3(a.pose.c[0], a.pose.c[1], a.pose.c[2]);
}

// Quadtree of direction cones, level 0 = cells, level n-1 = one root cone.
// Node arrays are concatenated: level l occupies [offset[l], offset[l] +
// gx[l] * gy[l]).
// A: (axis.xyz, cos phi); A.w > 1.5 marks an empty node.
// B: (sin phi, largest range, phi, number of points).
struct Levels {
    int n;
    uint32_t gx[kMaxLevels], gy[kMaxLevels], offset[kMaxLevels];
    const float4* A;
    const float4* B;
};

// Angle between two unit vectors from their chord, accurate at small angles.
__device__ __forceinline__ float unit_angle(float ax, float ay, float az, float bx, float by, float bz) {
    const float dx = ax - bx, dy = ay - by, dz = az - bz;
    const float chord = sqrtf(dx * dx + dy * dy + dz * dz);
    return 2.0f * asinf(fminf(1.0f, 0.5f * chord));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Conservative test: does the cap (unit direction v, cos/sin theta) meet the
// cone (A, B)?  Caps never exceed pi/2 (asin), and cones wider than
// kWideCone are treated as meeting everything, so theta + phi < pi.
__device__ __forceinline__ bool cap_meets_cone(float vx, float vy, float vz, float cosT, float sinT, float4 A,
                                               float4 B) {
    if (cosT < -1.5f || B.z >= kWideCone) return true;
    const float c = vx * A.x + vy * A.y + vz * A.z;
    return c >= cosT * A.w - sinT * B.x - kCosMargin;
}

// 1. Points: projection, pixel, mask, ray origin, range; key by pixel
// (reference preprocessPoints, opacityField.cuh:699-745, and
// preprocessActivePoints, bisectionTableImpl.inl:168-219).  Points of the
// bisection rounds that an earlier camera already put below 1/2 (active ==
// 0) are skipped, as the reference's compaction does.
__global__ __launch_bounds__(256) void k_field_points(CameraArgs a, const float* __restrict__ points, uint32_t Q,
                                                      const uint8_t* __restrict__ active,
                                                      uint32_t* __restrict__ pixKey, float4* __restrict__ info,
                                                      uint32_t* __restrict__ hist, uint32_t* __restrict__ err) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= Q) return;
    uint32_t key = kNoKey;
    if (active == nullptr || active[q] != 0u) {
        const V3 x = v3(points[3 * size_t(q)], points[3 * size_t(q) + 1], points[3 * size_t(q) + 2]);
        float u, v;
        if (project_world(a.cam, a.pose, x, u, v) && u >= 0.0f && v >= 0.0f && u < float(a.W) &&
            v < float(a.H)) {
            const int px = int(floorf(u)), py = int(floorf(v));
            if (px >= 0 && py >= 0 && uint32_t(px) < a.W && uint32_t(py) < a.H) {
                const size_t pix = size_t(px) + size_t(a.W) * size_t(py);
                if (a.mask == nullptr || a.mask[pix] != 0u) {
                    const V3 os = v3(a.rayO[3 * pix], a.rayO[3 * pix + 1], a.rayO[3 * pix + 2]);
                    const V3 os0 = v3(a.rayO[0], a.rayO[1], a.rayO[2]);
                    if (os.x != os0.x || os.y != os0.y || os.z != os0.z) atomicOr(err, 1u);
                    const V3 o = mat3(a.pose.Rinv, os) + v3(a.pose.c[0], a.pose.c[1], a.pose.c[2]);
                    const V3 delta = x - o;
                    const float range = sqrtf(dot3(delta, delta));
                    if (range > 0.0f && isfinite_f(range)) {
                        info[q] = make_float4(delta.x / range, delta.y / range, delta.z / range, range);
                        const uint32_t cell = (uint32_t(px) >> kCellShift) + a.gx * (uint32_t(py) >> kCellShift);
                        key = cell * kCellPixels + ((uint32_t(py) & (kCell - 1)) << kCellShift) +
                              (uint32_t(px) & (kCell - 1));
                        atomicAdd(&hist[key], 1u);
                    }
                }
            }
        }
    }
    pixKey[q] = key;
}

// 2. Counting-sort scatter: hist holds the per-key counts, start their
// exclusive scan; each point takes a slot by decrementing its count (order
// within one pixel is arbitrary: every point's result is independent of it).
__global__ __launch_bounds__(256) void k_field_scatter(const uint32_t* __restrict__ pixKey, uint32_t Q,
                                                       const uint32_t* __restrict__ start,
                                                       uint32_t* __restrict__ hist, uint32_t* __restrict__ sorted) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= Q) return;
    const uint32_t key = pixKey[q];
    if (key == kNoKey) return;
    sorted[start[key] + atomicSub(&hist[key], 1u) - 1u] = q;
}

// 3a. One warp per cell: cone of its point directions and largest range.
__global__ __launch_bounds__(256) void k_cell_cones(const uint32_t* __restrict__ start,
                                                    const uint32_t* __restrict__ sorted,
                                                    const float4* __restrict__ info, uint32_t cells,
                                                    float4* __restrict__ A, float4* __restrict__ B) {
    const uint32_t cell = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31u;
    if (cell >= cells) return;  // warp-uniform
    const uint32_t b = start[cell * kCellPixels], e = start[(cell + 1) * kCellPixels];
    if (e == b) {
        if (lane == 0) {
            A[cell] = make_float4(0.0f, 0.0f, 1.0f, 2.0f);
            B[cell] = make_float4(0.0f, -1.0f, 0.0f, 0.0f);
        }
        return;
    }
    float sx = 0.0f, sy = 0.0f, sz = 0.0f, mr = 0.0f;
    for (uint32_t i = b + lane; i < e; i += 32u) {
        const float4 d = info[sorted[i]];
        sx += d.x;
        sy += d.y;
        sz += d.z;
        mr = fmaxf(mr, d.w);
    }
    sx = warp_sum(sx);
    sy = warp_sum(sy);
    sz = warp_sum(sz);
    mr = warp_max(mr);
    const float n = sqrtf(sx * sx + sy * sy + sz * sz);
    float phi;
    float ax = 0.0f, ay = 0.0f, az = 1.0f;
    if (n > 1e-12f) {
        ax = sx / n;
        ay = sy / n;
        az = sz / n;
        float m = 0.0f;
        for (uint32_t i = b + lane; i < e; i += 32u) {
            const float4 d = info[sorted[i]];
            m = fmaxf(m, unit_angle(ax, ay, az, d.x, d.y, d.z));
        }
        phi = warp_max(m);
        phi = fminf(kPiF, phi * 1.0001f + kAngleMargin);
    } else {
        phi = kPiF;
    }
    if (lane == 0) {
        A[cell] = make_float4(ax, ay, az, cosf(phi));
        B[cell] = make_float4(sinf(phi), mr, phi, float(e - b));
    }
}

// 3b. One thread per parent node: cone containing its 4x4 children's cones.
__global__ __launch_bounds__(256) void k_cone_reduce(const float4* __restrict__ cA, const float4* __restrict__ cB,
                                                     uint32_t cgx, uint32_t cgy, float4* __restrict__ pA,
                                                     float4* __restrict__ pB, uint32_t pgx, uint32_t pgy) {
    const uint32_t node = blockIdx.x * blockDim.x + threadIdx.x;
    if (node >= pgx * pgy) return;
    const uint32_t px = node % pgx, py = node / pgx;
    float sx = 0.0f, sy = 0.0f, sz = 0.0f, cnt = 0.0f, mr = -1.0f;
    for (uint32_t j = 0; j < uint32_t(kFan); ++j) {
        for (uint32_t i = 0; i < uint32_t(kFan); ++i) {
            const uint32_t cx = px * kFan + i, cy = py * kFan + j;
            if (cx >= cgx || cy >= cgy) continue;
            const float4 a = cA[cy * cgx + cx];
            if (a.w > 1.5f) continue;
            const float4 b = cB[cy * cgx + cx];
            sx += a.x * b.w;
            sy += a.y * b.w;
            sz += a.z * b.w;
            cnt += b.w;
            mr = fmaxf(mr, b.y);
        }
    }
    if (!(cnt > 0.0f)) {
        pA[node] = make_float4(0.0f, 0.0f, 1.0f, 2.0f);
        pB[node] = make_float4(0.0f, -1.0f, 0.0f, 0.0f);
        return;
    }
    const float n = sqrtf(sx * sx + sy * sy + sz * sz);
    float ax = 0.0f, ay = 0.0f, az = 1.0f, phi = kPiF;
    if (n > 1e-12f) {
        ax = sx / n;
        ay = sy / n;
        az = sz / n;
        phi = 0.0f;
        for (uint32_t j = 0; j < uint32_t(kFan); ++j) {
            for (uint32_t i = 0; i < uint32_t(kFan); ++i) {
                const uint32_t cx = px * kFan + i, cy = py * kFan + j;
                if (cx >= cgx || cy >= cgy) continue;
                const float4 a = cA[cy * cgx + cx];
                if (a.w > 1.5f) continue;
                const float4 b = cB[cy * cgx + cx];
                phi = fmaxf(phi, unit_angle(ax, ay, az, a.x, a.y, a.z) + b.z);
            }
        }
        phi = fminf(kPiF, phi * 1.0001f + kAngleMargin);
    }
    pA[node] = make_float4(ax, ay, az, cosf(phi));
    pB[node] = make_float4(sinf(phi), mr, phi, cnt);
}

// Does the cap reach node c of level l: the node holds points, some of them
// beyond the support's lower range bound, and its cone meets the cap?
__device__ __forceinline__ bool node_passes(const Levels& L, int l, uint32_t c, float vx, float vy, float vz,
                                            float cosT, float sinT, float lower) {
    const uint32_t idx = L.offset[l] + c;
    const float4 A = L.A[idx];
    if (A.w > 1.5f) return false;
    const float4 B = L.B[idx];
    if (lower > B.y) return false;
    return cap_meets_cone(vx, vy, vz, cosT, sinT, A, B);
}

// Visits every cell the cap reaches, depth first from the root, testing
// children before pushing them.  Returns false, having visited only some
// cells, once more than kVisitBudget nodes were tested (such Gaussians are
// binned cooperatively by a warp instead).
template <typename Visit>
__device__ __forceinline__ bool for_cells(const Levels& L, float vx, float vy, float vz, float cosT, float sinT,
                                          float lower, Visit visit) {
    const int top = L.n - 1;
    if (!node_passes(L, top, 0u, vx, vy, vz, cosT, sinT, lower)) return true;
    if (top == 0) {
        visit(0u);
        return true;
    }
    uint32_t stack[kStack];
    int sp = 0, tests = 0;
    stack[sp++] = uint32_t(top) << 28;
    while (sp > 0) {
        const uint32_t e = stack[--sp];
        const int l = int(e >> 28);
        const uint32_t node = e & 0x0fffffffu;
        const uint32_t nx = node % L.gx[l], ny = node / L.gx[l];
        const int cl = l - 1;
        const uint32_t cgx = L.gx[cl], cgy = L.gy[cl];
        for (int j = 0; j < kFan; ++j) {
            for (int i = 0; i < kFan; ++i) {
                const uint32_t cx = nx * kFan + uint32_t(i), cy = ny * kFan + uint32_t(j);
                if (cx >= cgx || cy >= cgy) continue;
                if (++tests > kVisitBudget) return false;
                const uint32_t c = cy * cgx + cx;
                if (!node_passes(L, cl, c, vx, vy, vz, cosT, sinT, lower)) continue;
                if (cl == 0) {
                    visit(c);
                } else {
                    if (sp >= kStack) return false;
                    stack[sp++] = (uint32_t(cl) << 28) | c;
                }
            }
        }
    }
    return true;
}

// Warp-cooperative version for Gaussians over the budget: the warp tests the
// level-1 nodes 32 at a time and the 16 cells of every node that passes.
// Calls emit(k, cell) for the k-th cell found (k counts from 0 in the same
// order on every call) and returns the number of cells (warp-uniform).
template <typename Emit>
__device__ __forceinline__ uint32_t warp_cells(const Levels& L, float vx, float vy, float vz, float cosT, float sinT,
                                               float lower, uint32_t lane, Emit emit) {
    uint32_t n = 0;
    const uint32_t below = (1u << lane) - 1u;
    if (L.n == 1) {
        const uint32_t g0 = L.gx[0] * L.gy[0];
        for (uint32_t base = 0; base < g0; base += 32u) {
            const uint32_t c = base + lane;
            const bool ok = c < g0 && node_passes(L, 0, c, vx, vy, vz, cosT, sinT, lower);
            const uint32_t m = __ballot_sync(0xffffffffu, ok);
            if (ok) emit(n + uint32_t(__popc(m & below)), c);
            n += uint32_t(__popc(m));
        }
        return n;
    }
    const uint32_t g1 = L.gx[1] * L.gy[1], gx1 = L.gx[1], gx0 = L.gx[0], gy0 = L.gy[0];
    for (uint32_t base = 0; base < g1; base += 32u) {
        const uint32_t idx = base + lane;
        const bool pass = idx < g1 && node_passes(L, 1, idx, vx, vy, vz, cosT, sinT, lower);
        uint32_t m = __ballot_sync(0xffffffffu, pass);
        while (m != 0u) {
            const uint32_t n1 = base + uint32_t(__ffs(m) - 1);
            m &= m - 1u;
            const uint32_t cx = (n1 % gx1) * kFan + (lane & 3u), cy = (n1 / gx1) * kFan + (lane >> 2);
            const bool ok = lane < 16u && cx < gx0 && cy < gy0 &&
                            node_passes(L, 0, cy * gx0 + cx, vx, vy, vz, cosT, sinT, lower);
            const uint32_t cm = __ballot_sync(0xffffffffu, ok);
            if (ok) emit(n + uint32_t(__popc(cm & below)), cy * gx0 + cx);
            n += uint32_t(__popc(cm));
        }
    }
    return n;
}

// Compact per-Gaussian data, made once per context from the packed [N,32]
// rows: (position, density) and B^-1 rows with the support radius and the
// condition number of B^-1 in the spare slots.
__global__ __launch_bounds__(256) void k_field_pack(const float* __restrict__ particles, uint32_t N,
                                                    float4* __restrict__ posd, float4* __restrict__ binv) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N) return;
    const float* row = particles + 32 * size_t(i);
    posd[i] = make_float4(row[0], row[1], row[2], row[3]);
    float m[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) m[k] = row[21 + k];
    const float R = support_radius(m);
    // Condition number sqrt(lmax / lmin) of B^-T B^-1 via its trace bound:
    // lmax <= trace, so kappa <= sqrt(trace / lmin) = R * sqrt(trace) / 3.03.
    double tr = 0.0;
#pragma unroll
    for (int k = 0; k < 9; ++k) tr += double(m[k]) * double(m[k]);
    const float kappa = float(double(R) * sqrt(tr) / 3.03);
    binv[3 * size_t(i)] = make_float4(m[0], m[1], m[2], m[3]);
    binv[3 * size_t(i) + 1] = make_float4(m[4], m[5], m[6], m[7]);
    binv[3 * size_t(i) + 2] = make_float4(m[8], R, kappa, 0.0f);
}

struct ParticleArgs {
    const float4* posd;
    const float4* binv;
    uint32_t N;
};

// 4. Per camera and Gaussian: the cull record (cap direction, cos theta), the
// hit record (B^-1 (o - mu) exactly as the hit test computes it, density,
// B^-1, lower range bound, sin theta) and the number of cells it reaches.
// The support sphere's radius is inflated by 1e-5 * kappa * |mu - o|, far
// above the float error of evaluating the canonical closest point, so that
// no Gaussian the hit test could accept is culled.  Gaussians with density
// at most 1/255 can never pass the alpha test and reach no cell.
__global__ __launch_bounds__(256) void k_field_particles(CameraArgs a, ParticleArgs p, Levels L,
                                                         float4* __restrict__ cull, float4* __restrict__ hit,
                                                         uint32_t* __restrict__ counts, uint32_t* __restrict__ big,
                                                         uint32_t* __restrict__ bigCount) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= p.N) return;
    const float4 pd = p.posd[i];
    const float4 b0 = p.binv[3 * size_t(i)], b1 = p.binv[3 * size_t(i) + 1], b2 = p.binv[3 * size_t(i) + 2];
    V3 os0;
    const V3 origin = camera_centre(a, os0);
    const V3 v = v3(pd.x - origin.x, pd.y - origin.y, pd.z - origin.z);
    const float D = sqrtf(dot3(v, v));
    const float Rc = b2.y * 1.0001f + 1e-5f * b2.z * D + 1e-6f;
    float vx = 0.0f, vy = 0.0f, vz = 1.0f, cosT = kCapAll, sinT = 1.0f, lower = 0.0f;
    if (isfinite_f(D) && isfinite_f(Rc) && D > Rc) {
        vx = v.x / D;
        vy = v.y / D;
        vz = v.z / D;
        sinT = fminf(1.0f, (Rc / D) * 1.000001f);
        cosT = sqrtf(fmaxf(0.0f, 1.0f - sinT * sinT)) - kCosMargin;
        lower = fmaxf(0.0f, (D - Rc) * 0.999999f);
    }
    // o - mu and B^-1 (o - mu), in the hit test's order (half_ray).
    const V3 g = v3(origin.x - pd.x, origin.y - pd.y, origin.z - pd.z);
    const V3 gro = v3(__fmaf_rn(b0.z, g.z, __fmaf_rn(b0.y, g.y, b0.x * g.x)),
                      __fmaf_rn(b1.y, g.z, __fmaf_rn(b1.x, g.y, b0.w * g.x)),
                      __fmaf_rn(b2.x, g.z, __fmaf_rn(b1.w, g.y, b1.z * g.x)));
    uint32_t n = 0;
    bool small = true;
    if (!(pd.w <= kAlphaThreshold)) small = for_cells(L, vx, vy, vz, cosT, sinT, lower, [&](uint32_t) { ++n; });
    cull[i] = make_float4(vx, vy, vz, cosT);
    hit[4 * size_t(i)] = make_float4(gro.x, gro.y, gro.z, pd.w);
    hit[4 * size_t(i) + 1] = b0;
    hit[4 * size_t(i) + 2] = b1;
    hit[4 * size_t(i) + 3] = make_float4(b2.x, lower, sinT, small ? 0.0f : 1.0f);
    if (!small) big[atomicAdd(bigCount, 1u)] = i;
    counts[i] = small ? n : 0u;
}

// Cell counts (kEmit false) or keys (kEmit true) of the Gaussians over the
// traversal budget, one warp per Gaussian.
template <bool kEmit>
__global__ __launch_bounds__(256) void k_field_big(Levels L, const uint32_t* __restrict__ big,
                                                   const uint32_t* __restrict__ bigCount,
                                                   const float4* __restrict__ cull, const float4* __restrict__ hit,
                                                   uint32_t* __restrict__ counts, const uint64_t* __restrict__ offsets,
                                                   uint64_t* __restrict__ keys, uint32_t* __restrict__ ids) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    const uint32_t total = *bigCount;
    for (uint32_t w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total; w += warps) {
        const uint32_t i = big[w];
        const float4 c = cull[i];
        const float4 h3 = hit[4 * size_t(i) + 3];
        if (kEmit) {
            const uint64_t o = offsets[i];
            const uint32_t cap = counts[i];
            warp_cells(L, c.x, c.y, c.z, c.w, h3.z, h3.y, lane, [&](uint32_t k, uint32_t cell) {
                if (k < cap) {
                    keys[o + k] = (uint64_t(cell) << 32) | uint64_t(i);
                    ids[o + k] = i;
                }
            });
        } else {
            const uint32_t n = warp_cells(L, c.x, c.y, c.z, c.w, h3.z, h3.y, lane, [](uint32_t, uint32_t) {});
            if (lane == 0) counts[i] = n;
        }
    }
}

// 5. Emit (cell << 32 | id) keys at the scanned offsets, in id order.
__global__ __launch_bounds__(256) void k_field_emit(Levels L, uint32_t N, const float4* __restrict__ cull,
                                                    const float4* __restrict__ hit,
                                                    const uint32_t* __restrict__ counts,
                                                    const uint64_t* __restrict__ offsets, uint64_t* __restrict__ keys,
                                                    uint32_t* __restrict__ ids) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N || counts[i] == 0u) return;
    const float4 h3 = hit[4 * size_t(i) + 3];
    if (h3.w != 0.0f) return;  // binned by k_field_big
    const float4 c = cull[i];
    uint64_t o = offsets[i];
    const uint64_t end = o + counts[i];
    for_cells(L, c.x, c.y, c.z, c.w, h3.z, h3.y, [&](uint32_t cell) {
        if (o < end) {
            keys[o] = (uint64_t(cell) << 32) | uint64_t(i);
            ids[o] = i;
            ++o;
        }
    });
}

// Per-cell [begin, end) of the sorted candidate keys.
__global__ __launch_bounds__(256) void k_cell_ranges(const uint64_t* __restrict__ keys, uint32_t n,
                                                     uint2* __restrict__ ranges) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t c = uint32_t(keys[i] >> 32);
    if (i == 0 || uint32_t(keys[i - 1] >> 32) != c) ranges[c].x = i;
    if (i == n - 1 || uint32_t(keys[i + 1] >> 32) != c) ranges[c].y = i + 1;
}

// Integration blocks per cell: ceil(points / kBlock).
__global__ __launch_bounds__(256) void k_cell_blocks(const uint32_t* __restrict__ start, uint32_t cells,
                                                     uint32_t* __restrict__ blocks) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cells) return;
    const uint32_t n = start[(c + 1) * kCellPixels] - start[c * kCellPixels];
    blocks[c] = (n + kBlock - 1) / kBlock;
}

struct IntegrateArgs {
    const uint32_t* blockStart;  // exclusive scan of per-cell block counts
    uint32_t cells;
    const uint32_t* pointStart;  // exclusive scan of per-pixel-key point counts
    const uint32_t* sorted;
    const uint32_t* pixKey;
    const float4* info;
    const uint2* cellRanges;
    const uint32_t* candIds;
    const float4* cull;
    const float4* hit;
    float* minimum;     // field: camera-min opacity
    uint8_t* observed;  // field and rounds
    uint8_t* active;    // rounds: no camera below 1/2 yet
    uint8_t* exact;     // rounds: some camera exactly 1/2
    unsigned long long* counters;  // candidates staged, exact hit tests, hits, warp candidate iterations
};

// Alpha of one candidate for a point's segment [0, range] (0 when it is not
// a hit): the range and cap pre-tests, then the hit test with the arithmetic
// of half_ray / hit_test (gaussianParticles.slang hitInterval).
__device__ __forceinline__ float candidate_alpha(float4 c, float4 h0, float4 h1, float4 h2, float4 h3, float4 di,
                                                 uint32_t& tests) {
    if (h3.y > di.w) return 0.0f;                                                        // support beyond the point
    if (c.w > -1.5f && di.x * c.x + di.y * c.y + di.z * c.z < c.w) return 0.0f;        // ray misses the cap
    ++tests;
    const V3 grdu = v3(__fmaf_rn(h1.z, di.z, __fmaf_rn(h1.y, di.y, h1.x * di.x)),
                       __fmaf_rn(h2.y, di.z, __fmaf_rn(h2.x, di.y, h1.w * di.x)),
                       __fmaf_rn(h3.x, di.z, __fmaf_rn(h2.w, di.y, h2.z * di.x)));
    const float denom = fdot3(grdu, grdu);
    if (!(denom > 0.0f) || !isfinite_f(denom)) return 0.0f;
    const V3 gro = v3(h0.x, h0.y, h0.z);
    const float num = fdot3(gro, grdu);
    const float tauLine = -num / denom;
    const float tau = fminf(fmaxf(tauLine, 0.0f), di.w);
    const V3 pc = v3(__fmaf_rn(tau, grdu.x, gro.x), __fmaf_rn(tau, grdu.y, gro.y), __fmaf_rn(tau, grdu.z, gro.z));
    const float g2 = fdot3(pc, pc);
    if (g2 > kResponseCutoff2) return 0.0f;
    const float resp = gf_expf(-0.5f * g2);
    const float alpha = min_f(kMaxAlpha, resp * h0.w);
    return (resp > kMinKernelResponse && alpha > kAlphaThreshold) ? alpha : 0.0f;
}

// T <- T (1 - alpha).  Round lanes stop once the opacity 1 - T exceeds 1/2
// (the reference's threshold rounds do the same).  Field lanes stop once
// 1 - T rounds to exactly 1: later factors lie in [0.01, 1], so T can only
// shrink, and since rounding is monotone the final 1 - T is then exactly 1
// as well -- the full ordered product gives the same float.
template <bool kRound>
__device__ __forceinline__ void apply_alpha(float alpha, float& T, bool& done, bool& strictlyAbove) {
    T = T * (1.0f - alpha);
    if (kRound) {
        if (1.0f - T > 0.5f) {
            strictlyAbove = true;
            done = true;
        }
    } else if (1.0f - T == 1.0f) {
        done = true;
    }
}

// 6. Ordered integration (reference integratePoints, opacityField.cuh:775-829,
// and the threshold round, bisectionTableImpl.inl:222-304).  One block
// integrates up to kBlock points of one cell against the cell's candidates
// in ascending id.  Field mode keeps the exact float result (a lane stops
// only once 1 - T has rounded to 1, which no later factor can change); round
// mode stops a lane once 1 - T > 1/2 and classifies the camera as the
// reference's classifyCamera does.
template <bool kRound>
__global__ __launch_bounds__(kBlock) void k_field_integrate(IntegrateArgs a) {
    __shared__ float4 sCull[kBlock];
    __shared__ float4 sH0[kBlock], sH1[kBlock], sH2[kBlock], sH3[kBlock];
    __shared__ uint32_t sCell;
    __shared__ unsigned long long sKey[kBlock];
    __shared__ uint32_t sPoint[kBlock];
    const uint32_t tid = threadIdx.x, lane = tid & 31u;
    if (tid == 0) {
        // the last cell whose first block is at or before this one
        uint32_t lo = 0, hi = a.cells;
        while (hi - lo > 1u) {
            const uint32_t mid = (lo + hi) >> 1;
            if (a.blockStart[mid] <= blockIdx.x) lo = mid;
            else hi = mid;
        }
        sCell = lo;
    }
    __syncthreads();
    const uint32_t cell = sCell;
    const uint32_t pb = a.pointStart[cell * kCellPixels] + (blockIdx.x - a.blockStart[cell]) * kBlock;
    const uint32_t pe = min(pb + kBlock, a.pointStart[(cell + 1) * kCellPixels]);
    // Order the block's points by (pixel, range) so that each warp's points
    // share both a direction and a depth range (bitonic sort in shared memory).
    {
        const bool mine = pb + tid < pe;
        const uint32_t q0 = mine ? a.sorted[pb + tid] : 0u;
        sKey[tid] = mine ? (static_cast<unsigned long long>(a.pixKey[q0] & uint32_t(kCellPixels - 1)) << 32) |
                               __float_as_uint(a.info[q0].w)
                         : ~0ull;
        sPoint[tid] = q0;
        __syncthreads();
        for (uint32_t k = 2; k <= uint32_t(kBlock); k <<= 1) {
            for (uint32_t j = k >> 1; j > 0; j >>= 1) {
                const uint32_t ixj = tid ^ j;
                if (ixj > tid) {
                    const unsigned long long x = sKey[tid], y = sKey[ixj];
                    if ((x > y) == ((tid & k) == 0u)) {
                        sKey[tid] = y;
                        sKey[ixj] = x;
                        const uint32_t t = sPoint[tid];
                        sPoint[tid] = sPoint[ixj];
                        sPoint[ixj] = t;
                    }
                }
                __syncthreads();
            }
        }
    }
    const bool valid = sKey[tid] != ~0ull;
    const uint32_t q = valid ? sPoint[tid] : 0u;
    const float4 di = valid ? a.info[q] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);

    // The warp's direction cone (axis from all its points; half angle and
    // largest range refreshed per batch over the points still integrating).
    const float sx = warp_sum(di.x), sy = warp_sum(di.y), sz = warp_sum(di.z);
    const float sn = sqrtf(sx * sx + sy * sy + sz * sz);
    const bool axisOk = sn > 1e-12f;
    const float ax = axisOk ? sx / sn : 0.0f, ay = axisOk ? sy / sn : 0.0f, az = axisOk ? sz / sn : 1.0f;
    const float myAngle = valid ? unit_angle(ax, ay, az, di.x, di.y, di.z) : 0.0f;

    float T = 1.0f;
    bool done = !valid, strictlyAbove = false;
    uint32_t tests = 0, hits = 0, iterations = 0;
    const uint2 cr = a.cellRanges[cell];
    if (tid == 0) atomicAdd(&a.counters[0], static_cast<unsigned long long>(cr.y - cr.x));
    for (uint32_t base = cr.x; base < cr.y; base += kBlock) {
        if (__syncthreads_and(done)) break;
        const uint32_t idx = base + tid;
        if (idx < cr.y) {
            const uint32_t id = a.candIds[idx];
            sCull[tid] = a.cull[id];
            sH0[tid] = a.hit[4 * size_t(id)];
            sH1[tid] = a.hit[4 * size_t(id) + 1];
            sH2[tid] = a.hit[4 * size_t(id) + 2];
            sH3[tid] = a.hit[4 * size_t(id) + 3];
        }
        __syncthreads();
        const uint32_t n = min(uint32_t(kBlock), cr.y - base);
        float phi = warp_max(done ? 0.0f : myAngle);
        phi = axisOk ? phi * 1.0001f + kAngleMargin : kPiF;
        const bool wide = phi >= kWideCone;
        const float cphi = cosf(phi), sphi = sinf(phi);
        const float maxRange = warp_max(done ? 0.0f : di.w);
        for (uint32_t s = 0; s * 32u < n; ++s) {
            if (__all_sync(0xffffffffu, done)) break;
            const uint32_t k = s * 32u + lane;
            bool pass = false;
            if (k < n) {
                const float4 c = sCull[k];
                const float4 h3 = sH3[k];
                if (h3.y <= maxRange) {
                    pass = wide || c.w < -1.5f ||
                           ax * c.x + ay * c.y + az * c.z >= c.w * cphi - h3.z * sphi - kCosMargin;
                }
            }
            uint32_t m = __ballot_sync(0xffffffffu, pass);
            iterations += uint32_t(__popc(m));
            while (m != 0u) {
                const uint32_t slot = s * 32u + uint32_t(__ffs(m) - 1);
                m &= m - 1u;
                if (done) continue;
                const float alpha = candidate_alpha(sCull[slot], sH0[slot], sH1[slot], sH2[slot], sH3[slot], di,
                                                    tests);
                if (alpha > 0.0f) {
                    ++hits;
                    apply_alpha<kRound>(alpha, T, done, strictlyAbove);
                }
            }
        }
    }
    const uint32_t warpTests = __reduce_add_sync(0xffffffffu, tests);
    const uint32_t warpHits = __reduce_add_sync(0xffffffffu, hits);
    if (lane == 0) {
        atomicAdd(&a.counters[1], static_cast<unsigned long long>(warpTests));
        atomicAdd(&a.counters[2], static_cast<unsigned long long>(warpHits));
        atomicAdd(&a.counters[3], static_cast<unsigned long long>(iterations));
    }
    if (!valid) return;
    if (!kRound) {
        const float op = 1.0f - T;
        if (a.observed[q] != 0u) {
            a.minimum[q] = fminf(a.minimum[q], op);
        } else {
            a.minimum[q] = op;
            a.observed[q] = 1u;
        }
    } else {
        const float op = strictlyAbove ? 1.0f : 1.0f - T;
        a.observed[q] = 1u;
        if (op < 0.5f) {
            a.active[q] = 0u;
            a.exact[q] = 0u;
        } else if (op == 0.5f) {
            a.exact[q] = 1u;
        }
    }
}

// finish_opacity_field outputs (opacityFieldBinding.inl:318-338).
__global__ __launch_bounds__(256) void k_field_finish(const float* __restrict__ minimum,
                                                      const uint8_t* __restrict__ observed, uint32_t Q,
                                                      float* __restrict__ opacity, uint8_t* __restrict__ obsOut,
                                                      uint8_t* __restrict__ above) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= Q) return;
    const bool ob = observed[q] != 0u;
    const float op = ob ? minimum[q] : 0.0f;
    opacity[q] = op;
    obsOut[q] = ob ? 1u : 0u;
    above[q] = (ob && op >= 0.5f) ? 1u : 0u;
}

// Round decision vectors (finalizeDecisionVectors, bisectionTableImpl.inl:341-354).
__global__ __launch_bounds__(256) void k_round_finalize(const uint8_t* __restrict__ active,
                                                        const uint8_t* __restrict__ observed,
                                                        const uint8_t* __restrict__ exact, uint32_t Q,
                                                        uint8_t* __restrict__ aboveOut, uint8_t* __restrict__ obsOut,
                                                        uint8_t* __restrict__ exactOut) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= Q) return;
    const bool above = active[q] != 0u && observed[q] != 0u;
    aboveOut[q] = above ? 1u : 0u;
    obsOut[q] = observed[q] != 0u ? 1u : 0u;
    exactOut[q] = (above && exact[q] != 0u) ? 1u : 0u;
}

}  // namespace field
}  // namespace gf
