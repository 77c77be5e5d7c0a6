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
constexpr int kMaxTopNodes = 64;
constexpr int kMaxLevels = 6;
constexpr int kStack = 1 + (kFan * kFan - 1) * (kMaxLevels - 1) + 8;
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

// Quadtree of direction cones, level 0 = cells.  Node arrays are
// concatenated: level l occupies [offset[l], offset[l] + gx[l] * gy[l]).
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

// Visits every cell whose cone meets the cap and whose points reach the
// support's lower range bound (depth-first over the quadtree).
template <typename Visit>
__device__ __forceinline__ void for_cells(const Levels& L, float vx, float vy, float vz, float cosT, float sinT,
                                          float lower, Visit visit) {
    uint32_t stack[kStack];
    const int top = L.n - 1;
    const uint32_t topCount = L.gx[top] * L.gy[top];
    for (uint32_t t = 0; t < topCount; ++t) {
        int sp = 0;
        stack[sp++] = (uint32_t(top) << 28) | t;
        while (sp > 0) {
            const uint32_t e = stack[--sp];
            const int l = int(e >> 28);
            const uint32_t node = e & 0x0fffffffu;
            const uint32_t idx = L.offset[l] + node;
            const float4 A = L.A[idx];
            if (A.w > 1.5f) continue;
            const float4 B = L.B[idx];
            if (lower > B.y) continue;
            if (!cap_meets_cone(vx, vy, vz, cosT, sinT, A, B)) continue;
            if (l == 0) {
                visit(node);
                continue;
            }
            const uint32_t nx = node % L.gx[l], ny = node / L.gx[l];
            const uint32_t cgx = L.gx[l - 1], cgy = L.gy[l - 1];
            for (int j = kFan - 1; j >= 0; --j) {
                for (int i = kFan - 1; i >= 0; --i) {
                    const uint32_t cx = nx * kFan + uint32_t(i), cy = ny * kFan + uint32_t(j);
                    if (cx >= cgx || cy >= cgy) continue;
                    stack[sp++] = (uint32_t(l - 1) << 28) | (cy * cgx + cx);
                }
            }
        }
    }
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
                                                         uint32_t* __restrict__ counts) {
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
    cull[i] = make_float4(vx, vy, vz, cosT);
    hit[4 * size_t(i)] = make_float4(gro.x, gro.y, gro.z, pd.w);
    hit[4 * size_t(i) + 1] = b0;
    hit[4 * size_t(i) + 2] = b1;
    hit[4 * size_t(i) + 3] = make_float4(b2.x, lower, sinT, 0.0f);
    uint32_t n = 0;
    if (!(pd.w <= kAlphaThreshold)) for_cells(L, vx, vy, vz, cosT, sinT, lower, [&](uint32_t) { ++n; });
    counts[i] = n;
}

// 5. Emit (cell << 32 | id) keys at the scanned offsets, in id order.
__global__ __launch_bounds__(256) void k_field_emit(Levels L, uint32_t N, const float4* __restrict__ cull,
                                                    const float4* __restrict__ hit,
                                                    const uint32_t* __restrict__ counts,
                                                    const uint64_t* __restrict__ offsets, uint64_t* __restrict__ keys,
                                                    uint32_t* __restrict__ ids) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N || counts[i] == 0u) return;
    const float4 c = cull[i];
    const float4 h3 = hit[4 * size_t(i) + 3];
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
    const float4* info;
    const uint2* cellRanges;
    const uint32_t* candIds;
    const float4* cull;
    const float4* hit;
    float* minimum;     // field: camera-min opacity
    uint8_t* observed;  // field and rounds
    uint8_t* active;    // rounds: no camera below 1/2 yet
    uint8_t* exact;     // rounds: some camera exactly 1/2
};

// 6. Ordered integration (reference integratePoints, opacityField.cuh:775-829,
// and the threshold round, bisectionTableImpl.inl:222-304).  One block
// integrates up to kBlock points of one cell against the cell's candidates
// in ascending id.  Field mode keeps the exact product (a lane stops only
// when T reaches 0, after which it cannot change); round mode stops a lane
// once 1 - T > 1/2 and classifies the camera as the reference's
// classifyCamera does.
template <bool kRound>
__global__ __launch_bounds__(kBlock) void k_field_integrate(IntegrateArgs a) {
    __shared__ float4 sCull[kBlock];
    __shared__ float4 sH0[kBlock], sH1[kBlock], sH2[kBlock], sH3[kBlock];
    __shared__ uint32_t sCell;
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
    const bool valid = pb + tid < pe;
    const uint32_t q = valid ? a.sorted[pb + tid] : 0u;
    const float4 di = valid ? a.info[q] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);

    // The warp's direction cone and largest range.
    const float sx = warp_sum(di.x), sy = warp_sum(di.y), sz = warp_sum(di.z);
    const float sn = sqrtf(sx * sx + sy * sy + sz * sz);
    float ax = 0.0f, ay = 0.0f, az = 1.0f, phi = kPiF;
    if (sn > 1e-12f) {
        ax = sx / sn;
        ay = sy / sn;
        az = sz / sn;
        phi = warp_max(valid ? unit_angle(ax, ay, az, di.x, di.y, di.z) : 0.0f);
        phi = phi * 1.0001f + kAngleMargin;
    }
    const bool wide = phi >= kWideCone;
    const float cphi = cosf(phi), sphi = sinf(phi);
    const float maxRange = warp_max(valid ? di.w : 0.0f);

    float T = 1.0f;
    bool done = !valid, strictlyAbove = false;
    const uint2 cr = a.cellRanges[cell];
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
            while (m != 0u) {
                const uint32_t slot = s * 32u + uint32_t(__ffs(m) - 1);
                m &= m - 1u;
                if (done) continue;
                const float4 h3 = sH3[slot];
                if (h3.y > di.w) continue;  // support beyond the point
                const float4 c = sCull[slot];
                if (c.w > -1.5f && di.x * c.x + di.y * c.y + di.z * c.z < c.w) continue;  // ray misses the cap
                const float4 h0 = sH0[slot], h1 = sH1[slot], h2 = sH2[slot];
                // Hit test on [0, range], the arithmetic of half_ray / hit_test.
                const V3 grdu = v3(__fmaf_rn(h1.z, di.z, __fmaf_rn(h1.y, di.y, h1.x * di.x)),
                                   __fmaf_rn(h2.y, di.z, __fmaf_rn(h2.x, di.y, h1.w * di.x)),
                                   __fmaf_rn(h3.x, di.z, __fmaf_rn(h2.w, di.y, h2.z * di.x)));
                const float denom = fdot3(grdu, grdu);
                if (!(denom > 0.0f) || !isfinite_f(denom)) continue;
                const V3 gro = v3(h0.x, h0.y, h0.z);
                const float num = fdot3(gro, grdu);
                const float tauLine = -num / denom;
                const float tau = fminf(fmaxf(tauLine, 0.0f), di.w);
                const V3 pc = v3(__fmaf_rn(tau, grdu.x, gro.x), __fmaf_rn(tau, grdu.y, gro.y),
                                 __fmaf_rn(tau, grdu.z, gro.z));
                const float g2 = fdot3(pc, pc);
                if (g2 > kResponseCutoff2) continue;
                const float resp = gf_expf(-0.5f * g2);
                const float alpha = min_f(kMaxAlpha, resp * h0.w);
                if (!(resp > kMinKernelResponse && alpha > kAlphaThreshold)) continue;
                T = T * (1.0f - alpha);
                if (kRound) {
                    if (1.0f - T > 0.5f) {
                        strictlyAbove = true;
                        done = true;
                    }
                } else if (T == 0.0f) {
                    done = true;
                }
            }
        }
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
