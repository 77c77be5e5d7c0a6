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
    float utPartialScale2;  // partial UT covariance scale (0: off)
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

// ------------------------------------------------------------ cone fallback admission
// Particles whose unscented projection is invalid (wide-angle rim, near the
// camera, straddling the field-of-view boundary) are admitted by a
// conservative angular test of their bounding sphere against a quadtree of
// tile ray cones (reference fastFallbackTiles, gutProjector.cuh:100-183,
// render.gofish.fast_admission_fallback = "cone").  Leaf cone = the world
// directions of a retained tile's pixel rays; parents contain their 4x4
// children.  A tile is admitted when its cone and every ancestor's meet the
// particle's cap; a sphere that holds the camera centre admits every
// retained tile.  Only +, -, *, /, sqrt and the shared gf_logf enter these
// tests, in a fixed order, so the oracle admits exactly the same tiles.
namespace fb {

constexpr int kFan = 4;
constexpr int kMaxLevels = 8;
constexpr float kEps = 1e-6f;

enum CapMode : int { kNone = 0, kCone = 1, kAll = 2 };

struct TileTree {
    int n;
    int gx[kMaxLevels], gy[kMaxLevels];
    uint32_t offset[kMaxLevels];
    uint32_t second;  // offset of the leaves' second cones
    uint32_t sums;    // offset (in A) of each node's sum of unit pixel rays
    const float4* A;  // axis.xyz, cos phi (> 1.5: empty)
    const float* S;   // sin phi
    float optical[3]; // the camera's optical axis in world coordinates (third column of R^-1, not normalised)
};

struct Cap {
    float ux, uy, uz, cosA, sinA;
    int mode;
};

// Bounding sphere of the opacity support: sigma_max(B) (Gershgorin bound on
// the largest eigenvalue of B B^T) times the canonical radius where
// min(0.99, rho) exp(-r^2/2) falls to the minimum alpha (capped by the kernel
// cut-off), seen from the camera centre.
__device__ __forceinline__ Cap fallback_cap(const float B[9], V3 mu, float density, V3 cam) {
    Cap c{0.0f, 0.0f, 0.0f, 0.0f, 0.0f, kNone};
    const float m00 = B[0] * B[0] + B[1] * B[1] + B[2] * B[2];
    const float m01 = B[0] * B[3] + B[1] * B[4] + B[2] * B[5];
    const float m02 = B[0] * B[6] + B[1] * B[7] + B[2] * B[8];
    const float m11 = B[3] * B[3] + B[4] * B[4] + B[5] * B[5];
    const float m12 = B[3] * B[6] + B[4] * B[7] + B[5] * B[8];
    const float m22 = B[6] * B[6] + B[7] * B[7] + B[8] * B[8];
    const float g0 = m00 + abs_f(m01) + abs_f(m02);
    const float g1 = abs_f(m01) + m11 + abs_f(m12);
    const float g2 = abs_f(m02) + abs_f(m12) + m22;
    const float lam = max_f(g0, max_f(g1, g2));
    const float rho = min_f(kMaxAlpha, density);
    const float canonical = min_f(2.994f, __fsqrt_rn(max_f(0.0f, 2.0f * gf_logf(rho / kAlphaThreshold))));
    const float r = canonical * __fsqrt_rn(lam) * 1.001f;
    const V3 v = mu - cam;
    const float D = __fsqrt_rn(dot3(v, v));
    if (!(isfinite_f(r) && isfinite_f(D)) || !(r > 0.0f)) return c;
    if (D <= r) {
        c.mode = kAll;
        return c;
    }
    c.ux = v.x / D;
    c.uy = v.y / D;
    c.uz = v.z / D;
    c.sinA = min_f(1.0f, (r / D) * 1.0001f);
    c.cosA = __fsqrt_rn(max_f(0.0f, 1.0f - c.sinA * c.sinA));
    c.mode = kCone;
    return c;
}

// Cone (axis, phi) meets cap (u, alpha) iff angle(axis, u) <= phi + alpha:
// always when phi + alpha >= pi (sin(phi + alpha) < 0), else
// axis . u >= cos(phi + alpha) = cos phi cos alpha - sin phi sin alpha.
__device__ __forceinline__ bool cone_meets(const TileTree& t, uint32_t k, const Cap& c) {
    const float4 A = t.A[k];
    if (A.w > 1.5f) return false;
    const float S = t.S[k];
    if (S * c.cosA + A.w * c.sinA < 0.0f) return true;
    const float d = A.x * c.ux + A.y * c.uy + A.z * c.uz;
    return d >= A.w * c.cosA - S * c.sinA - kEps;
}

// A leaf (tile) holds two cones, one per cluster of its pixel rays; inner
// nodes hold one.
__device__ __forceinline__ bool node_pass(const TileTree& t, int l, uint32_t node, const Cap& c) {
    if (cone_meets(t, t.offset[l] + node, c)) return true;
    return l == 0 && cone_meets(t, t.second + node, c);
}

// Does every ancestor (levels >= 2) of level-1 node (x, y) meet the cap?
__device__ __forceinline__ bool ancestors_pass(const TileTree& t, uint32_t x, uint32_t y, const Cap& c) {
    for (int l = 2; l < t.n; ++l) {
        x /= kFan;
        y /= kFan;
        if (!node_pass(t, l, y * uint32_t(t.gx[l]) + x, c)) return false;
    }
    return true;
}

// The admitted tiles of one particle, found by one warp.  kAll: every
// retained tile.  kCone: every leaf that meets the cap together with all its
// ancestors, by a level-synchronous walk that keeps all 32 lanes testing:
// the frontier (nodes of one level whose path from the root passes) is kept
// in shared memory and its children are tested 32 at a time; from level 2
// the passing level-1 children of each batch of 32 are expanded at once into
// their leaves, two level-1 nodes (16 leaves each) per step.  A frontier
// larger than kFrontier entries (a raster beyond 4096x4096 pixels) falls back
// to the level-1 scan below, which yields the same set.  emit(k, tile)
// receives the k-th admitted tile (in an order the sorted output does not
// depend on: one particle's keys name distinct tiles); returns the number of
// tiles (warp-uniform).
constexpr int kFrontier = 256;
constexpr int kWarpScratch = 2 * kFrontier;

// Leaves of the level-1 nodes in `nodes` (bit i: level-1 node base1 + i of
// the candidate list `list`), two nodes per step.
template <typename Emit>
__device__ __forceinline__ void warp_leaves(const TileTree& t, const Cap& c, uint32_t lane, uint32_t below,
                                            uint32_t nodes, const uint32_t* list, uint32_t& n, Emit& emit) {
    const uint32_t gx1 = uint32_t(t.gx[1]);
    const uint32_t gx0 = uint32_t(t.gx[0]), gy0 = uint32_t(t.gy[0]);
    while (nodes != 0u) {
        const uint32_t a = uint32_t(__ffs(nodes) - 1);
        nodes &= nodes - 1u;
        uint32_t b = 32u;
        if (nodes != 0u) {
            b = uint32_t(__ffs(nodes) - 1);
            nodes &= nodes - 1u;
        }
        const uint32_t pick = lane < 16u ? a : b;
        bool ok = false;
        uint32_t leaf = 0u;
        if (pick < 32u) {
            const uint32_t n1 = list[pick];
            const uint32_t cx = (n1 % gx1) * kFan + (lane & 3u), cy = (n1 / gx1) * kFan + ((lane >> 2) & 3u);
            if (cx < gx0 && cy < gy0) {
                leaf = cy * gx0 + cx;
                ok = node_pass(t, 0, leaf, c);
            }
        }
        const uint32_t m = __ballot_sync(0xffffffffu, ok);
        if (ok) emit(n + uint32_t(__popc(m & below)), leaf);
        n += uint32_t(__popc(m));
    }
}

template <typename Emit>
__device__ __forceinline__ uint32_t warp_tiles(const TileTree& t, const uint8_t* __restrict__ mask, const Cap& c,
                                               uint32_t lane, uint32_t* __restrict__ scratch, Emit&& emit) {
    uint32_t n = 0;
    const uint32_t below = (1u << lane) - 1u;
    const uint32_t g0 = uint32_t(t.gx[0] * t.gy[0]);
    if (c.mode == kAll || t.n == 1) {
        for (uint32_t base = 0; base < g0; base += 32u) {
            const uint32_t tile = base + lane;
            bool ok = tile < g0 && mask[tile] != 0u;
            if (ok && c.mode != kAll) ok = node_pass(t, 0, tile, c);
            const uint32_t m = __ballot_sync(0xffffffffu, ok);
            if (ok) emit(n + uint32_t(__popc(m & below)), tile);
            n += uint32_t(__popc(m));
        }
        return n;
    }
    if (c.mode != kCone) return 0u;
    const int top = t.n - 1;
    if (!node_pass(t, top, 0u, c)) return 0u;
    uint32_t* cur = scratch;
    uint32_t* nxt = scratch + kFrontier;
    uint32_t* l1 = scratch + kFrontier;  // the level-1 batch reuses the spare frontier
    if (lane == 0) cur[0] = 0u;
    __syncwarp();
    uint32_t curN = 1;
    int level = top;
    bool overflow = false;
    // levels >= 3: expand the frontier one level down
    while (level >= 3 && !overflow) {
        const int cl = level - 1;
        const uint32_t pgx = uint32_t(t.gx[level]), cgx = uint32_t(t.gx[cl]), cgy = uint32_t(t.gy[cl]);
        const uint32_t total = curN * 16u;
        uint32_t nextN = 0;
        for (uint32_t base = 0; base < total; base += 32u) {
            const uint32_t idx = base + lane;
            bool pass = false;
            uint32_t child = 0u;
            if (idx < total) {
                const uint32_t node = cur[idx >> 4];
                const uint32_t cx = (node % pgx) * kFan + (idx & 3u), cy = (node / pgx) * kFan + ((idx >> 2) & 3u);
                if (cx < cgx && cy < cgy) {
                    child = cy * cgx + cx;
                    pass = node_pass(t, cl, child, c);
                }
            }
            const uint32_t m = __ballot_sync(0xffffffffu, pass);
            if (nextN + uint32_t(__popc(m)) > uint32_t(kFrontier)) {
                overflow = true;
                break;
            }
            if (pass) nxt[nextN + uint32_t(__popc(m & below))] = child;
            nextN += uint32_t(__popc(m));
        }
        __syncwarp();
        uint32_t* tmp = cur;
        cur = nxt;
        nxt = tmp;
        l1 = nxt;
        curN = nextN;
        level = cl;
    }
    if (!overflow) {
        if (level == 1) {
            // a two-level tree: the root is the only level-1 node
            warp_leaves(t, c, lane, below, 1u, cur, n, emit);
            return n;
        }
        // level 2: its level-1 children, 32 at a time, then their leaves
        const uint32_t pgx = uint32_t(t.gx[2]), cgx = uint32_t(t.gx[1]), cgy = uint32_t(t.gy[1]);
        const uint32_t total = curN * 16u;
        for (uint32_t base = 0; base < total; base += 32u) {
            const uint32_t idx = base + lane;
            bool pass = false;
            uint32_t child = 0u;
            if (idx < total) {
                const uint32_t node = cur[idx >> 4];
                const uint32_t cx = (node % pgx) * kFan + (idx & 3u), cy = (node / pgx) * kFan + ((idx >> 2) & 3u);
                if (cx < cgx && cy < cgy) {
                    child = cy * cgx + cx;
                    pass = node_pass(t, 1, child, c);
                }
            }
            const uint32_t m = __ballot_sync(0xffffffffu, pass);
            l1[lane] = child;
            __syncwarp();
            warp_leaves(t, c, lane, below, m, l1, n, emit);
            __syncwarp();
        }
        return n;
    }
    // Level-1 scan: nodes whose ancestors all pass, then their 16 leaves.
    n = 0;
    const uint32_t gx1 = uint32_t(t.gx[1]), g1 = gx1 * uint32_t(t.gy[1]);
    for (uint32_t base = 0; base < g1; base += 32u) {
        const uint32_t node = base + lane;
        const bool pass = node < g1 && node_pass(t, 1, node, c) && ancestors_pass(t, node % gx1, node / gx1, c);
        const uint32_t m = __ballot_sync(0xffffffffu, pass);
        __syncwarp();
        scratch[lane] = node;
        __syncwarp();
        warp_leaves(t, c, lane, below, m, scratch, n, emit);
    }
    return n;
}

// Leaf cones: one warp per tile, lane r < 16 walking pixel row r; row
// partials (sums, first minima) are combined in row order, so every value is
// the oracle's float for float.  The tile's rays are split in two clusters by
// the nearer of the two mutually farthest rays (far1 the farthest from the
// mean ray, far2 the farthest from far1; ties to far1), so that a tile mixing
// rim rays with the forward rays of pixels outside the image circle gets two
// narrow cones instead of one wide one.  Cone k: axis = normalised sum of its
// rays, cos phi = smallest cosine to the axis less kEps.
__device__ __forceinline__ bool pixel_dir(const FrameArgs& f, const float* __restrict__ rayD, int x, int y, V3& u) {
    const size_t p = size_t(x) + size_t(f.W) * size_t(y);
    const V3 d = v3(rayD[3 * p], rayD[3 * p + 1], rayD[3 * p + 2]);
    const float n2 = dot3(d, d);
    if (!(n2 > 0.0f) || !isfinite_f(n2)) return false;
    const V3 w = mat3(f.pose.Rinv, d);
    const float wn = __fsqrt_rn(dot3(w, w));
    u = v3(w.x / wn, w.y / wn, w.z / wn);
    return true;
}

__device__ __forceinline__ V3 shfl_v3(V3 v, int r) {
    return v3(__shfl_sync(0xffffffffu, v.x, r), __shfl_sync(0xffffffffu, v.y, r), __shfl_sync(0xffffffffu, v.z, r));
}

// Sum of the row partials in row order (rows with no ray skipped).
__device__ __forceinline__ V3 rows_sum(V3 part, int cnt, int& all) {
    V3 total = v3(0.0f, 0.0f, 0.0f);
    all = 0;
    for (int r = 0; r < kTile; ++r) {
        const V3 rs = shfl_v3(part, r);
        const int rc = __shfl_sync(0xffffffffu, cnt, r);
        if (rc > 0) total = total + rs;
        all += rc;
    }
    return total;
}

// Cone of axis a (or the whole sphere for a degenerate sum) from its minimum cosine.
__device__ __forceinline__ void store_cone(float4* A, float* S, uint32_t k, V3 a, float mn) {
    const float cphi = max_f(-1.0f, mn - kEps);
    A[k] = make_float4(a.x, a.y, a.z, cphi);
    S[k] = __fsqrt_rn(max_f(0.0f, 1.0f - cphi * cphi));
}

__global__ __launch_bounds__(128) void k_tile_cones(FrameArgs f, const uint8_t* __restrict__ mask,
                                                    const float* __restrict__ rayD, float4* __restrict__ A,
                                                    float* __restrict__ S, uint32_t second, uint32_t sums) {
    const int tile = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (tile >= f.gx * f.gy) return;  // warp-uniform
    const int tx = tile % f.gx, ty = tile / f.gx;
    const int x0 = tx * kTile, y0 = ty * kTile, x1 = min(f.W, x0 + kTile), y1 = min(f.H, y0 + kTile);
    const int y = y0 + lane;
    const bool row = lane < kTile && y < y1 && mask[tile] != 0u;
    const float4 empty = make_float4(0.0f, 0.0f, 1.0f, 2.0f);
    // the row's unit pixel directions, once (bit i of ok: pixel x0 + i has one);
    // every pass below visits them in x order, as a loop over the row would
    V3 ud[kTile];
    uint32_t ok = 0u;
    if (row) {
#pragma unroll
        for (int i = 0; i < kTile; ++i) {
            ud[i] = v3(0.0f, 0.0f, 1.0f);
            if (x0 + i < x1 && pixel_dir(f, rayD, x0 + i, y, ud[i])) ok |= 1u << i;
        }
    }
    // pass 0: the mean ray
    V3 sum = v3(0.0f, 0.0f, 0.0f);
    int count = 0;
#pragma unroll
    for (int i = 0; i < kTile; ++i) {
        if (!((ok >> i) & 1u)) continue;
        sum = sum + ud[i];
        ++count;
    }
    int all = 0;
    const V3 total = rows_sum(sum, count, all);
    if (lane == 0) A[sums + tile] = make_float4(total.x, total.y, total.z, 0.0f);
    if (mask[tile] == 0u || all == 0) {
        if (lane == 0) {
            A[tile] = empty;
            S[tile] = 0.0f;
            A[second + tile] = empty;
            S[second + tile] = 0.0f;
        }
        return;
    }
    const float sn = __fsqrt_rn(dot3(total, total));
    if (!(sn > 0.0f) || !isfinite_f(sn)) {
        if (lane == 0) {
            A[tile] = make_float4(0.0f, 0.0f, 1.0f, -1.0f);
            S[tile] = 0.0f;
            A[second + tile] = empty;
            S[second + tile] = 0.0f;
        }
        return;
    }
    const V3 mean = v3(total.x / sn, total.y / sn, total.z / sn);
    // passes 1, 2: the ray farthest from the mean, then the ray farthest from it
    V3 far1 = mean, far2 = mean;
    for (int pass = 0; pass < 2; ++pass) {
        const V3 ref = pass == 0 ? mean : far1;
        float best = 2.0f;
        V3 bu = ref;
#pragma unroll
        for (int i = 0; i < kTile; ++i) {
            if (!((ok >> i) & 1u)) continue;
            const float c = dot3(ref, ud[i]);
            if (c < best) {
                best = c;
                bu = ud[i];
            }
        }
        float gbest = 2.0f;
        V3 gu = ref;
        for (int r = 0; r < kTile; ++r) {
            const float rb = __shfl_sync(0xffffffffu, best, r);
            const V3 ru = shfl_v3(bu, r);
            if (rb < gbest) {
                gbest = rb;
                gu = ru;
            }
        }
        if (pass == 0) far1 = gu;
        else far2 = gu;
    }
    // pass 3: cluster sums
    V3 s0 = v3(0.0f, 0.0f, 0.0f), s1 = v3(0.0f, 0.0f, 0.0f);
    int n0 = 0, n1 = 0;
    uint32_t first = 0u;  // bit i: pixel x0 + i belongs to the first cluster
#pragma unroll
    for (int i = 0; i < kTile; ++i) {
        if (!((ok >> i) & 1u)) continue;
        if (dot3(far1, ud[i]) >= dot3(far2, ud[i])) {
            s0 = s0 + ud[i];
            ++n0;
            first |= 1u << i;
        } else {
            s1 = s1 + ud[i];
            ++n1;
        }
    }
    int all0 = 0, all1 = 0;
    const V3 t0 = rows_sum(s0, n0, all0);
    const V3 t1 = rows_sum(s1, n1, all1);
    const float l0 = __fsqrt_rn(dot3(t0, t0)), l1 = __fsqrt_rn(dot3(t1, t1));
    const bool ok0 = l0 > 0.0f && isfinite_f(l0), ok1 = l1 > 0.0f && isfinite_f(l1);
    const V3 a0 = ok0 ? v3(t0.x / l0, t0.y / l0, t0.z / l0) : mean;
    const V3 a1 = ok1 ? v3(t1.x / l1, t1.y / l1, t1.z / l1) : mean;
    // pass 4: the smallest cosine of each cluster to its axis
    float m0 = 1.0f, m1 = 1.0f;
#pragma unroll
    for (int i = 0; i < kTile; ++i) {
        if (!((ok >> i) & 1u)) continue;
        if ((first >> i) & 1u) m0 = min_f(m0, dot3(a0, ud[i]));
        else m1 = min_f(m1, dot3(a1, ud[i]));
    }
    for (int r = 0; r < kTile; ++r) {
        const float r0 = __shfl_sync(0xffffffffu, m0, r), r1 = __shfl_sync(0xffffffffu, m1, r);
        if (lane == 0) {
            m0 = min_f(m0, r0);
            m1 = min_f(m1, r1);
        }
    }
    if (lane != 0) return;
    if (ok0) store_cone(A, S, uint32_t(tile), a0, m0);
    else if (all0 > 0) A[tile] = make_float4(a0.x, a0.y, a0.z, -1.0f), S[tile] = 0.0f;
    else A[tile] = empty, S[tile] = 0.0f;
    if (ok1) store_cone(A, S, second + uint32_t(tile), a1, m1);
    else if (all1 > 0) A[second + tile] = make_float4(a1.x, a1.y, a1.z, -1.0f), S[second + tile] = 0.0f;
    else A[second + tile] = empty, S[second + tile] = 0.0f;
}

// Parent cones of level l >= 1, one block per node.  The node's ray sum is
// the sum of its 4x4 children's (row-major order).  Two axes are tried: the
// normalised ray sum (the mean direction of the pixel rays under the node)
// and the camera's optical axis; for each, cos phi = the smallest, over the
// non-empty cones of the leaves under the node, of cos(angle(axis, a) +
// phi_a) = (axis . a) cos phi_a - |axis x a| sin phi_a, and a cone reaching
// past pi makes the bound cover the sphere.  The node keeps the axis with the
// larger cos phi (the mean on ties), less kEps.  The mean alone fails for
// wide nodes: over a 200 deg field the rim rays can outweigh the centre and
// turn the sum backwards, so that the root would cover the whole sphere.  The
// node is empty when all its children are.  Minima are exact in any order, so
// the block reduction gives the oracle's values.
__device__ __forceinline__ void bound_cone(V3 ax, float4 a, float cs, float& mn, bool& full) {
    if (a.w > 1.5f) return;
    const V3 ca = v3(a.x, a.y, a.z);
    const V3 cr = v3(ax.y * ca.z - ax.z * ca.y, ax.z * ca.x - ax.x * ca.z, ax.x * ca.y - ax.y * ca.x);
    const float sang = __fsqrt_rn(dot3(cr, cr));
    const float cang = dot3(ax, ca);
    if (sang * a.w + cang * cs < 0.0f) full = true;
    else mn = min_f(mn, cang * a.w - sang * cs);
}

// One block per node of level l; any multiple of 32 threads up to 1024 (the
// bound is a min / or over the node's leaves, whatever their split over threads).
__host__ __device__ constexpr int cone_level_threads(int leaves) {
    return leaves >= 1024 ? 1024 : ((leaves + 31) / 32) * 32;
}

__global__ __launch_bounds__(1024) void k_tile_cone_level(TileTree t, int l, float4* __restrict__ A,
                                                          float* __restrict__ S) {
    __shared__ float axis[8];
    __shared__ float wmin[2][32];
    const int node = blockIdx.x;
    const int pgx = t.gx[l], cgx = t.gx[l - 1], cgy = t.gy[l - 1];
    const int px = node % pgx, py = node / pgx;
    if (threadIdx.x == 0) {
        V3 sum = v3(0.0f, 0.0f, 0.0f);
        bool any = false;
        for (int j = 0; j < kFan; ++j)
            for (int i = 0; i < kFan; ++i) {
                const int cx = px * kFan + i, cy = py * kFan + j;
                if (cx >= cgx || cy >= cgy) continue;
                const uint32_t child = t.offset[l - 1] + uint32_t(cy * cgx + cx);
                const float4 r = A[t.sums + child];
                sum = sum + v3(r.x, r.y, r.z);
                if (A[child].w <= 1.5f) any = true;
                if (l == 1 && A[t.second + uint32_t(cy * cgx + cx)].w <= 1.5f) any = true;
            }
        A[t.sums + t.offset[l] + uint32_t(node)] = make_float4(sum.x, sum.y, sum.z, 0.0f);
        const float sn = __fsqrt_rn(dot3(sum, sum));
        const bool ok = sn > 0.0f && isfinite_f(sn);
        axis[0] = ok ? sum.x / sn : 0.0f;
        axis[1] = ok ? sum.y / sn : 0.0f;
        axis[2] = ok ? sum.z / sn : 1.0f;
        axis[3] = !any ? 2.0f : (ok ? 1.0f : -1.0f);  // empty / mean usable / mean degenerate
        const V3 o = v3(t.optical[0], t.optical[1], t.optical[2]);
        const float on = __fsqrt_rn(dot3(o, o));
        const bool ook = on > 0.0f && isfinite_f(on);
        axis[4] = ook ? o.x / on : 0.0f;
        axis[5] = ook ? o.y / on : 0.0f;
        axis[6] = ook ? o.z / on : 1.0f;
        axis[7] = ook ? 1.0f : -1.0f;
    }
    __syncthreads();
    const float state = axis[3];
    if (state > 1.5f) {
        if (threadIdx.x == 0) {
            A[t.offset[l] + node] = make_float4(axis[0], axis[1], axis[2], 2.0f);
            S[t.offset[l] + node] = 0.0f;
        }
        return;
    }
    const V3 am = v3(axis[0], axis[1], axis[2]);
    const V3 ao = v3(axis[4], axis[5], axis[6]);
    int span = 1;
    for (int k = 0; k < l; ++k) span *= kFan;
    const int gx0 = t.gx[0], gy0 = t.gy[0];
    const int x0 = px * span, y0 = py * span, x1 = min(gx0, x0 + span), y1 = min(gy0, y0 + span);
    const int w = x1 - x0, cnt = w * (y1 - y0);
    float mm = 1.0f, mo = 1.0f;
    bool fm = state < 0.0f, fo = axis[7] < 0.0f;
    for (int k = threadIdx.x; k < cnt; k += blockDim.x) {
        const uint32_t leaf = uint32_t((y0 + k / w) * gx0 + x0 + k % w);
        const float4 a0 = A[leaf], a1 = A[t.second + leaf];
        const float s0 = S[leaf], s1 = S[t.second + leaf];
        bound_cone(am, a0, s0, mm, fm);
        bound_cone(am, a1, s1, mm, fm);
        bound_cone(ao, a0, s0, mo, fo);
        bound_cone(ao, a1, s1, mo, fo);
    }
    fm = __syncthreads_or(fm) != 0;
    fo = __syncthreads_or(fo) != 0;
    for (int o = 16; o > 0; o >>= 1) {
        mm = min_f(mm, __shfl_xor_sync(0xffffffffu, mm, o));
        mo = min_f(mo, __shfl_xor_sync(0xffffffffu, mo, o));
    }
    if ((threadIdx.x & 31) == 0) {
        wmin[0][threadIdx.x >> 5] = mm;
        wmin[1][threadIdx.x >> 5] = mo;
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int k = 0; k < int(blockDim.x >> 5); ++k) {
        mm = min_f(mm, wmin[0][k]);
        mo = min_f(mo, wmin[1][k]);
    }
    const float vm = fm ? -2.0f : mm, vo = fo ? -2.0f : mo;
    const bool useOptical = vo > vm;
    const V3 ax = useOptical ? ao : am;
    const float best = useOptical ? vo : vm;
    if (best < -1.5f) {
        A[t.offset[l] + node] = make_float4(ax.x, ax.y, ax.z, -1.0f);
        S[t.offset[l] + node] = 0.0f;
        return;
    }
    const float cphi = max_f(-1.0f, best - kEps);
    A[t.offset[l] + node] = make_float4(ax.x, ax.y, ax.z, cphi);
    S[t.offset[l] + node] = __fsqrt_rn(max_f(0.0f, 1.0f - cphi * cphi));
}

}  // namespace fb

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
struct FallbackArgs {
    int enabled;
    fb::TileTree tree;
    float4* caps;       // [N,2] for particles without a valid projection: (u, cos), (sin, mode, 0, 0)
    uint32_t* big;      // particles left to the warp kernel
    uint32_t* bigCount;
    uint32_t* bigCursor;  // [2] next list entry of k_fallback_big (count, emit), zeroed per frame
    uint32_t* wide;     // projected particles whose tile box exceeds kWideTiles, left to k_wide
    uint32_t* wideCount;
    const uint32_t* overflow;  // non-zero: the intersections exceed the key capacity, emit nothing (may be NULL)
    int complete;              // every particle takes the cone route (complete admission)
    int coneBig;               // "cone_big": no sphere holding the camera, cap sine in [sinMin, sinMax]
    float sinMin, sinMax;
    // Tile lists of the count pass's walks, read back by the emit pass: a
    // particle's admitted tiles (at most kCachedTiles, in walk order) at
    // cacheStart[i] of tileCache, kNotCached when they did not fit.
    uint32_t* tileCache;
    uint32_t cacheCapacity;
    uint32_t* cacheCursor;  // zeroed per frame
    uint32_t* cacheStart;   // [N], written for listed particles
};

constexpr uint32_t kCachedTiles = 256;
constexpr uint32_t kNotCached = 0xffffffffu;

__device__ __forceinline__ bool skip_emit(const FallbackArgs& fa) {
    return fa.overflow != nullptr && *fa.overflow != 0u;
}

// Projected particles whose tile bounding box holds more tiles than this are
// counted and emitted by one warp (k_wide) instead of one thread, so that a
// large Gaussian near the camera does not serialise thousands of tile tests
// and one thread's long box walk does not hold its warp's 31 others (on the
// 1M-Gaussian bench view: count + emit 0.84 ms at 64 tiles, 0.76 at 32,
// 0.69 at 16).
#ifndef GF_WIDE_TILES
#define GF_WIDE_TILES 16
#endif
constexpr int kWideTiles = GF_WIDE_TILES;

__device__ __forceinline__ bool wide_box(const TileBox& b) {
    return (b.x1 - b.x0) * (b.y1 - b.y0) > kWideTiles;
}

__global__ __launch_bounds__(256) void k_project(FrameArgs f, const float* __restrict__ particles,
                                                 const float* __restrict__ features,
                                                 const uint8_t* __restrict__ mask, float4* __restrict__ proj,
                                                 float4* __restrict__ records, uint32_t* __restrict__ counts,
                                                 uint32_t* __restrict__ visibility, float* __restrict__ bounds,
                                                 FallbackArgs fa) {
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
    bool valid = unscented_projection(f.cam, f.pose, mu, density, B, cx, cy, cov, f.utPartialScale2);
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
    // loops unrolled over all 16 coefficients with a predicate, so that the
    // basis stays in registers (a runtime bound would put it in local memory)
    if ((3u * f.shCoeffs) % 4u == 0u && (reinterpret_cast<uintptr_t>(features) & 15u) == 0u) {
        // rows of whole float4s: coefficient (k, channel) is float 3k + channel
        // of the row, read 4 at a time; each channel still sums in k order
        float acc[3] = {0.0f, 0.0f, 0.0f};
        const float4* c4 = reinterpret_cast<const float4*>(c);
#pragma unroll
        for (int q = 0; q < 12; ++q) {
            if (4 * q < 3 * nb) {
                const float4 v = __ldg(c4 + q);
                const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int k = (4 * q + r) / 3, ch = (4 * q + r) % 3;
                    if (k < nb) acc[ch] = k == 0 ? basis[0] * e[r] : __fmaf_rn(basis[k], e[r], acc[ch]);
                }
            }
        }
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) rgb[ch] = fmaxf(acc[ch] + 0.5f, 0.0f);
    } else {
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            float acc = basis[0] * __ldg(c + ch);
#pragma unroll
            for (int k = 1; k < 16; ++k)
                if (k < nb) acc = __fmaf_rn(basis[k], __ldg(c + 3 * k + ch), acc);
            rgb[ch] = fmaxf(acc + 0.5f, 0.0f);
        }
    }
    float4* rec = records + 4 * size_t(i);
    rec[0] = r0;
    rec[1] = make_float4(r5.y, r5.z, r5.w, r6.x);
    rec[2] = make_float4(r6.y, r6.z, r6.w, r7.x);
    rec[3] = make_float4(r7.y, rgb[0], rgb[1], rgb[2]);

    // complete admission: every particle takes the cone route, none its footprint
    const bool footprint = !fa.complete && fast_ut_valid(p);
    bool wide = false;
    if (footprint) wide = wide_box(tile_bbox(f.gx, f.gy, p.cx, p.cy, p.ex, p.ey));
    const uint32_t n = (wide || !footprint) ? 0u : for_admitted_tiles(f, mask, p, [](int, int, uint32_t) {});
    bool deferred = false;
    if (!footprint) {
        // Without a valid projection: the cone fallback, left to the warp
        // kernel once the cap meets the root cone.
        fb::Cap c{0.0f, 0.0f, 0.0f, 0.0f, 0.0f, fb::kNone};
        if (fa.enabled && density >= kAlphaThreshold) {
            c = fb::fallback_cap(B, mu, density, v3(f.pose.c[0], f.pose.c[1], f.pose.c[2]));
            // "cone_big" (gutProjector.cuh:145-154): only caps whose half-angle lies in the window, never a
            // sphere around the camera (the window compares sines: the half-angle is at most pi/2)
            if (fa.coneBig && !fa.complete &&
                (c.mode == fb::kAll || (c.mode == fb::kCone && (c.sinA < fa.sinMin || c.sinA > fa.sinMax))))
                c.mode = fb::kNone;
            if (c.mode == fb::kCone && !fb::node_pass(fa.tree, fa.tree.n - 1, 0u, c)) c.mode = fb::kNone;
            deferred = c.mode != fb::kNone;
        }
        fa.caps[2 * size_t(i)] = make_float4(c.ux, c.uy, c.uz, c.cosA);
        fa.caps[2 * size_t(i) + 1] = make_float4(c.sinA, float(c.mode), 0.0f, 0.0f);
    }
    // warp-aggregated append to the fallback list
    const uint32_t live = __activemask();
    const uint32_t dm = __ballot_sync(live, deferred);
    if (dm != 0u) {
        const uint32_t lane = threadIdx.x & 31u;
        const int leader = __ffs(dm) - 1;
        uint32_t base = 0u;
        if (int(lane) == leader) base = atomicAdd(fa.bigCount, uint32_t(__popc(dm)));
        base = __shfl_sync(live, base, leader);
        if (deferred) fa.big[base + uint32_t(__popc(dm & ((1u << lane) - 1u)))] = i;
    }
    // warp-aggregated append to the wide list
    const uint32_t wm = __ballot_sync(live, wide);
    if (wm != 0u) {
        const uint32_t lane = threadIdx.x & 31u;
        const int leader = __ffs(wm) - 1;
        uint32_t base = 0u;
        if (int(lane) == leader) base = atomicAdd(fa.wideCount, uint32_t(__popc(wm)));
        base = __shfl_sync(live, base, leader);
        if (wide) fa.wide[base + uint32_t(__popc(wm & ((1u << lane) - 1u)))] = i;
    }
    counts[i] = n;
    if (visibility != nullptr && !deferred && !wide) visibility[i] = n ? 1u : 0u;
    if (n != 0u || deferred || wide) {
        const float Binv[9] = {r5.y, r5.z, r5.w, r6.x, r6.y, r6.z, r6.w, r7.x, r7.y};
        bounds[i] = support_radius(Binv);
    }
}

// Per-tile sort key of particle i (per-tile max-response depth or radial depth).
__device__ __forceinline__ uint32_t tile_depth_key(int keyMode, V3 mu, const float Binv[9], float camRadial,
                                                   const float4* __restrict__ tileRays, uint32_t tile) {
    if (keyMode == GF_KEY_GLOBAL_DEPTH) return __float_as_uint(camRadial);
    return depth_key_per_tile(mu, Binv, camRadial, tileRays[2 * tile], tileRays[2 * tile + 1]);
}

// Cone-fallback particles (no valid projection, cap meeting the root cone or
// sphere holding the camera): one warp each, counting (kEmit false) or
// emitting keys at the scanned offsets.
template <bool kEmit>
__global__ __launch_bounds__(256) void k_fallback_big(FrameArgs f, FallbackArgs fa, const uint8_t* __restrict__ mask,
                                                      const float4* __restrict__ records,
                                                      const float4* __restrict__ tileRays,
                                                      uint32_t* __restrict__ counts, uint32_t* __restrict__ visibility,
                                                      const uint64_t* __restrict__ offsets,
                                                      uint64_t* __restrict__ keys, uint32_t* __restrict__ ids) {
    __shared__ uint32_t scratch[8][fb::kWarpScratch];
    __shared__ uint32_t walked[kEmit ? 1 : 8][kEmit ? 1 : kCachedTiles];
    const uint32_t lane = threadIdx.x & 31u;
    uint32_t* stack = scratch[threadIdx.x >> 5];
    if (kEmit && skip_emit(fa)) return;  // block-uniform
    const uint32_t total = *fa.bigCount;
    // each warp takes the next listed particle when it is done: the walks
    // differ by orders of magnitude (caps near the camera span most tiles)
    uint32_t* cursor = fa.bigCursor + (kEmit ? 1 : 0);
    const auto next = [&]() {
        uint32_t w = 0u;
        if (lane == 0) w = atomicAdd(cursor, 1u);
        return __shfl_sync(0xffffffffu, w, 0);
    };
    for (uint32_t w = next(); w < total; w = next()) {
        const uint32_t i = fa.big[w];
        const float4 c0 = fa.caps[2 * size_t(i)], c1 = fa.caps[2 * size_t(i) + 1];
        const fb::Cap c{c0.x, c0.y, c0.z, c0.w, c1.x, int(c1.y)};
        if constexpr (!kEmit) {
            uint32_t* list = walked[threadIdx.x >> 5];
            const uint32_t n = fb::warp_tiles(fa.tree, mask, c, lane, stack, [&](uint32_t k, uint32_t tile) {
                if (k < kCachedTiles) list[k] = tile;
            });
            __syncwarp();
            // keep the walk for the emit pass when it fits
            uint32_t start = kNotCached;
            if (n > 0u && n <= kCachedTiles) {
                if (lane == 0) start = atomicAdd(fa.cacheCursor, n);
                start = __shfl_sync(0xffffffffu, start, 0);
                if (start <= fa.cacheCapacity && n <= fa.cacheCapacity - start) {
                    for (uint32_t j = lane; j < n; j += 32u) fa.tileCache[start + j] = list[j];
                } else {
                    start = kNotCached;
                }
            }
            __syncwarp();
            if (lane == 0) {
                counts[i] = n;
                fa.cacheStart[i] = start;
                if (visibility != nullptr) visibility[i] = n ? 1u : 0u;
            }
        } else {
            const float4 a = records[4 * size_t(i)], b = records[4 * size_t(i) + 1], cc = records[4 * size_t(i) + 2],
                         d = records[4 * size_t(i) + 3];
            const V3 mu = v3(a.x, a.y, a.z);
            const float Binv[9] = {b.x, b.y, b.z, b.w, cc.x, cc.y, cc.z, cc.w, d.x};
            const V3 cv = mu - v3(f.pose.c[0], f.pose.c[1], f.pose.c[2]);
            const float camRadial = finite_nonneg(__fsqrt_rn(dot3(cv, cv)), kMaxDepthValue);
            const uint64_t begin = offsets[i];
            const uint32_t reserved = counts[i];
            const auto put = [&](uint32_t k, uint32_t tile) {
                if (k >= reserved) return;
                keys[begin + k] = (uint64_t(tile) << 32) | tile_depth_key(f.keyMode, mu, Binv, camRadial, tileRays, tile);
                ids[begin + k] = i;
            };
            const uint32_t start = fa.cacheStart[i];
            if (start != kNotCached) {
                for (uint32_t k = lane; k < reserved; k += 32u) put(k, fa.tileCache[start + k]);
            } else {
                fb::warp_tiles(fa.tree, mask, c, lane, stack, put);
            }
        }
    }
}

// Wide projected particles (tile box above kWideTiles): one warp each walks
// the box 32 tiles at a time with the same admission tests as
// for_admitted_tiles, counting (kEmit false) or emitting keys at the scanned
// offsets.  The admitted set is the per-thread walk's; only the order inside
// one particle's keys differs, and the sorted output does not depend on it
// (one particle's keys name distinct tiles).
template <bool kEmit>
__global__ __launch_bounds__(256) void k_wide(FrameArgs f, FallbackArgs fa, const uint8_t* __restrict__ mask,
                                              const float4* __restrict__ proj, const float4* __restrict__ records,
                                              const float4* __restrict__ tileRays, uint32_t* __restrict__ counts,
                                              uint32_t* __restrict__ visibility, const uint64_t* __restrict__ offsets,
                                              uint64_t* __restrict__ keys, uint32_t* __restrict__ ids) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t below = (1u << lane) - 1u;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    if (kEmit && skip_emit(fa)) return;  // block-uniform
    const uint32_t total = *fa.wideCount;
    for (uint32_t w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total; w += warps) {
        const uint32_t i = fa.wide[w];
        const float4 p0 = proj[2 * i], p1 = proj[2 * i + 1];
        Projected p;
        p.cx = p0.x; p.cy = p0.y; p.conic0 = p0.z; p.conic1 = p0.w;
        p.conic2 = p1.x; p.opacity = p1.y; p.ex = p1.z; p.ey = p1.w;
        const TileBox b = tile_bbox(f.gx, f.gy, p.cx, p.cy, p.ex, p.ey);
        const float maxPower = gf_logf(p.opacity / kAlphaThreshold) * 1.0f;
        const int bw = b.x1 - b.x0;
        const uint32_t area = uint32_t(bw * (b.y1 - b.y0));
        V3 mu{};
        float Binv[9] = {};
        float camRadial = 0.0f;
        uint64_t begin = 0;
        uint32_t reserved = 0;
        if constexpr (kEmit) {
            const float4 a = records[4 * size_t(i)], rb = records[4 * size_t(i) + 1], rc = records[4 * size_t(i) + 2],
                         rd = records[4 * size_t(i) + 3];
            mu = v3(a.x, a.y, a.z);
            const float bi[9] = {rb.x, rb.y, rb.z, rb.w, rc.x, rc.y, rc.z, rc.w, rd.x};
#pragma unroll
            for (int k = 0; k < 9; ++k) Binv[k] = bi[k];
            const V3 cv = mu - v3(f.pose.c[0], f.pose.c[1], f.pose.c[2]);
            camRadial = finite_nonneg(__fsqrt_rn(dot3(cv, cv)), kMaxDepthValue);
            begin = offsets[i];
            reserved = counts[i];
        }
        uint32_t n = 0;
        for (uint32_t base = 0; base < area; base += 32u) {
            const uint32_t t = base + lane;
            bool ok = false;
            int x = 0, y = 0;
            if (t < area) {
                x = b.x0 + int(t % uint32_t(bw));
                y = b.y0 + int(t / uint32_t(bw));
                ok = mask[y * f.gx + x] != 0u && tile_min_power(x, y, p) < maxPower;
            }
            const uint32_t m = __ballot_sync(0xffffffffu, ok);
            if constexpr (kEmit) {
                const uint32_t k = n + uint32_t(__popc(m & below));
                if (ok && k < reserved) {
                    const uint32_t tile = uint32_t(y * f.gx + x);
                    keys[begin + k] = (uint64_t(tile) << 32) | tile_depth_key(f.keyMode, mu, Binv, camRadial, tileRays, tile);
                    ids[begin + k] = i;
                }
            }
            n += uint32_t(__popc(m));
        }
        if (!kEmit && lane == 0) {
            counts[i] = n;
            if (visibility != nullptr) visibility[i] = n ? 1u : 0u;
        }
    }
}

// Emits (tile << 32 | depth bits) keys and particle ids at the scanned offsets
// (reference expandTileProjections, gutProjector.cuh:947-1113).
__global__ __launch_bounds__(256) void k_emit(FrameArgs f, const float4* __restrict__ proj,
                                              const float4* __restrict__ records, const uint8_t* __restrict__ mask,
                                              const float4* __restrict__ tileRays, const uint64_t* __restrict__ offsets,
                                              const uint32_t* __restrict__ counts, uint64_t* __restrict__ keys,
                                              uint32_t* __restrict__ ids, FallbackArgs fa) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= f.N || skip_emit(fa)) return;
    const float4 p0 = proj[2 * i], p1 = proj[2 * i + 1];
    Projected p;
    p.cx = p0.x; p.cy = p0.y; p.conic0 = p0.z; p.conic1 = p0.w;
    p.conic2 = p1.x; p.opacity = p1.y; p.ex = p1.z; p.ey = p1.w;
    if (fa.complete || !fast_ut_valid(p)) return;  // cone-route particles: k_fallback_big<true>
    if (wide_box(tile_bbox(f.gx, f.gy, p.cx, p.cy, p.ex, p.ey))) return;  // k_wide<true>
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
// The number of keys is read on the device (nDev, at most n, which sized the grid).
__global__ void k_tile_ranges(const uint64_t* __restrict__ keys, uint32_t n, uint2* __restrict__ ranges,
                              const uint32_t* __restrict__ nDev) {
    if (nDev != nullptr) n = min(n, *nDev);
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t tile = uint32_t(keys[i] >> 32);
    if (i == 0 || uint32_t(keys[i - 1] >> 32) != tile) ranges[tile].x = i;
    if (i == n - 1 || uint32_t(keys[i + 1] >> 32) != tile) ranges[tile].y = i + 1;
}

// Intersection plan of one forward, written after the count scan: the count,
// the fallback list size, whether the count exceeds the key capacity the host
// reserved (then nothing is emitted, sorted or composited, and the host
// reports the overflow), and the count the later kernels use.
struct FramePlan {
    unsigned long long intersections;
    uint32_t fallback;
    uint32_t overflow;
    uint32_t count;  // intersections, or 0 on overflow
    uint32_t pad;
};

__global__ void k_plan_intersections(const uint64_t* __restrict__ total, const uint32_t* __restrict__ fallbackCount,
                                     uint64_t capacity, FramePlan* __restrict__ plan) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const uint64_t I = *total;
    const bool over = I > capacity;
    plan->intersections = I;
    plan->fallback = fallbackCount != nullptr ? *fallbackCount : 0u;
    plan->overflow = over ? 1u : 0u;
    plan->count = over ? 0u : uint32_t(I);
    plan->pad = 0u;
}

// Projection backward: record gradients to the reference's [N,32] density
// gradient and [N,3*C] SH gradient (reference projectBackward,
// gutProjector.cuh:1171-1222; radianceFromSpHBwd, gaussianParticles.cuh:234-310).
// The block's SH rows (3 * shCoeffs floats per particle, contiguous over the
// block's particles) are staged in shared memory, one padded row per thread,
// so that their loads and the SH gradient stores are coalesced; each thread
// reads its row, then overwrites it with the gradient column by column.
constexpr int kProjectBwdThreads = 128;

__host__ __device__ constexpr size_t project_bwd_smem_bytes(uint32_t shCoeffs) {
    return sizeof(float) * kProjectBwdThreads * (3 * size_t(shCoeffs) + 1);
}

__global__ __launch_bounds__(kProjectBwdThreads) void k_project_bwd(FrameArgs f, const float* __restrict__ particles,
                                                                    const float* __restrict__ features,
                                                                    const uint32_t* __restrict__ counts,
                                                                    const float4* __restrict__ gradRecords,
                                                                    const float4* __restrict__ gradShape,
                                                                    const float4* __restrict__ gradIntrinsic,
                                                                    float* __restrict__ gradParticles,
                                                                    float* __restrict__ gradFeatures) {
    extern __shared__ float shRows[];  // [kProjectBwdThreads][3 * shCoeffs + 1]
    const uint32_t rowLen = 3 * f.shCoeffs, pitch = rowLen + 1;
    const uint32_t i0 = blockIdx.x * kProjectBwdThreads;
    const uint32_t blockRows = min(uint32_t(kProjectBwdThreads), f.N - i0);
    const float* src = features + size_t(i0) * rowLen;
    for (uint32_t e = threadIdx.x; e < blockRows * rowLen; e += kProjectBwdThreads) {
        const uint32_t p = e / rowLen;
        shRows[p * pitch + (e - p * rowLen)] = __ldg(src + e);
    }
    __syncthreads();
    const uint32_t i = i0 + threadIdx.x;
    if (i < f.N) {
        float* row = shRows + threadIdx.x * pitch;
        const float4 g0 = gradRecords[4 * size_t(i)], g1 = gradRecords[4 * size_t(i) + 1],
                     g2 = gradRecords[4 * size_t(i) + 2], g3 = gradRecords[4 * size_t(i) + 3];
        float gp0 = g0.x, gp1 = g0.y, gp2 = g0.z;
        float* gs = row;
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
            const float* c = row;
            const float gr[3] = {g3.y, g3.z, g3.w};
            V3 dg = v3(0.0f, 0.0f, 0.0f);
            // unrolled with predicates: the basis arrays stay in registers; column
            // ch of the row is read in full before its gradient overwrites it
    #pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                float acc = basis[0] * c[ch];
    #pragma unroll
                for (int k = 1; k < 16; ++k)
                    if (k < nb) acc = __fmaf_rn(basis[k], c[3 * k + ch], acc);
                const float m = (acc + 0.5f) > 0.0f ? gr[ch] : 0.0f;
    #pragma unroll
                for (int k = 1; k < 16; ++k) {
                    if (k < nb) {
                        const float ck = c[3 * k + ch] * m;
                        dg.x += bx[k] * ck;
                        dg.y += by[k] * ck;
                        dg.z += bz[k] * ck;
                    }
                }
    #pragma unroll
                for (int k = 0; k < 16; ++k)
                    if (k < nb) gs[3 * k + ch] = basis[k] * m;
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
        // rotation and intrinsic scale receive the extent channel's gradient (enable_normals)
        float4 gq = gradShape != nullptr ? gradShape[2 * size_t(i)] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float4 gsc = gradShape != nullptr ? gradShape[2 * size_t(i) + 1] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float gIntrinsicDensity = 0.0f;
        if (gradIntrinsic != nullptr) {
            // the SOF opacity field's gradient of the intrinsic Gaussian
            const float4 i0 = gradIntrinsic[4 * size_t(i)], i1 = gradIntrinsic[4 * size_t(i) + 1],
                         i2 = gradIntrinsic[4 * size_t(i) + 2];
            gp0 += i0.x;
            gp1 += i0.y;
            gp2 += i0.z;
            gIntrinsicDensity = i0.w;
            gq = make_float4(gq.x + i1.x, gq.y + i1.y, gq.z + i1.z, gq.w + i1.w);
            gsc = make_float4(gsc.x + i2.x, gsc.y + i2.y, gsc.z + i2.z, 0.0f);
        }
        out[0] = make_float4(gp0, gp1, gp2, g0.w);                      // pos, density
        out[1] = gq;                                                    // rotation
        out[2] = make_float4(gsc.x, gsc.y, gsc.z, gIntrinsicDensity);   // scale, intrinsic density
        out[3] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);                   // factor 0..3
        out[4] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);                   // factor 4..7
        out[5] = make_float4(0.0f, g1.x, g1.y, g1.z);                   // factor 8 | Binv 0..2
        out[6] = make_float4(g1.w, g2.x, g2.y, g2.z);                   // Binv 3..6
        out[7] = make_float4(g2.w, g3.x, 0.0f, 0.0f);                   // Binv 7..8 | padding
    }
    __syncthreads();
    float* dst = gradFeatures + size_t(i0) * rowLen;
    for (uint32_t e = threadIdx.x; e < blockRows * rowLen; e += kProjectBwdThreads) {
        const uint32_t p = e / rowLen;
        dst[e] = shRows[p * pitch + (e - p * rowLen)];
    }
}

}  // namespace gf
