// Marching tetrahedra and mesh filters of the mesh extraction on sm_100a
// (reference gofish/mesh/marching_tetrahedra.py:47-140, GOF's variant of
// Kaolin's marching tetrahedra that returns crossing-edge endpoints instead
// of interpolated vertices, and gofish/mesh/filters.py:15-58).
//
// Marching tetrahedra, as a pipeline of data-parallel passes:
//   1. classify: per tetrahedron the inside code (bit k: sdf[v_k] > 0), the
//      active flag (1-3 inside) and the triangle count of its code;
//   2. scan of the active flags; every active tetrahedron emits its six
//      (min << b | max) edge keys with the slot 6 * active + edge;
//   3. stable radix sort of the keys, head flags and a scan number the
//      distinct edges in lexicographic order; the crossing ones (one inside
//      endpoint) are numbered by a second scan and every slot learns its
//      crossing number (-1 otherwise);
//   4. the crossing edges write their endpoints, fields and scales; every
//      active tetrahedron writes its one or two faces from the case table at
//      a position fixed by the reference's order: chunk by chunk (ceil(T / n)
//      tetrahedra, n = T / chunk + 1 chunks when T exceeds the chunk size),
//      the one-triangle tetrahedra in order, then the two-triangle ones.
// Two host reads size the work (the active count) and the outputs (edges,
// faces).  Filters: SOF's vertex filter per crossing edge, GOF's cell filter
// per tetrahedron (six edges), each one thread per item.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/gofish_b200.h"
#include "gf_host.cuh"

namespace {

// Case table of marching tetrahedra: triangles of the 16 inside/outside
// codes as local edge indices over the edges (0-1, 0-2, 0-3, 1-2, 1-3, 2-3);
// it fixes the faces' order and winding, so it is the reference's table.
__constant__ int8_t kTriTable[16][6] = {
    {-1, -1, -1, -1, -1, -1}, {1, 0, 2, -1, -1, -1}, {4, 0, 3, -1, -1, -1}, {1, 4, 2, 1, 3, 4},
    {3, 1, 5, -1, -1, -1},    {2, 3, 0, 2, 5, 3},    {1, 4, 0, 1, 5, 4},    {4, 2, 5, -1, -1, -1},
    {4, 5, 2, -1, -1, -1},    {4, 1, 0, 4, 5, 1},    {3, 2, 0, 3, 5, 2},    {1, 3, 5, -1, -1, -1},
    {4, 1, 2, 4, 3, 1},       {3, 0, 4, -1, -1, -1}, {2, 0, 1, -1, -1, -1}, {-1, -1, -1, -1, -1, -1}};
__constant__ int8_t kTriCount[16] = {0, 1, 1, 2, 1, 2, 2, 1, 1, 2, 2, 1, 2, 1, 1, 0};
__constant__ int8_t kTetEdge[6][2] = {{0, 1}, {0, 2}, {0, 3}, {1, 2}, {1, 3}, {2, 3}};

__global__ void k_mt_classify(const int64_t* __restrict__ tets, uint64_t T, const float* __restrict__ sdf,
                              uint64_t V, uint8_t* __restrict__ code, uint32_t* __restrict__ active,
                              uint32_t* __restrict__ one, uint32_t* __restrict__ two, uint32_t* __restrict__ err) {
    const uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= T) return;
    uint32_t c = 0;
    for (int k = 0; k < 4; ++k) {
        const int64_t v = tets[4 * t + k];
        if (v < 0 || uint64_t(v) >= V) {
            atomicOr(err, 1u);
            c = 0;
            break;
        }
        c |= (sdf[v] > 0.0f ? 1u : 0u) << k;
    }
    const int n = kTriCount[c];
    code[t] = uint8_t(c);
    active[t] = n > 0 ? 1u : 0u;
    one[t] = n == 1 ? 1u : 0u;
    two[t] = n == 2 ? 1u : 0u;
}

__global__ void k_mt_emit_edges(const int64_t* __restrict__ tets, uint64_t T, const uint32_t* __restrict__ active,
                                const uint32_t* __restrict__ activeOffset, int bits, uint64_t* __restrict__ keys,
                                uint32_t* __restrict__ slots) {
    const uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= T || active[t] == 0u) return;
    const uint32_t a = activeOffset[t];
    for (int e = 0; e < 6; ++e) {
        const uint64_t p = uint64_t(tets[4 * t + kTetEdge[e][0]]), q = uint64_t(tets[4 * t + kTetEdge[e][1]]);
        const uint64_t lo = p < q ? p : q, hi = p < q ? q : p;
        keys[6 * size_t(a) + e] = (lo << bits) | hi;
        slots[6 * size_t(a) + e] = 6u * a + uint32_t(e);
    }
}

__global__ void k_mt_heads(const uint64_t* __restrict__ keys, uint32_t n, uint32_t* __restrict__ head) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) head[i] = (i == 0 || keys[i] != keys[i - 1]) ? 1u : 0u;
}

// Per distinct edge (at its head): the crossing flag.
__global__ void k_mt_crossing(const uint64_t* __restrict__ keys, uint32_t n, const uint32_t* __restrict__ head,
                              const uint32_t* __restrict__ headOffset, int bits, const float* __restrict__ sdf,
                              uint32_t* __restrict__ crossing, uint64_t* __restrict__ uniqueKey) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || head[i] == 0u) return;
    const uint64_t k = keys[i];
    const uint64_t lo = k >> bits, hi = k & ((uint64_t(1) << bits) - 1);
    const uint32_t u = headOffset[i];
    crossing[u] = ((sdf[lo] > 0.0f) != (sdf[hi] > 0.0f)) ? 1u : 0u;
    uniqueKey[u] = k;
}

// Crossing number of every slot (-1 for a non-crossing edge).
__global__ void k_mt_slot_numbers(const uint32_t* __restrict__ slots, uint32_t n, const uint32_t* __restrict__ head,
                                  const uint32_t* __restrict__ headOffset, const uint32_t* __restrict__ crossing,
                                  const uint32_t* __restrict__ crossOffset, int32_t* __restrict__ slotNumber) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t u = headOffset[i] + head[i] - 1u;  // distinct-edge index of sorted position i
    slotNumber[slots[i]] = crossing[u] ? int32_t(crossOffset[u]) : -1;
}

__global__ void k_mt_edge_outputs(const uint64_t* __restrict__ uniqueKey, uint32_t U,
                                  const uint32_t* __restrict__ crossing, const uint32_t* __restrict__ crossOffset,
                                  int bits, const float* __restrict__ vertices, const float* __restrict__ sdf,
                                  const float* __restrict__ scales, float* __restrict__ endpoints,
                                  float* __restrict__ endpointFields, float* __restrict__ endpointScales,
                                  int64_t* __restrict__ edges) {
    const uint32_t u = blockIdx.x * blockDim.x + threadIdx.x;
    if (u >= U || crossing[u] == 0u) return;
    const uint32_t f = crossOffset[u];
    const uint64_t k = uniqueKey[u];
    const uint64_t v[2] = {k >> bits, k & ((uint64_t(1) << bits) - 1)};
    for (int j = 0; j < 2; ++j) {
        edges[2 * size_t(f) + j] = int64_t(v[j]);
        for (int c = 0; c < 3; ++c) endpoints[6 * size_t(f) + 3 * j + c] = vertices[3 * v[j] + c];
        endpointFields[2 * size_t(f) + j] = sdf[v[j]];
        endpointScales[2 * size_t(f) + j] = scales[v[j]];
    }
}

// Faces of every active tetrahedron at the reference's position.  s1 / s2:
// exclusive scans (T + 1 entries) of the one- and two-triangle flags.
__global__ void k_mt_faces(const uint8_t* __restrict__ code, uint64_t T, const uint32_t* __restrict__ active,
                           const uint32_t* __restrict__ activeOffset, const uint32_t* __restrict__ s1,
                           const uint32_t* __restrict__ s2, uint64_t chunk, const int32_t* __restrict__ slotNumber,
                           int64_t* __restrict__ faces) {
    const uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= T || active[t] == 0u) return;
    const uint32_t c = code[t];
    const int n = kTriCount[c];
    const uint64_t cs = (t / chunk) * chunk;
    const uint64_t ce = cs + chunk < T ? cs + chunk : T;
    const uint64_t base = uint64_t(s1[cs]) + 2ull * s2[cs];
    uint64_t pos;
    if (n == 1) pos = base + (s1[t] - s1[cs]);
    else pos = base + (s1[ce] - s1[cs]) + 2ull * (s2[t] - s2[cs]);
    const uint32_t a = activeOffset[t];
    for (int k = 0; k < 3 * n; ++k) faces[3 * pos + k] = int64_t(slotNumber[6 * size_t(a) + kTriTable[c][k]]);
}

__global__ void k_sof_vertex_filter(const float* __restrict__ points, const float* __restrict__ scale,
                                    const int64_t* __restrict__ edges, uint64_t E, uint8_t* __restrict__ keep) {
    const uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= E) return;
    const int64_t a = edges[2 * e], b = edges[2 * e + 1];
    const float dx = points[3 * a] - points[3 * b], dy = points[3 * a + 1] - points[3 * b + 1],
                dz = points[3 * a + 2] - points[3 * b + 2];
    const float dist = sqrtf((dx * dx + dy * dy) + dz * dz);
    keep[e] = dist <= scale[a] + scale[b] ? 1u : 0u;
}

__global__ void k_gof_cell_filter(const int64_t* __restrict__ cells, uint64_t T, const float* __restrict__ points,
                                  const float* __restrict__ scale, const int64_t* __restrict__ owner,
                                  uint8_t* __restrict__ keep) {
    const uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= T) return;
    bool ok = true;
    for (int e = 0; e < 6 && ok; ++e) {
        const int64_t a = cells[4 * t + kTetEdge[e][0]], b = cells[4 * t + kTetEdge[e][1]];
        const float dx = points[3 * a] - points[3 * b], dy = points[3 * a + 1] - points[3 * b + 1],
                    dz = points[3 * a + 2] - points[3 * b + 2];
        const float dist = sqrtf((dx * dx + dy * dy) + dz * dz);
        if (owner[a] != owner[b] && dist > scale[a] + scale[b]) ok = false;
    }
    keep[t] = ok ? 1u : 0u;
}

uint32_t bits_for(uint64_t v) {
    uint32_t b = 1;
    while ((uint64_t(1) << b) < v) ++b;
    return b;
}

}  // namespace

struct gf_mesh_mt {
    DeviceBuffer code, active, one, two, activeOffset, s1, s2, keys[2], slots[2], hist, scanTiles, head, headOffset,
        crossing, crossOffset, uniqueKey, slotNumber, err;
    uint32_t* host = nullptr;  // pinned [4]
    uint64_t T = 0, V = 0, chunk = 0, edges = 0, faces = 0;
    uint32_t uniqueCount = 0, activeCount = 0;
    int finalBuf = 0, bits = 0;
    const float* vertices = nullptr;
    const float* sdf = nullptr;
    const float* scales = nullptr;
};

extern "C" {

gf_mesh_mt* gf_mesh_mt_create(void) { return new gf_mesh_mt(); }

void gf_mesh_mt_destroy(gf_mesh_mt* m) {
    if (m == nullptr) return;
    cudaDeviceSynchronize();
    DeviceBuffer* bufs[] = {&m->code, &m->active, &m->one, &m->two, &m->activeOffset, &m->s1, &m->s2,
                            &m->keys[0], &m->keys[1], &m->slots[0], &m->slots[1], &m->hist, &m->scanTiles,
                            &m->head, &m->headOffset, &m->crossing, &m->crossOffset, &m->uniqueKey,
                            &m->slotNumber, &m->err};
    for (DeviceBuffer* b : bufs) b->release();
    if (m->host != nullptr) cudaFreeHost(m->host);
    delete m;
}

int gf_mesh_mt_run(gf_mesh_mt* m, const float* vertices, uint64_t num_vertices, const int64_t* tets,
                   uint64_t num_tets, const float* sdf, const float* scales, uint64_t chunk_tets, uint64_t* num_edges,
                   uint64_t* num_faces, void* stream) {
    if (m == nullptr || num_edges == nullptr || num_faces == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL argument");
    if (num_tets > 0 && (vertices == nullptr || tets == nullptr || sdf == nullptr || scales == nullptr))
        return fail(GF_ERR_BAD_INPUT, "NULL input");
    if (num_vertices >= (uint64_t(1) << 31) || num_tets >= (uint64_t(1) << 31) / 6)
        return fail(GF_ERR_CAPACITY, "grid too large for 32-bit edge slots");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (m->host == nullptr) GF_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&m->host), 4 * sizeof(uint32_t), 0));
    const uint64_t T = num_tets, V = num_vertices;
    m->T = T;
    m->V = V;
    m->vertices = vertices;
    m->sdf = sdf;
    m->scales = scales;
    m->edges = m->faces = 0;
    m->uniqueCount = m->activeCount = 0;
    // the reference's chunking: n = T // chunk + 1 chunks of ceil(T / n) when T exceeds the chunk
    const uint64_t chunk = chunk_tets == 0 ? (uint64_t(32) << 20) : chunk_tets;
    m->chunk = T <= chunk ? (T > 0 ? T : 1) : (T + (T / chunk + 1) - 1) / (T / chunk + 1);
    *num_edges = *num_faces = 0;
    if (T == 0) return GF_OK;
    uint32_t launches = 0;
    if (int e = m->code.ensure(T, s)) return e;
    for (DeviceBuffer* b : {&m->active, &m->one, &m->two})
        if (int e = b->ensure(sizeof(uint32_t) * T, s)) return e;
    for (DeviceBuffer* b : {&m->activeOffset, &m->s1, &m->s2})
        if (int e = b->ensure(sizeof(uint32_t) * (T + 1), s)) return e;
    if (int e = m->err.ensure(sizeof(uint32_t), s)) return e;
    GF_CUDA(cudaMemsetAsync(m->err.ptr, 0, sizeof(uint32_t), s));
    const uint32_t blocks = uint32_t((T + 255) / 256);
    k_mt_classify<<<blocks, 256, 0, s>>>(tets, T, sdf, V, m->code.as<uint8_t>(), m->active.as<uint32_t>(),
                                         m->one.as<uint32_t>(), m->two.as<uint32_t>(), m->err.as<uint32_t>());
    GF_LAUNCH_CHECK();
    uint32_t* ao = m->activeOffset.as<uint32_t>();
    if (int e = scan_exclusive<uint32_t, uint32_t>(m->scanTiles, launches, m->active.as<uint32_t>(), T, ao, ao + T, s))
        return e;
    if (int e = scan_exclusive<uint32_t, uint32_t>(m->scanTiles, launches, m->one.as<uint32_t>(), T,
                                                   m->s1.as<uint32_t>(), m->s1.as<uint32_t>() + T, s))
        return e;
    if (int e = scan_exclusive<uint32_t, uint32_t>(m->scanTiles, launches, m->two.as<uint32_t>(), T,
                                                   m->s2.as<uint32_t>(), m->s2.as<uint32_t>() + T, s))
        return e;
    GF_CUDA(cudaMemcpyAsync(m->host, ao + T, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    GF_CUDA(cudaMemcpyAsync(m->host + 1, m->err.ptr, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    GF_CUDA(cudaStreamSynchronize(s));
    if (m->host[1] != 0u) return fail(GF_ERR_BAD_INPUT, "a tetrahedron names a vertex outside [0, %llu)",
                                      static_cast<unsigned long long>(V));
    const uint32_t A = m->host[0];
    m->activeCount = A;
    if (A == 0) return GF_OK;
    const uint32_t n = 6u * A;
    m->bits = int(bits_for(V));
    for (int b = 0; b < 2; ++b) {
        if (int e = m->keys[b].ensure(sizeof(uint64_t) * (size_t(n) + 1), s)) return e;
        if (int e = m->slots[b].ensure(sizeof(uint32_t) * (size_t(n) + 1), s)) return e;
    }
    k_mt_emit_edges<<<blocks, 256, 0, s>>>(tets, T, m->active.as<uint32_t>(), ao, m->bits, m->keys[0].as<uint64_t>(),
                                           m->slots[0].as<uint32_t>());
    GF_LAUNCH_CHECK();
    if (int e = sort_pairs(m->hist, m->scanTiles, launches, m->keys, m->slots, n, 0, 2 * m->bits, &m->finalBuf, s))
        return e;
    const uint64_t* sk = m->keys[m->finalBuf].as<uint64_t>();
    const uint32_t* ss = m->slots[m->finalBuf].as<uint32_t>();
    for (DeviceBuffer* b : {&m->head, &m->crossing})
        if (int e = b->ensure(sizeof(uint32_t) * n, s)) return e;
    for (DeviceBuffer* b : {&m->headOffset, &m->crossOffset})
        if (int e = b->ensure(sizeof(uint32_t) * (size_t(n) + 1), s)) return e;
    if (int e = m->uniqueKey.ensure(sizeof(uint64_t) * n, s)) return e;
    if (int e = m->slotNumber.ensure(sizeof(int32_t) * n, s)) return e;
    const uint32_t nb = (n + 255) / 256;
    k_mt_heads<<<nb, 256, 0, s>>>(sk, n, m->head.as<uint32_t>());
    GF_LAUNCH_CHECK();
    uint32_t* ho = m->headOffset.as<uint32_t>();
    if (int e = scan_exclusive<uint32_t, uint32_t>(m->scanTiles, launches, m->head.as<uint32_t>(), n, ho, ho + n, s))
        return e;
    GF_CUDA(cudaMemsetAsync(m->crossing.ptr, 0, sizeof(uint32_t) * n, s));
    k_mt_crossing<<<nb, 256, 0, s>>>(sk, n, m->head.as<uint32_t>(), ho, m->bits, sdf, m->crossing.as<uint32_t>(),
                                     m->uniqueKey.as<uint64_t>());
    GF_LAUNCH_CHECK();
    // the crossing numbering runs over all n slots of the flag array; entries
    // past the distinct-edge count are zero and do not move the totals
    uint32_t* co = m->crossOffset.as<uint32_t>();
    if (int e = scan_exclusive<uint32_t, uint32_t>(m->scanTiles, launches, m->crossing.as<uint32_t>(), n, co, co + n,
                                                   s))
        return e;
    k_mt_slot_numbers<<<nb, 256, 0, s>>>(ss, n, m->head.as<uint32_t>(), ho, m->crossing.as<uint32_t>(), co,
                                         m->slotNumber.as<int32_t>());
    GF_LAUNCH_CHECK();
    GF_CUDA(cudaMemcpyAsync(m->host, ho + n, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    GF_CUDA(cudaMemcpyAsync(m->host + 1, co + n, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    GF_CUDA(cudaMemcpyAsync(m->host + 2, m->s1.as<uint32_t>() + T, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    GF_CUDA(cudaMemcpyAsync(m->host + 3, m->s2.as<uint32_t>() + T, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    GF_CUDA(cudaStreamSynchronize(s));
    m->uniqueCount = m->host[0];
    m->edges = m->host[1];
    m->faces = uint64_t(m->host[2]) + 2ull * m->host[3];
    *num_edges = m->edges;
    *num_faces = m->faces;
    return GF_OK;
}

int gf_mesh_mt_outputs(gf_mesh_mt* m, float* endpoints, float* endpoint_fields, float* endpoint_scales,
                       int64_t* faces, int64_t* edges, void* stream) {
    if (m == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL argument");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (m->edges > 0) {
        if (endpoints == nullptr || endpoint_fields == nullptr || endpoint_scales == nullptr || edges == nullptr)
            return fail(GF_ERR_BAD_INPUT, "NULL edge output");
        k_mt_edge_outputs<<<(m->uniqueCount + 255) / 256, 256, 0, s>>>(
            m->uniqueKey.as<uint64_t>(), m->uniqueCount, m->crossing.as<uint32_t>(), m->crossOffset.as<uint32_t>(),
            m->bits, m->vertices, m->sdf, m->scales, endpoints, endpoint_fields, endpoint_scales, edges);
        GF_LAUNCH_CHECK();
    }
    if (m->faces > 0) {
        if (faces == nullptr) return fail(GF_ERR_BAD_INPUT, "NULL face output");
        k_mt_faces<<<uint32_t((m->T + 255) / 256), 256, 0, s>>>(
            m->code.as<uint8_t>(), m->T, m->active.as<uint32_t>(), m->activeOffset.as<uint32_t>(),
            m->s1.as<uint32_t>(), m->s2.as<uint32_t>(), m->chunk, m->slotNumber.as<int32_t>(), faces);
        GF_LAUNCH_CHECK();
    }
    return GF_OK;
}

int gf_mesh_sof_vertex_filter(const float* points, const float* scale, const int64_t* edges, uint64_t num_edges,
                              uint8_t* keep, void* stream) {
    if (num_edges == 0) return GF_OK;
    if (points == nullptr || scale == nullptr || edges == nullptr || keep == nullptr)
        return fail(GF_ERR_BAD_INPUT, "NULL argument");
    k_sof_vertex_filter<<<uint32_t((num_edges + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        points, scale, edges, num_edges, keep);
    GF_LAUNCH_CHECK();
    return GF_OK;
}

int gf_mesh_gof_cell_filter(const int64_t* cells, uint64_t num_cells, const float* points, const float* scale,
                            const int64_t* owner, uint8_t* keep, void* stream) {
    if (num_cells == 0) return GF_OK;
    if (cells == nullptr || points == nullptr || scale == nullptr || owner == nullptr || keep == nullptr)
        return fail(GF_ERR_BAD_INPUT, "NULL argument");
    k_gof_cell_filter<<<uint32_t((num_cells + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        cells, num_cells, points, scale, owner, keep);
    GF_LAUNCH_CHECK();
    return GF_OK;
}

}  // extern "C"
