// Host stand-ins for the CUDA built-ins used by the reference's per-hit
// device headers (threedgut_tracer/include/3dgut/kernels/cuda/models and
// common), so that those headers compile with g++ and run on the host cores.
// Test infrastructure only: it builds the golden-vector generator that pins
// the oracle's per-hit forward and backward to the reference's own code.
//
// Semantics: IEEE float arithmetic with no contraction (built with
// -ffp-contract=off), the C library's expf/logf/sqrtf, plain (non-atomic)
// read-modify-write for the atomics, which is exact for a single host thread.
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <cfloat>
#include <cfenv>
#include <cmath>
#include <limits>

#include "math_constants.h"

#define __device__
#define __host__
#define __global__
#define __forceinline__ inline
#define __inline__ inline
#define __restrict__
// mathUtils.cuh includes its float2/float3 operator header only under nvcc.
#ifndef __CUDACC__
#define __CUDACC__ 1
#endif

struct float2 { float x, y; };
struct float3 { float x, y, z; };
struct float4 { float x, y, z, w; };
struct int2 { int x, y; };
struct int3 { int x, y, z; };
struct uint2 { unsigned x, y; };
struct uint3 { unsigned x, y, z; };

// The launch built-ins, as host variables a driver sets before calling
// device code that reads them (one thread at a time).
struct dim3 {
    unsigned x = 0, y = 0, z = 0;
};
inline dim3 threadIdx, blockIdx, blockDim, gridDim;
constexpr int warpSize = 32;
#define __shared__ static
#define __constant__ static

// Block and warp intrinsics: declared only (a call would fail to link), so
// that the reference's kernel templates parse; the block barrier is a no-op
// for the one host thread.
inline void __syncthreads() {}  // one host thread: nothing to wait for
int __syncthreads_and(int);
int __syncthreads_or(int);
int __syncthreads_count(int);
void __syncwarp(unsigned = 0xffffffffu);
int __all_sync(unsigned, int);
int __any_sync(unsigned, int);
unsigned __ballot_sync(unsigned, int);
unsigned __activemask();
template <typename T> T __shfl_sync(unsigned, T, int, int = 32);
template <typename T> T __shfl_up_sync(unsigned, T, unsigned, int = 32);
template <typename T> T __shfl_down_sync(unsigned, T, unsigned, int = 32);
template <typename T> T __shfl_xor_sync(unsigned, T, int, int = 32);
template <typename T> unsigned __match_any_sync(unsigned, T);
int __ffs(int);
int __popc(unsigned);
int __clz(int);
using std::max;
using std::min;
// the mixed-sign integer overloads of the CUDA math header
inline unsigned min(unsigned a, int b) { return a < unsigned(b) ? a : unsigned(b); }
inline unsigned min(int a, unsigned b) { return unsigned(a) < b ? unsigned(a) : b; }
inline unsigned max(unsigned a, int b) { return a > unsigned(b) ? a : unsigned(b); }
inline unsigned max(int a, unsigned b) { return unsigned(a) > b ? unsigned(a) : b; }

// Directed-rounding arithmetic (the certified-admission headers' interval
// bounds): the operation evaluated under the requested rounding mode of the
// host FPU (built with -frounding-math).  The host drivers do not call the
// certified paths; their kernels, which the host build compiles as ordinary
// functions, reference these.
#define GF_SHIM_DIRECTED2(T, NAME, MODE, OP)                 \
    inline T NAME(T a, T b) {                                 \
        const int saved = std::fegetround();                  \
        std::fesetround(MODE);                                \
        volatile T r = a OP b;                                \
        std::fesetround(saved);                               \
        return r;                                             \
    }
#define GF_SHIM_DIRECTED_SET(SUFFIX, MODE)                    \
    GF_SHIM_DIRECTED2(double, __dadd_##SUFFIX, MODE, +)       \
    GF_SHIM_DIRECTED2(double, __dsub_##SUFFIX, MODE, -)       \
    GF_SHIM_DIRECTED2(double, __dmul_##SUFFIX, MODE, *)       \
    GF_SHIM_DIRECTED2(double, __ddiv_##SUFFIX, MODE, /)       \
    GF_SHIM_DIRECTED2(float, __fadd_##SUFFIX, MODE, +)        \
    GF_SHIM_DIRECTED2(float, __fsub_##SUFFIX, MODE, -)        \
    GF_SHIM_DIRECTED2(float, __fmul_##SUFFIX, MODE, *)        \
    GF_SHIM_DIRECTED2(float, __fdiv_##SUFFIX, MODE, /)        \
    inline double __dsqrt_##SUFFIX(double a) {               \
        const int saved = std::fegetround();                  \
        std::fesetround(MODE);                                \
        volatile double r = std::sqrt(a);                     \
        std::fesetround(saved);                               \
        return r;                                             \
    }                                                         \
    inline float __fsqrt_##SUFFIX(float a) {                  \
        const int saved = std::fegetround();                  \
        std::fesetround(MODE);                                \
        volatile float r = std::sqrt(a);                      \
        std::fesetround(saved);                               \
        return r;                                             \
    }                                                         \
    inline float __double2float_##SUFFIX(double a) {          \
        const int saved = std::fegetround();                  \
        std::fesetround(MODE);                                \
        volatile float r = float(a);                          \
        std::fesetround(saved);                               \
        return r;                                             \
    }                                                         \
    inline float __frcp_##SUFFIX(float a) { return __fdiv_##SUFFIX(1.0f, a); }
GF_SHIM_DIRECTED_SET(rd, FE_DOWNWARD)
GF_SHIM_DIRECTED_SET(ru, FE_UPWARD)
GF_SHIM_DIRECTED_SET(rz, FE_TOWARDZERO)
GF_SHIM_DIRECTED_SET(rn, FE_TONEAREST)
#undef GF_SHIM_DIRECTED_SET
#undef GF_SHIM_DIRECTED2


inline float2 make_float2(float x, float y) { return {x, y}; }
inline float3 make_float3(float x, float y, float z) { return {x, y, z}; }
inline float4 make_float4(float x, float y, float z, float w) { return {x, y, z, w}; }
inline float2 make_float2(float s) { return {s, s}; }
inline float3 make_float3(float s) { return {s, s, s}; }
inline float4 make_float4(float s) { return {s, s, s, s}; }
inline int2 make_int2(int x, int y) { return {x, y}; }
inline uint2 make_uint2(unsigned x, unsigned y) { return {x, y}; }

// Component-wise vector-vector arithmetic, negation and the scalar
// broadcasting constructors, which the reference headers take from the
// vector helper header of their CUDA build; the scalar and compound forms and
// float4 addition come from the reference's own mathUtils.cuh / cudaMath.cuh.
#define GF_SHIM_BINARY(T, OP)                                                     \
    inline T operator OP(const T& a, const T& b) {                               \
        T r;                                                                      \
        float* rp = &r.x;                                                         \
        const float* ap = &a.x;                                                   \
        const float* bp = &b.x;                                                   \
        for (unsigned i = 0; i < sizeof(T) / sizeof(float); ++i) rp[i] = ap[i] OP bp[i]; \
        return r;                                                                 \
    }
#define GF_SHIM_VECTOR(T)                                                         \
    GF_SHIM_BINARY(T, +)                                                          \
    GF_SHIM_BINARY(T, -)                                                          \
    GF_SHIM_BINARY(T, *)                                                          \
    GF_SHIM_BINARY(T, /)                                                          \
    inline T operator-(const T& a) {                                              \
        T r;                                                                      \
        float* rp = &r.x;                                                         \
        const float* ap = &a.x;                                                   \
        for (unsigned i = 0; i < sizeof(T) / sizeof(float); ++i) rp[i] = -ap[i];  \
        return r;                                                                 \
    }
GF_SHIM_VECTOR(float2)
GF_SHIM_VECTOR(float3)
GF_SHIM_BINARY(float4, -)
GF_SHIM_BINARY(float4, *)
GF_SHIM_BINARY(float4, /)
#undef GF_SHIM_VECTOR
#undef GF_SHIM_BINARY

// __saturatef: clamp to [0, 1]; NaN maps to 0.
inline float __saturatef(float x) { return (x > 0.0f) ? (x < 1.0f ? x : 1.0f) : 0.0f; }
inline float rsqrtf(float x) { return 1.0f / sqrtf(x); }

inline int __float_as_int(float f) { int i; memcpy(&i, &f, 4); return i; }
inline unsigned __float_as_uint(float f) { unsigned i; memcpy(&i, &f, 4); return i; }
inline float __int_as_float(int i) { float f; memcpy(&f, &i, 4); return f; }
inline float __uint_as_float(unsigned i) { float f; memcpy(&f, &i, 4); return f; }

template <typename T>
inline T atomicAdd(T* address, T value) { const T old = *address; *address = old + value; return old; }
template <typename T>
inline T atomicAnd(T* address, T value) { const T old = *address; *address = old & value; return old; }
template <typename T>
inline T atomicOr(T* address, T value) { const T old = *address; *address = old | value; return old; }
template <typename T>
inline T atomicExch(T* address, T value) { const T old = *address; *address = value; return old; }
template <typename T>
inline T atomicMax(T* address, T value) { const T old = *address; *address = std::max(old, value); return old; }
template <typename T>
inline T atomicMin(T* address, T value) { const T old = *address; *address = std::min(old, value); return old; }
