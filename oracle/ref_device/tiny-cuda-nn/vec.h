// Minimal host stand-in for the small-vector, matrix and quaternion types
// that the reference's camera headers (threedgut_tracer/include/3dgut/sensors/
// cameraModels.h, sensors.h, kernels/cuda/sensors/cameraProjections.cuh) take
// from the tiny-cuda-nn library, which is not vendored in the reference
// checkout.  Written for this test infrastructure from the mathematics of
// each operation (component-wise arithmetic, column-major 3x3 matrices,
// unit quaternions (w, x, y, z)); it reproduces only the interface those
// headers use, so that they compile unmodified with g++ and their projection
// functions run on the host cores to produce golden vectors.
#pragma once

#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include <type_traits>

#ifndef TCNN_HOST_DEVICE
#define TCNN_HOST_DEVICE
#endif

namespace tcnn {

// Storage: named members for 2-4 components (the headers read .x/.y/.z/.w),
// an array otherwise; element i is always ((T*)this)[i].
template <typename T, uint32_t N>
struct tvec_storage {
    T e[N];
};
template <typename T>
struct tvec_storage<T, 2> {
    T x, y;
};
template <typename T>
struct tvec_storage<T, 3> {
    T x, y, z;
};
template <typename T>
struct tvec_storage<T, 4> {
    T x, y, z, w;
};

template <typename T, uint32_t N, size_t A = sizeof(T)>
struct tvec : tvec_storage<T, N> {
    tvec() = default;
    explicit tvec(T s) {
        for (uint32_t i = 0; i < N; ++i) (*this)[i] = s;
    }
    template <typename... Ts, typename = typename std::enable_if<sizeof...(Ts) == N && (N > 1)>::type>
    tvec(Ts... v) {
        const T values[N] = {T(v)...};
        for (uint32_t i = 0; i < N; ++i) (*this)[i] = values[i];
    }
    template <typename U, size_t B>
    tvec(const tvec<U, N, B>& o) {
        for (uint32_t i = 0; i < N; ++i) (*this)[i] = T(o[i]);
    }
    // the leading N components of a longer vector (a 3-vector passed where a
    // 2-vector is expected reads its x and y)
    template <uint32_t M, size_t B, typename = typename std::enable_if<(M > N)>::type>
    tvec(const tvec<T, M, B>& o) {
        for (uint32_t i = 0; i < N; ++i) (*this)[i] = o[i];
    }
    T* data() { return reinterpret_cast<T*>(this); }
    const T* data() const { return reinterpret_cast<const T*>(this); }
    T& operator[](uint32_t i) { return data()[i]; }
    const T& operator[](uint32_t i) const { return data()[i]; }
    static tvec zero() { return tvec(T(0)); }
    tvec<T, 2> xy() const { return tvec<T, 2>((*this)[0], (*this)[1]); }
    // components [O, O + M) as a vector of M, aliasing this one
    template <uint32_t O, uint32_t M>
    tvec<T, M>& slice() {
        return *reinterpret_cast<tvec<T, M>*>(data() + O);
    }
    template <uint32_t O, uint32_t M>
    const tvec<T, M>& slice() const {
        return *reinterpret_cast<const tvec<T, M>*>(data() + O);
    }
    tvec& operator+=(const tvec& o) {
        for (uint32_t i = 0; i < N; ++i) (*this)[i] += o[i];
        return *this;
    }
    tvec& operator+=(T s) {
        for (uint32_t i = 0; i < N; ++i) (*this)[i] += s;
        return *this;
    }
    tvec& operator-=(const tvec& o) {
        for (uint32_t i = 0; i < N; ++i) (*this)[i] -= o[i];
        return *this;
    }
    tvec& operator*=(T s) {
        for (uint32_t i = 0; i < N; ++i) (*this)[i] *= s;
        return *this;
    }
};

#define GF_TCNN_VEC_BINARY(OP)                                                            \
    template <typename T, uint32_t N, size_t A>                                          \
    tvec<T, N, A> operator OP(const tvec<T, N, A>& a, const tvec<T, N, A>& b) {          \
        tvec<T, N, A> r;                                                                  \
        for (uint32_t i = 0; i < N; ++i) r[i] = a[i] OP b[i];                             \
        return r;                                                                         \
    }                                                                                     \
    template <typename T, uint32_t N, size_t A>                                          \
    tvec<T, N, A> operator OP(const tvec<T, N, A>& a, T s) {                             \
        tvec<T, N, A> r;                                                                  \
        for (uint32_t i = 0; i < N; ++i) r[i] = a[i] OP s;                                \
        return r;                                                                         \
    }                                                                                     \
    template <typename T, uint32_t N, size_t A>                                          \
    tvec<T, N, A> operator OP(T s, const tvec<T, N, A>& a) {                             \
        tvec<T, N, A> r;                                                                  \
        for (uint32_t i = 0; i < N; ++i) r[i] = s OP a[i];                                \
        return r;                                                                         \
    }
GF_TCNN_VEC_BINARY(+)
GF_TCNN_VEC_BINARY(-)
GF_TCNN_VEC_BINARY(*)
GF_TCNN_VEC_BINARY(/)
#undef GF_TCNN_VEC_BINARY

template <typename T, uint32_t N, size_t A>
tvec<T, N, A> operator-(const tvec<T, N, A>& a) {
    tvec<T, N, A> r;
    for (uint32_t i = 0; i < N; ++i) r[i] = -a[i];
    return r;
}

// Component-wise min, max, abs, sqrt; Euclidean length; swap.
template <typename T>
T min(T a, T b) { return b < a ? b : a; }
template <typename T>
T max(T a, T b) { return a < b ? b : a; }
template <typename T, uint32_t N, size_t A>
tvec<T, N, A> min(const tvec<T, N, A>& a, const tvec<T, N, A>& b) {
    tvec<T, N, A> r;
    for (uint32_t i = 0; i < N; ++i) r[i] = b[i] < a[i] ? b[i] : a[i];
    return r;
}
template <typename T, uint32_t N, size_t A>
tvec<T, N, A> max(const tvec<T, N, A>& a, const tvec<T, N, A>& b) {
    tvec<T, N, A> r;
    for (uint32_t i = 0; i < N; ++i) r[i] = a[i] < b[i] ? b[i] : a[i];
    return r;
}
template <typename T, uint32_t N, size_t A>
tvec<T, N, A> abs(const tvec<T, N, A>& a) {
    tvec<T, N, A> r;
    for (uint32_t i = 0; i < N; ++i) r[i] = a[i] < T(0) ? -a[i] : a[i];
    return r;
}
template <typename T, uint32_t N, size_t A>
tvec<T, N, A> sqrt(const tvec<T, N, A>& a) {
    tvec<T, N, A> r;
    for (uint32_t i = 0; i < N; ++i) r[i] = ::sqrt(a[i]);
    return r;
}
inline float sqrt(float x) { return ::sqrtf(x); }
template <typename T, uint32_t N, size_t A>
T dot(const tvec<T, N, A>& a, const tvec<T, N, A>& b) {
    T s = a[0] * b[0];
    for (uint32_t i = 1; i < N; ++i) s += a[i] * b[i];
    return s;
}
template <typename T, uint32_t N, size_t A>
T length2(const tvec<T, N, A>& a) {
    T s = T(0);
    for (uint32_t i = 0; i < N; ++i) s += a[i] * a[i];
    return s;
}
template <typename T, uint32_t N, size_t A>
T length(const tvec<T, N, A>& a) {
    return ::sqrt(length2(a));
}
template <typename T, uint32_t N, size_t A>
tvec<T, N, A> normalize(const tvec<T, N, A>& a) {
    return a / length(a);
}
template <typename T>
void host_device_swap(T& a, T& b) {
    T t = a;
    a = b;
    b = t;
}

template <uint32_t N>
using vec = tvec<float, N>;
using vec2 = tvec<float, 2>;
using vec3 = tvec<float, 3>;
using vec4 = tvec<float, 4>;
using ivec2 = tvec<int, 2>;
using uvec2 = tvec<uint32_t, 2>;
using uvec3 = tvec<uint32_t, 3>;

// largest component
template <typename T, uint32_t N, size_t A>
T max(const tvec<T, N, A>& a) {
    T m = a[0];
    for (uint32_t i = 1; i < N; ++i) m = a[i] > m ? a[i] : m;
    return m;
}
template <typename T, uint32_t N, size_t A>
T min(const tvec<T, N, A>& a) {
    T m = a[0];
    for (uint32_t i = 1; i < N; ++i) m = a[i] < m ? a[i] : m;
    return m;
}
template <typename T>
T div_round_up(T a, T b) { return (a + b - 1) / b; }

template <typename T, uint32_t N, size_t A>
tvec<T, N, A> mix(const tvec<T, N, A>& a, const tvec<T, N, A>& b, T t) {
    return a * (T(1) - t) + b * t;
}
template <typename T, uint32_t N, size_t A>
tvec<T, N, A> mix(const tvec<T, N, A>& a, const tvec<T, N, A>& b, const tvec<T, N, A>& t) {
    tvec<T, N, A> r;
    for (uint32_t i = 0; i < N; ++i) r[i] = a[i] * (T(1) - t[i]) + b[i] * t[i];
    return r;
}
template <typename T, uint32_t N, size_t A>
tvec<T, N, A> copysign(const tvec<T, N, A>& a, const tvec<T, N, A>& b) {
    tvec<T, N, A> r;
    for (uint32_t i = 0; i < N; ++i) r[i] = ::copysign(a[i], b[i]);
    return r;
}

// Column-major R x C matrix: m[c] is column c.
template <typename T, uint32_t C, uint32_t R>
struct tmat {
    tvec<T, R> col[C];
    tmat() = default;
    template <typename... Cs, typename = typename std::enable_if<sizeof...(Cs) == C>::type>
    tmat(const Cs&... cs) : col{cs...} {}
    // the leading C columns of a wider matrix (a 4x3 pose's rotation part)
    template <uint32_t C2, typename = typename std::enable_if<(C2 > C)>::type>
    explicit tmat(const tmat<T, C2, R>& o) {
        for (uint32_t c = 0; c < C; ++c) col[c] = o[c];
    }
    tvec<T, R>& operator[](uint32_t c) { return col[c]; }
    const tvec<T, R>& operator[](uint32_t c) const { return col[c]; }
};
using mat3 = tmat<float, 3, 3>;
using mat4x3 = tmat<float, 4, 3>;

template <typename T, uint32_t C, uint32_t R>
tvec<T, R> operator*(const tmat<T, C, R>& m, const tvec<T, C>& v) {
    tvec<T, R> r = tvec<T, R>::zero();
    for (uint32_t c = 0; c < C; ++c)
        for (uint32_t i = 0; i < R; ++i) r[i] += m[c][i] * v[c];
    return r;
}

template <typename T, uint32_t C, uint32_t R>
tmat<T, C, R> operator*(T s, const tmat<T, C, R>& m) {
    tmat<T, C, R> r;
    for (uint32_t c = 0; c < C; ++c) r[c] = s * m[c];
    return r;
}

template <typename T, uint32_t N>
tmat<T, N, N> transpose(const tmat<T, N, N>& m) {
    tmat<T, N, N> t;
    for (uint32_t c = 0; c < N; ++c)
        for (uint32_t r = 0; r < N; ++r) t[c][r] = m[r][c];
    return t;
}

// Unit quaternion w + x i + y j + z k, constructed as {w, x, y, z}.
template <typename T>
struct tquat {
    T x, y, z, w;
    tquat() = default;
    tquat(T w_, T x_, T y_, T z_) : x(x_), y(y_), z(z_), w(w_) {}
    // The quaternion of a rotation matrix (largest-diagonal branch).
    explicit tquat(const tmat<T, 3, 3>& m) {
        const T m00 = m[0][0], m11 = m[1][1], m22 = m[2][2];
        const T trace = m00 + m11 + m22;
        if (trace > T(0)) {
            const T s = T(2) * sqrt(trace + T(1));
            w = T(0.25) * s;
            x = (m[1][2] - m[2][1]) / s;
            y = (m[2][0] - m[0][2]) / s;
            z = (m[0][1] - m[1][0]) / s;
        } else if (m00 > m11 && m00 > m22) {
            const T s = T(2) * sqrt(T(1) + m00 - m11 - m22);
            w = (m[1][2] - m[2][1]) / s;
            x = T(0.25) * s;
            y = (m[1][0] + m[0][1]) / s;
            z = (m[2][0] + m[0][2]) / s;
        } else if (m11 > m22) {
            const T s = T(2) * sqrt(T(1) + m11 - m00 - m22);
            w = (m[2][0] - m[0][2]) / s;
            x = (m[1][0] + m[0][1]) / s;
            y = T(0.25) * s;
            z = (m[2][1] + m[1][2]) / s;
        } else {
            const T s = T(2) * sqrt(T(1) + m22 - m00 - m11);
            w = (m[0][1] - m[1][0]) / s;
            x = (m[2][0] + m[0][2]) / s;
            y = (m[2][1] + m[1][2]) / s;
            z = T(0.25) * s;
        }
    }
};
using quat = tquat<float>;

// Rotation matrix of a unit quaternion (columns are the rotated axes).
template <typename T>
tmat<T, 3, 3> to_mat3(const tquat<T>& q) {
    const T x = q.x, y = q.y, z = q.z, w = q.w;
    tmat<T, 3, 3> m;
    m[0] = tvec<T, 3>(T(1) - T(2) * (y * y + z * z), T(2) * (x * y + w * z), T(2) * (x * z - w * y));
    m[1] = tvec<T, 3>(T(2) * (x * y - w * z), T(1) - T(2) * (x * x + z * z), T(2) * (y * z + w * x));
    m[2] = tvec<T, 3>(T(2) * (x * z + w * y), T(2) * (y * z - w * x), T(1) - T(2) * (x * x + y * y));
    return m;
}

// Spherical linear interpolation along the shorter arc.
template <typename T>
tquat<T> slerp(const tquat<T>& a, tquat<T> b, T t) {
    T d = a.w * b.w + a.x * b.x + a.y * b.y + a.z * b.z;
    if (d < T(0)) {
        b = tquat<T>(-b.w, -b.x, -b.y, -b.z);
        d = -d;
    }
    T s0 = T(1) - t, s1 = t;
    if (d < T(0.9995)) {
        const T theta = acos(d);
        const T sn = sin(theta);
        s0 = sin((T(1) - t) * theta) / sn;
        s1 = sin(t * theta) / sn;
    }
    return tquat<T>(s0 * a.w + s1 * b.w, s0 * a.x + s1 * b.x, s0 * a.y + s1 * b.y, s0 * a.z + s1 * b.z);
}

}  // namespace tcnn
