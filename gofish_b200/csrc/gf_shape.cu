// Per-view full-shape operator on sm_100a (reference
// threedgut_tracer/view_observation_filter.py:64-330 current_view_q6,
// footprint_shape_operator.py + src/footprint_shape_operator_cuda.cu, and the
// fused inference kernel src/fast_shape.cu).
//
// For one camera view and every Gaussian: the world pixel Jacobian J (float64,
// rounded to float32 as the reference's operator receives it), the
// minimum-norm footprint Q = gamma J^+ J^+^T (column-pivoted modified
// Gram-Schmidt of J^T with one reorthogonalization), C = R S^2 R^T + Q, and
//   exact mode:    B = C^{1/2} R, B^-1 = R^T C^{-1/2}, from a 3x3 cyclic
//                  Jacobi eigendecomposition in float64 (no cuSOLVER, no
//                  float32/float64 escalation split: every row is float64);
//   cholesky mode: B = L (C = L L^T), B^-1 = L^-1, as the fused inference
//                  kernel does;
// the mass-preserving factor m = sqrt(det S0 / det(S0 + gamma I)),
// S0 = (J R S)(J R S)^T, and density' = m * density.  Rows the camera does
// not observe keep B = R S, B^-1 = S^-1 R^T, m = 1.  The VJP to (scale,
// quaternion, density) recomputes the forward state of each row instead of
// storing it, and uses the divided-difference form of the derivative of a
// symmetric matrix function: for f(C) = V f(L) V^T, dL/dC = V ((V^T G V) o K)
// V^T with K_ij = 1/(r_i + r_j) for the root and -1/(r_i r_j (r_i + r_j)) for
// the inverse root (r = sqrt of the eigenvalues), finite for repeated
// eigenvalues.  One thread per row, float64 throughout, no contraction.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "../../include/gofish_b200.h"
#include "gf_elementary.h"

int gf_record_error(int code, const char* message);

namespace {

constexpr int kThreads = 128;

struct Cam {
    double R[9];  // camera-to-world rotation, row-major
    double c[3];
    double fx, fy, k[4], maxAngle;
    int fisheye;
};

enum Status : int {
    kNotSpd = 1,            // C not strictly positive definite in float64
    kBadCompensation = 2,   // det(J Sigma J^T) not positive
    kNonFinite = 4,         // a non-finite output
};

__device__ __forceinline__ void record(int* status, unsigned long long* firstRow, int bit, int64_t row) {
    if (status == nullptr) return;
    atomicOr(status, bit);
    atomicMin(firstRow, static_cast<unsigned long long>(row));
}

// World pixel Jacobian rounded to float32, and the camera-chart validity
// (view_observation_filter.py:200-330).
__device__ bool view_jacobian(const Cam& cam, const float* p, float J[6]) {
    const double d0 = double(p[0]) - cam.c[0], d1 = double(p[1]) - cam.c[1], d2 = double(p[2]) - cam.c[2];
    const double x = d0 * cam.R[0] + d1 * cam.R[3] + d2 * cam.R[6];
    const double y = d0 * cam.R[1] + d1 * cam.R[4] + d2 * cam.R[7];
    const double z = d0 * cam.R[2] + d1 * cam.R[5] + d2 * cam.R[8];
    double Jc[6] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0};
    bool valid;
    if (cam.fisheye) {
        const double dist = sqrt(x * x + y * y + z * z);
        const double rho = gf::gf_hypotd(x, y);
        const double theta = gf::gf_atan2d(rho, z);
        const double t2 = theta * theta;
        const double rt = theta * (1.0 + t2 * (cam.k[0] + t2 * (cam.k[1] + t2 * (cam.k[2] + t2 * cam.k[3]))));
        const double rd =
            1.0 + t2 * (3.0 * cam.k[0] + t2 * (5.0 * cam.k[1] + t2 * (7.0 * cam.k[2] + t2 * 9.0 * cam.k[3])));
        const double rs = fmax(rho, sqrt(DBL_MIN));
        const double dd = fmax(dist * dist, DBL_MIN);
        const double cp = x / rs, sp = y / rs;
        const double gt[3] = {z * x / (rs * dd), z * y / (rs * dd), -rho / dd};
        const double gp[3] = {-y / (rs * rs), x / (rs * rs), 0.0};
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            Jc[a] = cam.fx * (rd * cp * gt[a] - rt * sp * gp[a]);
            Jc[3 + a] = cam.fy * (rd * sp * gt[a] + rt * cp * gp[a]);
        }
        if (rho <= 1.0e-12 && z > 0.0) {
#pragma unroll
            for (int a = 0; a < 6; ++a) Jc[a] = 0.0;
            Jc[0] = cam.fx / dist;
            Jc[4] = cam.fy / dist;
        }
        valid = dist > 0.2 && (rho > 1.0e-12 || z > 0.0) && theta < cam.maxAngle && rd > 0.0;
    } else {
        valid = z > 0.2;
        const double zs = valid ? z : 1.0;
        Jc[0] = cam.fx / zs;
        Jc[2] = -cam.fx * x / (zs * zs);
        Jc[4] = cam.fy / zs;
        Jc[5] = -cam.fy * y / (zs * zs);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int k = 0; k < 3; ++k)
            J[3 * i + k] = float(Jc[3 * i] * cam.R[3 * k] + Jc[3 * i + 1] * cam.R[3 * k + 1] +
                                 Jc[3 * i + 2] * cam.R[3 * k + 2]);
    return valid;
}

// Q = gamma J^+ J^+^T (view_observation_filter.py:90-163).  Q is row-major 3x3.
__device__ bool footprint_q(const float J[6], bool chartValid, double gamma, double Q[9]) {
    const double a[3] = {J[0], J[1], J[2]}, b[3] = {J[3], J[4], J[5]};
    bool finite = true;
#pragma unroll
    for (int i = 0; i < 6; ++i) finite = finite && gf::isfinite_d(double(J[i]));
    const bool swap = (b[0] * b[0] + b[1] * b[1] + b[2] * b[2]) > (a[0] * a[0] + a[1] * a[1] + a[2] * a[2]);
    const double* lead = swap ? b : a;
    const double* trail = swap ? a : b;
    const double p0 = sqrt(lead[0] * lead[0] + lead[1] * lead[1] + lead[2] * lead[2]);
    const bool ok0 = gf::isfinite_d(p0) && p0 > 0.0;
    const double s0 = ok0 ? p0 : 1.0;
    double u0[3], r[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) u0[i] = lead[i] / s0;
    double coef = u0[0] * trail[0] + u0[1] * trail[1] + u0[2] * trail[2];
#pragma unroll
    for (int i = 0; i < 3; ++i) r[i] = trail[i] - coef * u0[i];
    const double corr = u0[0] * r[0] + u0[1] * r[1] + u0[2] * r[2];
#pragma unroll
    for (int i = 0; i < 3; ++i) r[i] = r[i] - corr * u0[i];
    coef = coef + corr;
    const double p1 = sqrt(r[0] * r[0] + r[1] * r[1] + r[2] * r[2]);
    const bool ok1 = gf::isfinite_d(p1) && p1 > 0.0;
    const double s1 = ok1 ? p1 : 1.0;
    double u1[3], c0[3], c1[3];
    const double i00 = 1.0 / s0, i10 = -coef / (s0 * s1), i11 = 1.0 / s1;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        u1[i] = r[i] / s1;
        c0[i] = u0[i] * i00 + u1[i] * i10;
        c1[i] = u1[i] * i11;
    }
    bool valid = chartValid && finite && ok0 && ok1 && gf::isfinite_d(coef);
#pragma unroll
    for (int i = 0; i < 3; ++i) valid = valid && gf::isfinite_d(u0[i]) && gf::isfinite_d(u1[i]);
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            Q[3 * i + j] = gamma * (c0[i] * c0[j] + c1[i] * c1[j]);
            valid = valid && gf::isfinite_d(Q[3 * i + j]);
        }
    if (!valid)
#pragma unroll
        for (int i = 0; i < 9; ++i) Q[i] = 0.0;
    return valid;
}

__device__ __forceinline__ void quat_rotation(const float* q, double R[9]) {
    const double w = q[0], x = q[1], y = q[2], z = q[3];
    R[0] = 1.0 - 2.0 * (y * y + z * z);
    R[1] = 2.0 * (x * y - z * w);
    R[2] = 2.0 * (x * z + y * w);
    R[3] = 2.0 * (x * y + z * w);
    R[4] = 1.0 - 2.0 * (x * x + z * z);
    R[5] = 2.0 * (y * z - x * w);
    R[6] = 2.0 * (x * z - y * w);
    R[7] = 2.0 * (y * z + x * w);
    R[8] = 1.0 - 2.0 * (x * x + y * y);
}

// Symmetric 3x3 eigendecomposition by cyclic Jacobi rotations: A = V diag(l) V^T
// (A row-major, overwritten; V column k is the k-th eigenvector).
__device__ void jacobi3(double A[9], double V[9], double l[3]) {
#pragma unroll
    for (int i = 0; i < 9; ++i) V[i] = (i % 4 == 0) ? 1.0 : 0.0;
    for (int sweep = 0; sweep < 20; ++sweep) {
        const double off = A[1] * A[1] + A[2] * A[2] + A[5] * A[5];
        const double diag = A[0] * A[0] + A[4] * A[4] + A[8] * A[8];
        if (!(off > 1e-34 * diag)) break;
#pragma unroll
        for (int pair = 0; pair < 3; ++pair) {
            const int p = pair == 2 ? 1 : 0;
            const int q = pair == 0 ? 1 : 2;
            const double apq = A[3 * p + q];
            if (apq == 0.0) continue;
            const double app = A[4 * p], aqq = A[4 * q];
            const double theta = (aqq - app) / (2.0 * apq);
            const double at = fabs(theta);
            double t = at > 1e150 ? 0.5 / at : 1.0 / (at + sqrt(theta * theta + 1.0));
            if (theta < 0.0) t = -t;
            const double c = 1.0 / sqrt(t * t + 1.0);
            const double s = t * c;
            A[4 * p] = app - t * apq;
            A[4 * q] = aqq + t * apq;
            A[3 * p + q] = 0.0;
            A[3 * q + p] = 0.0;
            const int r = 3 - p - q;
            const double arp = A[3 * r + p], arq = A[3 * r + q];
            A[3 * r + p] = c * arp - s * arq;
            A[3 * p + r] = A[3 * r + p];
            A[3 * r + q] = s * arp + c * arq;
            A[3 * q + r] = A[3 * r + q];
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                const double vp = V[3 * k + p], vq = V[3 * k + q];
                V[3 * k + p] = c * vp - s * vq;
                V[3 * k + q] = s * vp + c * vq;
            }
        }
    }
    l[0] = A[0];
    l[1] = A[4];
    l[2] = A[8];
}

// M = V diag(f) V^T
__device__ __forceinline__ void spectral(const double V[9], const double f[3], double M[9]) {
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            M[3 * i + j] = V[3 * i] * f[0] * V[3 * j] + V[3 * i + 1] * f[1] * V[3 * j + 1] +
                           V[3 * i + 2] * f[2] * V[3 * j + 2];
}

__device__ __forceinline__ void matmul3(const double* A, const double* B, double* C) {
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) C[3 * i + j] = A[3 * i] * B[j] + A[3 * i + 1] * B[3 + j] + A[3 * i + 2] * B[6 + j];
}

// F = J R S (2x3), S0 = F F^T; m = sqrt(det S0 / det(S0 + gamma I)).
__device__ bool compensation(const float J[6], const double R[9], const double s[3], double gamma, double& m,
                             double S0[3]) {
    double F[6];
#pragma unroll
    for (int px = 0; px < 2; ++px)
#pragma unroll
        for (int ax = 0; ax < 3; ++ax)
            F[3 * px + ax] = (double(J[3 * px]) * R[ax] + double(J[3 * px + 1]) * R[3 + ax] +
                              double(J[3 * px + 2]) * R[6 + ax]) * s[ax];
    S0[0] = F[0] * F[0] + F[1] * F[1] + F[2] * F[2];
    S0[1] = F[0] * F[3] + F[1] * F[4] + F[2] * F[5];
    S0[2] = F[3] * F[3] + F[4] * F[4] + F[5] * F[5];
    const double det0 = S0[0] * S0[2] - S0[1] * S0[1];
    const double det1 = (S0[0] + gamma) * (S0[2] + gamma) - S0[1] * S0[1];
    m = sqrt(det0 / det1);
    return gf::isfinite_d(m) && det0 > 0.0 && det1 > 0.0;
}

struct RowState {
    double R[9], s[3], o;
    double C[9];         // covariance output (C or Sigma)
    double B[9], Bi[9];  // factor, inverse factor
    double V[9], r[3];   // eigenvectors and square roots of the eigenvalues (exact mode, observed rows)
    double m, S0[3];
    bool observed;
    int error;
};

// The forward of one row; mode 0 exact (symmetric root), 1 Cholesky.
__device__ void shape_row(const float* scale, const float* quat, float density, const double Q[9], const float J[6],
                          bool observed, double gamma, int mode, bool fallback, RowState& st) {
    quat_rotation(quat, st.R);
#pragma unroll
    for (int k = 0; k < 3; ++k) st.s[k] = scale[k];
    st.o = density;
    st.error = 0;
    st.m = 1.0;
    double sigma[9];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            sigma[3 * i + j] = st.R[3 * i] * st.s[0] * st.s[0] * st.R[3 * j] +
                               st.R[3 * i + 1] * st.s[1] * st.s[1] * st.R[3 * j + 1] +
                               st.R[3 * i + 2] * st.s[2] * st.s[2] * st.R[3 * j + 2];
    bool shaped = false;
    if (observed) {
#pragma unroll
        for (int i = 0; i < 9; ++i) st.C[i] = sigma[i] + Q[i];
        if (!compensation(J, st.R, st.s, gamma, st.m, st.S0)) {
            st.error |= kBadCompensation;
        } else if (mode == 0) {
            double A[9], l[3];
#pragma unroll
            for (int i = 0; i < 9; ++i) A[i] = st.C[i];
            jacobi3(A, st.V, l);
            if (gf::isfinite_d(l[0]) && gf::isfinite_d(l[1]) && gf::isfinite_d(l[2]) && l[0] > 0.0 && l[1] > 0.0 &&
                l[2] > 0.0) {
                double root[9], iroot[9], ir[3];
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    st.r[k] = sqrt(l[k]);
                    ir[k] = 1.0 / st.r[k];
                }
                spectral(st.V, st.r, root);
                spectral(st.V, ir, iroot);
                matmul3(root, st.R, st.B);
                double Rt[9];
#pragma unroll
                for (int i = 0; i < 3; ++i)
#pragma unroll
                    for (int j = 0; j < 3; ++j) Rt[3 * i + j] = st.R[3 * j + i];
                matmul3(Rt, iroot, st.Bi);
                shaped = true;
            } else {
                st.error |= kNotSpd;
            }
        } else {
            const double* C = st.C;
            const double l00 = C[0] > 0.0 ? sqrt(C[0]) : -1.0;
            if (l00 > 0.0) {
                const double l10 = C[3] / l00, l20 = C[6] / l00;
                const double t11 = C[4] - l10 * l10;
                const double l11 = t11 > 0.0 ? sqrt(t11) : -1.0;
                if (l11 > 0.0) {
                    const double l21 = (C[7] - l20 * l10) / l11;
                    const double t22 = C[8] - l20 * l20 - l21 * l21;
                    const double l22 = t22 > 0.0 ? sqrt(t22) : -1.0;
                    if (l22 > 0.0) {
                        const double a00 = 1.0 / l00, a11 = 1.0 / l11, a22 = 1.0 / l22;
                        const double a10 = -l10 * a00 * a11;
                        const double a21 = -l21 * a11 * a22;
                        const double a20 = -(l20 * a00 + l21 * a10) * a22;
                        const double B[9] = {l00, 0.0, 0.0, l10, l11, 0.0, l20, l21, l22};
                        const double Bi[9] = {a00, 0.0, 0.0, a10, a11, 0.0, a20, a21, a22};
#pragma unroll
                        for (int i = 0; i < 9; ++i) {
                            st.B[i] = B[i];
                            st.Bi[i] = Bi[i];
                        }
                        shaped = true;
                    }
                }
            }
            if (!shaped) st.error |= kNotSpd;
        }
    }
    st.observed = shaped;
    if (!shaped && (!observed || fallback || st.error == 0)) {
        // stored shape: B = R S, B^-1 = S^-1 R^T, C = Sigma, m = 1
        st.m = 1.0;
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                st.B[3 * i + j] = st.R[3 * i + j] * st.s[j];
                st.Bi[3 * i + j] = st.R[3 * j + i] / st.s[i];
            }
#pragma unroll
        for (int i = 0; i < 9; ++i) st.C[i] = sigma[i];
        if (fallback) st.error = 0;
    }
}

__device__ __forceinline__ void q_from6(const double* q6, double Q[9]) {
    Q[0] = q6[0];
    Q[1] = Q[3] = q6[1];
    Q[2] = Q[6] = q6[2];
    Q[4] = q6[3];
    Q[5] = Q[7] = q6[4];
    Q[8] = q6[5];
}

struct ViewArgs {
    int64_t N;
    const float* positions;
    Cam cam;
    double gamma;
    double* q6;
    float* jacobian;
    uint8_t* observed;
};

__global__ __launch_bounds__(kThreads) void k_view_q6(ViewArgs a) {
    const int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x;
    if (i >= a.N) return;
    float J[6];
    const bool chart = view_jacobian(a.cam, a.positions + 3 * i, J);
    double Q[9];
    const bool ob = footprint_q(J, chart, a.gamma, Q);
    double* q6 = a.q6 + 6 * i;
    q6[0] = Q[0];
    q6[1] = Q[1];
    q6[2] = Q[2];
    q6[3] = Q[4];
    q6[4] = Q[5];
    q6[5] = Q[8];
#pragma unroll
    for (int k = 0; k < 6; ++k) a.jacobian[6 * i + k] = ob ? J[k] : 0.0f;
    a.observed[i] = ob ? 1u : 0u;
}

struct ShapeArgs {
    int64_t N;
    const float* scales;
    const float* quats;
    const float* density;
    const double* q6;
    const float* jacobian;
    const uint8_t* observed;
    double gamma;
    int mode;
    int massPreserving;
    float* covariance;
    float* factor;
    float* inverseFactor;
    float* compensation;
    float* outDensity;
    int* status;
    unsigned long long* firstRow;
};

// Four blocks (16 warps) per SM: the float64 eigen-solve is latency-bound,
// and the extra warps hide more than the few register spills this costs
// (measured on 1M Gaussians together with the VJP below: 0.15 ms a step).
__global__ __launch_bounds__(kThreads, 4) void k_full_shape(ShapeArgs a) {
    const int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x;
    if (i >= a.N) return;
    double Q[9];
    q_from6(a.q6 + 6 * i, Q);
    RowState st;
    shape_row(a.scales + 3 * i, a.quats + 4 * i, a.density[i], Q, a.jacobian + 6 * i, a.observed[i] != 0, a.gamma,
              a.mode, false, st);
    if (st.error != 0) {
        record(a.status, a.firstRow, st.error, i);
        return;
    }
    const double d = a.massPreserving ? st.m * st.o : st.o;
    bool finite = gf::isfinite_d(d) && gf::isfinite_d(st.m);
    for (int k = 0; k < 9; ++k) {
        a.covariance[9 * i + k] = float(st.C[k]);
        a.factor[9 * i + k] = float(st.B[k]);
        a.inverseFactor[9 * i + k] = float(st.Bi[k]);
        finite = finite && gf::isfinite_d(st.B[k]) && gf::isfinite_d(st.Bi[k]);
    }
    a.compensation[i] = float(st.m);
    a.outDensity[i] = float(d);
    if (!finite) record(a.status, a.firstRow, kNonFinite, i);
}

struct ShapeBwdArgs {
    ShapeArgs f;
    const float* gC;
    const float* gB;
    const float* gBi;
    const float* gm;
    const float* gd;
    float* gScales;
    float* gQuats;
    float* gDensity;
};

__device__ __forceinline__ double ld(const float* p, int64_t k) { return p == nullptr ? 0.0 : double(p[k]); }

// Four blocks per SM as for k_full_shape (226 registers, 8 warps per SM, unbounded).
__global__ __launch_bounds__(kThreads, 4) void k_full_shape_bwd(ShapeBwdArgs a) {
    const int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x;
    if (i >= a.f.N) return;
    double Q[9];
    q_from6(a.f.q6 + 6 * i, Q);
    const float* J = a.f.jacobian + 6 * i;
    RowState st;
    shape_row(a.f.scales + 3 * i, a.f.quats + 4 * i, a.f.density[i], Q, J, a.f.observed[i] != 0, a.f.gamma, 0,
              false, st);
    double gC[9], gB[9], gBi[9];
    for (int k = 0; k < 9; ++k) {
        gC[k] = ld(a.gC, 9 * i + k);
        gB[k] = ld(a.gB, 9 * i + k);
        gBi[k] = ld(a.gBi, 9 * i + k);
    }
    const double gm = ld(a.gm, i), gd = ld(a.gd, i);
    double gR[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0}, gs[3] = {0, 0, 0}, gS[9];
    double go = gd;
    const double* R = st.R;
    const double* s = st.s;
#pragma unroll
    for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int q = 0; q < 3; ++q) gS[3 * p + q] = 0.5 * (gC[3 * p + q] + gC[3 * q + p]);
    if (!st.observed || st.error != 0) {
        // B = R S, B^-1 = S^-1 R^T, C = Sigma, m = 1, density' = density
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                gR[3 * p + q] += gB[3 * p + q] * s[q] + gBi[3 * q + p] / s[q];
                gs[q] += gB[3 * p + q] * R[3 * p + q];
                gs[p] -= gBi[3 * p + q] * R[3 * q + p] / (s[p] * s[p]);
            }
    } else {
        const double m = st.m;
        double gmt = gm;
        if (a.f.massPreserving) {
            gmt += gd * st.o;
            go = gd * m;
        }
        // root and inverse root from the eigen pairs
        double root[9], iroot[9], ir[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) ir[k] = 1.0 / st.r[k];
        spectral(st.V, st.r, root);
        spectral(st.V, ir, iroot);
        // explicit R terms: B = root R, B^-1 = R^T iroot
        double G1[9], G2[9];  // dL/droot = gB R^T, dL/diroot = R gBi
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                G1[3 * p + q] = gB[3 * p] * R[3 * q] + gB[3 * p + 1] * R[3 * q + 1] + gB[3 * p + 2] * R[3 * q + 2];
                G2[3 * p + q] = R[3 * p] * gBi[q] + R[3 * p + 1] * gBi[3 + q] + R[3 * p + 2] * gBi[6 + q];
                gR[3 * p + q] += root[3 * p] * gB[q] + root[3 * p + 1] * gB[3 + q] + root[3 * p + 2] * gB[6 + q] +
                                 iroot[3 * p] * gBi[3 * q] + iroot[3 * p + 1] * gBi[3 * q + 1] +
                                 iroot[3 * p + 2] * gBi[3 * q + 2];
            }
        // V^T sym(G) V, weighted by the divided differences, back to V (.) V^T
        double H[9];
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                double h1 = 0.0, h2 = 0.0;
#pragma unroll
                for (int u = 0; u < 3; ++u)
#pragma unroll
                    for (int v = 0; v < 3; ++v) {
                        const double w = st.V[3 * u + p] * st.V[3 * v + q];
                        h1 += w * 0.5 * (G1[3 * u + v] + G1[3 * v + u]);
                        h2 += w * 0.5 * (G2[3 * u + v] + G2[3 * v + u]);
                    }
                const double k1 = 1.0 / (st.r[p] + st.r[q]);
                const double k2 = -k1 / (st.r[p] * st.r[q]);
                H[3 * p + q] = h1 * k1 + h2 * k2;
            }
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                double v = 0.0;
#pragma unroll
                for (int u = 0; u < 3; ++u)
#pragma unroll
                    for (int w = 0; w < 3; ++w) v += st.V[3 * p + u] * H[3 * u + w] * st.V[3 * q + w];
                gS[3 * p + q] += v;
            }
        // m through Sigma: dm/dSigma = m/2 J^T (S0^-1 - (S0 + gamma I)^-1) J
        const double g = a.f.gamma;
        const double det0 = st.S0[0] * st.S0[2] - st.S0[1] * st.S0[1];
        const double det1 = (st.S0[0] + g) * (st.S0[2] + g) - st.S0[1] * st.S0[1];
        const double in00 = st.S0[2] / det0 - (st.S0[2] + g) / det1;
        const double in01 = -st.S0[1] / det0 + st.S0[1] / det1;
        const double in11 = st.S0[0] / det0 - (st.S0[0] + g) / det1;
        const double scale = gmt * m * 0.5;
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                const double jp0 = J[p], jp1 = J[3 + p], jq0 = J[q], jq1 = J[3 + q];
                gS[3 * p + q] += scale * (jp0 * (in00 * jq0 + in01 * jq1) + jp1 * (in01 * jq0 + in11 * jq1));
            }
    }
    // Sigma = R S^2 R^T (gS symmetric)
#pragma unroll
    for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const double v = gS[3 * p] * R[k] + gS[3 * p + 1] * R[3 + k] + gS[3 * p + 2] * R[6 + k];
            gR[3 * p + k] += 2.0 * v * s[k] * s[k];
        }
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        double v = 0.0;
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int q = 0; q < 3; ++q) v += R[3 * p + k] * gS[3 * p + q] * R[3 * q + k];
        gs[k] += 2.0 * s[k] * v;
    }
    // R(q), q = (w, x, y, z)
    const float* qq = a.f.quats + 4 * i;
    const double w = qq[0], x = qq[1], y = qq[2], z = qq[3];
    const double* G = gR;
    const double gw = 2.0 * (-z * G[1] + y * G[2] + z * G[3] - x * G[5] - y * G[6] + x * G[7]);
    const double gx = 2.0 * (y * G[1] + z * G[2] + y * G[3] - 2.0 * x * G[4] - w * G[5] + z * G[6] + w * G[7] -
                             2.0 * x * G[8]);
    const double gy = 2.0 * (-2.0 * y * G[0] + x * G[1] + w * G[2] + x * G[3] + z * G[5] - w * G[6] + z * G[7] -
                             2.0 * y * G[8]);
    const double gz = 2.0 * (-2.0 * z * G[0] - w * G[1] + x * G[2] + w * G[3] - 2.0 * z * G[4] + y * G[5] +
                             x * G[6] + y * G[7]);
    a.gScales[3 * i] = float(gs[0]);
    a.gScales[3 * i + 1] = float(gs[1]);
    a.gScales[3 * i + 2] = float(gs[2]);
    a.gQuats[4 * i] = float(gw);
    a.gQuats[4 * i + 1] = float(gx);
    a.gQuats[4 * i + 2] = float(gy);
    a.gQuats[4 * i + 3] = float(gz);
    a.gDensity[i] = float(go);
}

struct PackedArgs {
    int64_t N;
    const float* positions;
    const float* quats;
    const float* scales;
    const float* density;
    Cam cam;
    double gamma;
    int mode;
    float* packed;
    int* status;
    unsigned long long* firstRow;
};

// One frame of the inference renderer: everything above, written into the
// packed [N,32] rows (density 3, B 12-20, B^-1 21-29).
__global__ __launch_bounds__(kThreads) void k_view_shape_packed(PackedArgs a) {
    const int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x;
    if (i >= a.N) return;
    float J[6];
    double Q[9];
    bool ob = false;
    if (a.gamma > 0.0) {
        const bool chart = view_jacobian(a.cam, a.positions + 3 * i, J);
        ob = footprint_q(J, chart, a.gamma, Q);
    } else {
#pragma unroll
        for (int k = 0; k < 9; ++k) Q[k] = 0.0;
#pragma unroll
        for (int k = 0; k < 6; ++k) J[k] = 0.0f;
    }
    RowState st;
    // the Cholesky mode falls back to the stored shape as the fused kernel does
    shape_row(a.scales + 3 * i, a.quats + 4 * i, a.density[i], Q, J, ob, a.gamma, a.mode, a.mode == 1, st);
    if (st.error != 0) {
        record(a.status, a.firstRow, st.error, i);
        return;
    }
    float* out = a.packed + 32 * i;
    out[3] = float(st.m * st.o);
#pragma unroll
    for (int k = 0; k < 9; ++k) {
        out[12 + k] = float(st.B[k]);
        out[21 + k] = float(st.Bi[k]);
    }
}

bool make_cam(const gf_shape_camera* c, Cam& cam) {
    if (c == nullptr) return false;
    for (int r = 0; r < 3; ++r) {
        for (int k = 0; k < 3; ++k) cam.R[3 * r + k] = c->c2w[4 * r + k];
        cam.c[r] = c->c2w[4 * r + 3];
    }
    cam.fx = c->focal_length[0];
    cam.fy = c->focal_length[1];
    for (int k = 0; k < 4; ++k) cam.k[k] = c->radial[k];
    cam.maxAngle = c->max_angle;
    cam.fisheye = c->fisheye != 0;
    return true;
}

int launch_check() {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return gf_record_error(GF_ERR_CUDA, cudaGetErrorString(e));
    return GF_OK;
}

unsigned blocks_for(int64_t n) { return unsigned((n + kThreads - 1) / kThreads); }

// ------------------------------------------------------------------ row packing
// The training renderer's [N,32] particle rows from the model's per-slot
// tensors, and the row gradient back to them (reference tracer.py:171-179,
// :334-343).  One thread per row; the row is written and read as 8 float4.
struct PackPtrs {
    const float* pos;      // [N,3]
    const float* dens;     // [N]
    const float* rot;      // [N,4]
    const float* scale;    // [N,3]
    const float* idens;    // [N]
    const float* factor;   // [N,9]
    const float* inverse;  // [N,9]
};

// The block's kThreads rows pass through shared memory (pitch 33 floats), so
// that the [N,32] rows and every per-slot array are read and written with
// consecutive threads on consecutive words.
constexpr int kRowPitch = 33;

__global__ __launch_bounds__(kThreads) void k_pack_rows(PackPtrs p, int64_t n, float4* __restrict__ out) {
    __shared__ float rows[kThreads * kRowPitch];
    const int64_t i0 = int64_t(blockIdx.x) * kThreads;
    const int cnt = int(n - i0 < kThreads ? n - i0 : kThreads);
    const int tid = threadIdx.x;
    // slot s of the row <- width-w array, for the block's particles
    auto gather = [&](const float* src, int w, int s0) {
        for (int e = tid; e < w * cnt; e += kThreads) {
            const int r = e / w;
            rows[r * kRowPitch + s0 + (e - r * w)] = src[w * i0 + e];
        }
    };
    gather(p.pos, 3, 0);
    gather(p.dens, 1, 3);
    gather(p.rot, 4, 4);
    gather(p.scale, 3, 8);
    gather(p.idens, 1, 11);
    gather(p.factor, 9, 12);
    gather(p.inverse, 9, 21);
    for (int r = tid; r < cnt; r += kThreads) rows[r * kRowPitch + 30] = rows[r * kRowPitch + 31] = 0.0f;
    __syncthreads();
    for (int e = tid; e < 8 * cnt; e += kThreads) {
        const float* q = rows + (e >> 3) * kRowPitch + 4 * (e & 7);
        out[8 * i0 + e] = make_float4(q[0], q[1], q[2], q[3]);
    }
}

struct UnpackPtrs {
    float* pos;
    float* dens;
    float* rot;
    float* scale;
    float* idens;
    float* factor;
    float* inverse;
};

__global__ __launch_bounds__(kThreads) void k_unpack_rows(const float4* __restrict__ in, int64_t n, UnpackPtrs p) {
    __shared__ float rows[kThreads * kRowPitch];
    const int64_t i0 = int64_t(blockIdx.x) * kThreads;
    const int cnt = int(n - i0 < kThreads ? n - i0 : kThreads);
    const int tid = threadIdx.x;
    for (int e = tid; e < 8 * cnt; e += kThreads) {
        const float4 v = in[8 * i0 + e];
        float* q = rows + (e >> 3) * kRowPitch + 4 * (e & 7);
        q[0] = v.x;
        q[1] = v.y;
        q[2] = v.z;
        q[3] = v.w;
    }
    __syncthreads();
    // width-w array <- slot s of the row, for the block's particles
    auto scatter = [&](float* dst, int w, int s0) {
        for (int e = tid; e < w * cnt; e += kThreads) {
            const int r = e / w;
            dst[w * i0 + e] = rows[r * kRowPitch + s0 + (e - r * w)];
        }
    };
    scatter(p.pos, 3, 0);
    scatter(p.dens, 1, 3);
    scatter(p.rot, 4, 4);
    scatter(p.scale, 3, 8);
    scatter(p.idens, 1, 11);
    scatter(p.factor, 9, 12);
    scatter(p.inverse, 9, 21);
}

}  // namespace

extern "C" {

int gf_view_q6(const float* positions, int64_t n, const gf_shape_camera* camera, double gamma, double* q6,
               float* jacobian, uint8_t* observed, void* stream) {
    if (n < 0 || (n > 0 && (positions == nullptr || q6 == nullptr || jacobian == nullptr || observed == nullptr)))
        return gf_record_error(GF_ERR_BAD_INPUT, "current_view_q6: bad buffers");
    ViewArgs a{};
    if (!make_cam(camera, a.cam)) return gf_record_error(GF_ERR_BAD_INPUT, "current_view_q6: camera is NULL");
    if (n == 0) return GF_OK;
    a.N = n;
    a.positions = positions;
    a.gamma = gamma;
    a.q6 = q6;
    a.jacobian = jacobian;
    a.observed = observed;
    k_view_q6<<<blocks_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    return launch_check();
}

int gf_full_shape(const float* scales, const float* quaternions, const float* density, const double* q6,
                  const float* jacobian, const uint8_t* observed, int64_t n, double gamma, int mass_preserving,
                  int mode, float* covariance, float* factor, float* inverse_factor, float* compensation,
                  float* out_density, int32_t* status, void* stream) {
    if (n < 0 || (mode != 0 && mode != 1) || status == nullptr)
        return gf_record_error(GF_ERR_BAD_INPUT, "full shape: bad arguments");
    if (n > 0 && (scales == nullptr || quaternions == nullptr || density == nullptr || q6 == nullptr ||
                  jacobian == nullptr || observed == nullptr || covariance == nullptr || factor == nullptr ||
                  inverse_factor == nullptr || compensation == nullptr || out_density == nullptr))
        return gf_record_error(GF_ERR_BAD_INPUT, "full shape: buffers must not be NULL");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // status: int32 flags, pad, then the first failing row as u64
    if (cudaMemsetAsync(status, 0, 4, s) != cudaSuccess || cudaMemsetAsync(status + 2, 0xff, 8, s) != cudaSuccess)
        return gf_record_error(GF_ERR_CUDA, "full shape: status reset failed");
    if (n == 0) return GF_OK;
    ShapeArgs a{n, scales, quaternions, density, q6, jacobian, observed, gamma, mode, mass_preserving != 0,
                covariance, factor, inverse_factor, compensation, out_density, status,
                reinterpret_cast<unsigned long long*>(status + 2)};
    k_full_shape<<<blocks_for(n), kThreads, 0, s>>>(a);
    return launch_check();
}

int gf_full_shape_bwd(const float* scales, const float* quaternions, const float* density, const double* q6,
                      const float* jacobian, const uint8_t* observed, int64_t n, double gamma, int mass_preserving,
                      const float* grad_covariance, const float* grad_factor, const float* grad_inverse_factor,
                      const float* grad_compensation, const float* grad_density, float* grad_scales,
                      float* grad_quaternions, float* grad_density_in, void* stream) {
    if (n < 0) return gf_record_error(GF_ERR_BAD_INPUT, "full shape backward: bad arguments");
    if (n > 0 && (scales == nullptr || quaternions == nullptr || density == nullptr || q6 == nullptr ||
                  jacobian == nullptr || observed == nullptr || grad_scales == nullptr ||
                  grad_quaternions == nullptr || grad_density_in == nullptr))
        return gf_record_error(GF_ERR_BAD_INPUT, "full shape backward: buffers must not be NULL");
    if (n == 0) return GF_OK;
    ShapeBwdArgs a{};
    a.f = ShapeArgs{n, scales, quaternions, density, q6, jacobian, observed, gamma, 0, mass_preserving != 0,
                    nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    a.gC = grad_covariance;
    a.gB = grad_factor;
    a.gBi = grad_inverse_factor;
    a.gm = grad_compensation;
    a.gd = grad_density;
    a.gScales = grad_scales;
    a.gQuats = grad_quaternions;
    a.gDensity = grad_density_in;
    k_full_shape_bwd<<<blocks_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    return launch_check();
}

int gf_view_shape_packed(const float* positions, const float* quaternions, const float* scales,
                         const float* density, int64_t n, const gf_shape_camera* camera, double gamma, int mode,
                         float* packed, int32_t* status, void* stream) {
    if (n < 0 || (mode != 0 && mode != 1) || status == nullptr)
        return gf_record_error(GF_ERR_BAD_INPUT, "view shape: bad arguments");
    if (n > 0 && (positions == nullptr || quaternions == nullptr || scales == nullptr || density == nullptr ||
                  packed == nullptr))
        return gf_record_error(GF_ERR_BAD_INPUT, "view shape: buffers must not be NULL");
    PackedArgs a{};
    if (!make_cam(camera, a.cam)) return gf_record_error(GF_ERR_BAD_INPUT, "view shape: camera is NULL");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(status, 0, 4, s) != cudaSuccess || cudaMemsetAsync(status + 2, 0xff, 8, s) != cudaSuccess)
        return gf_record_error(GF_ERR_CUDA, "view shape: status reset failed");
    if (n == 0) return GF_OK;
    a.N = n;
    a.positions = positions;
    a.quats = quaternions;
    a.scales = scales;
    a.density = density;
    a.gamma = gamma;
    a.mode = mode;
    a.packed = packed;
    a.status = status;
    a.firstRow = reinterpret_cast<unsigned long long*>(status + 2);
    k_view_shape_packed<<<blocks_for(n), kThreads, 0, s>>>(a);
    return launch_check();
}

int gf_pack_particle_rows(const float* positions, const float* density, const float* rotations,
                          const float* scales, const float* intrinsic_density, const float* factor,
                          const float* inverse_factor, int64_t n, float* rows, void* stream) {
    if (n < 0) return gf_record_error(GF_ERR_BAD_INPUT, "pack rows: negative row count");
    if (n == 0) return GF_OK;
    if (positions == nullptr || density == nullptr || rotations == nullptr || scales == nullptr ||
        intrinsic_density == nullptr || factor == nullptr || inverse_factor == nullptr || rows == nullptr)
        return gf_record_error(GF_ERR_BAD_INPUT, "pack rows: buffers must not be NULL");
    if ((reinterpret_cast<uintptr_t>(rows) & 15u) != 0u)
        return gf_record_error(GF_ERR_BAD_INPUT, "pack rows: output rows must be 16-byte aligned");
    PackPtrs p{positions, density, rotations, scales, intrinsic_density, factor, inverse_factor};
    k_pack_rows<<<blocks_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p, n,
                                                                                  reinterpret_cast<float4*>(rows));
    return launch_check();
}

int gf_unpack_particle_rows(const float* rows, int64_t n, float* positions, float* density, float* rotations,
                            float* scales, float* intrinsic_density, float* factor, float* inverse_factor,
                            void* stream) {
    if (n < 0) return gf_record_error(GF_ERR_BAD_INPUT, "unpack rows: negative row count");
    if (n == 0) return GF_OK;
    if (positions == nullptr || density == nullptr || rotations == nullptr || scales == nullptr ||
        intrinsic_density == nullptr || factor == nullptr || inverse_factor == nullptr || rows == nullptr)
        return gf_record_error(GF_ERR_BAD_INPUT, "unpack rows: buffers must not be NULL");
    if ((reinterpret_cast<uintptr_t>(rows) & 15u) != 0u)
        return gf_record_error(GF_ERR_BAD_INPUT, "unpack rows: input rows must be 16-byte aligned");
    UnpackPtrs p{positions, density, rotations, scales, intrinsic_density, factor, inverse_factor};
    k_unpack_rows<<<blocks_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const float4*>(rows), n, p);
    return launch_check();
}

}  // extern "C"
