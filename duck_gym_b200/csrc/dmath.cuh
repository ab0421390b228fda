// Device vector / quaternion algebra for the AVBD kernels.
//
// Two families:
//  * plain operators (V3 + V3, dot, rotate, ...): the compiler may contract
//    them into FMAs.  Used by the primal/dual solve, whose parity bound is a
//    tolerance (1e-4 m / rad per substep).
//  * x-prefixed functions (xadd, xdot, xrotate, ...): every multiply and add
//    is rounded separately (__fmul_rn / __fadd_rn never contract), in the
//    same order as the reference's C++ (src/cuda/kernel.cuh:86-160), and the
//    thresholds compare in double exactly like the reference's implicit
//    promotions.  Used by contact generation, whose parity bound is bit
//    equality of the contact sets.
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace duckb200 {

template <class R> struct V3 { R x, y, z; };
template <class R> struct Q4 { R w, x, y, z; };

// ---------------------------------------------------------------- scalar ops
__device__ __forceinline__ float xadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float xsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float xmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double xadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double xsub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double xmul(double a, double b) { return __dmul_rn(a, b); }

template <class R> __device__ __forceinline__ R rmin(R a, R b) { return a < b ? a : b; }
template <class R> __device__ __forceinline__ R rmax(R a, R b) { return a > b ? a : b; }
template <class R> __device__ __forceinline__ R rclamp(R v, R a, R b) { return rmin(rmax(v, a), b); }

// hypot(float, float) of the reference's host build is correctly rounded; the
// double evaluation below reproduces it (exact squares, one rounding each for
// the sum, the root and the final narrowing).
__device__ __forceinline__ float xhypot(float x, float y) {
  double dx = x, dy = y;
  return float(__dsqrt_rn(__dadd_rn(__dmul_rn(dx, dx), __dmul_rn(dy, dy))));
}
__device__ __forceinline__ double xhypot(double x, double y) { return hypot(x, y); }

// Approximate square root (PTX sqrt.approx) for stiffness majorizers.
__device__ __forceinline__ float fsqrt(float x) {
  float r;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ double fsqrt(double x) { return sqrt(x); }

// ---------------------------------------------------------------- fast V3
template <class R> __device__ __forceinline__ V3<R> operator+(V3<R> a, V3<R> b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
template <class R> __device__ __forceinline__ V3<R> operator-(V3<R> a, V3<R> b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
template <class R> __device__ __forceinline__ V3<R> operator-(V3<R> a) { return {-a.x, -a.y, -a.z}; }
template <class R> __device__ __forceinline__ V3<R> operator*(V3<R> a, R s) { return {a.x * s, a.y * s, a.z * s}; }
template <class R> __device__ __forceinline__ R dot(V3<R> a, V3<R> b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
template <class R> __device__ __forceinline__ V3<R> cross(V3<R> a, V3<R> b) {
  return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}
template <class R> __device__ __forceinline__ R norm(V3<R> a) { return sqrt(dot(a, a)); }
template <class R> __device__ __forceinline__ R comp(V3<R> a, int k) { return k == 0 ? a.x : (k == 1 ? a.y : a.z); }
template <class R> __device__ __forceinline__ Q4<R> conj(Q4<R> q) { return {q.w, -q.x, -q.y, -q.z}; }
template <class R> __device__ __forceinline__ Q4<R> qmul(Q4<R> a, Q4<R> b) {
  return {a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z,
          a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y,
          a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x,
          a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w};
}
template <class R> __device__ __forceinline__ Q4<R> qnormalized(Q4<R> q) {
  R n = sqrt(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
  if (!(n >= R(1e-15))) return {R(NAN), R(NAN), R(NAN), R(NAN)};
  R inv = R(1) / n;
  return {q.w * inv, q.x * inv, q.y * inv, q.z * inv};
}
// v + 2 u x (u x v + w v): the reference's rotation (kernel.cuh:132-135).
template <class R> __device__ __forceinline__ V3<R> rotate(Q4<R> q, V3<R> v) {
  V3<R> u{q.x, q.y, q.z};
  return v + cross(u, cross(u, v) + v * q.w) * R(2);
}
template <class R> __device__ __forceinline__ V3<R> rotateInv(Q4<R> q, V3<R> v) { return rotate(conj(q), v); }

__device__ __forceinline__ void sincosT(float a, float *s, float *c) { sincosf(a, s, c); }
__device__ __forceinline__ void sincosT(double a, double *s, double *c) { sincos(a, s, c); }

// Exponential map of a rotation vector (kernel.cuh:136-145).
template <class R> __device__ __forceinline__ Q4<R> qexp(V3<R> v) {
  R a = norm(v), s, c;
  sincosT(a * R(0.5), &s, &c);
  R k = a < R(1e-8) ? R(0.5) - a * a / R(48) : s / a;
  return qnormalized(Q4<R>{c, k * v.x, k * v.y, k * v.z});
}
// Logarithm of a unit quaternion (kernel.cuh:146-153).
template <class R> __device__ __forceinline__ V3<R> qlog(Q4<R> q) {
  q = qnormalized(q);
  if (q.w < R(0)) q = {-q.w, -q.x, -q.y, -q.z};
  V3<R> v{q.x, q.y, q.z};
  R s = norm(v);
  return v * (s < R(1e-10) ? R(2) : R(2) * atan2(s, q.w) / s);
}
// remainder(a, 2 pi) as the reference computes it, in double
// (kernel.cuh:154-160).  Angles already inside (-pi, pi) are returned as is,
// which is exactly what the double remainder gives for them.
template <class R> __device__ __forceinline__ R wrapAngle(R a) {
  const double pi = 3.14159265358979311600;
  double d = double(a);
  if (fabs(d) < pi) return a;
  return R(remainder(d, 2.0 * pi));
}

// ---------------------------------------------------------------- exact V3
template <class R> __device__ __forceinline__ V3<R> xadd(V3<R> a, V3<R> b) { return {xadd(a.x, b.x), xadd(a.y, b.y), xadd(a.z, b.z)}; }
template <class R> __device__ __forceinline__ V3<R> xsub(V3<R> a, V3<R> b) { return {xsub(a.x, b.x), xsub(a.y, b.y), xsub(a.z, b.z)}; }
template <class R> __device__ __forceinline__ V3<R> xscale(V3<R> a, R s) { return {xmul(a.x, s), xmul(a.y, s), xmul(a.z, s)}; }
template <class R> __device__ __forceinline__ R xdot(V3<R> a, V3<R> b) {
  return xadd(xadd(xmul(a.x, b.x), xmul(a.y, b.y)), xmul(a.z, b.z));
}
template <class R> __device__ __forceinline__ V3<R> xcross(V3<R> a, V3<R> b) {
  return {xsub(xmul(a.y, b.z), xmul(a.z, b.y)), xsub(xmul(a.z, b.x), xmul(a.x, b.z)),
          xsub(xmul(a.x, b.y), xmul(a.y, b.x))};
}
template <class R> __device__ __forceinline__ R xnorm(V3<R> a) { return sqrt(xdot(a, a)); }
// Vec3 / s is a multiplication by the reciprocal in the reference (kernel.cuh:100).
template <class R> __device__ __forceinline__ V3<R> xdiv(V3<R> a, R s) { return xscale(a, R(1) / s); }
template <class R> __device__ __forceinline__ V3<R> xunit(V3<R> a) {
  R n = xnorm(a);
  if (double(n) < 1e-15) return {R(NAN), R(NAN), R(NAN)};
  return xdiv(a, n);
}
template <class R> __device__ __forceinline__ V3<R> xrotate(Q4<R> q, V3<R> v) {
  V3<R> u{q.x, q.y, q.z};
  return xadd(v, xscale(xcross(u, xadd(xcross(u, v), xscale(v, q.w))), R(2)));
}

}  // namespace duckb200

namespace duckb200 {
// ---------------------------------------------------------------- fast path
// Approximate reciprocal square root / reciprocal / square root (PTX .approx,
// a few ulp) for the primal/dual solve, whose parity bound is a tolerance.
__device__ __forceinline__ float frsqrt(float x) { return rsqrtf(x); }
__device__ __forceinline__ double frsqrt(double x) { return rsqrt(x); }
__device__ __forceinline__ float frcp(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ double frcp(double x) { return 1.0 / x; }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdividef(a, b); }
__device__ __forceinline__ double fdiv(double a, double b) { return a / b; }
template <class R> __device__ __forceinline__ R fnorm(V3<R> a) { return fsqrt(dot(a, a)); }
template <class R> __device__ __forceinline__ Q4<R> fnormalized(Q4<R> q) {
  R n2 = q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z;
  if (!(n2 >= R(1e-30))) return {R(NAN), R(NAN), R(NAN), R(NAN)};
  R inv = frsqrt(n2);
  return {q.w * inv, q.x * inv, q.y * inv, q.z * inv};
}
// Rotation matrix of a unit quaternion, row major.
template <class R> __device__ __forceinline__ void quatToMatrix(Q4<R> q, R *m) {
  R xx = q.x * q.x, yy = q.y * q.y, zz = q.z * q.z, xy = q.x * q.y, xz = q.x * q.z, yz = q.y * q.z;
  R wx = q.w * q.x, wy = q.w * q.y, wz = q.w * q.z;
  m[0] = R(1) - R(2) * (yy + zz); m[1] = R(2) * (xy - wz); m[2] = R(2) * (xz + wy);
  m[3] = R(2) * (xy + wz); m[4] = R(1) - R(2) * (xx + zz); m[5] = R(2) * (yz - wx);
  m[6] = R(2) * (xz - wy); m[7] = R(2) * (yz + wx); m[8] = R(1) - R(2) * (xx + yy);
}
template <class M, class R> __device__ __forceinline__ V3<R> matVec(const M &m, V3<R> v) {
  return {m[0] * v.x + m[1] * v.y + m[2] * v.z, m[3] * v.x + m[4] * v.y + m[5] * v.z,
          m[6] * v.x + m[7] * v.y + m[8] * v.z};
}
// atan2 for the solver's hinge angles and rotation logarithms, whose parity
// bound is a tolerance: the ratio min(|x|, |y|) / max(|x|, |y|) in [0, 1], an
// odd polynomial t P(t^2) for atan on [0, 1], then the octant and quadrant
// restored.  P (degree 7 in t^2) was fitted for this file by iteratively
// reweighted least squares on the relative error of atan(t) / t over
// [0, 1]; evaluated in float its error is at most 1.6e-7 rad
// (tests/test_fatan2.py checks it again over all four quadrants).
__device__ __forceinline__ float fatan2(float y, float x) {
  const float ax = fabsf(x), ay = fabsf(y);
  const float mx = fmaxf(ax, ay), mn = fminf(ax, ay);
  const float t = mx > 0.f ? mn * frcp(mx) : 0.f;
  const float s = t * t;
  float p = -0x1.33932ep-8f;
  p = p * s + 0x1.8d589cp-6f;
  p = p * s - 0x1.e74ea8p-5f;
  p = p * s + 0x1.961640p-4f;
  p = p * s - 0x1.1f1e4cp-3f;
  p = p * s + 0x1.98fad4p-3f;
  p = p * s - 0x1.5551d0p-2f;
  p = p * s + 0x1.fffffcp-1f;
  p *= t;
  if (ay > ax) p = 1.57079632679489662f - p;
  if (x < 0.f) p = 3.14159265358979324f - p;
  return copysignf(p, y);
}
__device__ __forceinline__ double fatan2(double y, double x) { return atan2(y, x); }
// Exponential map with fast normalisation (kernel.cuh:136-145).
// Below 0.25 rad (every clamped Gauss-Seidel step, whose rotation is at most
// 0.25 rad, and the predictor at ordinary spin rates) cos(a/2) and
// sin(a/2)/a come from their Taylor series in a^2 to the a^6 terms, in float,
// with no square root (truncation error below 1e-11); above, sincos.
// fqexpRaw leaves the result unnormalised, for callers that normalise the
// product they form with it; fqexp normalises.
template <class R> __device__ __forceinline__ Q4<R> fqexpRaw(V3<R> v);
template <class R> __device__ __forceinline__ Q4<R> fqexp(V3<R> v) { return fnormalized(fqexpRaw(v)); }
template <class R> __device__ __forceinline__ Q4<R> fqexpRaw(V3<R> v) {
  const R a2 = dot(v, v);
  R c, k;
  if (sizeof(R) == 4 && a2 <= R(0.0625)) {
    const R h2 = R(0.25) * a2;
    k = R(0.5) * (R(1) + h2 * (R(-1.0 / 6) + h2 * (R(1.0 / 120) - h2 * R(1.0 / 5040))));
    c = R(1) + h2 * (R(-0.5) + h2 * (R(1.0 / 24) - h2 * R(1.0 / 720)));
  } else {
    const R a = fsqrt(a2);
    R s;
    sincosT(a * R(0.5), &s, &c);
    k = a < R(1e-8) ? R(0.5) - a2 / R(48) : s * frcp(a);
  }
  return Q4<R>{c, k * v.x, k * v.y, k * v.z};
}
// Logarithm of a (near) unit quaternion (kernel.cuh:146-153).  The result
// depends on q only through the direction of its vector part and the angle
// atan2(|v|, w), both unchanged by a positive scale, so q is not normalised
// first.
template <class R> __device__ __forceinline__ V3<R> fqlog(Q4<R> q) {
  if (q.w < R(0)) q = {-q.w, -q.x, -q.y, -q.z};
  V3<R> v{q.x, q.y, q.z};
  R s = fnorm(v);
  return v * (s < R(1e-10) ? R(2) : R(2) * fatan2(s, q.w) * frcp(s));
}
}  // namespace duckb200
