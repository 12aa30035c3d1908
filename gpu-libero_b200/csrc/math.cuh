// Small precision-generic helpers for the physics kernels (float or double).
#pragma once
#include <cuda_runtime.h>
#include <cmath>

namespace b200 {

__device__ __forceinline__ float msqrt(float x) { return sqrtf(x); }
__device__ __forceinline__ double msqrt(double x) { return sqrt(x); }
__device__ __forceinline__ float msin(float x) { return sinf(x); }
__device__ __forceinline__ double msin(double x) { return sin(x); }
__device__ __forceinline__ float mcos(float x) { return cosf(x); }
__device__ __forceinline__ double mcos(double x) { return cos(x); }
__device__ __forceinline__ float mpow(float a, float b) { return powf(a, b); }
__device__ __forceinline__ double mpow(double a, double b) { return pow(a, b); }
__device__ __forceinline__ float mabs(float x) { return fabsf(x); }
__device__ __forceinline__ double mabs(double x) { return fabs(x); }
template <class R> __device__ __forceinline__ R mmin(R a, R b) { return a < b ? a : b; }
template <class R> __device__ __forceinline__ R mmax(R a, R b) { return a > b ? a : b; }
template <class R> __device__ __forceinline__ R mclamp(R x, R lo, R hi) { return mmax(lo, mmin(hi, x)); }
template <class R> __device__ __forceinline__ R safe_div(R x, R y) { return x / (y != R(0) ? y : R(1e-15)); }

template <class R> struct V3 {
  R x, y, z;
  __device__ R &operator[](int i) { return i == 0 ? x : (i == 1 ? y : z); }
  __device__ R operator[](int i) const { return i == 0 ? x : (i == 1 ? y : z); }
};
template <class R> __device__ __forceinline__ V3<R> v3(R x, R y, R z) { return {x, y, z}; }
template <class R> __device__ __forceinline__ V3<R> ld3(const R *p) { return {p[0], p[1], p[2]}; }
template <class R> __device__ __forceinline__ void st3(R *p, V3<R> a) { p[0] = a.x; p[1] = a.y; p[2] = a.z; }
template <class R> __device__ __forceinline__ V3<R> operator+(V3<R> a, V3<R> b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
template <class R> __device__ __forceinline__ V3<R> operator-(V3<R> a, V3<R> b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
template <class R> __device__ __forceinline__ V3<R> operator-(V3<R> a) { return {-a.x, -a.y, -a.z}; }
template <class R> __device__ __forceinline__ V3<R> operator*(V3<R> a, R s) { return {a.x * s, a.y * s, a.z * s}; }
template <class R> __device__ __forceinline__ R dot(V3<R> a, V3<R> b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
template <class R> __device__ __forceinline__ V3<R> cross(V3<R> a, V3<R> b) {
  return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}
template <class R> __device__ __forceinline__ V3<R> normalize(V3<R> a) {
  R n = msqrt(dot(a, a));
  return n > R(0) ? a * (R(1) / n) : v3<R>(0, 0, 0);
}
// row-major 3x3
template <class R> __device__ __forceinline__ V3<R> rot(const R *r, V3<R> x) {
  return {r[0] * x.x + r[1] * x.y + r[2] * x.z, r[3] * x.x + r[4] * x.y + r[5] * x.z,
          r[6] * x.x + r[7] * x.y + r[8] * x.z};
}
template <class R> __device__ __forceinline__ V3<R> rotT(const R *r, V3<R> x) {
  return {r[0] * x.x + r[3] * x.y + r[6] * x.z, r[1] * x.x + r[4] * x.y + r[7] * x.z,
          r[2] * x.x + r[5] * x.y + r[8] * x.z};
}
template <class R> __device__ __forceinline__ V3<R> col(const R *r, int k) { return {r[k], r[3 + k], r[6 + k]}; }

template <class R> struct Q4 { R w, x, y, z; };
template <class R> __device__ __forceinline__ Q4<R> ldq(const R *p) { return {p[0], p[1], p[2], p[3]}; }
template <class R> __device__ __forceinline__ void stq(R *p, Q4<R> q) { p[0] = q.w; p[1] = q.x; p[2] = q.y; p[3] = q.z; }
template <class R> __device__ __forceinline__ Q4<R> qnormalize(Q4<R> q) {
  R n = msqrt(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
  if (n > R(0)) {
    R r = R(1) / n;
    return {q.w * r, q.x * r, q.y * r, q.z * r};
  }
  return {R(0), R(0), R(0), R(1)};
}
template <class R> __device__ __forceinline__ Q4<R> qmul(Q4<R> a, Q4<R> b) {
  return {a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z, a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y,
          a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x, a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w};
}
template <class R> __device__ __forceinline__ V3<R> qrot(V3<R> v, Q4<R> q) {
  V3<R> u = {q.x, q.y, q.z};
  V3<R> r = u * (R(2) * dot(u, v)) + v * (q.w * q.w - dot(u, u));
  return r + cross(u, v) * (R(2) * q.w);
}
template <class R> __device__ __forceinline__ void qmat(R *p, Q4<R> q) {
  R a = q.w * q.w, b = q.w * q.x, c = q.w * q.y, d = q.w * q.z;
  R e = q.x * q.x, f = q.x * q.y, h = q.x * q.z, j = q.y * q.y, k = q.y * q.z, l = q.z * q.z;
  p[0] = a + e - j - l; p[1] = R(2) * (f - d); p[2] = R(2) * (h + c);
  p[3] = R(2) * (f + d); p[4] = a - e + j - l; p[5] = R(2) * (k - b);
  p[6] = R(2) * (h - c); p[7] = R(2) * (k + b); p[8] = a - e - j + l;
}

// spatial inertia (vec10: I00 I11 I22 I01 I02 I12, m*c, m) times motion (ang, lin)
template <class R> __device__ __forceinline__ void inert_mul(const R *i, const R *v, R *r) {
  r[0] = i[0] * v[0] + i[3] * v[1] + i[4] * v[2] - i[8] * v[4] + i[7] * v[5];
  r[1] = i[3] * v[0] + i[1] * v[1] + i[5] * v[2] + i[8] * v[3] - i[6] * v[5];
  r[2] = i[4] * v[0] + i[5] * v[1] + i[2] * v[2] - i[7] * v[3] + i[6] * v[4];
  r[3] = i[8] * v[1] - i[7] * v[2] + i[9] * v[3];
  r[4] = i[6] * v[2] - i[8] * v[0] + i[9] * v[4];
  r[5] = i[7] * v[0] - i[6] * v[1] + i[9] * v[5];
}

}  // namespace b200
