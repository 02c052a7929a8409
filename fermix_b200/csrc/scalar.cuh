// Scalar field of one call: float, double, complex<float>, complex<double>.
//
// Conventions follow the reference's value layer (src/fermix/_field.py):
//   abs1(x)  = |x| for real, |re| + |im| for complex: the pivot metric (_field.py:131-136)
//   mag(x)   = the modulus |x| (log|pivot|, _field.py:139-143)
//   unit(x)  = x / |x|, 0 -> 0 (the sign contribution of a pivot, _field.py:165-170)
//   recip(x) = 1 / x, 0 -> 0 (the guarded reciprocal, _field.py:152-162)
// Complex values are (re, im) pairs of the real component type, stored interleaved in
// HBM exactly like numpy / torch / XLA complex arrays.
//
// Every multiply-add that updates a matrix entry goes through fms() (acc - l * u as an
// explicit chain of fused multiply-adds in a fixed order). Two rows that hold the same
// bits and receive the same multipliers therefore stay bitwise equal, which is what makes
// a duplicated row come out as an exactly zero pivot.
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace fx {

template <typename R>
struct cplx {
  R re, im;
};

typedef cplx<float> c64_t;
typedef cplx<double> c128_t;

template <typename T>
struct Sc;

template <>
struct Sc<float> {
  typedef float R;
  static constexpr bool cx = false;
};
template <>
struct Sc<double> {
  typedef double R;
  static constexpr bool cx = false;
};
template <>
struct Sc<c64_t> {
  typedef float R;
  static constexpr bool cx = true;
};
template <>
struct Sc<c128_t> {
  typedef double R;
  static constexpr bool cx = true;
};

__device__ __forceinline__ float rfma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double rfma(double a, double b, double c) { return __fma_rn(a, b, c); }
__device__ __forceinline__ float rmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double rmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float rdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double rdiv(double a, double b) { return __ddiv_rn(a, b); }
__device__ __forceinline__ float rlog(float a) { return logf(a); }
__device__ __forceinline__ double rlog(double a) { return log(a); }
__device__ __forceinline__ float rexp(float a) { return expf(a); }
__device__ __forceinline__ double rexp(double a) { return exp(a); }
__device__ __forceinline__ float rhypot(float a, float b) { return hypotf(a, b); }
__device__ __forceinline__ double rhypot(double a, double b) { return hypot(a, b); }
__device__ __forceinline__ float rsqrt_(float a) { return sqrtf(a); }
__device__ __forceinline__ double rsqrt_(double a) { return sqrt(a); }
__device__ __forceinline__ bool risfinite(float a) { return isfinite(a); }
__device__ __forceinline__ bool risfinite(double a) { return isfinite(a); }

// ---------------------------------------------------------------- real ops
__device__ __forceinline__ float zero_of(float) { return 0.f; }
__device__ __forceinline__ double zero_of(double) { return 0.0; }
__device__ __forceinline__ c64_t zero_of(c64_t) { return {0.f, 0.f}; }
__device__ __forceinline__ c128_t zero_of(c128_t) { return {0.0, 0.0}; }

template <typename T>
__device__ __forceinline__ T s_zero() {
  return zero_of(T());
}
template <typename T>
__device__ __forceinline__ T s_one();
template <>
__device__ __forceinline__ float s_one<float>() {
  return 1.f;
}
template <>
__device__ __forceinline__ double s_one<double>() {
  return 1.0;
}
template <>
__device__ __forceinline__ c64_t s_one<c64_t>() {
  return {1.f, 0.f};
}
template <>
__device__ __forceinline__ c128_t s_one<c128_t>() {
  return {1.0, 0.0};
}

template <typename R>
__device__ __forceinline__ R s_from_real(R x, R*) {
  return x;
}

// real: acc - l * u
__device__ __forceinline__ float fms(float acc, float l, float u) { return rfma(-l, u, acc); }
__device__ __forceinline__ double fms(double acc, double l, double u) { return rfma(-l, u, acc); }
// complex: the same four real FMAs in a fixed order
template <typename R>
__device__ __forceinline__ cplx<R> fms(cplx<R> acc, cplx<R> l, cplx<R> u) {
  R re = rfma(-l.re, u.re, acc.re);
  re = rfma(l.im, u.im, re);
  R im = rfma(-l.re, u.im, acc.im);
  im = rfma(-l.im, u.re, im);
  return {re, im};
}
// acc + a * b
__device__ __forceinline__ float fma_(float a, float b, float acc) { return rfma(a, b, acc); }
__device__ __forceinline__ double fma_(double a, double b, double acc) { return rfma(a, b, acc); }
template <typename R>
__device__ __forceinline__ cplx<R> fma_(cplx<R> a, cplx<R> b, cplx<R> acc) {
  R re = rfma(a.re, b.re, acc.re);
  re = rfma(-a.im, b.im, re);
  R im = rfma(a.re, b.im, acc.im);
  im = rfma(a.im, b.re, im);
  return {re, im};
}

__device__ __forceinline__ float mul(float a, float b) { return rmul(a, b); }
__device__ __forceinline__ double mul(double a, double b) { return rmul(a, b); }
template <typename R>
__device__ __forceinline__ cplx<R> mul(cplx<R> a, cplx<R> b) {
  return {rfma(a.re, b.re, -rmul(a.im, b.im)), rfma(a.re, b.im, rmul(a.im, b.re))};
}
__device__ __forceinline__ float add(float a, float b) { return a + b; }
__device__ __forceinline__ double add(double a, double b) { return a + b; }
template <typename R>
__device__ __forceinline__ cplx<R> add(cplx<R> a, cplx<R> b) {
  return {a.re + b.re, a.im + b.im};
}
__device__ __forceinline__ float sub(float a, float b) { return a - b; }
__device__ __forceinline__ double sub(double a, double b) { return a - b; }
template <typename R>
__device__ __forceinline__ cplx<R> sub(cplx<R> a, cplx<R> b) {
  return {a.re - b.re, a.im - b.im};
}
__device__ __forceinline__ float neg(float a) { return -a; }
__device__ __forceinline__ double neg(double a) { return -a; }
template <typename R>
__device__ __forceinline__ cplx<R> neg(cplx<R> a) {
  return {-a.re, -a.im};
}
__device__ __forceinline__ float scale(float a, float s) { return rmul(a, s); }
__device__ __forceinline__ double scale(double a, double s) { return rmul(a, s); }
template <typename R>
__device__ __forceinline__ cplx<R> scale(cplx<R> a, R s) {
  return {rmul(a.re, s), rmul(a.im, s)};
}
__device__ __forceinline__ float conj_(float a) { return a; }
__device__ __forceinline__ double conj_(double a) { return a; }
template <typename R>
__device__ __forceinline__ cplx<R> conj_(cplx<R> a) {
  return {a.re, -a.im};
}

__device__ __forceinline__ float abs1(float a) { return fabsf(a); }
__device__ __forceinline__ double abs1(double a) { return fabs(a); }
template <typename R>
__device__ __forceinline__ R abs1(cplx<R> a) {
  return fabs(a.re) + fabs(a.im);
}
__device__ __forceinline__ float mag(float a) { return fabsf(a); }
__device__ __forceinline__ double mag(double a) { return fabs(a); }
template <typename R>
__device__ __forceinline__ R mag(cplx<R> a) {
  return rhypot(a.re, a.im);
}
__device__ __forceinline__ bool is_zero(float a) { return a == 0.f; }
__device__ __forceinline__ bool is_zero(double a) { return a == 0.0; }
template <typename R>
__device__ __forceinline__ bool is_zero(cplx<R> a) {
  return a.re == R(0) && a.im == R(0);
}
__device__ __forceinline__ bool is_finite(float a) { return isfinite(a); }
__device__ __forceinline__ bool is_finite(double a) { return isfinite(a); }
template <typename R>
__device__ __forceinline__ bool is_finite(cplx<R> a) {
  return risfinite(a.re) && risfinite(a.im);
}
__device__ __forceinline__ float re_(float a) { return a; }
__device__ __forceinline__ double re_(double a) { return a; }
template <typename R>
__device__ __forceinline__ R re_(cplx<R> a) {
  return a.re;
}

// x / y, correctly rounded for real; for complex the form that returns exactly 1 for
// x == y (no fused product in the cross term, so b*c - a*d cancels exactly).
__device__ __forceinline__ float sdiv(float x, float y) { return rdiv(x, y); }
__device__ __forceinline__ double sdiv(double x, double y) { return rdiv(x, y); }
template <typename R>
__device__ __forceinline__ cplx<R> sdiv(cplx<R> x, cplx<R> y) {
  R den = rfma(y.re, y.re, rmul(y.im, y.im));
  R nre = rfma(x.re, y.re, rmul(x.im, y.im));
  R nim = rmul(x.im, y.re) - rmul(x.re, y.im);
  return {rdiv(nre, den), rdiv(nim, den)};
}
// guarded reciprocal (0 -> 0)
__device__ __forceinline__ float recip(float x) { return x == 0.f ? 0.f : rdiv(1.f, x); }
__device__ __forceinline__ double recip(double x) { return x == 0.0 ? 0.0 : rdiv(1.0, x); }
template <typename R>
__device__ __forceinline__ cplx<R> recip(cplx<R> x) {
  R m2 = rfma(x.re, x.re, rmul(x.im, x.im));
  R inv = m2 == R(0) ? R(0) : rdiv(R(1), m2);
  return {rmul(x.re, inv), -rmul(x.im, inv)};
}
// x / |x|, 0 -> 0
__device__ __forceinline__ float unit(float x) { return x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f); }
__device__ __forceinline__ double unit(double x) { return x > 0.0 ? 1.0 : (x < 0.0 ? -1.0 : 0.0); }
template <typename R>
__device__ __forceinline__ cplx<R> unit(cplx<R> x) {
  R m = rhypot(x.re, x.im);
  if (m == R(0)) return {R(0), R(0)};
  return {rdiv(x.re, m), rdiv(x.im, m)};
}

// --------------------------------------------------------------- warp helpers
template <typename R>
__device__ __forceinline__ R shfl_xor_r(R v, int m) {
  return __shfl_xor_sync(0xffffffffu, v, m);
}
template <typename T>
__device__ __forceinline__ T shfl_idx(T v, int src);
template <>
__device__ __forceinline__ float shfl_idx<float>(float v, int src) {
  return __shfl_sync(0xffffffffu, v, src);
}
template <>
__device__ __forceinline__ double shfl_idx<double>(double v, int src) {
  return __shfl_sync(0xffffffffu, v, src);
}
template <>
__device__ __forceinline__ c64_t shfl_idx<c64_t>(c64_t v, int src) {
  return {__shfl_sync(0xffffffffu, v.re, src), __shfl_sync(0xffffffffu, v.im, src)};
}
template <>
__device__ __forceinline__ c128_t shfl_idx<c128_t>(c128_t v, int src) {
  return {__shfl_sync(0xffffffffu, v.re, src), __shfl_sync(0xffffffffu, v.im, src)};
}

// Warp argmax of (value, index): the largest value, ties -> the smallest index.
template <typename R>
__device__ __forceinline__ void warp_argmax(R& v, int& i) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    R ov = __shfl_xor_sync(0xffffffffu, v, off);
    int oi = __shfl_xor_sync(0xffffffffu, i, off);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

// Neumaier-compensated running sum (the log of |det| / |pf| over n pivots).
template <typename R>
struct KSum {
  R s, c;
  __device__ __forceinline__ void init() {
    s = R(0);
    c = R(0);
  }
  __device__ __forceinline__ void add(R x) {
    R t = s + x;
    if (fabs(s) >= fabs(x))
      c += (s - t) + x;
    else
      c += (x - t) + s;
    s = t;
  }
  __device__ __forceinline__ R value() const {
    // -inf / nan propagate through s; the compensation is finite only when s is
    return isfinite(s) ? s + c : s;
  }
};

// Optional per-phase cycle counters for profiling builds (-DFX_PHASE_TIMERS): thread 0
// of each block adds clock64() deltas into fx_phase_cycles[phase].
#ifdef FX_PHASE_TIMERS
static __device__ unsigned long long fx_phase_cycles[16];
#define FX_TIC(var) long long var = clock64()
#define FX_TOC(var, ph)                                                              \
  do {                                                                               \
    if (threadIdx.x == 0) atomicAdd(&fx_phase_cycles[ph], (unsigned long long)(clock64() - var)); \
    var = clock64();                                                                 \
  } while (0)
#else
#define FX_TIC(var)
#define FX_TOC(var, ph)
#endif

}  // namespace fx
