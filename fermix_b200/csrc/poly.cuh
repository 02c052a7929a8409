// Closed forms for tiny matrices: det for n <= 4 and pf for even n <= 6, with their
// exact (polynomial) gradients. One thread per matrix.
//
// Reference: src/fermix/_poly.py:10-60 (the same expressions: 2x2 minors, the 3x3
// expansion along row 0, the Laplace expansion along rows (0, 1) at n = 4, the
// perfect-matching sums for pf) and the derivative rules of src/fermix/_diff.py:114-119,
// :143-149, :290-292, :321-324 (the adjugate / minor Pfaffians, finite for any input).
#pragma once
#include "fused_lu.cuh"

namespace fx {

constexpr int DET_POLY_MAX = 4;
constexpr int PF_POLY_MAX = 6;

// det of the k x k submatrix (rows ri[], cols ci[]) of the n x n matrix M (row-major).
template <typename T>
__device__ T det_poly(const T* M, int n, const int* ri, const int* ci, int k) {
  auto a = [&](int i, int j) { return M[ri[i] * n + ci[j]]; };
  auto m2 = [&](int r, int s, int i, int j) { return sub(mul(a(r, i), a(s, j)), mul(a(r, j), a(s, i))); };
  if (k == 0) return s_one<T>();
  if (k == 1) return a(0, 0);
  if (k == 2) return m2(0, 1, 0, 1);
  if (k == 3) {
    T c0 = mul(a(0, 0), m2(1, 2, 1, 2));
    T c1 = mul(a(0, 1), m2(1, 2, 0, 2));
    T c2 = mul(a(0, 2), m2(1, 2, 0, 1));
    return add(sub(c0, c1), c2);
  }
  T p01 = mul(m2(0, 1, 0, 1), m2(2, 3, 2, 3));
  T p02 = mul(m2(0, 1, 0, 2), m2(2, 3, 1, 3));
  T p03 = mul(m2(0, 1, 0, 3), m2(2, 3, 1, 2));
  T p12 = mul(m2(0, 1, 1, 2), m2(2, 3, 0, 3));
  T p13 = mul(m2(0, 1, 1, 3), m2(2, 3, 0, 2));
  T p23 = mul(m2(0, 1, 2, 3), m2(2, 3, 0, 1));
  return add(sub(add(add(sub(p01, p02), p03), p12), p13), p23);
}

// pf of the k x k principal submatrix (indices ix[]) of the skew n x n matrix S.
template <typename T>
__device__ T pf_poly(const T* S, int n, const int* ix, int k) {
  auto s = [&](int i, int j) { return S[ix[i] * n + ix[j]]; };
  auto pf4 = [&](int a, int b, int c, int d) {
    return add(sub(mul(s(a, b), s(c, d)), mul(s(a, c), s(b, d))), mul(s(a, d), s(b, c)));
  };
  if (k == 0) return s_one<T>();
  if (k == 2) return s(0, 1);
  if (k == 4) return pf4(0, 1, 2, 3);
  T t1 = mul(s(0, 1), pf4(2, 3, 4, 5));
  T t2 = mul(s(0, 2), pf4(1, 3, 4, 5));
  T t3 = mul(s(0, 3), pf4(1, 2, 4, 5));
  T t4 = mul(s(0, 4), pf4(1, 2, 3, 5));
  T t5 = mul(s(0, 5), pf4(1, 2, 3, 4));
  return add(sub(add(sub(t1, t2), t3), t4), t5);
}

template <typename T>
__device__ __forceinline__ void sign_log(T x, T& s, typename Sc<T>::R& l) {
  s = unit(x);
  l = rlog(mag(x));
}

// 1 / x with 1 / 0 -> 0 (_poly.py:67-71)
template <typename T>
__device__ __forceinline__ T safe_recip(T x) {
  return is_zero(x) ? s_zero<T>() : sdiv(s_one<T>(), x);
}

// is_pf: pf / slogpf on the (optionally skew-symmetrised) input, else det / slogdet.
// mode as in Job; a 6 x 6 scratch copy per thread holds the matrix.
template <typename T>
__global__ void poly_kernel(Job<T> J, int is_pf) {
  typedef typename Sc<T>::R R;
  const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (b >= J.B) return;
  const int n = J.n;
  T M[36];
  const T* src = J.a + b * (int64_t)n * n;
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < n; ++j) {
      T v = src[i * n + j];
      if (is_pf && J.skew) v = scale(sub(v, src[j * n + i]), R(0.5));
      M[i * n + j] = v;
    }
  int ix[6] = {0, 1, 2, 3, 4, 5};
  const T val = is_pf ? pf_poly(M, n, ix, n) : det_poly(M, n, ix, ix, n);
  T s;
  R l;
  sign_log(val, s, l);
  J.sign[b] = s;
  J.logabs[b] = l;
  if (J.value) J.value[b] = val;
  if (J.mode == MODE_FWD) return;
  const T cf = J.coef ? J.coef[b] : s_one<T>();
  T f = cf;
  if (J.mode == MODE_SLOG_GRAD) f = mul(cf, safe_recip(val));
  T* G = J.g + b * (int64_t)n * n;
  if (!is_pf) {
    // d det / dA = adj(A)^T: the signed complementary minors
    for (int i = 0; i < n; ++i)
      for (int j = 0; j < n; ++j) {
        int ri[3], ci[3];
        int a = 0, c = 0;
        for (int t = 0; t < n; ++t) {
          if (t != i) ri[a++] = t;
          if (t != j) ci[c++] = t;
        }
        T m = n == 1 ? s_one<T>() : det_poly(M, n, ri, ci, n - 1);
        if ((i + j) & 1) m = neg(m);
        T v = mul(f, m);
        G[i * n + j] = J.conj_out ? conj_(v) : v;
      }
  } else {
    // d pf / d s_ij (i < j) = (-1)^(i+j+1) pf(S without i, j); the gradient w.r.t. a
    // skew (or skew-symmetrised) input is (D - D^T) / 2
    for (int i = 0; i < n; ++i) G[i * n + i] = s_zero<T>();
    for (int i = 0; i < n; ++i)
      for (int j = i + 1; j < n; ++j) {
        int kx[4];
        int a = 0;
        for (int t = 0; t < n; ++t)
          if (t != i && t != j) kx[a++] = t;
        T m = pf_poly(M, n, kx, n - 2);
        if (((i + j + 1) & 1)) m = neg(m);
        T v = mul(f, scale(m, R(0.5)));
        G[i * n + j] = J.conj_out ? conj_(v) : v;
        T vn = neg(mul(f, scale(m, R(0.5))));
        G[j * n + i] = J.conj_out ? conj_(vn) : vn;
      }
  }
}

// Odd n for pf / slogpf: (0, -inf), value 0, zero gradient (src/fermix/api.py:122-123).
template <typename T>
__global__ void pf_odd_kernel(Job<T> J) {
  const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (b >= J.B) return;
  J.sign[b] = s_zero<T>();
  J.logabs[b] = -INFINITY;
  if (J.value) J.value[b] = s_zero<T>();
}

}  // namespace fx
