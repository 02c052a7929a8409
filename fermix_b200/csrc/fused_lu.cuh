// Batched LU with partial pivoting: slogdet / det forward and their gradients, one
// thread block per matrix, the whole factorisation and the inverse on chip.
//
// Reference behaviour (ChenAo-Phys/fermix, paths relative to that project):
//   forward  : src/fermix/_lu.py:543-611 (_lu_core), pivot = first-occurrence argmax
//              of abs1 over the unassigned rows (_lu.py:151-152), sign = prod unit(pivot)
//              times (-1)^swaps, logabs = sum log|pivot|, a zero pivot gives a zero L
//              column, sign 0 and logabs -inf (_lu.py:167-174)
//   gradient : src/fermix/_inverse.py:502-531 (_lu_parts): A^-T = (U~^-1 L^-1 P)^T with
//              zero pivots replaced by 1, zeroed for singular / non-finite members;
//              det: src/fermix/_diff.py:205-246 (_det_gradT) incl. the Woodbury branch
//              for one or two exact zero pivots.
//
// Design (B200): the matrix sits in shared memory (227 KB per block) when it fits and
// otherwise in a per-block global workspace slot (L2 resident while the block works on
// it). LAPACK-style blocked right-looking factorisation with physical row swaps: one
// warp factors a panel of FX_NB columns, then the block applies the interchanges, the
// U-row triangular solve and a register-tiled trailing update. Every entry is updated by
// one sequential FMA chain over the panel columns (same order in the panel, the U-row
// solve and the trailing update), so a duplicated row becomes an exactly zero row and
// the matrix reports (0, -inf) as an exactly singular input must.
#pragma once
#include "scalar.cuh"

namespace fx {

#ifndef FX_NB
#define FX_NB 16
#endif

enum { MODE_FWD = 0, MODE_SLOG_GRAD = 1, MODE_VALUE_GRAD = 2 };

template <typename T>
struct Job {
  const T* a;                  // (B, n, n) input, row-major, complex interleaved
  T* sign;                     // (B,) sign (input dtype)
  typename Sc<T>::R* logabs;   // (B,) log|det| / log|pf|
  T* g;                        // (B, n, n) gradient output (modes 1, 2) or null
  T* value;                    // (B,) det / pf value or null
  const T* coef;               // (B,) per-matrix gradient coefficient or null (= 1)
  int conj_out;                // write conj(coef * D)
  int skew;                    // pf: skew-symmetrise the input as (a - a^T) / 2
  int64_t B;
  int n;
  int mode;
  int prec;                    // FX_PREC_* of the call (the blocked engines' update kind)
  int ld;                      // leading dimension of the work buffers
  int in_smem;                 // work buffers in dynamic shared memory
  T* ws;                       // global work slots (gridDim.x * nbuf * n * ld) otherwise
  uint32_t wait_polls;         // polls of each bounded wait (tensor-memory kernels)
  // complex input / gradient as split real and imaginary planes (B, n, n) each: when a_re
  // is set it replaces a, and when g_re is set it replaces g (read and written only by the
  // blocked engines' copy-in and gradient kernels)
  const typename Sc<T>::R* a_re;
  const typename Sc<T>::R* a_im;
  typename Sc<T>::R* g_re;
  typename Sc<T>::R* g_im;
  // row gather (tensor-memory LU only): matrix b row i = gbase[gidx[b * n + i] * gld + 0 .. n),
  // NaN for an index outside [0, grows)
  const int* gidx;
  const T* gbase;
  int64_t gld, grows;
};

// ---------------------------------------------------------------- block helpers
__device__ __forceinline__ int nthr() { return blockDim.x; }

template <typename T>
__device__ __forceinline__ void swap_(T& a, T& b) {
  T t = a;
  a = b;
  b = t;
}

// Load matrix b into the work buffer (pf: optionally (a - a^T) / 2).
template <typename T>
__device__ void load_matrix(const Job<T>& J, int64_t b, T* A, int ld, bool skew) {
  const int n = J.n;
  const T* src = J.a + b * (int64_t)n * n;
  const int nn = n * n;
  if (!skew) {
    for (int idx = threadIdx.x; idx < nn; idx += nthr()) {
      int r = idx / n, c = idx - r * n;
      A[r * ld + c] = src[idx];
    }
  } else {
    typedef typename Sc<T>::R R;
    for (int idx = threadIdx.x; idx < nn; idx += nthr()) {
      int r = idx / n, c = idx - r * n;
      A[r * ld + c] = scale(sub(src[idx], src[c * n + r]), R(0.5));
    }
  }
}

// Trailing update A[r][c] -= sum_s A[r][k0+s] * A[k0+s][c] for r, c in [r0, n), one FMA
// chain per entry in the order s = 0 .. kb-1. Threads form a TR x 16 grid with a cyclic
// assignment of rows and columns (consecutive lanes -> consecutive columns).
template <typename T, int MI, int MJ>
__device__ void lu_trailing(T* A, int ld, int r0, int n, int k0, int kb) {
  const int m = n - r0;
  if (m <= 0) return;
  const int TC = 16;
  const int TR = nthr() / TC;
  const int ti = threadIdx.x / TC, tj = threadIdx.x % TC;
  for (int bi = 0; bi < m; bi += TR * MI) {
    for (int bj = 0; bj < m; bj += TC * MJ) {
      int rr[MI], cc[MJ];
      bool rv[MI], cv[MJ];
#pragma unroll
      for (int i = 0; i < MI; ++i) {
        rr[i] = r0 + bi + ti + TR * i;
        rv[i] = rr[i] < n;
      }
#pragma unroll
      for (int j = 0; j < MJ; ++j) {
        cc[j] = r0 + bj + tj + TC * j;
        cv[j] = cc[j] < n;
      }
      bool any = false;
#pragma unroll
      for (int i = 0; i < MI; ++i) any |= rv[i];
      bool anyc = false;
#pragma unroll
      for (int j = 0; j < MJ; ++j) anyc |= cv[j];
      if (!any || !anyc) continue;
      T acc[MI][MJ];
#pragma unroll
      for (int i = 0; i < MI; ++i)
#pragma unroll
        for (int j = 0; j < MJ; ++j) acc[i][j] = (rv[i] && cv[j]) ? A[rr[i] * ld + cc[j]] : s_zero<T>();
      for (int s = 0; s < kb; ++s) {
        T l[MI], u[MJ];
#pragma unroll
        for (int i = 0; i < MI; ++i) l[i] = rv[i] ? A[rr[i] * ld + k0 + s] : s_zero<T>();
#pragma unroll
        for (int j = 0; j < MJ; ++j) u[j] = cv[j] ? A[(k0 + s) * ld + cc[j]] : s_zero<T>();
#pragma unroll
        for (int i = 0; i < MI; ++i)
#pragma unroll
          for (int j = 0; j < MJ; ++j) acc[i][j] = fms(acc[i][j], l[i], u[j]);
      }
#pragma unroll
      for (int i = 0; i < MI; ++i)
#pragma unroll
        for (int j = 0; j < MJ; ++j)
          if (rv[i] && cv[j]) A[rr[i] * ld + cc[j]] = acc[i][j];
    }
  }
}

template <typename T>
struct TileShape {
  static constexpr int MI = Sc<T>::cx ? 2 : 4;
  static constexpr int MJ = Sc<T>::cx ? 2 : 4;
};

// Shared per-matrix scalars of the factorisation.
template <typename T>
struct FacState {
  T sign;
  typename Sc<T>::R logabs;
  int parity;
  int nzero;  // number of exactly zero pivots
  int k1, k2; // first / last zero pivot
  int bad;    // non-finite inverse entry seen
};

// Blocked LU of the n x n matrix in A (leading dimension ld), in place: L (unit, strictly
// below the diagonal) and U; ipiv[j] = the row interchanged with j at step j (LAPACK).
// The scalars go to st (written by thread 0).
template <typename T>
__device__ void lu_factor(T* A, int ld, int n, int* ipiv, FacState<T>* st) {
  typedef typename Sc<T>::R R;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  T sgn = s_one<T>();
  KSum<R> ls;
  ls.init();
  int par = 0, nzero = 0, k1 = -1, k2 = -1;
  for (int k0 = 0; k0 < n; k0 += FX_NB) {
    const int kb = min(FX_NB, n - k0);
    if (warp == 0) {
      for (int jj = 0; jj < kb; ++jj) {
        const int j = k0 + jj;
        R best = R(-1);
        int bi = 0x7fffffff;
        for (int r = j + lane; r < n; r += 32) {
          R v = abs1(A[r * ld + j]);
          if (v > best) {
            best = v;
            bi = r;
          }
        }
        warp_argmax(best, bi);
        const int p = (bi == 0x7fffffff) ? j : bi;
        if (p != j) {
          for (int c = k0 + lane; c < k0 + kb; c += 32) swap_(A[j * ld + c], A[p * ld + c]);
        }
        __syncwarp();
        const T piv = A[j * ld + j];
        const bool z = is_zero(piv);
        if (lane == 0) {
          ipiv[j] = p;
          par ^= (p != j);
          sgn = mul(sgn, unit(piv));
          ls.add(rlog(mag(piv)));
          if (z) {
            if (k1 < 0) k1 = j;
            k2 = j;
            ++nzero;
          }
        }
        for (int r = j + 1 + lane; r < n; r += 32) {
          const T l = z ? s_zero<T>() : sdiv(A[r * ld + j], piv);
          A[r * ld + j] = l;
          for (int c = j + 1; c < k0 + kb; ++c) A[r * ld + c] = fms(A[r * ld + c], l, A[j * ld + c]);
        }
        __syncwarp();
      }
    }
    __syncthreads();
    // interchanges outside the panel, then U_k = L_kk^-1 A[k rows, trailing cols]
    for (int c = tid; c < n; c += nthr()) {
      if (c >= k0 && c < k0 + kb) continue;
      for (int jj = 0; jj < kb; ++jj) {
        const int j = k0 + jj, p = ipiv[j];
        if (p != j) swap_(A[j * ld + c], A[p * ld + c]);
      }
      if (c >= k0 + kb) {
        for (int t = 1; t < kb; ++t) {
          T acc = A[(k0 + t) * ld + c];
          for (int s = 0; s < t; ++s) acc = fms(acc, A[(k0 + t) * ld + k0 + s], A[(k0 + s) * ld + c]);
          A[(k0 + t) * ld + c] = acc;
        }
      }
    }
    __syncthreads();
    lu_trailing<T, TileShape<T>::MI, TileShape<T>::MJ>(A, ld, k0 + kb, n, k0, kb);
    __syncthreads();
  }
  if (tid == 0) {
    if (par) sgn = neg(sgn);
    if (nzero) sgn = s_zero<T>();
    if constexpr (Sc<T>::cx) {
      // renormalise the product of unit phases (drifts by ~n ulp; _lu.py:614-621)
      R m = rhypot(sgn.re, sgn.im);
      if (m != R(0)) sgn = {rdiv(sgn.re, m), rdiv(sgn.im, m)};
    }
    st->sign = sgn;
    st->logabs = nzero ? -INFINITY : ls.value();
    st->parity = par;
    st->nzero = nzero;
    st->k1 = k1;
    st->k2 = k2;
    st->bad = 0;
  }
  __syncthreads();
}

// X = U~^-1 L^-1 (U~: U with exact zero pivots replaced by 1) into W (leading dimension
// ld), one column per thread: forward substitution with the unit lower L, then back
// substitution with U~. Reads the packed LU in A only.
template <typename T>
__device__ void lu_inverse_cols(const T* A, T* W, int ld, int n, FacState<T>* st) {
  for (int j = threadIdx.x; j < n; j += nthr()) {
    // L y = e_j: y[i] = 0 (i < j), 1 (i == j)
    for (int i = 0; i < j; ++i) W[i * ld + j] = s_zero<T>();
    W[j * ld + j] = s_one<T>();
    for (int i = j + 1; i < n; ++i) {
      T acc0 = s_zero<T>(), acc1 = s_zero<T>();
      int k = j;
      for (; k + 1 < i; k += 2) {
        acc0 = fma_(A[i * ld + k], W[k * ld + j], acc0);
        acc1 = fma_(A[i * ld + k + 1], W[(k + 1) * ld + j], acc1);
      }
      if (k < i) acc0 = fma_(A[i * ld + k], W[k * ld + j], acc0);
      W[i * ld + j] = neg(add(acc0, acc1));
    }
    // U~ x = y, bottom-up
    bool bad = false;
    for (int i = n - 1; i >= 0; --i) {
      T acc0 = W[i * ld + j], acc1 = s_zero<T>();
      int k = i + 1;
      for (; k + 1 < n; k += 2) {
        acc0 = fms(acc0, A[i * ld + k], W[k * ld + j]);
        acc1 = fms(acc1, A[i * ld + k + 1], W[(k + 1) * ld + j]);
      }
      if (k < n) acc0 = fms(acc0, A[i * ld + k], W[k * ld + j]);
      T u = A[i * ld + i];
      if (is_zero(u)) u = s_one<T>();
      T x = sdiv(add(acc0, acc1), u);
      bad |= !is_finite(x);
      W[i * ld + j] = x;
    }
    if (bad) st->bad = 1;
  }
}

// U~^-1 e_k (one warp): back substitution with the row sums spread over the lanes.
template <typename T>
__device__ void lu_upper_solve_unit(const T* A, int ld, int n, int k, T* out) {
  const int lane = threadIdx.x & 31;
  for (int i = n - 1; i >= 0; --i) {
    T acc = s_zero<T>();
    for (int c = i + 1 + lane; c < n; c += 32) acc = fma_(A[i * ld + c], out[c], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      T o = shfl_idx(acc, (lane ^ off));
      acc = add(acc, o);
    }
    if (lane == 0) {
      T u = A[i * ld + i];
      if (is_zero(u)) u = s_one<T>();
      T rhs = (i == k) ? s_one<T>() : s_zero<T>();
      out[i] = sdiv(sub(rhs, acc), u);
    }
    __syncwarp();
  }
}

template <typename T>
__device__ __forceinline__ T coef_of(const Job<T>& J, int64_t b) {
  return J.coef ? J.coef[b] : s_one<T>();
}

template <typename T>
__device__ __forceinline__ T maybe_conj(const Job<T>& J, T v) {
  return J.conj_out ? conj_(v) : v;
}

// Dynamic shared memory carve-up of one block.
template <typename T>
struct SmemLayout {
  static __host__ __device__ size_t scalars_bytes(int n) {
    // ipiv / perm (2n ints), two n-vectors of T, the FacState, padding
    return 2 * (size_t)n * sizeof(int) + 2 * (size_t)n * sizeof(T) + sizeof(FacState<T>) + 64;
  }
  static __host__ __device__ size_t bytes(int n, int ld, int nbuf, bool in_smem) {
    size_t s = scalars_bytes(n);
    if (in_smem) s += (size_t)nbuf * n * ld * sizeof(T);
    return (s + 15) & ~(size_t)15;
  }
};

// Gradient epilogue after the factorisation (A: packed LU in LAPACK order, ipiv the
// interchanges): X = U~^-1 L^-1 into W, then
//   slogdet: G = coef * A^-T (zero for singular / non-finite members),
//   det:     G = coef * adj(A)^T (det * A^-T, or the Woodbury rank-1 form for one or two
//            exact zero pivots, _diff.py:205-246),
// and the forward's (sign, logabs, value).
template <typename T>
__device__ void lu_gradient_epilogue(const Job<T>& J, int64_t b, T* A, T* W, int ld, int n, const int* ipiv,
                                     int* sigma, T* vec0, T* vec1, FacState<T>* st) {
  typedef typename Sc<T>::R R;
    // ---- gradient: X = U~^-1 L^-1, then A^-T[i][j] = X[j][sigma(i)]
    if (threadIdx.x == 0) {
      for (int j = 0; j < n; ++j) sigma[j] = j;
      for (int j = n - 1; j >= 0; --j) {
        int p = ipiv[j];
        if (p != j) {
          int t = sigma[j];
          sigma[j] = sigma[p];
          sigma[p] = t;
        }
      }
    }
    const bool det_sing = (J.mode == MODE_VALUE_GRAD) && st->nzero > 0 && st->nzero < 3;
    if (det_sing) {
      // Woodbury branch (_diff.py:222-246): u1 = U~^-1 e_k1 (vec0), c = (U~^-1 e_k2)[k1]
      const int warp = threadIdx.x >> 5;
      if (warp == 0) lu_upper_solve_unit(A, ld, n, st->k1, vec0);
      if (warp == 1 || (nthr() == 32)) {
        if (nthr() == 32) __syncwarp();
        lu_upper_solve_unit(A, ld, n, st->k2, vec1);
      }
    }
    lu_inverse_cols(A, W, ld, n, st);
    __syncthreads();
    const T cf = coef_of(J, b);
    T scale_all;
    bool zero_all = false;
    const FacState<T> s = *st;
    if (J.mode == MODE_SLOG_GRAD) {
      zero_all = s.nzero > 0 || s.bad;
      scale_all = cf;
    } else {
      zero_all = s.bad && s.nzero == 0;
      if (s.nzero == 0) {
        // det from the very pivots of this LU (_diff.py:184-202)
        T det = scale(s.sign, rexp(s.logabs));
        scale_all = mul(cf, det);
      } else {
        scale_all = cf;
      }
    }
    T* G = J.g + b * (int64_t)n * n;
    const int nn = n * n;
    if (J.mode == MODE_VALUE_GRAD && s.nzero > 0) {
      // G[i][j] = s * X[k2][sigma(i)] * u1[j]; s = sgn(P) d_K (m >= 2 ? c : 1), 0 for m >= 3
      T sK = s_zero<T>();
      if (s.nzero < 3) {
        // d_K: the product of the nonzero pivots, phase times exp(sum log|d|) -- the
        // factorisation's own logabs without the -inf terms
        T ph = s_one<T>();
        KSum<R> lsum;
        lsum.init();
        for (int k = 0; k < n; ++k) {
          T d = A[k * ld + k];
          if (!is_zero(d)) {
            ph = mul(ph, unit(d));
            lsum.add(rlog(mag(d)));
          }
        }
        T dK = scale(ph, rexp(lsum.value()));
        if (s.parity) dK = neg(dK);
        T c = (s.nzero >= 2) ? vec1[s.k1] : s_one<T>();
        sK = mul(dK, c);
      }
      const T f = mul(cf, sK);
      for (int idx = threadIdx.x; idx < nn; idx += nthr()) {
        int i = idx / n, j = idx - i * n;
        T v = mul(f, mul(W[s.k2 * ld + sigma[i]], vec0[j]));
        G[idx] = maybe_conj(J, v);
      }
    } else {
      for (int idx = threadIdx.x; idx < nn; idx += nthr()) {
        int i = idx / n, j = idx - i * n;
        T v = zero_all ? s_zero<T>() : mul(scale_all, W[j * ld + sigma[i]]);
        G[idx] = maybe_conj(J, v);
      }
    }
    if (threadIdx.x == 0) {
      J.sign[b] = s.sign;
      J.logabs[b] = s.logabs;
      if (J.value) J.value[b] = scale(s.sign, rexp(s.logabs));
    }
    __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(256) lu_fused_kernel(Job<T> J) {
  typedef typename Sc<T>::R R;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int n = J.n, ld = J.ld;
  const int nbuf = J.mode == MODE_FWD ? 1 : 2;
  T* bufs = J.in_smem ? reinterpret_cast<T*>(smem_raw) : J.ws + (int64_t)blockIdx.x * nbuf * n * ld;
  unsigned char* tail = smem_raw + (J.in_smem ? (size_t)nbuf * n * ld * sizeof(T) : 0);
  T* vec0 = reinterpret_cast<T*>(tail);
  T* vec1 = vec0 + n;
  FacState<T>* st = reinterpret_cast<FacState<T>*>(vec1 + n);
  int* ipiv = reinterpret_cast<int*>(st + 1);
  int* sigma = ipiv + n;
  T* A = bufs;
  T* W = bufs + (size_t)n * ld;

  for (int64_t b = blockIdx.x; b < J.B; b += gridDim.x) {
    load_matrix(J, b, A, ld, false);
    __syncthreads();
    lu_factor(A, ld, n, ipiv, st);
    if (J.mode == MODE_FWD) {
      if (threadIdx.x == 0) {
        J.sign[b] = st->sign;
        J.logabs[b] = st->logabs;
        if (J.value) J.value[b] = scale(st->sign, rexp(st->logabs));
      }
      __syncthreads();
      continue;
    }
    lu_gradient_epilogue(J, b, A, W, ld, n, ipiv, sigma, vec0, vec1, st);
  }
}

}  // namespace fx
