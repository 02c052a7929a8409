// Batched Parlett-Reid skew tridiagonalisation: slogpf / pf forward and their
// gradients, one thread block per matrix, on chip.
//
// Reference behaviour (ChenAo-Phys/fermix):
//   forward  : src/fermix/_fallback.py:266-300 (the pair step: pivot = first-occurrence
//              argmax |S[r, c]| over r > c, swap into c+1, d = S[c, c+1],
//              tau = -S[:, c] / d, w = S[:, c+1], S += tau w^T - w tau^T on the trailing
//              rows / columns), blocked as in src/fermix/_pf.py:516-570 (a panel of
//              FX_NB / 2 pair steps with corrected columns, then one rank-FX_NB update of
//              the lower triangle mirrored into the upper one, _pf.py:352-358)
//   gradient : src/fermix/_pfinv.py:1-36 and _fallback.py:101-263: with L~ the factor
//              (column a_K not scaled by 1 / d_K), Y = L~^-1, R = Y^T D~^-1 Y, w = R e_aK,
//              v = Y^T e_aK: S^-1 = -[R + c (w v^T - v w^T)] and
//              pf(S) S^-1 = -D_K [d_K R + (1 - d_K)(w v^T - v w^T)]; a second exact zero
//              pivot is lifted to +-1 and the two evaluations averaged (_fallback.py:142-154).
//
// Design (B200): the matrix lives in shared memory (or a global workspace slot), with
// physical symmetric row / column interchanges so that the factor ends up in position
// order. The L factor is stored in place: column 2s holds w_s, column 2s + 1 holds tau_s
// (rows > 2s + 1), exactly the columns the pair step consumed.
#pragma once
#include "fused_lu.cuh"

namespace fx {

template <typename T>
struct PfState {
  T sign;
  typename Sc<T>::R logabs;
  int parity;
  int nzero;
  int K;     // pivot of smallest modulus (first occurrence)
  int s2;    // a second exact zero pivot (first one other than K), -1 if none
  int bad;
};

// Lower-triangle trailing update of rows / columns [r0, n) by the np pair steps of the
// block at k0; each entry: acc += tau_t[i] w_t[j]; acc -= w_t[i] tau_t[j] (t ascending),
// stored at (i, j) and negated at (j, i).
template <typename T, int MI, int MJ>
__device__ void pf_trailing(T* A, int ld, int r0, int n, int k0, int np) {
  const int m = n - r0;
  if (m <= 1) return;
  const int TC = 16;
  const int TR = nthr() / TC;
  const int ti = threadIdx.x / TC, tj = threadIdx.x % TC;
  for (int bi = 0; bi < m; bi += TR * MI) {
    for (int bj = 0; bj <= bi + TR * MI - 1 && bj < m; bj += TC * MJ) {
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
      for (int i = 0; i < MI; ++i)
#pragma unroll
        for (int j = 0; j < MJ; ++j) any |= (rv[i] && cv[j] && rr[i] > cc[j]);
      if (!any) continue;
      T acc[MI][MJ];
#pragma unroll
      for (int i = 0; i < MI; ++i)
#pragma unroll
        for (int j = 0; j < MJ; ++j)
          acc[i][j] = (rv[i] && cv[j] && rr[i] > cc[j]) ? A[rr[i] * ld + cc[j]] : s_zero<T>();
      for (int t = 0; t < np; ++t) {
        const int cw = k0 + 2 * t, ct = cw + 1;
        T wi[MI], ti_[MI], wj[MJ], tj_[MJ];
#pragma unroll
        for (int i = 0; i < MI; ++i) {
          wi[i] = rv[i] ? A[rr[i] * ld + cw] : s_zero<T>();
          ti_[i] = rv[i] ? A[rr[i] * ld + ct] : s_zero<T>();
        }
#pragma unroll
        for (int j = 0; j < MJ; ++j) {
          wj[j] = cv[j] ? A[cc[j] * ld + cw] : s_zero<T>();
          tj_[j] = cv[j] ? A[cc[j] * ld + ct] : s_zero<T>();
        }
#pragma unroll
        for (int i = 0; i < MI; ++i)
#pragma unroll
          for (int j = 0; j < MJ; ++j) {
            acc[i][j] = fma_(ti_[i], wj[j], acc[i][j]);
            acc[i][j] = fms(acc[i][j], wi[i], tj_[j]);
          }
      }
#pragma unroll
      for (int i = 0; i < MI; ++i)
#pragma unroll
        for (int j = 0; j < MJ; ++j)
          if (rv[i] && cv[j] && rr[i] > cc[j]) {
            A[rr[i] * ld + cc[j]] = acc[i][j];
            A[cc[j] * ld + rr[i]] = neg(acc[i][j]);
          }
    }
  }
}

// Blocked Parlett-Reid of the skew n x n matrix in A (n even), in place. perm[f] = the
// original index at final position f; dvec[s] = the pivot of pair s.
template <typename T>
__device__ void pf_factor(T* A, int ld, int n, int* perm, T* dvec, T* cvec, PfState<T>* st) {
  typedef typename Sc<T>::R R;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < n; i += nthr()) perm[i] = i;
  __syncthreads();
  T sgn = s_one<T>();
  KSum<R> ls;
  ls.init();
  int par = 0, nzero = 0;
  for (int k0 = 0; k0 < n; k0 += FX_NB) {
    const int np = min(FX_NB, n - k0) / 2;
    if (warp == 0) {
      for (int s = 0; s < np; ++s) {
        const int c = k0 + 2 * s;
        // corrected column c on rows > c
        R best = R(-1);
        int bi = 0x7fffffff;
        for (int r = c + 1 + lane; r < n; r += 32) {
          T v = A[r * ld + c];
          for (int t = 0; t < s; ++t) {
            const int cw = k0 + 2 * t, ct = cw + 1;
            v = fma_(A[r * ld + ct], A[c * ld + cw], v);
            v = fms(v, A[r * ld + cw], A[c * ld + ct]);
          }
          cvec[r] = v;
          R a = abs1(v);
          if (a > best) {
            best = a;
            bi = r;
          }
        }
        warp_argmax(best, bi);
        const int p = (bi == 0x7fffffff) ? c + 1 : bi;
        __syncwarp();
        if (p != c + 1) {
          const int q = c + 1;
          for (int x = lane; x < n; x += 32) swap_(A[q * ld + x], A[p * ld + x]);
          __syncwarp();
          for (int x = lane; x < n; x += 32) swap_(A[x * ld + q], A[x * ld + p]);
          if (lane == 0) {
            swap_(cvec[q], cvec[p]);
            int t = perm[q];
            perm[q] = perm[p];
            perm[p] = t;
          }
        }
        __syncwarp();
        const T d = neg(cvec[c + 1]);
        const T inv = recip(d);
        // corrected column c+1 on rows > c+1 -> w; tau = -col_c / d; store L in place
        for (int r = c + 2 + lane; r < n; r += 32) {
          T v = A[r * ld + c + 1];
          for (int t = 0; t < s; ++t) {
            const int cw = k0 + 2 * t, ct = cw + 1;
            v = fma_(A[r * ld + ct], A[(c + 1) * ld + cw], v);
            v = fms(v, A[r * ld + cw], A[(c + 1) * ld + ct]);
          }
          A[r * ld + c] = v;                              // w
          A[r * ld + c + 1] = neg(mul(cvec[r], inv));     // tau
        }
        if (lane == 0) {
          dvec[c / 2] = d;
          par ^= (p != c + 1);
          sgn = mul(sgn, unit(d));
          ls.add(rlog(mag(d)));
          nzero += is_zero(d);
        }
        __syncwarp();
      }
    }
    __syncthreads();
    pf_trailing<T, TileShape<T>::MI, TileShape<T>::MJ>(A, ld, k0 + 2 * np, n, k0, np);
    __syncthreads();
  }
  if (tid == 0) {
    if (par) sgn = neg(sgn);
    if (nzero) sgn = s_zero<T>();
    if constexpr (Sc<T>::cx) {
      R m = rhypot(sgn.re, sgn.im);
      if (m != R(0)) sgn = {rdiv(sgn.re, m), rdiv(sgn.im, m)};
    }
    st->sign = sgn;
    st->logabs = nzero ? -INFINITY : ls.value();
    st->parity = par;
    st->nzero = nzero;
    // K = argmin |d| (first occurrence, _fallback.py:101-108); s2 = first zero != K
    const int h = n / 2;
    int K = 0;
    R bm = R(INFINITY);
    for (int s = 0; s < h; ++s) {
      R a = mag(dvec[s]);
      if (a < bm) {
        bm = a;
        K = s;
      }
    }
    int s2 = -1;
    for (int s = 0; s < h; ++s)
      if (s != K && is_zero(dvec[s])) {
        s2 = s;
        break;
      }
    st->K = K;
    st->s2 = s2;
    st->bad = 0;
  }
  __syncthreads();
}

// One evaluation of the inverse / adjugate formula for the pivots dd (dvec with an
// optional lifted entry `lift_s` set to `lift_v`). A holds the factor (consumed: R is
// written over it), W receives Y. Writes out[i][j] = f * PT[pos[i]][pos[j]] (accumulate
// adds to the existing output).
template <typename T>
__device__ void pf_evaluate(T* A, T* W, int ld, int n, const T* dvec, int lift_s, T lift_v, const int* perm,
                            int* pos, T* dinv, PfState<T>* st, bool adjugate, T f, bool accumulate, bool conj_out,
                            T* out, T* coefs) {
  typedef typename Sc<T>::R R;
  const int h = n / 2;
  const int K = st->K;
  for (int s = threadIdx.x; s < h; s += nthr()) {
    T d = (s == lift_s) ? lift_v : dvec[s];
    T dt = (s == K || is_zero(d)) ? s_one<T>() : d;
    dinv[s] = sdiv(s_one<T>(), dt);
  }
  for (int i = threadIdx.x; i < n; i += nthr()) pos[perm[i]] = i;
  __syncthreads();
  // Y = L~^-1, one column per thread (L~[i][2s] = w_s[i] / d~_s, L~[i][2s+1] = tau_s[i])
  for (int j = threadIdx.x; j < n; j += nthr()) {
    for (int i = 0; i < j; ++i) W[i * ld + j] = s_zero<T>();
    W[j * ld + j] = s_one<T>();
    for (int i = j + 1; i < n; ++i) {
      T acc = s_zero<T>();
      for (int k = j; k < i; ++k) {
        T l;
        if ((k & 1) == 0) {
          if (i == k + 1) continue;
          l = mul(A[i * ld + k], dinv[k >> 1]);
        } else {
          l = A[i * ld + k];
        }
        acc = fma_(l, W[k * ld + j], acc);
      }
      W[i * ld + j] = neg(acc);
    }
  }
  __syncthreads();
  // R = Y^T D~^-1 Y (skew): R[i][j] = sum_s dinv_s (Y[2s][i] Y[2s+1][j] - Y[2s+1][i] Y[2s][j])
  {
    const int TC = 16, MI = TileShape<T>::MI, MJ = TileShape<T>::MJ;
    const int TR = nthr() / TC;
    const int ti = threadIdx.x / TC, tj = threadIdx.x % TC;
    bool bad = false;
    for (int bi = 0; bi < n; bi += TR * MI) {
      for (int bj = 0; bj < n && bj <= bi + TR * MI - 1; bj += TC * MJ) {
        int rr[MI], cc[MJ];
#pragma unroll
        for (int i = 0; i < MI; ++i) rr[i] = bi + ti + TR * i;
#pragma unroll
        for (int j = 0; j < MJ; ++j) cc[j] = bj + tj + TC * j;
        T acc[MI][MJ];
#pragma unroll
        for (int i = 0; i < MI; ++i)
#pragma unroll
          for (int j = 0; j < MJ; ++j) acc[i][j] = s_zero<T>();
        const int s0 = bi >= 1 ? (bi - 1) / 2 : 0;
        for (int s = s0; s < h; ++s) {
          const int ka = 2 * s, kb = ka + 1;
          const T di = dinv[s];
          T ya[MI], yb[MI], za[MJ], zb[MJ];
#pragma unroll
          for (int i = 0; i < MI; ++i) {
            ya[i] = rr[i] < n ? W[ka * ld + rr[i]] : s_zero<T>();
            yb[i] = rr[i] < n ? W[kb * ld + rr[i]] : s_zero<T>();
          }
#pragma unroll
          for (int j = 0; j < MJ; ++j) {
            za[j] = cc[j] < n ? mul(W[kb * ld + cc[j]], di) : s_zero<T>();
            zb[j] = cc[j] < n ? mul(W[ka * ld + cc[j]], di) : s_zero<T>();
          }
#pragma unroll
          for (int i = 0; i < MI; ++i)
#pragma unroll
            for (int j = 0; j < MJ; ++j) {
              acc[i][j] = fma_(ya[i], za[j], acc[i][j]);
              acc[i][j] = fms(acc[i][j], yb[i], zb[j]);
            }
        }
#pragma unroll
        for (int i = 0; i < MI; ++i)
#pragma unroll
          for (int j = 0; j < MJ; ++j) {
            if (rr[i] < n && cc[j] < n && rr[i] > cc[j]) {
              bad |= !is_finite(acc[i][j]);
              A[rr[i] * ld + cc[j]] = acc[i][j];
              A[cc[j] * ld + rr[i]] = neg(acc[i][j]);
            }
          }
      }
    }
    for (int i = threadIdx.x; i < n; i += nthr()) A[i * ld + i] = s_zero<T>();
    if (bad) st->bad = 1;
  }
  __syncthreads();
  // coefficients (a1, a2) of _fallback._pf_adj_coeffs, and w = R e_aK, v = Y^T e_aK
  if (threadIdx.x == 0) {
    T dK = (K == lift_s) ? lift_v : dvec[K];
    if (adjugate) {
      T ph = s_one<T>();
      KSum<R> lsum;
      lsum.init();
      for (int s = 0; s < h; ++s) {
        if (s == K) continue;
        T d = (s == lift_s) ? lift_v : dvec[s];
        ph = mul(ph, unit(d));
        if (!is_zero(d)) lsum.add(rlog(mag(d)));
      }
      T D = scale(ph, rexp(lsum.value()));
      if (st->parity) D = neg(D);
      coefs[0] = mul(D, dK);
      coefs[1] = mul(D, sub(s_one<T>(), dK));
    } else {
      coefs[0] = s_one<T>();
      coefs[1] = is_zero(dK) ? s_zero<T>() : sdiv(sub(s_one<T>(), dK), dK);
    }
  }
  __syncthreads();
  const T a1 = coefs[0], a2 = coefs[1];
  const int aK = 2 * K;
  const int nn = n * n;
  for (int idx = threadIdx.x; idx < nn; idx += nthr()) {
    const int i = idx / n, j = idx - i * n;
    const int fi = pos[i], fj = pos[j];
    const T r = A[fi * ld + fj];
    const T wi = A[fi * ld + aK], wj = A[fj * ld + aK];
    const T vi = W[aK * ld + fi], vj = W[aK * ld + fj];
    // -(a1 R + a2 (w v^T - v w^T)) with products kept unfused so the result is exactly skew
    const T rk = sub(mul(wi, vj), mul(vi, wj));
    T v = neg(add(mul(a1, r), mul(a2, rk)));
    v = mul(f, v);
    if (conj_out) v = conj_(v);
    if (accumulate) v = add(out[idx], v);
    out[idx] = v;
  }
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(256) pf_fused_kernel(Job<T> J) {
  typedef typename Sc<T>::R R;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int n = J.n, ld = J.ld;
  const int nbuf = J.mode == MODE_FWD ? 1 : 2;
  T* bufs = J.in_smem ? reinterpret_cast<T*>(smem_raw) : J.ws + (int64_t)blockIdx.x * nbuf * n * ld;
  unsigned char* tail = smem_raw + (J.in_smem ? (size_t)nbuf * n * ld * sizeof(T) : 0);
  T* dvec = reinterpret_cast<T*>(tail);  // n/2 pivots, then n/2 inverse pivots
  T* dinv = dvec + n / 2;
  T* cvec = dvec + n;                    // n scratch entries (+ 2 coefficients at the end)
  PfState<T>* st = reinterpret_cast<PfState<T>*>(cvec + n);
  int* perm = reinterpret_cast<int*>(st + 1);
  int* pos = perm + n;
  T* A = bufs;
  T* W = bufs + (size_t)n * ld;

  for (int64_t b = blockIdx.x; b < J.B; b += gridDim.x) {
    load_matrix(J, b, A, ld, J.skew != 0);
    __syncthreads();
    pf_factor(A, ld, n, perm, dvec, cvec, st);
    if (threadIdx.x == 0) {
      J.sign[b] = st->sign;
      J.logabs[b] = st->logabs;
      if (J.value) J.value[b] = scale(st->sign, rexp(st->logabs));
    }
    if (J.mode == MODE_FWD) {
      __syncthreads();
      continue;
    }
    const bool adjugate = J.mode == MODE_VALUE_GRAD;
    T* G = J.g + b * (int64_t)n * n;
    // gradient of sum(logabs) = -S^-1 / 2 (slogpf), of pf = -pf S^-1 / 2
    const T f = scale(coef_of(J, b), R(-0.5));
    // cvec doubles as the two-entry coefficient scratch once the factorisation is done
    T* coefs = cvec;
    const int s2 = st->s2;
    if (!adjugate || s2 < 0) {
      pf_evaluate(A, W, ld, n, dvec, -1, s_zero<T>(), perm, pos, dinv, st, adjugate, f, false, J.conj_out != 0, G,
                  coefs);
      if (!adjugate) {
        const PfState<T> s = *st;
        const bool zero_all = is_zero(dvec[s.K]) || s.bad;
        if (zero_all) {
          const int nn = n * n;
          for (int idx = threadIdx.x; idx < nn; idx += nthr()) G[idx] = s_zero<T>();
        }
      }
    } else {
      // second exact zero pivot: mean of the evaluations with it lifted to +1 and -1
      const T half_f = scale(f, R(0.5));
      pf_evaluate(A, W, ld, n, dvec, s2, s_one<T>(), perm, pos, dinv, st, true, half_f, false, J.conj_out != 0, G,
                  coefs);
      load_matrix(J, b, A, ld, J.skew != 0);
      __syncthreads();
      pf_factor(A, ld, n, perm, dvec, cvec, st);
      pf_evaluate(A, W, ld, n, dvec, s2, neg(s_one<T>()), perm, pos, dinv, st, true, half_f, true,
                  J.conj_out != 0, G, coefs);
    }
    __syncthreads();
  }
}

}  // namespace fx
