// k-index Pfaffian moves (no reference counterpart; the multi-electron move of a Pfaffian
// wavefunction, on the gradient the Pfaffian path exports -- _pf_parts,
// src/fermix/_pfinv.py:196-269). G = S^-T / 2 per matrix; the move replaces rows idx[r] of
// the skew S by rows[r] and columns idx[r] by -rows[r], applied in order r = 0 .. k - 1 (on the
// idx x idx block the later row wins; rows[r][idx[r]] is ignored), i.e. k one-index moves.
//
// With G_t the gradient after t one-index moves, u_t the new row (its idx_t entry zero),
// g_t = row idx_t of G_t, rho_t = 2 g_t . u_t and y_t = e_idx_t - 2 G_t u_t:
//   pf(S') / pf(S) = prod_t rho_t,   G' = G + sum_t (y_t g_t^T - g_t y_t^T) / rho_t.
// Every G_t u_s and every row of G_t follow from V = G U^T and the rows idx of G by the
// earlier rank-2 corrections, so the move is three passes:
//   pfk_v_kernel:    V[t][j] = G_j . u_t (one read of G; one warp per row, k dot products)
//   pfk_prep_kernel: per matrix (one block), t = 0 .. k - 1: g_t, y_t and the dot products
//                    g_t . u_s, y_t . u_s (s >= t) they feed, O(n k^2); the ratio and the
//                    per-matrix action
//   pfk_rows_kernel: G_j += sum_t (y_t[j] g_t - g_t[j] y_t) / rho_t (one read and one write
//                    of G; one warp per row)
// so G crosses HBM three times (3 n^2 s bytes), against 2 n^2 s for the one-index move whose
// ratio needs only one row.
#pragma once
#include "update.cuh"

namespace fx {

template <typename T>
struct PfkArgs {
  T* g;                         // (B, n, n) G = S^-T / 2, updated in place by pfk_rows_kernel
  const T* u;                   // (B, k, n) the new rows of S
  const int* idx;               // (B, k) the moved indices (distinct)
  const unsigned char* accept;  // (B,) or null = all
  T* sign;                      // (B,) sign of pf(S') / pf(S)
  typename Sc<T>::R* logabs;    // (B,) log |pf(S') / pf(S)|
  T* v;                         // (B, k, n) workspace: G u_t
  T* gv;                        // (B, k, n) workspace: g_t
  T* yv;                        // (B, k, n) workspace: y_t
  T* rinv;                      // (B, k) workspace: 1 / rho_t
  int* act;                     // (B,) workspace: UPD_KEEP / UPD_APPLY / UPD_ZERO
  int64_t B;
  int n, k;
};

constexpr int kPfkPrepThreads = 128;

// V[t][j] = G_j . u_t, u_t with entry idx_t left out; KM (a power of two >= k) bounds the
// unrolled coefficient loops
template <typename T, int KM>
__global__ void __launch_bounds__(kUpdRowThreads, 2) pfk_v_kernel(PfkArgs<T> A) {
  const int lane = threadIdx.x & 31;
  const int n = A.n, k = A.k;
  const int64_t nw = (int64_t)gridDim.x * (kUpdRowThreads / 32);
  for (int64_t w = (int64_t)blockIdx.x * (kUpdRowThreads / 32) + (threadIdx.x >> 5); w < A.B * n; w += nw) {
    const int64_t b = w / n;
    const int j = (int)(w % n);
    const T* gj = A.g + (b * n + j) * (int64_t)n;
    const T* ub = A.u + b * (int64_t)k * n;
    const int* ib = A.idx + b * k;
    int id[KM];
#pragma unroll
    for (int t = 0; t < KM; ++t) id[t] = t < k ? ib[t] : -1;
    T acc[KM];
#pragma unroll
    for (int t = 0; t < KM; ++t) acc[t] = s_zero<T>();
#pragma unroll 1
    for (int c = lane; c < n; c += 32) {
      const T gv = gj[c];
#pragma unroll
      for (int t = 0; t < KM; ++t)
        if (t < k && c != id[t]) acc[t] = fma_(gv, ub[(int64_t)t * n + c], acc[t]);
    }
    const T s = warp_reduce_scatter<T, KM>(acc, lane);
    if (lane < k) A.v[(b * k + lane) * (int64_t)n + j] = s;
  }
}

template <typename T>
struct PfkSmem {
  T dg[kUpdMaxK][kUpdMaxK];  // dg[q][s] = g_q . u_s
  T dy[kUpdMaxK][kUpdMaxK];  // dy[q][s] = y_q . u_s
  T red[kPfkPrepThreads / 32][2 * kUpdMaxK];
  T ri[kUpdMaxK];            // 1 / rho_q
  T gi[kUpdMaxK][kUpdMaxK];  // gi[q][t] = g_q[idx_t]
  T yi[kUpdMaxK][kUpdMaxK];  // yi[q][t] = y_q[idx_t]
  int id[kUpdMaxK];
  int bad, zero;
};

// One block per matrix: the recurrence over t, the ratio and the action.
template <typename T>
__global__ void __launch_bounds__(kPfkPrepThreads) pfk_prep_kernel(PfkArgs<T> A) {
  using R = typename Sc<T>::R;
  __shared__ PfkSmem<T> S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NW = kPfkPrepThreads / 32;
  const int n = A.n, k = A.k;
  for (int64_t b = blockIdx.x; b < A.B; b += gridDim.x) {
    if (tid == 0) {
      S.bad = 0;
      S.zero = 0;
    }
    __syncthreads();
    if (tid < k) {
      const int i = A.idx[b * k + tid];
      S.id[tid] = i;
      if (i < 0 || i >= n) atomicOr(&S.bad, 1);
    }
    __syncthreads();
    const bool bad = S.bad != 0;
    const T* Gb = A.g + b * (int64_t)n * n;
    const T* ub = A.u + b * (int64_t)k * n;
    const T* vb = A.v + b * (int64_t)k * n;
    T* gvb = A.gv + b * (int64_t)k * n;
    T* yvb = A.yv + b * (int64_t)k * n;
    T sgn = s_one<T>();
    KSum<R> ls;
    ls.init();
    for (int t = 0; t < k && !bad; ++t) {
      const int i = S.id[t];
      const bool z = S.zero != 0;
      // g_t, y_t elementwise, with the partial dot products against u_s, s >= t
      T pg[kUpdMaxK], py[kUpdMaxK];
#pragma unroll
      for (int s = 0; s < kUpdMaxK; ++s) pg[s] = py[s] = s_zero<T>();
      for (int c = tid; c < n; c += kPfkPrepThreads) {
        T gval = Gb[(int64_t)i * n + c], w = vb[(int64_t)t * n + c];
        for (int q = 0; q < t && !z; ++q) {
          const T gq = gvb[(int64_t)q * n + c], yq = yvb[(int64_t)q * n + c];
          gval = add(gval, mul(S.ri[q], sub(mul(S.yi[q][t], gq), mul(S.gi[q][t], yq))));
          w = add(w, mul(S.ri[q], sub(mul(yq, S.dg[q][t]), mul(gq, S.dy[q][t]))));
        }
        T y = neg(add(w, w));
        if (c == i) y = add(y, s_one<T>());
        gvb[(int64_t)t * n + c] = gval;
        yvb[(int64_t)t * n + c] = y;
#pragma unroll
        for (int s = 0; s < kUpdMaxK; ++s)
          if (s >= t && s < k && c != S.id[s]) {
            const T us = ub[(int64_t)s * n + c];
            pg[s] = fma_(gval, us, pg[s]);
            py[s] = fma_(y, us, py[s]);
          }
      }
      // block sums of pg[s], py[s]
#pragma unroll
      for (int s = 0; s < kUpdMaxK; ++s) {
        if (s >= t && s < k) {
          const T a = warp_sum_t<T>(pg[s]), c2 = warp_sum_t<T>(py[s]);
          if (lane == 0) {
            S.red[warp][s] = a;
            S.red[warp][kUpdMaxK + s] = c2;
          }
        }
      }
      __syncthreads();  // also: g_t, y_t of this step visible to the block
      if (tid < k && tid >= t) {
        T a = s_zero<T>(), c2 = s_zero<T>();
#pragma unroll
        for (int w2 = 0; w2 < NW; ++w2) {
          a = add(a, S.red[w2][tid]);
          c2 = add(c2, S.red[w2][kUpdMaxK + tid]);
        }
        S.dg[t][tid] = a;
        S.dy[t][tid] = c2;
      }
      if (tid >= 32 && tid < 32 + k) {  // the moved entries of g_t, y_t for the later steps
        const int s = tid - 32;
        S.gi[t][s] = gvb[(int64_t)t * n + S.id[s]];
        S.yi[t][s] = yvb[(int64_t)t * n + S.id[s]];
      }
      __syncthreads();
      if (tid == 0) {
        const T rho = add(S.dg[t][t], S.dg[t][t]);
        if (is_zero(rho)) {
          S.zero = 1;
          S.ri[t] = s_zero<T>();
        } else {
          S.ri[t] = recip(rho);
        }
      }
      __syncthreads();
      if (!z) {
        const T rho = add(S.dg[t][t], S.dg[t][t]);
        sgn = mul(sgn, unit(rho));
        ls.add(rlog(mag(rho)));
      }
    }
    if (tid == 0) {
      const bool acc = A.accept == nullptr || A.accept[b] != 0;
      const bool zero = S.zero != 0;
      if (bad) {
        A.sign[b] = upd_nan<T>();
        A.logabs[b] = R(NAN);
      } else {
        A.sign[b] = zero ? s_zero<T>() : sgn;
        A.logabs[b] = zero ? -R(INFINITY) : ls.value();
      }
      if (A.act) A.act[b] = (bad || !acc) ? UPD_KEEP : (zero ? UPD_ZERO : UPD_APPLY);
    }
    if (A.rinv && tid < k) A.rinv[b * k + tid] = S.ri[tid];
    __syncthreads();
  }
}

// G_j += sum_t (y_t[j] g_t - g_t[j] y_t) / rho_t; one warp per row; KM as pfk_v_kernel
template <typename T, int KM>
__global__ void __launch_bounds__(kUpdRowThreads, 2) pfk_rows_kernel(PfkArgs<T> A) {
  const int lane = threadIdx.x & 31;
  const int n = A.n, k = A.k;
  const int64_t nw = (int64_t)gridDim.x * (kUpdRowThreads / 32);
  for (int64_t w = (int64_t)blockIdx.x * (kUpdRowThreads / 32) + (threadIdx.x >> 5); w < A.B * n; w += nw) {
    const int64_t b = w / n;
    const int j = (int)(w % n);
    const int act = A.act[b];
    if (act == UPD_KEEP) continue;
    T* gj = A.g + (b * n + j) * (int64_t)n;
    if (act == UPD_ZERO) {
      for (int c = lane; c < n; c += 32) gj[c] = s_zero<T>();
      continue;
    }
    const T* gvb = A.gv + b * (int64_t)k * n;
    const T* yvb = A.yv + b * (int64_t)k * n;
    T ca[KM], cb[KM];
#pragma unroll
    for (int t = 0; t < KM; ++t) {
      ca[t] = cb[t] = s_zero<T>();
      if (t < k) {
        const T ri = A.rinv[b * k + t];
        ca[t] = mul(yvb[(int64_t)t * n + j], ri);
        cb[t] = mul(gvb[(int64_t)t * n + j], ri);
      }
    }
#pragma unroll 1
    for (int c = lane; c < n; c += 32) {
      T x = gj[c];
#pragma unroll
      for (int t = 0; t < KM; ++t)
        if (t < k) x = fma_(ca[t], gvb[(int64_t)t * n + c], fms(x, cb[t], yvb[(int64_t)t * n + c]));
      gj[c] = x;
    }
  }
}

}  // namespace fx
