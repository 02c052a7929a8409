// Register-panel variants of the fused kernels for n <= 256 (RS = ceil(n / 32) rows per
// lane): the panel of each block is factored by one warp with its rows held in
// registers and virtual pivoting (rows never move during the panel); the panel's
// interchanges are then applied to the whole matrix at once, so everything after the
// panel works on a position-ordered matrix with contiguous tiles.
//
// Parlett-Reid (pf2_*): the factor is stored in place -- column 2s holds w_s, column
// 2s + 1 holds tau_s (the columns the pair step consumed) -- and the gradient runs in
// the same buffer: L~ is scaled in place, Y = L~^-1 overwrites it (blocked triangular
// inverse, right to left), R = Y^T D~^-1 Y goes to the free upper triangle, and the
// output gathers the permuted adjugate / inverse. One n x n buffer serves forward and
// backward, so three 128 x 128 float blocks fit on one SM.
//
// Arithmetic is the same as fused_pf.cuh / fused_lu.cuh (same update chains, same
// pivoting rule up to tie-breaking), see those files for the reference citations.
#pragma once
#include "fused_pf.cuh"

namespace fx {

template <typename T, int RS>
__device__ __forceinline__ T pick_slot(const T (&v)[RS], int slot) {
  T r = v[0];
#pragma unroll
  for (int i = 1; i < RS; ++i)
    if (slot == i) r = v[i];
  return r;
}

// First unassigned row of the warp (fallback pivot when no candidate compares, e.g. NaN).
template <int RS>
__device__ __forceinline__ int first_unassigned(uint32_t unas, int lane) {
  unsigned cand = 0xffffffffu;
#pragma unroll
  for (int i = RS - 1; i >= 0; --i)
    if ((unas >> i) & 1u) cand = (unsigned)(lane + 32 * i);
  return (int)__reduce_min_sync(0xffffffffu, cand);
}


// (sign, logabs, nzero) of prod_k d_k (k < cnt, d_k = piv(k)), reduced by warp 0 in a
// fixed order (lanes stride the pivots, then a butterfly), so every kernel that calls it
// on the same pivots returns the same bits. Real signs are products of +-1 (exact).
template <typename T, typename F>
__device__ void warp_sign_log(int cnt, F piv, int parity, PfState<T>* out_pf, FacState<T>* out_lu) {
  typedef typename Sc<T>::R R;
  const int lane = threadIdx.x & 31;
  if ((threadIdx.x >> 5) != 0) return;
  T sg = s_one<T>();
  KSum<R> ls;
  ls.init();
  int nz = 0;
  for (int k = lane; k < cnt; k += 32) {
    const T d = piv(k);
    sg = mul(sg, unit(d));
    ls.add(rlog(mag(d)));
    nz += is_zero(d);
  }
  R lsum = ls.value();
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const T o = shfl_idx(sg, lane ^ off);
    sg = mul(sg, o);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
    nz += __shfl_xor_sync(0xffffffffu, nz, off);
  }
  if (lane == 0) {
    if (parity) sg = neg(sg);
    if (nz) sg = s_zero<T>();
    if constexpr (Sc<T>::cx) {
      R m = rhypot(sg.re, sg.im);
      if (m != R(0)) sg = {rdiv(sg.re, m), rdiv(sg.im, m)};
    }
    const R la = nz ? R(-INFINITY) : lsum;
    if (out_pf) {
      out_pf->sign = sg;
      out_pf->logabs = la;
      out_pf->nzero = nz;
    }
    if (out_lu) {
      out_lu->sign = sg;
      out_lu->logabs = la;
      out_lu->nzero = nz;
    }
  }
}

// ------------------------------------------------------------------ Parlett-Reid
template <typename T, int RS>
struct PfNP {
  // pairs per panel: keep the panel's tau / w registers at <= 64 32-bit words per lane
  static constexpr int words = sizeof(T) / 4;
  static constexpr int v = 64 / (RS * 2 * words);
  static constexpr int NP = v >= 8 ? 8 : (v >= 4 ? 4 : (v >= 2 ? 2 : 1));
};

// Blocked Parlett-Reid in place, position-ordered on return: M[i][2s] = w_s[i],
// M[i][2s+1] = tau_s[i] (i > 2s + 1), M[2s+1][2s] = 0; dvec[s] = d_s; perm[f] = the
// input index at position f. at / pof / ipiv are n-int scratch arrays.
template <typename T, int RS, int NP>
__device__ void pf2_factor(T* M, int ld, int n, int* perm, int* at, int* pof, int* ipiv, T* dvec, PfState<T>* st) {
  typedef typename Sc<T>::R R;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < n; i += nthr()) perm[i] = i;
  int par = 0;
  __syncthreads();
  FX_TIC(tp0);
  for (int k0 = 0; k0 < n; k0 += 2 * NP) {
    const int np = min(NP, (n - k0) / 2);
    if (warp == 0) {
      for (int x = k0 + lane; x < n; x += 32) {
        at[x] = x;
        pof[x] = x;
      }
      __syncwarp();
      T tw[RS][2 * NP];
      uint32_t unas = 0;
#pragma unroll
      for (int i = 0; i < RS; ++i) {
        const int r = lane + 32 * i;
        if (r >= k0 && r < n) unas |= 1u << i;
#pragma unroll
        for (int t = 0; t < 2 * NP; ++t) tw[i][t] = s_zero<T>();
      }
      int ap[NP], pp[NP];
#pragma unroll
      for (int s = 0; s < NP; ++s) {
        ap[s] = 0;
        pp[s] = 0;
      }
#pragma unroll
      for (int s = 0; s < NP; ++s) {
        if (s < np) {
          const int c = k0 + 2 * s;
          const int a = at[c];
          if ((a & 31) == lane) unas &= ~(1u << (a >> 5));
          T wa[NP], ta[NP];
#pragma unroll
          for (int t = 0; t < NP; ++t)
            if (t < s) {
              wa[t] = M[a * ld + ap[t]];
              ta[t] = M[a * ld + pp[t]];
            }
          T colA[RS];
          R best = R(-1);
          int bi = 0x7fffffff;
#pragma unroll
          for (int i = 0; i < RS; ++i) {
            const int r = lane + 32 * i;
            T v = (r < n) ? M[r * ld + a] : s_zero<T>();
#pragma unroll
            for (int t = 0; t < NP; ++t)
              if (t < s) {
                v = fma_(tw[i][2 * t + 1], wa[t], v);
                v = fms(v, tw[i][2 * t], ta[t]);
              }
            colA[i] = v;
            if ((unas >> i) & 1u) {
              const R m = abs1(v);
              if (m > best) {
                best = m;
                bi = r;
              }
            }
          }
          warp_argmax(best, bi);
          const int p = (bi == 0x7fffffff) ? first_unassigned<RS>(unas, lane) : bi;
          const T d = neg(shfl_idx(pick_slot<T, RS>(colA, p >> 5), p & 31));
          const T inv = recip(d);
          if ((p & 31) == lane) unas &= ~(1u << (p >> 5));
          T wp[NP], tp[NP];
#pragma unroll
          for (int t = 0; t < NP; ++t)
            if (t < s) {
              wp[t] = M[p * ld + ap[t]];
              tp[t] = M[p * ld + pp[t]];
            }
#pragma unroll
          for (int i = 0; i < RS; ++i) {
            const int r = lane + 32 * i;
            T v = (r < n) ? M[r * ld + p] : s_zero<T>();
#pragma unroll
            for (int t = 0; t < NP; ++t)
              if (t < s) {
                v = fma_(tw[i][2 * t + 1], wp[t], v);
                v = fms(v, tw[i][2 * t], tp[t]);
              }
            const bool u = (unas >> i) & 1u;
            const T w = u ? v : s_zero<T>();
            const T tau = u ? neg(mul(colA[i], inv)) : s_zero<T>();
            tw[i][2 * s] = w;
            tw[i][2 * s + 1] = tau;
            if (u) {
              M[r * ld + a] = w;
              M[r * ld + p] = tau;
            }
          }
          if ((p & 31) == lane) M[p * ld + a] = s_zero<T>();
          ap[s] = a;
          pp[s] = p;
          if (lane == 0) {
            const int q = pof[p];
            ipiv[c + 1] = q;
            dvec[c >> 1] = d;
            if (q != c + 1) {
              const int x = at[c + 1];
              at[c + 1] = p;
              at[q] = x;
              pof[p] = c + 1;
              pof[x] = q;
              const int t = perm[c + 1];
              perm[c + 1] = perm[q];
              perm[q] = t;
              par ^= 1;
            }
          }
          __syncwarp();
        }
      }
    }
    __syncthreads();
    FX_TOC(tp0, 0);
    // the panel's interchanges, rows (all columns) then columns (rows >= k0)
    for (int x = tid; x < n; x += nthr()) {
      for (int s = 0; s < np; ++s) {
        const int c1 = k0 + 2 * s + 1, q = ipiv[c1];
        if (q != c1) swap_(M[c1 * ld + x], M[q * ld + x]);
      }
    }
    __syncthreads();
    for (int y = k0 + tid; y < n; y += nthr()) {
      for (int s = 0; s < np; ++s) {
        const int c1 = k0 + 2 * s + 1, q = ipiv[c1];
        if (q != c1) swap_(M[y * ld + c1], M[y * ld + q]);
      }
    }
    __syncthreads();
    FX_TOC(tp0, 1);
    pf_trailing<T, TileShape<T>::MI, TileShape<T>::MJ>(M, ld, k0 + 2 * np, n, k0, np);
    __syncthreads();
    FX_TOC(tp0, 2);
  }
  warp_sign_log<T>(n / 2, [&](int k) { return dvec[k]; }, par, st, (FacState<T>*)nullptr);
  __syncwarp();
  if (tid == 0) {
    st->parity = par;
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

// In-place unit-lower-triangular inverse of the position-ordered n x n matrix (lower
// part, diagonal implicit 1): blocks of 16 columns from right to left; for block J the
// diagonal block is inverted first, then B <- -Y_trail B Y_JJ with C = Y_trail B staged
// transposed in the (free) upper part of the block's rows.
template <typename T>
__device__ void tri_inv_unit_lower_inplace(T* M, int ld, int n) {
  const int tid = threadIdx.x;
  const int nbk = (n + 15) / 16;
  for (int J = nbk - 1; J >= 0; --J) {
    const int j0 = 16 * J, bs = min(16, n - j0), j1 = j0 + bs;
    // diagonal block: warp 0, one lane per column q (all reads before any write)
    if (tid < 32) {
      const int q = tid;
      T y[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) y[i] = s_zero<T>();
      if (q < bs) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (i > q && i < bs) {
            T acc = M[(j0 + i) * ld + j0 + q];  // m = q (y[q] = 1)
#pragma unroll
            for (int m = 0; m < 16; ++m)
              if (m > q && m < i) acc = fma_(M[(j0 + i) * ld + j0 + m], y[m], acc);
            y[i] = neg(acc);
          }
        }
      }
      __syncwarp();
      if (q < bs) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i > q && i < bs) M[(j0 + i) * ld + j0 + q] = y[i];
      }
    }
    __syncthreads();
    if (j1 < n) {
      const int rows = n - j1;
      // C[i][q] = B[i][q] + sum_{m=j1}^{i-1} Y[i][m] B[m][q]  ->  M[j0+q][i]
      for (int it = tid; it < rows * bs; it += nthr()) {
        const int i = j1 + it / bs, q = it - (it / bs) * bs;
        T acc0 = M[i * ld + j0 + q], acc1 = s_zero<T>();
        int m = j1;
        for (; m + 1 < i; m += 2) {
          acc0 = fma_(M[i * ld + m], M[m * ld + j0 + q], acc0);
          acc1 = fma_(M[i * ld + m + 1], M[(m + 1) * ld + j0 + q], acc1);
        }
        if (m < i) acc0 = fma_(M[i * ld + m], M[m * ld + j0 + q], acc0);
        M[(j0 + q) * ld + i] = add(acc0, acc1);
      }
      __syncthreads();
      // B[i][q] = -sum_{q' >= q} C[i][q'] Y_JJ[q'][q]
      for (int it = tid; it < rows * bs; it += nthr()) {
        const int i = j1 + it / bs, q = it - (it / bs) * bs;
        T acc = M[(j0 + q) * ld + i];
        for (int q2 = q + 1; q2 < bs; ++q2) acc = fma_(M[(j0 + q2) * ld + i], M[(j0 + q2) * ld + j0 + q], acc);
        M[i * ld + j0 + q] = neg(acc);
      }
      __syncthreads();
    }
  }
}

// One evaluation of the inverse / adjugate formula on the position-ordered factor in M
// (consumed). dvec, perm from pf2_factor; pos = n-int scratch. Writes
// out[r][q] = f * PT[pos[r]][pos[q]] (accumulating into out when requested).
template <typename T>
__device__ void pf2_evaluate(T* M, int ld, int n, const T* dvec, int lift_s, T lift_v, const int* perm, int* pos,
                             T* dinv, T* wv, PfState<T>* st, bool adjugate, T f, bool accumulate, bool conj_out,
                             T* out, T* coefs) {
  typedef typename Sc<T>::R R;
  const int h = n / 2;
  const int K = st->K;
  for (int s = threadIdx.x; s < h; s += nthr()) {
    const T d = (s == lift_s) ? lift_v : dvec[s];
    const T dt = (s == K || is_zero(d)) ? s_one<T>() : d;
    dinv[s] = sdiv(s_one<T>(), dt);
  }
  for (int i = threadIdx.x; i < n; i += nthr()) pos[perm[i]] = i;
  __syncthreads();
  FX_TIC(te0);
  // L~: column 2s (w_s) scaled by 1 / d~_s
  for (int idx = threadIdx.x; idx < h * n; idx += nthr()) {
    const int s = idx / n, i = idx - s * n;
    if (i > 2 * s + 1) M[i * ld + 2 * s] = mul(M[i * ld + 2 * s], dinv[s]);
  }
  __syncthreads();
  FX_TOC(te0, 3);
  tri_inv_unit_lower_inplace(M, ld, n);
  FX_TOC(te0, 4);
  // R = Y^T D~^-1 Y, lower triangle R[i][j] (i > j) stored at M[j][i]
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
          // Y[k][x] = M[k][x] (k > x), 1 (k == x), 0 (k < x)
#pragma unroll
          for (int i = 0; i < MI; ++i) {
            const int x = rr[i];
            ya[i] = (x < n && ka > x) ? M[ka * ld + x] : (ka == x ? s_one<T>() : s_zero<T>());
            yb[i] = (x < n && kb > x) ? M[kb * ld + x] : (kb == x ? s_one<T>() : s_zero<T>());
          }
#pragma unroll
          for (int j = 0; j < MJ; ++j) {
            const int x = cc[j];
            const T y1 = (x < n && kb > x) ? M[kb * ld + x] : (kb == x ? s_one<T>() : s_zero<T>());
            const T y0 = (x < n && ka > x) ? M[ka * ld + x] : (ka == x ? s_one<T>() : s_zero<T>());
            za[j] = mul(y1, di);
            zb[j] = mul(y0, di);
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
          for (int j = 0; j < MJ; ++j)
            if (rr[i] < n && cc[j] < n && rr[i] > cc[j]) {
              bad |= !is_finite(acc[i][j]);
              M[cc[j] * ld + rr[i]] = acc[i][j];
            }
      }
    }
    if (bad) st->bad = 1;
  }
  __syncthreads();
  FX_TOC(te0, 5);
  const int aK = 2 * K;
  // w[i] = R[i][aK], v[i] = Y[aK][i] (position order)
  T* wvec = wv;
  T* vvec = wv + n;
  for (int i = threadIdx.x; i < n; i += nthr()) {
    wvec[i] = i > aK ? M[aK * ld + i] : (i < aK ? neg(M[i * ld + aK]) : s_zero<T>());
    vvec[i] = i < aK ? M[aK * ld + i] : (i == aK ? s_one<T>() : s_zero<T>());
  }
  if (threadIdx.x == 0) {
    const T dK = (K == lift_s) ? lift_v : dvec[K];
    if (adjugate) {
      T ph = s_one<T>();
      KSum<R> lsum;
      lsum.init();
      for (int s = 0; s < h; ++s) {
        if (s == K) continue;
        const T d = (s == lift_s) ? lift_v : dvec[s];
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
  const int nn = n * n;
  for (int idx = threadIdx.x; idx < nn; idx += nthr()) {
    const int r = idx / n, q = idx - r * n;
    const int fi = pos[r], fj = pos[q];
    const T rv = fi > fj ? M[fj * ld + fi] : (fi < fj ? neg(M[fi * ld + fj]) : s_zero<T>());
    const T rk = sub(mul(wvec[fi], vvec[fj]), mul(vvec[fi], wvec[fj]));
    T v = neg(add(mul(a1, rv), mul(a2, rk)));
    v = mul(f, v);
    if (conj_out) v = conj_(v);
    if (accumulate) v = add(out[idx], v);
    out[idx] = v;
  }
  __syncthreads();
  FX_TOC(te0, 6);
}

template <typename T>
struct Small {
  // n-int arrays: perm, at, pof, ipiv/pos; T arrays: dvec (n/2), dinv (n/2), wv (2n), coefs (2)
  static __host__ __device__ size_t scalars_bytes(int n) {
    return 4 * (size_t)n * sizeof(int) + (3 * (size_t)n + 4) * sizeof(T) + sizeof(FacState<T>) + 64;
  }
  static __host__ __device__ size_t bytes(int n, int ld, bool in_smem) {
    size_t s = scalars_bytes(n);
    if (in_smem) s += (size_t)n * ld * sizeof(T);
    return (s + 15) & ~(size_t)15;
  }
};

template <typename T, int RS>
__global__ void __launch_bounds__(256) pf_small_kernel(Job<T> J) {
  typedef typename Sc<T>::R R;
  constexpr int NP = PfNP<T, RS>::NP;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int n = J.n, ld = J.ld;
  T* M = J.in_smem ? reinterpret_cast<T*>(smem_raw) : J.ws + (int64_t)blockIdx.x * n * ld;
  unsigned char* tail = smem_raw + (J.in_smem ? (size_t)n * ld * sizeof(T) : 0);
  T* dvec = reinterpret_cast<T*>(tail);  // n/2
  T* dinv = dvec + n / 2;                // n/2
  T* wv = dinv + n / 2 + (n & 1);        // 2n
  T* coefs = wv + 2 * n;                 // 4
  PfState<T>* st = reinterpret_cast<PfState<T>*>(coefs + 4);
  int* perm = reinterpret_cast<int*>(st + 1);
  int* at = perm + n;
  int* pof = at + n;
  int* ipiv = pof + n;
  int* pos = at;  // at / pof are free after the factorisation

  for (int64_t b = blockIdx.x; b < J.B; b += gridDim.x) {
    load_matrix(J, b, M, ld, J.skew != 0);
    __syncthreads();
    pf2_factor<T, RS, NP>(M, ld, n, perm, at, pof, ipiv, dvec, st);
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
    const T f = scale(coef_of(J, b), R(-0.5));
    const int s2 = st->s2;
    if (!adjugate || s2 < 0) {
      pf2_evaluate(M, ld, n, dvec, -1, s_zero<T>(), perm, pos, dinv, wv, st, adjugate, f, false, J.conj_out != 0, G,
                   coefs);
      if (!adjugate) {
        const bool zero_all = is_zero(dvec[st->K]) || st->bad;
        if (zero_all) {
          const int nn = n * n;
          for (int idx = threadIdx.x; idx < nn; idx += nthr()) G[idx] = s_zero<T>();
        }
      }
    } else {
      const T half_f = scale(f, R(0.5));
      pf2_evaluate(M, ld, n, dvec, s2, s_one<T>(), perm, pos, dinv, wv, st, true, half_f, false, J.conj_out != 0, G,
                   coefs);
      load_matrix(J, b, M, ld, J.skew != 0);
      __syncthreads();
      pf2_factor<T, RS, NP>(M, ld, n, perm, at, pof, ipiv, dvec, st);
      pf2_evaluate(M, ld, n, dvec, s2, neg(s_one<T>()), perm, pos, dinv, wv, st, true, half_f, true,
                   J.conj_out != 0, G, coefs);
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ LU
template <typename T, int RS>
struct LuNB {
  static constexpr int words = sizeof(T) / 4;
  static constexpr int v = 64 / (RS * words);
  static constexpr int NB = v >= 16 ? 16 : (v >= 8 ? 8 : (v >= 4 ? 4 : 2));
};

// Blocked LU in place with the register panel; on return M is the packed LU in LAPACK
// order (P A = L U) and ipiv[j] the row interchanged with j at step j.
template <typename T, int RS, int NB>
__device__ void lu2_factor(T* M, int ld, int n, int* ipiv, int* at, int* pof, FacState<T>* st) {
  typedef typename Sc<T>::R R;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int par = 0, k1z = -1, k2z = -1;
  for (int k0 = 0; k0 < n; k0 += NB) {
    const int kb = min(NB, n - k0);
    if (warp == 0) {
      for (int x = k0 + lane; x < n; x += 32) {
        at[x] = x;
        pof[x] = x;
      }
      T P[RS][NB];
      uint32_t unas = 0;
#pragma unroll
      for (int i = 0; i < RS; ++i) {
        const int r = lane + 32 * i;
        const bool live = r >= k0 && r < n;
        if (live) unas |= 1u << i;
#pragma unroll
        for (int jj = 0; jj < NB; ++jj) P[i][jj] = (live && jj < kb) ? M[r * ld + k0 + jj] : s_zero<T>();
      }
      __syncwarp();
#pragma unroll
      for (int jj = 0; jj < NB; ++jj) {
        if (jj < kb) {
          const int j = k0 + jj;
          R best = R(-1);
          int bi = 0x7fffffff;
#pragma unroll
          for (int i = 0; i < RS; ++i)
            if ((unas >> i) & 1u) {
              const R m = abs1(P[i][jj]);
              if (m > best) {
                best = m;
                bi = lane + 32 * i;
              }
            }
          warp_argmax(best, bi);
          const int p = (bi == 0x7fffffff) ? first_unassigned<RS>(unas, lane) : bi;
          const int ps = p >> 5, pl = p & 31;
          T prow[NB];
#pragma unroll
          for (int j2 = 0; j2 < NB; ++j2) {
            if (j2 >= jj) {
              T v = P[0][j2];
#pragma unroll
              for (int i = 1; i < RS; ++i)
                if (ps == i) v = P[i][j2];
              prow[j2] = shfl_idx(v, pl);
            }
          }
          const T piv = prow[jj];
          if (pl == lane) unas &= ~(1u << ps);
          const bool z = is_zero(piv);
#pragma unroll
          for (int i = 0; i < RS; ++i) {
            if ((unas >> i) & 1u) {
              const T l = z ? s_zero<T>() : sdiv(P[i][jj], piv);
              P[i][jj] = l;
#pragma unroll
              for (int j2 = 0; j2 < NB; ++j2)
                if (j2 > jj) P[i][j2] = fms(P[i][j2], l, prow[j2]);
            }
          }
          if (lane == 0) {
            const int q = pof[p];
            ipiv[j] = q;
            if (q != j) {
              const int x = at[j];
              at[j] = p;
              at[q] = x;
              pof[p] = j;
              pof[x] = q;
              par ^= 1;
            }
            if (z) {
              if (k1z < 0) k1z = j;
              k2z = j;
            }
          }
          __syncwarp();
        }
      }
      // the panel goes back in its final row order (pof: panel-start row -> position),
      // so the interchange pass below leaves the panel columns alone
#pragma unroll
      for (int i = 0; i < RS; ++i) {
        const int r = lane + 32 * i;
        if (r >= k0 && r < n) {
          const int dst = pof[r];
#pragma unroll
          for (int jj = 0; jj < NB; ++jj)
            if (jj < kb) M[dst * ld + k0 + jj] = P[i][jj];
        }
      }
    }
    __syncthreads();
    // interchanges on the columns outside the panel, then U_k = L_kk^-1 A[k rows, trailing cols]
    for (int c = tid; c < n; c += nthr()) {
      if (c >= k0 && c < k0 + kb) continue;
      for (int jj = 0; jj < kb; ++jj) {
        const int j = k0 + jj, q = ipiv[j];
        if (q != j) swap_(M[j * ld + c], M[q * ld + c]);
      }
      if (c >= k0 + kb) {
        for (int t = 1; t < kb; ++t) {
          T acc = M[(k0 + t) * ld + c];
          for (int s = 0; s < t; ++s) acc = fms(acc, M[(k0 + t) * ld + k0 + s], M[(k0 + s) * ld + c]);
          M[(k0 + t) * ld + c] = acc;
        }
      }
    }
    __syncthreads();
    lu_trailing<T, TileShape<T>::MI, TileShape<T>::MJ>(M, ld, k0 + kb, n, k0, kb);
    __syncthreads();
  }
  // the pivots are U's diagonal
  warp_sign_log<T>(n, [&](int k) { return M[k * ld + k]; }, par, (PfState<T>*)nullptr, st);
  __syncwarp();
  if (tid == 0) {
    st->parity = par;
    st->k1 = k1z;
    st->k2 = k2z;
    st->bad = 0;
  }
  __syncthreads();
}

template <typename T>
struct LuSmall {
  // T arrays vec0, vec1 (n each); n-int arrays ipiv, sigma, at, pof
  static __host__ __device__ size_t scalars_bytes(int n) {
    return 4 * (size_t)n * sizeof(int) + 2 * (size_t)n * sizeof(T) + sizeof(FacState<T>) + 64;
  }
  static __host__ __device__ size_t bytes(int n, int ld, int nbuf, bool in_smem) {
    size_t s = scalars_bytes(n);
    if (in_smem) s += (size_t)nbuf * n * ld * sizeof(T);
    return (s + 15) & ~(size_t)15;
  }
};

template <typename T, int RS>
__global__ void __launch_bounds__(256) lu_small_kernel(Job<T> J) {
  typedef typename Sc<T>::R R;
  constexpr int NB = LuNB<T, RS>::NB;
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
  int* at = sigma + n;
  int* pof = at + n;
  T* A = bufs;
  T* W = bufs + (size_t)n * ld;

  for (int64_t b = blockIdx.x; b < J.B; b += gridDim.x) {
    load_matrix(J, b, A, ld, false);
    __syncthreads();
    lu2_factor<T, RS, NB>(A, ld, n, ipiv, at, pof, st);
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
