// Rank-k row replacement of determinants from the exported inverse (no reference
// counterpart: the single- and multi-electron move of a QMC caller, built on the inverse
// the gradient path exports -- _lu_parts, src/fermix/_inverse.py:502-531 -- and on the
// reference's sign / logabs conventions for the ratio, src/fermix/_lu.py:614-621).
//
// State: G = A^-T, the slogdet gradient (fermix_slogdet_grad with coef = 1). A move
// replaces rows idx[0 .. k) of A by the rows of U (k x n). With E = columns idx of I:
//   R = U A^-1 E,  R[r][s] = U_r . G_{idx_s}           det(A') / det(A) = det(R)
//   V = U A^-1,    V[r][j] = U_r . G_j
//   G' = A'^-T = G - (V^T - E) H,  H = R^-T G[idx, :]   (Woodbury)
// so row j of G' is G_j - sum_r (V[r][j] - [j == idx_r]) H_r.
//
// upd_prep1_kernel (k = 1): one warp per matrix: R = U . G_idx, the ratio, H = G_idx / R.
// upd_prep_kernel (k > 1): one 128-thread block per matrix. R by k^2 dot products (fixed-order lane
//   partials and an xor tree, four per warp at a time), then one warp runs Gauss-Jordan with
//   partial pivoting on [R | I] (k <= 16, first-occurrence argmax of abs1 as the reference's
//   LU; lane j holds column j), giving the ratio's (sign, logabs) and R^-1; then H into the
//   workspace, and the matrix's row-kernel action.
// upd_rows_vec_kernel: rows of up to 4 KB whose bytes are a multiple of 16 (16-byte aligned
//   arrays): one warp holds RW rows of one matrix in registers as 16-byte pieces (lane l owns
//   pieces l, l + 32, ...), forms their k dot products V[.][j] from the same registers, updates
//   them and stores them. Each G element is read once and written once; U and H, shared by
//   the matrix's rows, stay L1 / L2 resident. HBM-bound at n^2 (read) + n^2 (write) elements.
// upd_rows_kernel: any other shape: one warp per row, scalar column loop, the row read twice
//   (the second read hits L1 / L2).
#pragma once
#include "scalar.cuh"
#include "umma.cuh"

namespace fx {

constexpr int kUpdMaxK = 16;  // largest rank of one move
constexpr int kUpdPrepThreads = 128;
constexpr int kUpdRowThreads = 256;

enum : int { UPD_KEEP = 0, UPD_APPLY = 1, UPD_ZERO = 2 };

template <typename T>
struct UpdArgs {
  T* g;                         // (B, n, n) G = A^-T; updated in place by the rows kernel
  const T* u;                   // (B, k, n) replacement rows
  const int* idx;               // (B, k) replaced row indices
  const unsigned char* accept;  // (B,) apply the move where nonzero; null = every matrix
  T* sign;                      // (B,) sign of det(A') / det(A) (input dtype)
  typename Sc<T>::R* logabs;    // (B,) log |det(A') / det(A)|
  T* h;                         // (B, k, n) workspace: H = R^-T G[idx, :]; null = ratio only
  int* act;                     // (B,) workspace: UPD_KEEP / UPD_APPLY / UPD_ZERO
  int64_t B;
  int n, k;
};

// 16 bytes of consecutive elements: the unit of the vector row kernel
template <typename T>
struct alignas(16) UpdPiece {
  T v[16 / sizeof(T)];
};

template <typename T>
__device__ __forceinline__ void upd_swap(T& a, T& b) {
  const T t = a;
  a = b;
  b = t;
}

// NaN of the field (both parts for complex)
template <typename T>
__device__ __forceinline__ T upd_nan() {
  using R = typename Sc<T>::R;
  T v = s_zero<T>();
  if constexpr (Sc<T>::cx) {
    v.re = R(NAN);
    v.im = R(NAN);
  } else {
    v = R(NAN);
  }
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_sum_t(T v);
template <>
__device__ __forceinline__ float warp_sum_t<float>(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <>
__device__ __forceinline__ double warp_sum_t<double>(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <>
__device__ __forceinline__ c64_t warp_sum_t<c64_t>(c64_t v) {
  return {warp_sum_t<float>(v.re), warp_sum_t<float>(v.im)};
}
template <>
__device__ __forceinline__ c128_t warp_sum_t<c128_t>(c128_t v) {
  return {warp_sum_t<double>(v.re), warp_sum_t<double>(v.im)};
}

template <typename T>
__device__ __forceinline__ T upd_shfl_xor(T v, int m) {
  if constexpr (Sc<T>::cx) {
    v.re = __shfl_xor_sync(0xffffffffu, v.re, m);
    v.im = __shfl_xor_sync(0xffffffffu, v.im, m);
    return v;
  } else {
    return __shfl_xor_sync(0xffffffffu, v, m);
  }
}

// Warp sums of KM per-lane partials (KM a power of two <= 16) at once: halving exchanges
// over lane bits KM/2 .. 1 (the lane with the bit set keeps the upper half), then plain xor
// sums over the remaining bits. Returns, in every lane, the full sum of index lane % KM;
// (KM - 1) + (5 - log2 KM) shuffles instead of 5 KM. a is clobbered.
template <typename T, int KM>
__device__ __forceinline__ T warp_reduce_scatter(T (&a)[KM], int lane) {
#pragma unroll
  for (int half = KM / 2; half >= 1; half >>= 1) {
    const bool up = (lane & half) != 0;
#pragma unroll
    for (int t = 0; t < half; ++t) {
      const T send = up ? a[t] : a[t + half];
      const T keep = up ? a[t + half] : a[t];
      a[t] = add(keep, upd_shfl_xor<T>(send, half));
    }
  }
  T v = a[0];
#pragma unroll
  for (int o = KM; o < 32; o <<= 1) v = add(v, upd_shfl_xor<T>(v, o));
  return v;
}

// x . y over n entries: lane partials in column order, then the xor tree (every lane
// returns the same bits).
template <typename T>
__device__ __forceinline__ T warp_dot(const T* __restrict__ x, const T* __restrict__ y, int n, int lane) {
  T acc = s_zero<T>();
  for (int c = lane; c < n; c += 32) acc = fma_(x[c], y[c], acc);
  return warp_sum_t<T>(acc);
}

template <typename T>
struct UpdSmem {
  T r[kUpdMaxK][kUpdMaxK + 1];   // R
  T ri[kUpdMaxK][kUpdMaxK + 1];  // R^-1
  int id[kUpdMaxK];
  int bad, sing;
};

// k = 1: one warp per matrix. R = U . G_idx (the lane-partial / xor-tree dot), the ratio's
// (sign, logabs) = (unit(R), log|R|), and H = R^-1 G_idx.
template <typename T>
__global__ void __launch_bounds__(kUpdRowThreads) upd_prep1_kernel(UpdArgs<T> A) {
  using R = typename Sc<T>::R;
  const int lane = threadIdx.x & 31;
  const int n = A.n;
  const int64_t wstride = (int64_t)gridDim.x * (kUpdRowThreads / 32);
  for (int64_t b = (int64_t)blockIdx.x * (kUpdRowThreads / 32) + (threadIdx.x >> 5); b < A.B; b += wstride) {
    const int i = A.idx[b];
    const bool bad = i < 0 || i >= n;
    const T* Gi = A.g + (b * n + (bad ? 0 : i)) * (int64_t)n;
    T d = s_zero<T>();
    if (!bad) d = warp_dot(A.u + b * (int64_t)n, Gi, n, lane);
    const bool sing = !bad && is_zero(d);
    const bool acc = A.accept == nullptr || A.accept[b] != 0;
    if (lane == 0) {
      A.sign[b] = bad ? upd_nan<T>() : (sing ? s_zero<T>() : unit(d));
      A.logabs[b] = bad ? R(NAN) : (sing ? -R(INFINITY) : rlog(mag(d)));
      if (A.h) A.act[b] = (!acc || bad) ? UPD_KEEP : (sing ? UPD_ZERO : UPD_APPLY);
    }
    if (A.h && acc && !bad && !sing) {
      const T ri = recip(d);
      T* H = A.h + b * (int64_t)n;
      for (int c = lane; c < n; c += 32) H[c] = mul(ri, Gi[c]);
    }
  }
}

// a[i] with i only known at run time, over a register array indexed by constants
template <typename T>
__device__ __forceinline__ T upd_pick(const T (&a)[kUpdMaxK], int i) {
  T v = a[0];
#pragma unroll
  for (int q = 1; q < kUpdMaxK; ++q)
    if (q == i) v = a[q];
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kUpdPrepThreads) upd_prep_kernel(UpdArgs<T> A) {
  using R = typename Sc<T>::R;
  __shared__ UpdSmem<T> S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = A.n, k = A.k, kk = A.k * A.k;
  for (int64_t b = blockIdx.x; b < A.B; b += gridDim.x) {
    const T* G = A.g + b * (int64_t)n * n;
    const T* U = A.u + b * (int64_t)k * n;
    if (tid == 0) S.bad = 0;
    __syncthreads();
    if (tid < k) {
      const int v = A.idx[b * k + tid];
      S.id[tid] = v;
      if (v < 0 || v >= n) S.bad = 1;
    }
    __syncthreads();
    const bool bad = S.bad != 0;
    if (!bad) {
      // R[r][s] = U_r . G_{idx_s}: four dot products per warp at a time (lane partials in
      // column order, then the xor tree)
      for (int p0 = warp * 4; p0 < kk; p0 += kUpdPrepThreads / 32 * 4) {
        T acc[4];
        const T* ur[4];
        const T* gr[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int p = p0 + q < kk ? p0 + q : 0;
          const int r = p / k, sc = p - r * k;
          ur[q] = U + (int64_t)r * n;
          gr[q] = G + (int64_t)S.id[sc] * n;
          acc[q] = s_zero<T>();
        }
        for (int c = lane; c < n; c += 32)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[q] = fma_(ur[q][c], gr[q][c], acc[q]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const T v = warp_sum_t<T>(acc[q]);
          const int p = p0 + q;
          if (lane == 0 && p < kk) S.r[p / k][p - (p / k) * k] = v;
        }
      }
    }
    __syncthreads();
    if (warp == 0) {
      // Gauss-Jordan with partial pivoting on [R | I], lane j holding column j: pivot = the
      // first largest abs1 of column c in rows c .. k - 1 (lane c's registers); rows below c
      // get the LU update a_i -= (a_ic / d) a_c, so the pivots, sign and logabs are those of
      // the LU of R; the rows above get the same update, leaving [D | D R^-1] (row-permuted).
      // sign = prod unit(pivot) * (-1)^swaps, logabs = sum log|pivot| in column order.
      T a[kUpdMaxK], dd[kUpdMaxK];
#pragma unroll
      for (int i = 0; i < kUpdMaxK; ++i) {
        T v = s_zero<T>();
        if (!bad && i < k) {
          if (lane < k) v = S.r[i][lane];
          else if (lane - k == i) v = s_one<T>();
        }
        a[i] = v;
        dd[i] = s_one<T>();
      }
      T sg = s_one<T>();
      KSum<R> ls;
      ls.init();
      int sing = 0;
#pragma unroll
      for (int c = 0; c < kUpdMaxK; ++c) {
        if (bad || c >= k) continue;
        int p = c;
        if (lane == c) {
          R best = abs1(a[c]);
#pragma unroll
          for (int i = c + 1; i < kUpdMaxK; ++i) {
            if (i < k) {
              const R m = abs1(a[i]);
              if (m > best) {
                best = m;
                p = i;
              }
            }
          }
        }
        p = __shfl_sync(0xffffffffu, p, c);
        if (p != c) {
          const T t = upd_pick(a, p);
#pragma unroll
          for (int i = c + 1; i < kUpdMaxK; ++i)
            if (i == p) a[i] = a[c];
          a[c] = t;
          sg = neg(sg);
        }
        const T d = shfl_idx<T>(a[c], c);
        dd[c] = d;
        if (is_zero(d)) {
          sing = 1;
          continue;
        }
        sg = mul(sg, unit(d));
        ls.add(rlog(mag(d)));
        const T dinv = recip(d);
#pragma unroll
        for (int i = 0; i < kUpdMaxK; ++i) {
          if (i != c && i < k) {
            const T l = shfl_idx<T>(mul(a[i], dinv), c);  // lane c holds a_ic
            a[i] = fms(a[i], l, a[c]);
          }
        }
      }
      R la = ls.value();
      if (bad) {
        sg = upd_nan<T>();
        la = R(NAN);
      } else if (sing) {
        sg = s_zero<T>();
        la = -R(INFINITY);
      }
      const bool acc = A.accept == nullptr || A.accept[b] != 0;
      if (lane == 0) {
        A.sign[b] = sg;
        A.logabs[b] = la;
        S.sing = sing;
        if (A.h) A.act[b] = (!acc || bad) ? UPD_KEEP : (sing ? UPD_ZERO : UPD_APPLY);
      }
      if (A.h && acc && !bad && !sing && lane >= k && lane < 2 * k) {
#pragma unroll
        for (int i = 0; i < kUpdMaxK; ++i)
          if (i < k) S.ri[i][lane - k] = mul(a[i], recip(dd[i]));  // row i of R^-1 = row i / d_i
      }
    }
    __syncthreads();
    if (A.h && !bad && !S.sing && (A.accept == nullptr || A.accept[b] != 0)) {
      // H[r][c] = sum_s R^-1[s][r] G[idx_s][c], coalesced over c
      T* H = A.h + b * (int64_t)k * n;
      for (int c = tid; c < n; c += kUpdPrepThreads) {
        T gs[kUpdMaxK];
#pragma unroll
        for (int s2 = 0; s2 < kUpdMaxK; ++s2)
          if (s2 < k) gs[s2] = G[(int64_t)S.id[s2] * n + c];
        for (int r = 0; r < k; ++r) {
          T acc = s_zero<T>();
#pragma unroll
          for (int s2 = 0; s2 < kUpdMaxK; ++s2)
            if (s2 < k) acc = fma_(S.ri[s2][r], gs[s2], acc);
          H[(int64_t)r * n + c] = acc;
        }
      }
    }
    __syncthreads();
  }
}

template <typename T>
__global__ void __launch_bounds__(kUpdRowThreads) upd_rows_kernel(UpdArgs<T> A) {
  const int lane = threadIdx.x & 31;
  const int n = A.n, k = A.k;
  const int64_t rows = A.B * (int64_t)n;
  const int64_t wstride = (int64_t)gridDim.x * (kUpdRowThreads / 32);
  for (int64_t q = (int64_t)blockIdx.x * (kUpdRowThreads / 32) + (threadIdx.x >> 5); q < rows; q += wstride) {
    const int64_t b = q / n;
    const int j = (int)(q - b * n);
    const int act = A.act[b];
    if (act == UPD_KEEP) continue;
    T* Gj = A.g + q * n;
    if (act == UPD_ZERO) {
      for (int c = lane; c < n; c += 32) Gj[c] = s_zero<T>();
      continue;
    }
    const T* U = A.u + b * (int64_t)k * n;
    const T* H = A.h + b * (int64_t)k * n;
    const int* id = A.idx + b * k;
    T cf[kUpdMaxK];
#pragma unroll
    for (int r = 0; r < kUpdMaxK; ++r) {
      cf[r] = s_zero<T>();
      if (r < k) {
        T v = warp_dot(U + (int64_t)r * n, Gj, n, lane);
        if (__ldg(id + r) == j) v = sub(v, s_one<T>());
        cf[r] = v;
      }
    }
    for (int c = lane; c < n; c += 32) {
      T x = Gj[c];
#pragma unroll
      for (int r = 0; r < kUpdMaxK; ++r)
        if (r < k) x = fms(x, cf[r], H[(int64_t)r * n + c]);
      Gj[c] = x;
    }
  }
}

// k > 1 with U and H of a matrix staged in shared memory (2 k n s <= kUpdBlkSmem bytes): one
// block per matrix at a time; its warps sweep the matrix's rows RW at a time, reading U and H
// from shared memory instead of once per row from L2.
constexpr int kUpdBlkSmem = 100 * 1024;  // two blocks per SM

template <typename T, int CH, int RW, int KM>
__global__ void __launch_bounds__(kUpdRowThreads, 2) upd_rows_blk_kernel(UpdArgs<T> A) {
  constexpr int E = 16 / (int)sizeof(T);
  constexpr int NWP = kUpdRowThreads / 32;
  extern __shared__ __align__(16) unsigned char upd_raw[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = A.n, k = A.k, np = n / E;
  UpdPiece<T>* Us = reinterpret_cast<UpdPiece<T>*>(upd_raw);  // k x np
  UpdPiece<T>* Hs = Us + (size_t)k * np;                       // k x np
  __shared__ int ids[kUpdMaxK];
  for (int64_t b = blockIdx.x; b < A.B; b += gridDim.x) {
    const int act = A.act[b];
    if (act == UPD_KEEP) continue;  // block-uniform
    UpdPiece<T>* Gp = reinterpret_cast<UpdPiece<T>*>(A.g + b * (int64_t)n * n);
    if (act == UPD_ZERO) {
      UpdPiece<T> z;
#pragma unroll
      for (int e = 0; e < E; ++e) z.v[e] = s_zero<T>();
      for (int64_t e = tid; e < (int64_t)n * np; e += kUpdRowThreads) Gp[e] = z;
      continue;
    }
    const UpdPiece<T>* Up = reinterpret_cast<const UpdPiece<T>*>(A.u + b * (int64_t)k * n);
    const UpdPiece<T>* Hp = reinterpret_cast<const UpdPiece<T>*>(A.h + b * (int64_t)k * n);
    for (int e = tid; e < k * np; e += kUpdRowThreads) {
      Us[e] = Up[e];
      Hs[e] = Hp[e];
    }
    if (tid < k) ids[tid] = A.idx[b * k + tid];
    __syncthreads();
    for (int j0 = warp * RW; j0 < n; j0 += NWP * RW) {
      UpdPiece<T> x[RW][CH];
#pragma unroll
      for (int w = 0; w < RW; ++w)
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int p = c * 32 + lane;
          if (p < np && j0 + w < n) {
            x[w][c] = Gp[(int64_t)(j0 + w) * np + p];
          } else {
#pragma unroll
            for (int e = 0; e < E; ++e) x[w][c].v[e] = s_zero<T>();
          }
        }
      T cf[RW][KM];
#pragma unroll
      for (int w = 0; w < RW; ++w)
#pragma unroll
        for (int r = 0; r < KM; ++r) cf[w][r] = s_zero<T>();
#pragma unroll
      for (int r = 0; r < KM; ++r) {
        if (r < k) {
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            const int p = c * 32 + lane;
            if (p < np) {
              const UpdPiece<T> u = Us[r * np + p];
#pragma unroll
              for (int e = 0; e < E; ++e)
#pragma unroll
                for (int w = 0; w < RW; ++w) cf[w][r] = fma_(u.v[e], x[w][c].v[e], cf[w][r]);
            }
          }
        }
      }
#pragma unroll
      for (int w = 0; w < RW; ++w) {
        const T tot = warp_reduce_scatter<T, KM>(cf[w], lane);
#pragma unroll
        for (int r = 0; r < KM; ++r) cf[w][r] = shfl_idx<T>(tot, r);
#pragma unroll
        for (int r = 0; r < KM; ++r)
          if (r < k && ids[r] == j0 + w) cf[w][r] = sub(cf[w][r], s_one<T>());
      }
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int p = c * 32 + lane;
        if (p < np) {
#pragma unroll
          for (int r = 0; r < KM; ++r) {
            if (r < k) {
              const UpdPiece<T> h = Hs[r * np + p];
#pragma unroll
              for (int w = 0; w < RW; ++w)
#pragma unroll
                for (int e = 0; e < E; ++e) x[w][c].v[e] = fms(x[w][c].v[e], cf[w][r], h.v[e]);
            }
          }
#pragma unroll
          for (int w = 0; w < RW; ++w)
            if (j0 + w < n) Gp[(int64_t)(j0 + w) * np + p] = x[w][c];
        }
      }
    }
    __syncthreads();  // Us, Hs, ids free for the next matrix
  }
}

// ---------------------------------------------------------------- Pfaffian moves (k = 1)
// A one-electron move of a Pfaffian wavefunction replaces row and column i of the skew S by
// u and -u (u_i is ignored: the skew diagonal stays 0). The state is the slogpf gradient
// G = S^-T / 2 = -S^-1 / 2 (fermix_slogpf_grad, adjugate 0). With g_i = row i of G and
// v = G u, the rank-2 skew Woodbury identity gives
//   pf(S') / pf(S) = rho = 2 g_i . u,
//   G' = G + (y g_i^T - g_i y^T) / rho,  y = e_i - 2 v,
// i.e. row j of G' is G_j + ((d_ij - 2 v_j) g_i - g_ij y) / rho. Every row needs the whole
// of v, so the update takes three launches: the ratio (and a snapshot of g_i), v, the rows.
template <typename T>
struct PfMoveArgs {
  T* g;                         // (B, n, n) G = S^-T / 2, updated in place
  const T* u;                   // (B, n) the new row of S
  const int* idx;               // (B,) the moved index i
  const unsigned char* accept;  // (B,) or null = all
  T* sign;                      // (B,) sign of pf(S') / pf(S)
  typename Sc<T>::R* logabs;    // (B,) log |pf(S') / pf(S)|
  T* h;                         // (B, n) workspace: g_i
  T* v;                         // (B, n) workspace: G u
  T* rho;                       // (B,) workspace: the ratio
  int* act;                     // (B,) workspace: UPD_KEEP / UPD_APPLY / UPD_ZERO
  int64_t B;
  int n;
  uint32_t wait_polls;          // polls of the bounded copy wait (pfm_smem_kernel)
};

// x . y over n entries with entry `skip` left out
template <typename T>
__device__ __forceinline__ T warp_dot_skip(const T* __restrict__ x, const T* __restrict__ y, int n, int skip,
                                           int lane) {
  T acc = s_zero<T>();
  for (int c = lane; c < n; c += 32)
    if (c != skip) acc = fma_(x[c], y[c], acc);
  return warp_sum_t<T>(acc);
}

template <typename T>
__global__ void __launch_bounds__(kUpdRowThreads) pfm_prep_kernel(PfMoveArgs<T> A) {
  using R = typename Sc<T>::R;
  const int lane = threadIdx.x & 31;
  const int n = A.n;
  const int64_t wstride = (int64_t)gridDim.x * (kUpdRowThreads / 32);
  for (int64_t b = (int64_t)blockIdx.x * (kUpdRowThreads / 32) + (threadIdx.x >> 5); b < A.B; b += wstride) {
    const int i = A.idx[b];
    const bool bad = i < 0 || i >= n;
    const T* Gi = A.g + (b * n + (bad ? 0 : i)) * (int64_t)n;
    T d = s_zero<T>();
    if (!bad) {
      d = warp_dot_skip(Gi, A.u + b * (int64_t)n, n, i, lane);
      d = add(d, d);
    }
    const bool sing = !bad && is_zero(d);
    const bool acc = A.accept == nullptr || A.accept[b] != 0;
    if (lane == 0) {
      A.sign[b] = bad ? upd_nan<T>() : (sing ? s_zero<T>() : unit(d));
      A.logabs[b] = bad ? R(NAN) : (sing ? -R(INFINITY) : rlog(mag(d)));
      if (A.h) {
        A.act[b] = (!acc || bad) ? UPD_KEEP : (sing ? UPD_ZERO : UPD_APPLY);
        A.rho[b] = d;
      }
    }
    if (A.h && acc && !bad && !sing)
      for (int c = lane; c < n; c += 32) A.h[b * (int64_t)n + c] = Gi[c];
  }
}

// v_j = G_j . u (u_i left out), one warp per row of the matrices that apply the move
template <typename T>
__global__ void __launch_bounds__(kUpdRowThreads) pfm_v_kernel(PfMoveArgs<T> A) {
  const int lane = threadIdx.x & 31;
  const int n = A.n;
  const int64_t rows = A.B * (int64_t)n;
  const int64_t wstride = (int64_t)gridDim.x * (kUpdRowThreads / 32);
  for (int64_t q = (int64_t)blockIdx.x * (kUpdRowThreads / 32) + (threadIdx.x >> 5); q < rows; q += wstride) {
    const int64_t b = q / n;
    if (A.act[b] != UPD_APPLY) continue;
    const T vj = warp_dot_skip(A.g + q * n, A.u + b * (int64_t)n, n, A.idx[b], lane);
    if (lane == 0) A.v[q] = vj;
  }
}

// G_j += ((d_ij - 2 v_j) g_i - g_ij (e_i - 2 v)) / rho, in place, one warp per row
template <typename T>
__global__ void __launch_bounds__(kUpdRowThreads) pfm_rows_kernel(PfMoveArgs<T> A) {
  const int lane = threadIdx.x & 31;
  const int n = A.n;
  const int64_t rows = A.B * (int64_t)n;
  const int64_t wstride = (int64_t)gridDim.x * (kUpdRowThreads / 32);
  for (int64_t q = (int64_t)blockIdx.x * (kUpdRowThreads / 32) + (threadIdx.x >> 5); q < rows; q += wstride) {
    const int64_t b = q / n;
    const int j = (int)(q - b * n);
    const int act = A.act[b];
    if (act == UPD_KEEP) continue;
    T* Gj = A.g + q * n;
    if (act == UPD_ZERO) {
      for (int c = lane; c < n; c += 32) Gj[c] = s_zero<T>();
      continue;
    }
    const int i = A.idx[b];
    const T ri = recip(A.rho[b]);
    const T* h = A.h + b * (int64_t)n;
    const T* v = A.v + b * (int64_t)n;
    T c1 = neg(add(v[j], v[j]));
    if (j == i) c1 = add(c1, s_one<T>());
    c1 = mul(c1, ri);                 // (d_ij - 2 v_j) / rho
    const T c2 = neg(mul(h[j], ri));  // -g_ij / rho
    for (int c = lane; c < n; c += 32) {
      T y = neg(add(v[c], v[c]));
      if (c == i) y = add(y, s_one<T>());
      Gj[c] = fma_(c2, y, fma_(c1, h[c], Gj[c]));
    }
  }
}

// Pfaffian move with G held in shared memory (n^2 s <= kPfmSmemMax bytes, n s a multiple of
// 16): one block per matrix, the whole move in one launch. Thread 0 brings G in with one bulk
// copy (cp.async.bulk, completing on an mbarrier; the wait is bounded and a timeout turns
// the block's remaining outputs into NaN), then the ratio rho = 2 g_i . u, v = G u, y = e_i - 2v
// and the updated rows (written straight to global) all read shared memory, so G crosses HBM
// once each way: the 2 n^2 s roofline.
constexpr int kPfmSmemMax = 64 * 1024;
constexpr int kPfmThreads = 256;
constexpr uint32_t kPfmWaitIters = 1u << 24;

template <typename T>
__global__ void __launch_bounds__(kPfmThreads) pfm_smem_kernel(PfMoveArgs<T> A) {
  using R = typename Sc<T>::R;
  extern __shared__ __align__(16) unsigned char pfm_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NW = kPfmThreads / 32;
  const int n = A.n;
  T* Gs = reinterpret_cast<T*>(pfm_raw);  // n x n
  T* us = Gs + (size_t)n * n;              // u with u_i = 0
  T* ys = us + n;                          // y = e_i - 2 G u
  T* red = ys + n;                         // red[NW]: the ratio
  uint64_t* mbar = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(red + NW + 1) + 7) & ~(uintptr_t)7);
  __shared__ int s_dead, s_skip;
  if (tid == 0) {
    umma::mbar_init(mbar, 1);
    umma::fence_mbar_init();
    s_dead = 0;
  }
  __syncthreads();
  uint32_t phase = 0;
  const uint32_t bytes = (uint32_t)((size_t)n * n * sizeof(T));
  for (int64_t b = blockIdx.x; b < A.B; b += gridDim.x) {
    const int i = A.idx[b];
    const bool bad = i < 0 || i >= n;
    const bool acc = A.accept == nullptr || A.accept[b] != 0;
    T* Gg = A.g + b * (int64_t)n * n;
    const bool dead = s_dead != 0;
    // rejected members need only the ratio (row i of G from global); the others load G
    const bool load = !dead && !bad && acc;
    if (load && tid == 0) {
      umma::fence_proxy_async_smem();  // earlier generic reads of Gs before the async write
      umma::mbar_arrive_expect_tx(mbar, bytes);
      umma::bulk_g2s(Gs, Gg, bytes, mbar);
    }
    for (int c = tid; c < n; c += kPfmThreads) us[c] = (c == i || bad) ? s_zero<T>() : A.u[b * (int64_t)n + c];
    if (load) {
      if (!umma::mbar_wait(mbar, phase, A.wait_polls)) {
        s_dead = 1;  // give the copy one more bounded wait; no later matrix loads into Gs
        (void)umma::mbar_wait(mbar, phase, kPfmWaitIters);
      }
      phase ^= 1;
    }
    __syncthreads();
    const bool fail = s_dead != 0;
    // the ratio rho = 2 g_i . u by warp 0, in the order of pfm_prep_kernel (so that the
    // ratio and update calls give the same bits)
    const T* gi = load && !fail ? Gs + (size_t)i * n : Gg + (size_t)(bad ? 0 : i) * n;
    T d = s_zero<T>();
    if (warp == 0 && !bad && !fail) {
      d = warp_dot_skip(gi, us, n, i, lane);
      d = add(d, d);
    }
    if (tid == 0) {
      const bool sing = !bad && is_zero(d);
      A.sign[b] = (bad || fail) ? upd_nan<T>() : (sing ? s_zero<T>() : unit(d));
      A.logabs[b] = (bad || fail) ? R(NAN) : (sing ? -R(INFINITY) : rlog(mag(d)));
      red[NW] = d;
      s_skip = (!load || fail) ? 1 : (sing ? 2 : 0);
      if (fail) umma::record_status(8);  // FX_ERR_TIMEOUT: G is left as it was
    }
    __syncthreads();
    const int skip = s_skip;
    if (skip == 2) {  // accepted move with ratio exactly 0: G' = 0
      for (int64_t e = tid; e < (int64_t)n * n; e += kPfmThreads) Gg[e] = s_zero<T>();
    } else if (skip == 0) {
      // y = e_i - 2 G u, one warp per row of the shared copy
      for (int j = warp; j < n; j += NW) {
        T acc2 = s_zero<T>();
        for (int c = lane; c < n; c += 32) acc2 = fma_(Gs[(size_t)j * n + c], us[c], acc2);
        acc2 = warp_sum_t<T>(acc2);
        if (lane == 0) {
          T yv = neg(add(acc2, acc2));
          if (j == i) yv = add(yv, s_one<T>());
          ys[j] = yv;
        }
      }
      __syncthreads();
      // G'_j = G_j + (y_j g_i - g_ij y) / rho
      const T ri = recip(red[NW]);
      const T* h = Gs + (size_t)i * n;
      for (int j = warp; j < n; j += NW) {
        const T c1 = mul(ys[j], ri), c2 = neg(mul(h[j], ri));
        for (int c = lane; c < n; c += 32)
          Gg[(size_t)j * n + c] = fma_(c2, ys[c], fma_(c1, h[c], Gs[(size_t)j * n + c]));
      }
    }
    __syncthreads();  // Gs, us, ys, red free for the next matrix
  }
}

// Gs, us, ys, red[9], then the mbarrier at the next 8-byte boundary
inline size_t pfm_smem_bytes(int n, size_t s) { return (size_t)n * n * s + 2 * (size_t)n * s + 9 * s + 32; }

// CH: 16-byte pieces per lane (row bytes <= CH * 512); RW: rows per warp; KM: the largest k
template <typename T, int CH, int RW, int KM>
__global__ void __launch_bounds__(kUpdRowThreads, KM <= 4 ? 2 : 1) upd_rows_vec_kernel(UpdArgs<T> A) {
  constexpr int E = 16 / (int)sizeof(T);
  const int lane = threadIdx.x & 31;
  const int n = A.n, k = A.k;
  const int np = n / E;  // pieces per row
  const int gpm = (n + RW - 1) / RW;
  const int64_t groups = A.B * gpm;
  const int64_t wstride = (int64_t)gridDim.x * (kUpdRowThreads / 32);
  // U and H do not depend on G: where registers allow they are loaded together with the rows
  constexpr bool HOIST = KM * CH <= 4 && (KM == 1 || sizeof(T) <= 8);
  int64_t q = (int64_t)blockIdx.x * (kUpdRowThreads / 32) + (threadIdx.x >> 5);
  int act_next = q < groups ? A.act[q / gpm] : UPD_KEEP;
  for (; q < groups; q += wstride) {
    const int64_t b = q / gpm;
    const int j0 = (int)(q - b * gpm) * RW;
    const int act = act_next;
    if (q + wstride < groups) act_next = A.act[(q + wstride) / gpm];  // in flight meanwhile
    if (act == UPD_KEEP) continue;
    UpdPiece<T>* Gp = reinterpret_cast<UpdPiece<T>*>(A.g + (b * n + j0) * (int64_t)n);
    UpdPiece<T> x[RW][CH];
#pragma unroll
    for (int w = 0; w < RW; ++w)
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int p = c * 32 + lane;
        if (p < np && j0 + w < n) {
          x[w][c] = Gp[(int64_t)w * np + p];
        } else {
#pragma unroll
          for (int e = 0; e < E; ++e) x[w][c].v[e] = s_zero<T>();
        }
      }
    if (act == UPD_APPLY) {
      const UpdPiece<T>* Up = reinterpret_cast<const UpdPiece<T>*>(A.u + b * (int64_t)k * n);
      const UpdPiece<T>* Hp = reinterpret_cast<const UpdPiece<T>*>(A.h + b * (int64_t)k * n);
      const int* id = A.idx + b * k;
      UpdPiece<T> uu[HOIST ? KM : 1][HOIST ? CH : 1], hh[HOIST ? KM : 1][HOIST ? CH : 1];
      if constexpr (HOIST) {
#pragma unroll
        for (int r = 0; r < KM; ++r)
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            const int p = c * 32 + lane;
            if (r < k && p < np) {
              uu[r][c] = Up[(int64_t)r * np + p];
              hh[r][c] = Hp[(int64_t)r * np + p];
            }
          }
      }
      // lane partials of the k dot products of each row, then one reduce-scatter per row
      T cf[RW][KM];
#pragma unroll
      for (int w = 0; w < RW; ++w)
#pragma unroll
        for (int r = 0; r < KM; ++r) cf[w][r] = s_zero<T>();
#pragma unroll
      for (int r = 0; r < KM; ++r) {
        if (r < k) {
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            const int p = c * 32 + lane;
            if (p < np) {
              const UpdPiece<T> u = HOIST ? uu[HOIST ? r : 0][HOIST ? c : 0] : Up[(int64_t)r * np + p];
#pragma unroll
              for (int e = 0; e < E; ++e)
#pragma unroll
                for (int w = 0; w < RW; ++w) cf[w][r] = fma_(u.v[e], x[w][c].v[e], cf[w][r]);
            }
          }
        }
      }
#pragma unroll
      for (int w = 0; w < RW; ++w) {
        if constexpr (KM == 1) {
          cf[w][0] = warp_sum_t<T>(cf[w][0]);
        } else {
          const T tot = warp_reduce_scatter<T, KM>(cf[w], lane);  // the sum of index lane % KM
#pragma unroll
          for (int r = 0; r < KM; ++r) cf[w][r] = shfl_idx<T>(tot, r);
        }
#pragma unroll
        for (int r = 0; r < KM; ++r)
          if (r < k && __ldg(id + r) == j0 + w) cf[w][r] = sub(cf[w][r], s_one<T>());
      }
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int p = c * 32 + lane;
        if (p < np) {
#pragma unroll
          for (int r = 0; r < KM; ++r) {
            if (r < k) {
              const UpdPiece<T> h = HOIST ? hh[HOIST ? r : 0][HOIST ? c : 0] : Hp[(int64_t)r * np + p];
#pragma unroll
              for (int w = 0; w < RW; ++w)
#pragma unroll
                for (int e = 0; e < E; ++e) x[w][c].v[e] = fms(x[w][c].v[e], cf[w][r], h.v[e]);
            }
          }
        }
      }
    } else {  // UPD_ZERO
#pragma unroll
      for (int w = 0; w < RW; ++w)
#pragma unroll
        for (int c = 0; c < CH; ++c)
#pragma unroll
          for (int e = 0; e < E; ++e) x[w][c].v[e] = s_zero<T>();
    }
#pragma unroll
    for (int w = 0; w < RW; ++w)
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int p = c * 32 + lane;
        if (p < np && j0 + w < n) Gp[(int64_t)w * np + p] = x[w][c];
      }
  }
}

// Vector forms of the Pfaffian move's two row passes (rows of up to 4 KB, a multiple of 16
// bytes): RW rows of one matrix per warp as 16-byte pieces in registers, as upd_rows_vec_kernel.
template <typename T, int CH, int RW>
__global__ void __launch_bounds__(kUpdRowThreads, 2) pfm_v_vec_kernel(PfMoveArgs<T> A) {
  constexpr int E = 16 / (int)sizeof(T);
  const int lane = threadIdx.x & 31;
  const int n = A.n, np = n / E, gpm = (n + RW - 1) / RW;
  const int64_t groups = A.B * gpm;
  const int64_t wstride = (int64_t)gridDim.x * (kUpdRowThreads / 32);
  for (int64_t q = (int64_t)blockIdx.x * (kUpdRowThreads / 32) + (threadIdx.x >> 5); q < groups; q += wstride) {
    const int64_t b = q / gpm;
    const int j0 = (int)(q - b * gpm) * RW;
    if (A.act[b] != UPD_APPLY) continue;
    const int i = A.idx[b];
    const UpdPiece<T>* Gp = reinterpret_cast<const UpdPiece<T>*>(A.g + (b * n + j0) * (int64_t)n);
    const UpdPiece<T>* Up = reinterpret_cast<const UpdPiece<T>*>(A.u + b * (int64_t)n);
    T acc[RW];
#pragma unroll
    for (int w = 0; w < RW; ++w) acc[w] = s_zero<T>();
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int p = c * 32 + lane;
      if (p < np) {
        UpdPiece<T> u = Up[p];
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (p * E + e == i) u.v[e] = s_zero<T>();  // u_i is not part of the move
#pragma unroll
        for (int w = 0; w < RW; ++w) {
          if (j0 + w < n) {
            const UpdPiece<T> x = Gp[(int64_t)w * np + p];
#pragma unroll
            for (int e = 0; e < E; ++e) acc[w] = fma_(u.v[e], x.v[e], acc[w]);
          }
        }
      }
    }
#pragma unroll
    for (int w = 0; w < RW; ++w) {
      const T vj = warp_sum_t<T>(acc[w]);
      if (lane == 0 && j0 + w < n) A.v[b * (int64_t)n + j0 + w] = vj;
    }
  }
}

template <typename T, int CH, int RW>
__global__ void __launch_bounds__(kUpdRowThreads, 2) pfm_rows_vec_kernel(PfMoveArgs<T> A) {
  constexpr int E = 16 / (int)sizeof(T);
  const int lane = threadIdx.x & 31;
  const int n = A.n, np = n / E, gpm = (n + RW - 1) / RW;
  const int64_t groups = A.B * gpm;
  const int64_t wstride = (int64_t)gridDim.x * (kUpdRowThreads / 32);
  int64_t q = (int64_t)blockIdx.x * (kUpdRowThreads / 32) + (threadIdx.x >> 5);
  int act_next = q < groups ? A.act[q / gpm] : UPD_KEEP;
  for (; q < groups; q += wstride) {
    const int64_t b = q / gpm;
    const int j0 = (int)(q - b * gpm) * RW;
    const int act = act_next;
    if (q + wstride < groups) act_next = A.act[(q + wstride) / gpm];
    if (act == UPD_KEEP) continue;
    UpdPiece<T>* Gp = reinterpret_cast<UpdPiece<T>*>(A.g + (b * n + j0) * (int64_t)n);
    if (act == UPD_ZERO) {
      UpdPiece<T> z;
#pragma unroll
      for (int e = 0; e < E; ++e) z.v[e] = s_zero<T>();
#pragma unroll
      for (int w = 0; w < RW; ++w)
#pragma unroll
        for (int c = 0; c < CH; ++c)
          if (c * 32 + lane < np && j0 + w < n) Gp[(int64_t)w * np + c * 32 + lane] = z;
      continue;
    }
    const int i = A.idx[b];
    const T* h = A.h + b * (int64_t)n;
    const T* v = A.v + b * (int64_t)n;
    const UpdPiece<T>* Hp = reinterpret_cast<const UpdPiece<T>*>(h);
    const UpdPiece<T>* Vp = reinterpret_cast<const UpdPiece<T>*>(v);
    const T ri = recip(A.rho[b]);
    T c1[RW], c2[RW];
#pragma unroll
    for (int w = 0; w < RW; ++w) {
      const int j = j0 + w < n ? j0 + w : j0;
      T t = neg(add(v[j], v[j]));
      if (j == i) t = add(t, s_one<T>());
      c1[w] = mul(t, ri);            // (d_ij - 2 v_j) / rho
      c2[w] = neg(mul(h[j], ri));    // -g_ij / rho
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int p = c * 32 + lane;
      if (p < np) {
        const UpdPiece<T> hp = Hp[p];
        UpdPiece<T> y = Vp[p];
#pragma unroll
        for (int e = 0; e < E; ++e) {
          T t = neg(add(y.v[e], y.v[e]));
          if (p * E + e == i) t = add(t, s_one<T>());
          y.v[e] = t;  // y = e_i - 2 v
        }
#pragma unroll
        for (int w = 0; w < RW; ++w) {
          if (j0 + w < n) {
            UpdPiece<T> x = Gp[(int64_t)w * np + p];
#pragma unroll
            for (int e = 0; e < E; ++e) x.v[e] = fma_(c2[w], y.v[e], fma_(c1[w], hp.v[e], x.v[e]));
            Gp[(int64_t)w * np + p] = x;
          }
        }
      }
    }
  }
}

}  // namespace fx
