// Blocked LU / Gauss-Jordan engine for slogdet and its gradient at n > 256, every dtype:
// a host-driven loop over panels of NB columns, each panel a short sequence of batched
// kernels (grid = the batch slice x tiles), the matrices in the caller's workspace.
//
// Reference behaviour: the blocked LU of src/fermix/_lu.py:51-120 (panel) and :153-217
// (trailing update) with sign / log|det| as in :543-611 (pivot = largest abs1 entry of
// the column, first occurrence; a zero pivot gives a zero multiplier column, sign 0 and
// logabs -inf); gradient A^-T (src/fermix/_inverse.py:502-531), zero for an exactly
// singular or non-finite member.
//
// Per panel K = [k0, k0 + kw):
//   1. pivots by tall-skinny LU: every chunk of 512 rows runs partial pivoting on its
//      panel rows in registers (lg_leaf_kernel); the chunks' pivot rows then compete in
//      one more partial-pivoting pass that also yields L11 / U11 (lg_tree_kernel). With a
//      single chunk (n - k0 <= 512) this IS partial pivoting; above, the pivot order is
//      the tournament's (a documented deviation, same determinant);
//   2. the row interchanges on the whole rows, and a snapshot Pb of the pivot rows
//      (lg_swap_kernel);
//   3. per row, the coefficients C_x = l_x L11^-1 with l_x = M_xK U11^-1 -- forward then
//      back substitution, the same sequential FMA chains as the elimination, so that a
//      row duplicating pivot row s gets exactly e_s (lg_coef_kernel);
//   4. M -= C Pb over the trailing block (forward) or the whole matrix outside K
//      (gradient), one FMA chain per entry in panel-column order (lg_update_kernel).
// Gradient mode is the Gauss-Jordan exchange: pivot rows take C = e_j + (A_PK^-1)_j,
// rows above the panel take their C as well, and the panel columns are replaced by C
// (and A_PK^-1 for the pivot rows). After the last panel the workspace holds
// (P A)^-1 = A^-1 P^T; lg_grad_kernel writes grad[perm[k]][j] = M[j][k].
#pragma once
#include "fused_lu.cuh"

namespace fx {

constexpr int kLgChunk = 512;  // rows per tall-skinny leaf (one thread per row)

template <typename T>
struct LgCfg {
  static constexpr int NB = sizeof(T) <= 8 ? 32 : 16;  // panel width (registers per row)
};

// Per-matrix state of the engine, all in the workspace (bs = matrices in the slice).
template <typename T>
struct LgArgs {
  T* M;          // bs x n x n, the matrices being factorised (row-major)
  T* C;          // bs x n x NB coefficients of the current panel
  T* P;          // bs x NB x n snapshot of the current pivot rows
  T* LU11;       // bs x 3 x NB x NB: L11 (strict lower), U11 (upper), A_PK^-1 (gradient)
  T* piv;        // bs x n pivots
  int* ipiv;     // bs x n interchanges (LAPACK order: row k swapped with ipiv[k])
  int* cand;     // bs x nchunk x NB leaf pivot rows
  int* perm;     // bs x n row permutation (gradient)
  int* flag;     // bs: non-finite entry seen in the inverse (gradient)
  int n, k0, kw, nchunk;
  int grad;  // gradient mode (the tree kernel also forms A_PK^-1)
  // caller options: write (sign, logabs, value) (slogdet) or not (the Pfaffian gradient,
  // whose primal comes from the Parlett-Reid forward); scale of the gradient (1 for
  // slogdet, 1/2 for slogpf: d log pf / dS = S^-T / 2); zsign: a zero entry zeroes that
  // member's gradient (the Pfaffian forward's exact singularity)
  int primal;
  typename Sc<T>::R gscale;
  const T* zsign;
  uint32_t wait_polls;  // polls of the tensor-core update's bounded completion wait
};

// Element reader of the caller's input: interleaved values, or split real / imaginary
// planes for complex dtypes (re set).
template <typename T>
struct SrcMat {
  typedef typename Sc<T>::R R;
  const T* a;
  const R* re;
  const R* im;
  __device__ __forceinline__ T at(size_t off) const {
    if constexpr (Sc<T>::cx) {
      if (re) return T{re[off], im[off]};
    }
    return a[off];
  }
  __host__ __device__ SrcMat offset(size_t off) const {
    return SrcMat{a ? a + off : nullptr, re ? re + off : nullptr, im ? im + off : nullptr};
  }
};

template <typename T>
__host__ __device__ inline SrcMat<T> src_of(const Job<T>& J) {
  return SrcMat<T>{J.a, J.a_re, J.a_im};
}

// M = (a - a^T) / 2 of matrix blockIdx.z (32 x 32 tiles through shared memory)
template <typename T>
__global__ void __launch_bounds__(256) lg_skew_copy_kernel(T* M, SrcMat<T> a, int n) {
  __shared__ T tile[32][33];
  typedef typename Sc<T>::R R;
  const int b = blockIdx.z, i0 = blockIdx.y * 32, j0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const SrcMat<T> ab = a.offset((size_t)b * n * n);
  // tile of a^T: rows j0.., columns i0..
  for (int r = ty; r < 32; r += 8) {
    const int j = j0 + r, i = i0 + tx;
    tile[r][tx] = (j < n && i < n) ? ab.at((size_t)j * n + i) : s_zero<T>();
  }
  __syncthreads();
  T* Mb = M + (size_t)b * n * n;
  for (int r = ty; r < 32; r += 8) {
    const int i = i0 + r, j = j0 + tx;
    if (i < n && j < n) Mb[(size_t)i * n + j] = scale(sub(ab.at((size_t)i * n + j), tile[tx][r]), R(0.5));
  }
}

// M = a for `count` elements from split planes (complex dtypes only)
template <typename T>
__global__ void __launch_bounds__(256) lg_planar_copy_kernel(T* M, SrcMat<T> a, size_t count) {
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < count; e += (size_t)gridDim.x * blockDim.x)
    M[e] = a.at(e);
}

template <typename T>
__device__ __forceinline__ typename Sc<T>::R lg_key(T v, bool live) {
  typedef typename Sc<T>::R R;
  if (!live) return R(-1);
  const R a = abs1(v);
  return a != a ? R(-0.5) : a;  // NaN: a candidate only when every candidate is NaN
}

// Order key of a pivot candidate as 64 bits: 0 = not a candidate, 1 = NaN (a candidate
// only when every candidate is NaN), else the bits of abs1(v) (a non-negative float orders as
// its bit pattern) plus 2.
template <typename T>
__device__ __forceinline__ uint64_t lg_key64(T v, bool live) {
  typedef typename Sc<T>::R R;
  if (!live) return 0ull;
  const R a = abs1(v);
  if (a != a) return 1ull;
  if constexpr (sizeof(R) == 8) return (uint64_t)__double_as_longlong(a) + 2ull;
  else return (uint64_t)__float_as_uint(a) + 2ull;
}

// Warp argmax over (key, then the smallest pos) with redux.sync: every lane gets the
// winning key and pos.
__device__ __forceinline__ void lg_warp_argmax(uint64_t key, int pos, uint64_t& km, int& pm) {
  const unsigned hi = (unsigned)(key >> 32), lo = (unsigned)key;
  const unsigned mh = __reduce_max_sync(0xffffffffu, hi);
  const unsigned ml = __reduce_max_sync(0xffffffffu, hi == mh ? lo : 0u);
  km = ((uint64_t)mh << 32) | ml;
  pm = __reduce_min_sync(0xffffffffu, key == km ? pos : 0x7fffffff);
}

// Partial pivoting on the panel columns [k0, k0 + kw) of up to 512 listed rows (thread i
// holds row rows[i] in registers). Writes the kw pivot rows in order to out[]; with
// want_lu also L11 / U11 and the pivots. Every block thread must call it. Per column: each
// warp reduces its candidates with redux.sync, the warp winners go to shared memory with
// their rows, and after one barrier every warp reduces the 16 warp winners the same way.
template <typename T, int NB>
__device__ void lg_gepp(const T* __restrict__ Mb, int n, int k0, int kw, const int* rows, int count, int* out,
                        T* L11, T* U11, T* pivs, bool want_lu, unsigned char* smem) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NW = kLgChunk / 32;
  unsigned long long* skey = reinterpret_cast<unsigned long long*>(smem);  // [2][NW]
  int* spos = reinterpret_cast<int*>(skey + 2 * NW);                        // [2][NW] row position
  int* sidx = spos + 2 * NW;                                                // [2][NW] list index
  T* srow = reinterpret_cast<T*>(sidx + 2 * NW + (2 * NW) % 4);             // [2][NW][NB]
  const bool have = tid < count;
  const int myrow = have ? rows[tid] : 0x7fffffff;
  T pr[NB];
#pragma unroll
  for (int t = 0; t < NB; ++t) pr[t] = (have && t < kw) ? Mb[(size_t)myrow * n + k0 + t] : s_zero<T>();
  int mystep = have ? -1 : NB;
#pragma unroll
  for (int s = 0; s < NB; ++s) {
    if (s < kw) {
      const bool live = mystep < 0;
      const uint64_t key = lg_key64(pr[s], live);
      const int pos = live ? myrow : 0x7fffffff;
      uint64_t wk;
      int wp;
      lg_warp_argmax(key, pos, wk, wp);
      const unsigned win = __ballot_sync(0xffffffffu, key == wk && pos == wp);
      const int par = s & 1;
      if (lane == __ffs(win) - 1) {
        skey[par * NW + warp] = wk;
        spos[par * NW + warp] = wp;
        sidx[par * NW + warp] = tid;
#pragma unroll
        for (int t = 0; t < NB; ++t) srow[(par * NW + warp) * NB + t] = pr[t];
      }
      __syncthreads();
      const uint64_t ck = lane < NW ? (uint64_t)skey[par * NW + lane] : 0ull;
      const int cp = lane < NW ? spos[par * NW + lane] : 0x7fffffff;
      uint64_t kv;
      int kp;
      lg_warp_argmax(ck, cp, kv, kp);
      const unsigned wwin = __ballot_sync(0xffffffffu, lane < NW && ck == kv && cp == kp);
      const int w0 = __ffs(wwin) - 1;
      const bool valid = kp != 0x7fffffff;  // false once fewer rows than steps remain
      const int wi = sidx[par * NW + w0];
      const T* u = srow + (par * NW + w0) * NB;
      const T pv = u[s];
      if (valid && tid == wi) {
        mystep = s;
      } else if (valid && mystep < 0) {
        const T l = is_zero(pv) ? s_zero<T>() : sdiv(pr[s], pv);
        pr[s] = l;
#pragma unroll
        for (int t = 0; t < NB; ++t)
          if (t > s) pr[t] = fms(pr[t], l, u[t]);
      }
      if (tid == 0) {
        out[s] = valid ? kp : -1;
        if (want_lu) pivs[s] = pv;
      }
    }
  }
  if (want_lu && mystep >= 0 && mystep < kw) {
    const int j = mystep;
#pragma unroll
    for (int t = 0; t < NB; ++t) {
      if (t < j) L11[j * NB + t] = pr[t];
      else U11[j * NB + t] = pr[t];
    }
  }
  __syncthreads();
}

template <typename T>
constexpr size_t lg_gepp_smem() {
  constexpr int NW = kLgChunk / 32;
  return 2 * NW * sizeof(unsigned long long) + 4 * NW * sizeof(int) + 64 + 2 * NW * LgCfg<T>::NB * sizeof(T) + 64;
}

// 1. leaf: chunk blockIdx.x of the rows [k0, n) of matrix blockIdx.y
template <typename T>
__global__ void __launch_bounds__(kLgChunk) lg_leaf_kernel(LgArgs<T> A) {
  constexpr int NB = LgCfg<T>::NB;
  extern __shared__ __align__(16) unsigned char smem[];
  int* rows = reinterpret_cast<int*>(smem);
  const int b = blockIdx.y, c = blockIdx.x, n = A.n;
  const int r0 = A.k0 + c * kLgChunk;
  const int count = min(kLgChunk, n - r0);
  rows[threadIdx.x] = r0 + threadIdx.x;
  __syncthreads();
  lg_gepp<T, NB>(A.M + (size_t)b * n * n, n, A.k0, A.kw, rows, count, A.cand + ((size_t)b * A.nchunk + c) * NB,
                 nullptr, nullptr, nullptr, false, smem + kLgChunk * sizeof(int));
}

// 2. tree: partial pivoting over the leaves' candidates (in chunk order, at most 512 rows
// per pass: winners of a pass compete again with the next candidates) gives the panel's
// pivot rows, L11, U11 and the pivots; thread 0 turns the rows into LAPACK-order
// interchanges.
template <typename T>
__global__ void __launch_bounds__(kLgChunk) lg_tree_kernel(LgArgs<T> A) {
  constexpr int NB = LgCfg<T>::NB;
  extern __shared__ __align__(16) unsigned char smem[];
  int* rows = reinterpret_cast<int*>(smem);  // [512] current pass
  int* sel = rows + kLgChunk;                // [NB] winners
  const int nc = A.nchunk * NB > kLgChunk ? A.nchunk * NB : kLgChunk;
  int* allc = sel + NB;                      // [nc] compacted candidates
  int* ntot = allc + nc;                     // [1]
  unsigned char* scratch = smem + (size_t)(kLgChunk + NB + nc + 4) * sizeof(int);
  const int b = blockIdx.x, n = A.n, kw = A.kw, k0 = A.k0;
  const int* cb = A.cand + (size_t)b * A.nchunk * NB;
  if (A.nchunk == 1) {
    // one chunk (n - k0 <= 512): no leaf ran; every row of [k0, n) is a candidate and
    // this pass is plain partial pivoting
    for (int i = threadIdx.x; i < n - k0; i += blockDim.x) allc[i] = k0 + i;
    if (threadIdx.x == 0) *ntot = n - k0;
  }
  __syncthreads();
  int total = 0;
  if (A.nchunk == 1) {
    total = *ntot;
  } else {
    // the leaves' pivot rows in chunk order; every chunk but the last has 512 rows and always
    // yields kw of them, and a chunk's valid entries come first (-1 once its rows run out), so
    // the valid candidates form a prefix of the list: copy in parallel and count them
    for (int base = 0; base < A.nchunk * kw; base += blockDim.x) {
      const int i = base + threadIdx.x;
      int r = -1;
      if (i < A.nchunk * kw) {
        r = cb[(i / kw) * NB + i % kw];
        allc[i] = r;
      }
      total += __syncthreads_count(r >= 0);
    }
  }
  int count = min(total, kLgChunk);
  for (int i = threadIdx.x; i < count; i += blockDim.x) rows[i] = allc[i];
  int consumed = count;
  const T* Mb = A.M + (size_t)b * n * n;
  while (consumed < total) {
    __syncthreads();
    lg_gepp<T, NB>(Mb, n, k0, kw, rows, count, sel, nullptr, nullptr, nullptr, false, scratch);
    const int more = min(total - consumed, kLgChunk - kw);
    if (threadIdx.x < kw) rows[threadIdx.x] = sel[threadIdx.x];
    for (int i = threadIdx.x; i < more; i += blockDim.x) rows[kw + i] = allc[consumed + i];
    count = kw + more;
    consumed += more;
  }
  __syncthreads();
  T* LU = A.LU11 + (size_t)b * 3 * NB * NB;
  lg_gepp<T, NB>(Mb, n, k0, kw, rows, count, sel, LU, LU + NB * NB, A.piv + (size_t)b * n + k0, true, scratch);
  if (A.grad) {
    // A_PK^-1 = U11^-1 L11^-1 for the gradient's pivot rows and swept rows: columns of
    // L11^-1 (threads 0 .. kw-1) and rows of U11^-1 (threads 32 .. 32 + kw-1) in parallel,
    // then the product, two entries per thread
    __syncthreads();  // L11 / U11 written by lg_gepp
    T* Li = reinterpret_cast<T*>(scratch);  // [NB][NB] L11^-1, then reused
    T* Ui = Li + NB * NB;                   // [NB][NB] U11^-1
    const T* L = LU;
    const T* U = LU + NB * NB;
    const int tid = threadIdx.x;
    if (tid < kw) {
      const int t = tid;  // column t of L11^-1: unit lower forward substitution
      T y[NB];
#pragma unroll
      for (int r = 0; r < NB; ++r) {
        T acc = (r == t) ? s_one<T>() : s_zero<T>();
#pragma unroll
        for (int q = 0; q < NB; ++q)
          if (q < r) acc = fms(acc, L[r * NB + q], y[q]);
        y[r] = (r >= t && r < kw) ? acc : s_zero<T>();
        Li[r * NB + t] = y[r];
      }
    } else if (tid >= 32 && tid < 32 + kw) {
      const int j = tid - 32;  // row j of U11^-1: w U11 = e_j
      T w[NB];
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        T acc = (t == j) ? s_one<T>() : s_zero<T>();
#pragma unroll
        for (int q = 0; q < NB; ++q)
          if (q < t) acc = fms(acc, w[q], U[q * NB + t]);
        const T d = U[t * NB + t];
        w[t] = (t < kw && t >= j && !is_zero(d)) ? sdiv(acc, d) : s_zero<T>();
        Ui[j * NB + t] = w[t];
      }
    }
    __syncthreads();
    T* Ai = LU + 2 * NB * NB;
    for (int e = tid; e < NB * NB; e += blockDim.x) {
      const int j = e / NB, t = e % NB;
      T acc = s_zero<T>();
      if (j < kw && t < kw)
        for (int r = 0; r < kw; ++r) acc = fma_(Ui[j * NB + r], Li[r * NB + t], acc);
      Ai[e] = acc;
    }
  }
  if (threadIdx.x == 0) {
    // positions of the chosen rows as earlier interchanges move them
    int cur[NB];
    for (int j = 0; j < kw; ++j) cur[j] = sel[j];
    int* ip = A.ipiv + (size_t)b * n;
    for (int j = 0; j < kw; ++j) {
      const int t = cur[j];
      ip[k0 + j] = t;
      for (int q = j + 1; q < kw; ++q)
        if (cur[q] == k0 + j) cur[q] = t;
    }
  }
}

// allc holds max(nchunk * NB, 512) candidates (all rows of a single chunk); the scratch
// behind it serves lg_gepp, then L11^-1 and U11^-1 (2 NB^2 entries) in gradient mode
template <typename T>
inline size_t lg_tree_smem(int nchunk) {
  constexpr int NB = LgCfg<T>::NB;
  const int nc = nchunk * NB > kLgChunk ? nchunk * NB : kLgChunk;
  const size_t inv = 2 * (size_t)NB * NB * sizeof(T);
  const size_t scratch = lg_gepp_smem<T>() > inv ? lg_gepp_smem<T>() : inv;
  return (size_t)(kLgChunk + NB + nc + 4) * sizeof(int) + scratch;
}

// 3. interchanges on the columns [c_lo, n) of the whole rows, then the pivot-row snapshot
template <typename T>
__global__ void __launch_bounds__(256) lg_swap_kernel(LgArgs<T> A, int c_lo) {
  constexpr int NB = LgCfg<T>::NB;
  const int b = blockIdx.y, n = A.n, k0 = A.k0, kw = A.kw;
  const int c = c_lo + blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  T* Mb = A.M + (size_t)b * n * n;
  const int* ip = A.ipiv + (size_t)b * n;
  for (int j = 0; j < kw; ++j) {
    const int p = ip[k0 + j];
    if (p != k0 + j) {
      const T x = Mb[(size_t)(k0 + j) * n + c];
      Mb[(size_t)(k0 + j) * n + c] = Mb[(size_t)p * n + c];
      Mb[(size_t)p * n + c] = x;
    }
  }
  T* Pb = A.P + (size_t)b * NB * n;
  for (int j = 0; j < kw; ++j) Pb[(size_t)j * n + c] = Mb[(size_t)(k0 + j) * n + c];
}

// 4. coefficients of rows [r_lo, n) (one thread per row)
template <typename T, bool GRAD>
__global__ void __launch_bounds__(256) lg_coef_kernel(LgArgs<T> A, int r_lo) {
  constexpr int NB = LgCfg<T>::NB;
  __shared__ T sL[NB * NB], sU[NB * NB], sAi[GRAD ? NB * NB : 1];
  const int b = blockIdx.y, n = A.n, k0 = A.k0, kw = A.kw;
  const T* LU = A.LU11 + (size_t)b * 3 * NB * NB;
  for (int i = threadIdx.x; i < NB * NB; i += blockDim.x) {
    sL[i] = LU[i];
    sU[i] = LU[NB * NB + i];
    if (GRAD) sAi[i] = LU[2 * NB * NB + i];
  }
  __syncthreads();
  const int r = r_lo + blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  T* Mb = A.M + (size_t)b * n * n;
  T* row = Mb + (size_t)r * n + k0;
  T c[NB];
  if (r >= k0 && r < k0 + kw) {
    if (!GRAD) return;
    // pivot row j: the exchanged block gets row j of A_PK^-1, the coefficient e_j + it
    const int j = r - k0;
#pragma unroll
    for (int t = 0; t < NB; ++t) c[t] = t < kw ? sAi[j * NB + t] : s_zero<T>();
#pragma unroll
    for (int t = 0; t < NB; ++t)
      if (t < kw) row[t] = c[t];
#pragma unroll
    for (int t = 0; t < NB; ++t)
      if (t == j) c[t] = add(c[t], s_one<T>());
  } else if (GRAD && r < k0) {
    // a row above the panel (already exchanged): C = M_xK A_PK^-1, a plain product (these
    // rows never feed the pivots)
    T a[NB];
#pragma unroll
    for (int q = 0; q < NB; ++q) a[q] = q < kw ? row[q] : s_zero<T>();
#pragma unroll
    for (int t = 0; t < NB; ++t) {
      T acc = s_zero<T>();
#pragma unroll
      for (int q = 0; q < NB; ++q)
        if (q < kw) acc = fma_(a[q], sAi[q * NB + t], acc);
      c[t] = t < kw ? acc : s_zero<T>();
    }
#pragma unroll
    for (int t = 0; t < NB; ++t)
      if (t < kw) row[t] = c[t];
  } else {
    // l = M_xK U11^-1 (the elimination's FMA chains), then C L11 = l
    T l[NB];
#pragma unroll
    for (int t = 0; t < NB; ++t) {
      T acc = t < kw ? row[t] : s_zero<T>();
#pragma unroll
      for (int q = 0; q < NB; ++q)
        if (q < t) acc = fms(acc, l[q], sU[q * NB + t]);
      const T d = sU[t * NB + t];
      l[t] = (t < kw && !is_zero(d)) ? sdiv(acc, d) : s_zero<T>();
    }
#pragma unroll
    for (int t = NB - 1; t >= 0; --t) {
      T acc = l[t];
#pragma unroll
      for (int q = 0; q < NB; ++q)
        if (q > t && q < kw) acc = fms(acc, c[q], sL[q * NB + t]);
      c[t] = t < kw ? acc : s_zero<T>();
    }
    if (GRAD) {
#pragma unroll
      for (int t = 0; t < NB; ++t)
        if (t < kw) row[t] = c[t];
    }
  }
  T* cr = A.C + ((size_t)b * n + r) * NB;
#pragma unroll
  for (int t = 0; t < NB; ++t) cr[t] = c[t];
}

// 5. M[x][y] -= sum_s C[x][s] P[s][y] (s < kw) over rows [r_lo, n) x columns [c_lo, n)
// minus the panel columns [k0, k0 + kw); 64 x 64 tiles, 256 threads, 4 x 4 entries per
// thread, one FMA chain per entry in panel-column order. SKEW: only entries below the
// diagonal are computed, and M[y][x] = -M[x][y] is written beside them.
// Four 256-thread blocks per SM for the 4- and 8-byte types: more loads of M in flight (the
// kernel is bound by their latency).
template <typename T, bool SKEW = false>
__global__ void __launch_bounds__(256, sizeof(T) <= 8 ? 4 : 2) lg_update_kernel(LgArgs<T> A, int r_lo, int c_lo) {
  constexpr int NB = LgCfg<T>::NB;
  constexpr int TM = 64, TN = 64;
  __shared__ T sC[TM][NB + 1];
  __shared__ T sP[NB][TN];
  const int b = blockIdx.z, n = A.n, k0 = A.k0, kw = A.kw;
  const int r0 = r_lo + blockIdx.y * TM, c0 = c_lo + blockIdx.x * TN;
  if (SKEW && c0 >= r0 + TM) return;  // tile entirely above the diagonal
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  T* Mb = A.M + (size_t)b * n * n;
  const T* Cb = A.C + (size_t)b * n * NB;
  const T* Pb = A.P + (size_t)b * NB * n;
  for (int i = tid; i < TM * NB; i += 256) {
    const int rr = i / NB, s = i % NB, r = r0 + rr;
    sC[rr][s] = (r < n && s < kw) ? Cb[(size_t)r * NB + s] : s_zero<T>();
  }
  for (int i = tid; i < NB * TN; i += 256) {
    const int s = i / TN, cc = i % TN, c = c0 + cc;
    sP[s][cc] = (c < n && s < kw) ? Pb[(size_t)s * n + c] : s_zero<T>();
  }
  __syncthreads();
  int rr[4], cc[4];
  bool rv[4], cv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    rr[i] = r0 + ty + 16 * i;
    rv[i] = rr[i] < n;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    cc[j] = c0 + tx + 16 * j;
    cv[j] = cc[j] < n && (cc[j] < k0 || cc[j] >= k0 + kw);
  }
  T acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      acc[i][j] = (rv[i] && cv[j] && (!SKEW || rr[i] > cc[j])) ? Mb[(size_t)rr[i] * n + cc[j]] : s_zero<T>();
  for (int s = 0; s < kw; ++s) {
    T a[4], p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = sC[ty + 16 * i][s];
#pragma unroll
    for (int j = 0; j < 4; ++j) p[j] = sP[s][tx + 16 * j];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = fms(acc[i][j], a[i], p[j]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (rv[i] && cv[j] && (!SKEW || rr[i] > cc[j])) {
        Mb[(size_t)rr[i] * n + cc[j]] = acc[i][j];
        if (SKEW) Mb[(size_t)cc[j] * n + rr[i]] = neg(acc[i][j]);
      }
}

// 6. (sign, logabs) from the pivots and interchanges; gradient mode also the row
// permutation for the output (one warp per matrix)
template <typename T>
__global__ void __launch_bounds__(32) lg_finish_kernel(LgArgs<T> A, Job<T> J, int64_t b0, int grad) {
  typedef typename Sc<T>::R R;
  const int b = blockIdx.x, n = A.n, lane = threadIdx.x;
  const T* pv = A.piv + (size_t)b * n;
  const int* ip = A.ipiv + (size_t)b * n;
  if (lane == 0) {
    T sgn = s_one<T>();
    KSum<R> ls;
    ls.init();
    int par = 0, nz = 0;
    for (int k = 0; k < n; ++k) {
      const T d = pv[k];
      par ^= ip[k] != k;
      sgn = mul(sgn, unit(d));
      ls.add(rlog(mag(d)));
      nz += is_zero(d);
    }
    if (par) sgn = neg(sgn);
    if (nz) sgn = s_zero<T>();
    if constexpr (Sc<T>::cx) {
      R m = rhypot(sgn.re, sgn.im);
      if (m != R(0)) sgn = {rdiv(sgn.re, m), rdiv(sgn.im, m)};
    }
    const R la = nz ? -INFINITY : ls.value();
    if (A.primal) {
      J.sign[b0 + b] = sgn;
      J.logabs[b0 + b] = la;
      if (J.value) J.value[b0 + b] = scale(sgn, rexp(la));
    }
    A.flag[b] = (nz ? 1 : 0) | ((A.zsign && is_zero(A.zsign[b0 + b])) ? 4 : 0);
    if (grad) {
      int* pm = A.perm + (size_t)b * n;
      for (int k = 0; k < n; ++k) pm[k] = k;
      for (int k = 0; k < n; ++k) {
        const int p = ip[k];
        const int x = pm[k];
        pm[k] = pm[p];
        pm[p] = x;
      }
    }
  }
}

// 7. non-finite entries of the inverse (gradient mode): flag the matrix
template <typename T>
__global__ void __launch_bounds__(256) lg_check_kernel(LgArgs<T> A) {
  const int b = blockIdx.y, n = A.n;
  const size_t nn = (size_t)n * n;
  const T* Mb = A.M + (size_t)b * nn;
  bool bad = false;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nn; i += (size_t)gridDim.x * blockDim.x)
    bad |= !is_finite(Mb[i]);
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(A.flag + b, 2);
}

// 8. grad[perm[k]][j] = f * M[j][k] (f = coef, conjugated on request; zero when flagged),
// through a 32 x 32 shared-memory transpose
template <typename T>
__global__ void __launch_bounds__(256) lg_grad_kernel(LgArgs<T> A, Job<T> J, int64_t b0) {
  __shared__ T tile[32][33];
  const int b = blockIdx.z, n = A.n;
  const int j0 = blockIdx.y * 32, k0 = blockIdx.x * 32;
  const T* Mb = A.M + (size_t)b * n * n;
  const int* pm = A.perm + (size_t)b * n;
  const bool zero = A.flag[b] != 0;
  const T f = J.coef ? J.coef[b0 + b] : s_one<T>();
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int jj = ty; jj < 32; jj += 8) {
    const int j = j0 + jj, k = k0 + tx;
    tile[jj][tx] = (j < n && k < n) ? Mb[(size_t)j * n + k] : s_zero<T>();
  }
  __syncthreads();
  const size_t gb = (size_t)(b0 + b) * n * n;
  for (int kk = ty; kk < 32; kk += 8) {
    const int k = k0 + kk, j = j0 + tx;
    if (k < n && j < n) {
      T v = zero ? s_zero<T>() : scale(mul(f, tile[tx][kk]), A.gscale);
      v = maybe_conj(J, v);
      const size_t o = gb + (size_t)pm[k] * n + j;
      if constexpr (Sc<T>::cx) {
        if (J.g_re) {  // split planes
          J.g_re[o] = v.re;
          J.g_im[o] = v.im;
          continue;
        }
      }
      J.g[o] = v;
    }
  }
}

}  // namespace fx
