// Blocked Parlett-Reid engine for the slogpf forward at 256 < n <= 8192, every dtype: a
// host-driven loop over panels of NP pairs, each panel three batched kernels, the
// matrices in the caller's workspace (skew-symmetrised copies).
//
// Reference behaviour: the pair steps and pivoting of src/fermix/_fallback.py:266-300
// (pivot = largest abs1 entry of column a among the unassigned rows, first occurrence;
// d = -S[p, a]), blocked as in src/fermix/_pf.py:516-570; sign = prod unit(d) times
// (-1)^interchanges, logabs = sum log|d| (src/fermix/_pf.py:497-502).
//
// Per panel (positions k0 .. k0 + 2 np):
//   1. pfl_panel_kernel: one block per matrix, thread x owns the row at position k0 + x.
//      Pair step s reads the corrected columns a and p of the current matrix (the stored
//      column plus this panel's earlier pair corrections, the same FMA chains as the
//      register-panel kernel) with virtual pivoting; the trailing block is kept exactly skew
//      (mirrored updates, symmetric interchanges), so column a is read as minus row a, one
//      coalesced row instead of a strided column, and keeps each row's pair factors
//      (w_t, tau_t) in shared memory; at the end the factors go out by final position as
//      the update operands C = (-tau_t, w_t) and P = (w_t; tau_t);
//   2. pfl_swap_rows_kernel / pfl_swap_cols_kernel: the panel's symmetric interchanges
//      on the trailing rows and columns;
//   3. lg_update_kernel<SKEW = true>: S -= C P on the lower triangle of the trailing block,
//      mirrored (the update S += tau w^T - w tau^T keeps S exactly skew).
#pragma once
#include "large_lu.cuh"
#include "umma.cuh"

namespace fx {

constexpr int kPflRows = 1024;  // rows per panel block (one thread each): n <= 1024

template <typename T>
struct PflCfg {
  static constexpr int NP = sizeof(T) <= 8 ? 8 : 4;         // pairs per panel, 1024-row blocks
  static constexpr int NP_SMALL = LgCfg<T>::NB / 2;         // pairs per panel, n <= 512 (512-row blocks)
};

template <typename T>
struct PflArgs {
  T* M;        // bs x n x n skew matrices (row-major)
  T* C;        // bs x n x LgCfg<T>::NB update coefficients (by position; 2 NP used)
  T* P;        // bs x LgCfg<T>::NB x n update rows (by position; 2 NP used)
  T* dvec;     // bs x n/2 pair pivots
  int* ipiv;   // bs x n: position c1 = k0 + 2 s + 1 interchanged with ipiv[c1]
  int n, k0, np;
};

// 1. panel: block b factors pairs k0 / 2 .. k0 / 2 + np - 1 of matrix b (ROWS threads,
// n - k0 <= ROWS; NP pairs at most)
template <typename T, int NP, int ROWS>
__global__ void __launch_bounds__(ROWS) pfl_panel_kernel(PflArgs<T> A) {
  typedef typename Sc<T>::R R;
  constexpr int WL = 2 * NP + 1;
  constexpr int NW = ROWS / 32;
  extern __shared__ __align__(16) unsigned char smem[];
  T* W = reinterpret_cast<T*>(smem);                      // [m][WL] pair factors by row offset
  int* at = reinterpret_cast<int*>(W + (size_t)ROWS * WL);  // [m] position offset -> row offset
  int* pof = at + ROWS;                                   // [m] row offset -> position offset
  R* skey = reinterpret_cast<R*>(pof + ROWS);                 // [NW] best |colA| per warp
  int* srow = reinterpret_cast<int*>(skey + NW);              // [NW] its row offset
  int* sfir = srow + NW;                                      // [NW] first unassigned row offset
  T* sval = reinterpret_cast<T*>(sfir + NW + (NW % 4));       // [2][NW] colA of the best / first
  const int b = blockIdx.x, n = A.n, k0 = A.k0, np = A.np;
  const int m = n - k0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int x = tid;
  const bool have = x < m;
  T* Mb = A.M + (size_t)b * n * n;
  if (have) {
    at[x] = x;
    pof[x] = x;
  }
  bool unas = have;
  __syncthreads();
  for (int s = 0; s < np; ++s) {
    const int c = 2 * s;  // position offset of the pair
    const int a = at[c];
    if (x == a) unas = false;
    // column a of the current matrix at this row, with the panel's earlier corrections
    T colA = s_zero<T>();
    if (have) {
      colA = neg(Mb[(size_t)(k0 + a) * n + k0 + x]);  // S[x][a] = -S[a][x]: row a, coalesced
      for (int t = 0; t < s; ++t) {
        colA = fma_(W[x * WL + 2 * t + 1], W[a * WL + 2 * t], colA);
        colA = fms(colA, W[x * WL + 2 * t], W[a * WL + 2 * t + 1]);
      }
    }
    // pivot: largest abs1 over the unassigned rows (first occurrence); none comparable
    // (NaN) -> the first unassigned row
    R best = unas ? abs1(colA) : R(-1);
    if (!(best >= R(0))) best = R(-1);
    int bi = (unas && best >= R(0)) ? x : 0x7fffffff;
    T bv = colA;
    int fi = unas ? x : 0x7fffffff;
    T fv = colA;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const R ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      const T ov = shfl_idx(bv, lane ^ off);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
        bv = ov;
      }
      const int of = __shfl_xor_sync(0xffffffffu, fi, off);
      const T ofv = shfl_idx(fv, lane ^ off);
      if (of < fi) {
        fi = of;
        fv = ofv;
      }
    }
    if (lane == 0) {
      skey[warp] = best;
      srow[warp] = bi;
      sfir[warp] = fi;
      sval[warp] = bv;
      sval[NW + warp] = fv;
    }
    __syncthreads();
    R pb = skey[0];
    int p = srow[0];
    T pv = sval[0];
    int pfi = sfir[0];
    T pfv = sval[NW];
    for (int w = 1; w < NW; ++w) {
      const R ob = skey[w];
      const int oi = srow[w];
      if (ob > pb || (ob == pb && oi < p)) {
        pb = ob;
        p = oi;
        pv = sval[w];
      }
      if (sfir[w] < pfi) {
        pfi = sfir[w];
        pfv = sval[NW + w];
      }
    }
    if (p == 0x7fffffff) {
      p = pfi;
      pv = pfv;
    }
    const T d = neg(pv);
    const T inv = recip(d);
    if (x == p) unas = false;
    if (have) {
      T colP = neg(Mb[(size_t)(k0 + p) * n + k0 + x]);
      for (int t = 0; t < s; ++t) {
        colP = fma_(W[x * WL + 2 * t + 1], W[p * WL + 2 * t], colP);
        colP = fms(colP, W[x * WL + 2 * t], W[p * WL + 2 * t + 1]);
      }
      W[x * WL + 2 * s] = unas ? colP : s_zero<T>();
      W[x * WL + 2 * s + 1] = unas ? neg(mul(colA, inv)) : s_zero<T>();
    }
    if (tid == 0) {
      const int q = pof[p];
      A.ipiv[(size_t)b * n + k0 + c + 1] = k0 + q;
      A.dvec[(size_t)b * (n / 2) + (k0 + c) / 2] = d;
      if (q != c + 1) {
        const int y = at[c + 1];
        at[c + 1] = p;
        at[q] = y;
        pof[p] = c + 1;
        pof[y] = q;
      }
    }
    __syncthreads();
  }
  // operands by final position: C[pos] = (-tau_t, w_t), P[.][pos] = (w_t; tau_t), in the
  // update kernel's layout (row stride / rows per matrix LgCfg<T>::NB >= 2 NP)
  if (have) {
    constexpr int LD = LgCfg<T>::NB;
    const int pos = k0 + pof[x];
    T* cr = A.C + ((size_t)b * n + pos) * LD;
    T* pb = A.P + (size_t)b * LD * n;
#pragma unroll
    for (int t = 0; t < NP; ++t) {
      const T w = t < np ? W[x * WL + 2 * t] : s_zero<T>();
      const T tau = t < np ? W[x * WL + 2 * t + 1] : s_zero<T>();
      cr[2 * t] = neg(tau);
      cr[2 * t + 1] = w;
      pb[(size_t)(2 * t) * n + pos] = w;
      pb[(size_t)(2 * t + 1) * n + pos] = tau;
    }
  }
}

template <typename T, int NP, int ROWS>
inline size_t pfl_panel_smem() {
  typedef typename Sc<T>::R R;
  constexpr int NW = ROWS / 32;
  return (size_t)ROWS * (2 * NP + 1) * sizeof(T) + 2 * ROWS * sizeof(int) + NW * sizeof(R) + (3 * NW) * sizeof(int) +
         2 * NW * sizeof(T) + 64;
}

// ---------------------------------------------------------------- cluster panel
// 1024 < n - k0 <= 8192: the panel's rows split over a cluster of CL <= 8 blocks (1024
// rows each; 8 is the portable cluster size). Every block keeps its rows' pair factors and a full copy of the position
// bookkeeping; the pivot search combines the blocks' candidates through distributed
// shared memory, and the pivot rows' factors are read from the block that owns them. Two
// cluster barriers per pair step, executed by every thread of every block.
constexpr int kPflMaxN = 8 * kPflRows;

__device__ __forceinline__ uint32_t cl_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cl_sync() {
  asm volatile("barrier.cluster.arrive.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}
// shared::cluster address of this block's shared variable p as seen in block `rank`
__device__ __forceinline__ uint32_t cl_map(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(umma::smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ float cl_ld(uint32_t a, float*) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ double cl_ld(uint32_t a, double*) {
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ int cl_ld(uint32_t a, int*) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
template <typename R>
__device__ __forceinline__ cplx<R> cl_ld(uint32_t a, cplx<R>*) {
  return {cl_ld(a, (R*)nullptr), cl_ld(a + (uint32_t)sizeof(R), (R*)nullptr)};
}
template <typename V>
__device__ __forceinline__ V cl_get(const V* p, uint32_t rank) {
  return cl_ld(cl_map(p, rank), (V*)nullptr);
}

template <typename T>
struct PflClSlot {
  typename Sc<T>::R key[2];
  int row[2], fi[2];
  T val[2], fval[2];
};

// Column x of the pivot row's pair corrections: col += tau_x w_r - w_x tau_r over this panel's
// earlier pairs t < s, the pivot row's factors (w_r, tau_r) read from block `rank`. BATCH (the
// 512-row blocks, 128 registers a thread): four pairs' remote reads are issued before the
// first is used; otherwise one pair's two reads at a time (the 1024-row blocks' 64 registers).
template <typename T, int NP, bool BATCH>
__device__ __forceinline__ T pfl_cl_correct(T col, const T* Wr, uint32_t rank, int s, const T* Wme, bool have) {
  if constexpr (BATCH) {
    // groups of four pairs: eight remote reads in flight, then their FMAs
    const uint32_t base = cl_map(Wr, rank);
#pragma unroll
    for (int t0 = 0; t0 < NP; t0 += 4) {
      if (t0 < s) {
        T w[4], tau[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (t0 + j < s) {
            w[j] = cl_ld(base + (uint32_t)(2 * (t0 + j) * sizeof(T)), (T*)nullptr);
            tau[j] = cl_ld(base + (uint32_t)((2 * (t0 + j) + 1) * sizeof(T)), (T*)nullptr);
          }
        }
        if (have) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (t0 + j < s) {
              col = fma_(Wme[2 * (t0 + j) + 1], w[j], col);
              col = fms(col, Wme[2 * (t0 + j)], tau[j]);
            }
          }
        }
      }
    }
  } else {
    for (int t = 0; t < s; ++t) {
      const T w = cl_get(Wr + 2 * t, rank), tau = cl_get(Wr + 2 * t + 1, rank);
      if (have) {
        col = fma_(Wme[2 * t + 1], w, col);
        col = fms(col, Wme[2 * t], tau);
      }
    }
  }
  return col;
}

// ROWS rows per block (512 or 1024), NP pairs per panel, CL * ROWS >= n - k0.
template <typename T, int CL, int ROWS, int NP>
__global__ void __launch_bounds__(ROWS) pfl_panel_cl_kernel(PflArgs<T> A) {
  typedef typename Sc<T>::R R;
  constexpr int WL = 2 * NP + 1;
  constexpr int NW = ROWS / 32;
  static_assert(NW <= 32, "one warp merges the block's warp candidates");
  extern __shared__ __align__(16) unsigned char smem[];
  T* W = reinterpret_cast<T*>(smem);                               // [ROWS][WL] this block's rows
  PflClSlot<T>* cs = reinterpret_cast<PflClSlot<T>*>(W + (size_t)ROWS * WL);  // block candidate
  T* wval = reinterpret_cast<T*>(cs + 1);                          // [2][NW] warp candidates' values
  R* wkey = reinterpret_cast<R*>(wval + 2 * NW);                   // [NW]
  int* wrow = reinterpret_cast<int*>(wkey + NW);                   // [NW]
  int* wfi = wrow + NW;                                            // [NW]
  int* at = wfi + NW;                                              // [m] position offset -> row offset
  int* pof = at + kPflMaxN;                                        // [m] row offset -> position offset
  const uint32_t rank = cl_rank();
  const int b = blockIdx.x / CL, n = A.n, k0 = A.k0, np = A.np;
  const int m = n - k0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int xr = (int)rank * ROWS + tid;  // this thread's row offset
  const bool have = xr < m;
  T* Mb = A.M + (size_t)b * n * n;
  for (int i = tid; i < m; i += ROWS) {
    at[i] = i;
    pof[i] = i;
  }
  bool unas = have;
  cl_sync();
  for (int s = 0; s < np; ++s) {
    const int par = s & 1;
    const int c = 2 * s;
    const int a = at[c];
    if (xr == a) unas = false;
    T colA = s_zero<T>();
    if (have) colA = neg(Mb[(size_t)(k0 + a) * n + k0 + xr]);  // S[x][a] = -S[a][x]: row a, coalesced
    colA = pfl_cl_correct<T, NP, (ROWS <= 512)>(colA, W + (a % ROWS) * WL, (uint32_t)(a / ROWS), s, W + tid * WL, have);
    R best = unas ? abs1(colA) : R(-1);
    if (!(best >= R(0))) best = R(-1);
    int bi = (unas && best >= R(0)) ? xr : 0x7fffffff;
    T bv = colA;
    int fi = unas ? xr : 0x7fffffff;
    T fv = colA;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const R ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      const T ov = shfl_idx(bv, lane ^ off);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
        bv = ov;
      }
      const int of = __shfl_xor_sync(0xffffffffu, fi, off);
      const T ofv = shfl_idx(fv, lane ^ off);
      if (of < fi) {
        fi = of;
        fv = ofv;
      }
    }
    if (lane == 0) {
      wkey[warp] = best;
      wrow[warp] = bi;
      wfi[warp] = fi;
      wval[warp] = bv;
      wval[NW + warp] = fv;
    }
    __syncthreads();
    if (warp == 0) {
      // this block's candidate: lane w takes warp w's (lanes past the block's warps hold none)
      const bool in = lane < NW;
      best = in ? wkey[lane] : R(-1);
      bi = in ? wrow[lane] : 0x7fffffff;
      bv = in ? wval[lane] : s_zero<T>();
      fi = in ? wfi[lane] : 0x7fffffff;
      fv = in ? wval[NW + lane] : s_zero<T>();
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const R ob = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        const T ov = shfl_idx(bv, lane ^ off);
        if (ob > best || (ob == best && oi < bi)) {
          best = ob;
          bi = oi;
          bv = ov;
        }
        const int of = __shfl_xor_sync(0xffffffffu, fi, off);
        const T ofv = shfl_idx(fv, lane ^ off);
        if (of < fi) {
          fi = of;
          fv = ofv;
        }
      }
      if (lane == 0) {
        cs->key[par] = best;
        cs->row[par] = bi;
        cs->val[par] = bv;
        cs->fi[par] = fi;
        cs->fval[par] = fv;
      }
    }
    cl_sync();
    // the cluster's pivot: the blocks' candidates in block order
    R pb = R(-1);
    int p = 0x7fffffff, pfi = 0x7fffffff;
    T pv = s_zero<T>(), pfv = s_zero<T>();
#pragma unroll
    for (int r = 0; r < CL; ++r) {
      const R ob = cl_get(&cs->key[par], (uint32_t)r);
      const int oi = cl_get(&cs->row[par], (uint32_t)r);
      if (ob > pb || (ob == pb && oi < p)) {
        pb = ob;
        p = oi;
        pv = cl_get(&cs->val[par], (uint32_t)r);
      }
      const int of = cl_get(&cs->fi[par], (uint32_t)r);
      if (of < pfi) {
        pfi = of;
        pfv = cl_get(&cs->fval[par], (uint32_t)r);
      }
    }
    if (p == 0x7fffffff) {
      p = pfi;
      pv = pfv;
    }
    const T d = neg(pv);
    const T inv = recip(d);
    if (xr == p) unas = false;
    T colP = s_zero<T>();
    if (have) colP = neg(Mb[(size_t)(k0 + p) * n + k0 + xr]);
    colP = pfl_cl_correct<T, NP, (ROWS <= 512)>(colP, W + (p % ROWS) * WL, (uint32_t)(p / ROWS), s, W + tid * WL, have);
    if (have) {
      W[tid * WL + 2 * s] = unas ? colP : s_zero<T>();
      W[tid * WL + 2 * s + 1] = unas ? neg(mul(colA, inv)) : s_zero<T>();
    }
    if (tid == 0) {
      const int q = pof[p];
      if (rank == 0) {
        A.ipiv[(size_t)b * n + k0 + c + 1] = k0 + q;
        A.dvec[(size_t)b * (n / 2) + (k0 + c) / 2] = d;
      }
      if (q != c + 1) {
        const int y = at[c + 1];
        at[c + 1] = p;
        at[q] = y;
        pof[p] = c + 1;
        pof[y] = q;
      }
    }
    cl_sync();
  }
  if (have) {
    constexpr int LD = LgCfg<T>::NB;
    static_assert(2 * NP <= LD, "the update operands hold 2 NP columns");
    const int pos = k0 + pof[xr];
    T* cr = A.C + ((size_t)b * n + pos) * LD;
    T* pb = A.P + (size_t)b * LD * n;
#pragma unroll
    for (int t = 0; t < NP; ++t) {
      const T w = t < np ? W[tid * WL + 2 * t] : s_zero<T>();
      const T tau = t < np ? W[tid * WL + 2 * t + 1] : s_zero<T>();
      cr[2 * t] = neg(tau);
      cr[2 * t + 1] = w;
      pb[(size_t)(2 * t) * n + pos] = w;
      pb[(size_t)(2 * t + 1) * n + pos] = tau;
    }
  }
}

template <typename T, int ROWS, int NP>
inline size_t pfl_panel_cl_smem() {
  typedef typename Sc<T>::R R;
  constexpr int NW = ROWS / 32;
  return (size_t)ROWS * (2 * NP + 1) * sizeof(T) + sizeof(PflClSlot<T>) + 2 * NW * sizeof(T) + NW * sizeof(R) +
         2 * NW * sizeof(int) + 2 * kPflMaxN * sizeof(int) + 64;
}

// complex128 panels of 8 pairs (the update kernel's full K = 16) on 512-row cluster blocks,
// for n - k0 <= 8 * 512; wider trailing blocks keep 4 pairs on 1024-row blocks
template <typename T>
struct PflWide {
  static constexpr bool on = std::is_same<T, c128_t>::value;
  static constexpr int ROWS = 512, NP = LgCfg<T>::NB / 2, MAXM = 8 * ROWS;
};

// 2a. the panel's row interchanges on columns [k0, n)
template <typename T>
__global__ void __launch_bounds__(256) pfl_swap_rows_kernel(PflArgs<T> A) {
  const int b = blockIdx.y, n = A.n, k0 = A.k0;
  const int col = k0 + blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= n) return;
  T* Mb = A.M + (size_t)b * n * n;
  const int* ip = A.ipiv + (size_t)b * n;
  for (int s = 0; s < A.np; ++s) {
    const int c1 = k0 + 2 * s + 1, q = ip[c1];
    if (q != c1) {
      const T t = Mb[(size_t)c1 * n + col];
      Mb[(size_t)c1 * n + col] = Mb[(size_t)q * n + col];
      Mb[(size_t)q * n + col] = t;
    }
  }
}

// 2b. then the column interchanges on rows [k0, n)
template <typename T>
__global__ void __launch_bounds__(256) pfl_swap_cols_kernel(PflArgs<T> A) {
  const int b = blockIdx.y, n = A.n, k0 = A.k0;
  const int row = k0 + blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  T* r = A.M + (size_t)b * n * n + (size_t)row * n;
  const int* ip = A.ipiv + (size_t)b * n;
  for (int s = 0; s < A.np; ++s) {
    const int c1 = k0 + 2 * s + 1, q = ip[c1];
    if (q != c1) {
      const T t = r[c1];
      r[c1] = r[q];
      r[q] = t;
    }
  }
}

// 4. (sign, logabs, value) from the pair pivots and the interchanges (one warp per matrix)
template <typename T>
__global__ void __launch_bounds__(32) pfl_finish_kernel(PflArgs<T> A, Job<T> J, int64_t b0) {
  typedef typename Sc<T>::R R;
  const int b = blockIdx.x, n = A.n, h = n / 2, lane = threadIdx.x;
  const T* dv = A.dvec + (size_t)b * h;
  const int* ip = A.ipiv + (size_t)b * n;
  T sg = s_one<T>();
  KSum<R> ls;
  ls.init();
  int nz = 0, par = 0;
  for (int k = lane; k < h; k += 32) {
    const T d = dv[k];
    sg = mul(sg, unit(d));
    ls.add(rlog(mag(d)));
    nz += is_zero(d);
    par ^= ip[2 * k + 1] != 2 * k + 1;
  }
  R lsum = ls.value();
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const T o = shfl_idx(sg, lane ^ off);
    sg = mul(sg, o);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
    nz += __shfl_xor_sync(0xffffffffu, nz, off);
    par ^= __shfl_xor_sync(0xffffffffu, par, off);
  }
  if (lane == 0) {
    if (par) sg = neg(sg);
    if (nz) sg = s_zero<T>();
    if constexpr (Sc<T>::cx) {
      R mm = rhypot(sg.re, sg.im);
      if (mm != R(0)) sg = {rdiv(sg.re, mm), rdiv(sg.im, mm)};
    }
    const R la = nz ? R(-INFINITY) : lsum;
    J.sign[b0 + b] = sg;
    J.logabs[b0 + b] = la;
    if (J.value) J.value[b0 + b] = scale(sg, rexp(la));
  }
}

}  // namespace fx
