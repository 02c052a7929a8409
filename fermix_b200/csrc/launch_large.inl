// Blocked engines for n > 256 (large_lu.cuh, large_pf.cuh): workspace layout, batch
// slices and the host-side panel loops. Included by launch_large_real.cu and
// launch_large_complex.cu, which instantiate it for their dtypes.
#pragma once
#include <type_traits>

#include "dispatch.cuh"
#include "large_pf.cuh"
#include "large_tc.cuh"

namespace fxh {

// ---------------------------------------------------------------- large-n LU engine
// n > kSmallMax, slogdet forward and gradient: the panel loop of large_lu.cuh over slices
// of the batch. Workspace per matrix: the matrix itself, the panel coefficients and
// pivot-row snapshot, L11 / U11, pivots and index arrays; each array 256-byte aligned.
// Matrices [b0, b0 + cnt) of the caller's input into the slice buffer M: a plain copy, or
// (a - a^T) / 2 when skew; from interleaved values or from split planes (Job::a_re).
template <typename T>
int lg_copy_in(cudaStream_t s, T* M, const Job<T>& J, int64_t b0, int cnt, int n, bool skew) {
  const SrcMat<T> src = src_of(J).offset((size_t)b0 * n * n);
  const size_t count = (size_t)cnt * n * n;
  if (skew) {
    lg_skew_copy_kernel<T><<<dim3((n + 31) / 32, (n + 31) / 32, cnt), 256, 0, s>>>(M, src, n);
  } else if (src.re) {
    const size_t blocks = (count + 255) / 256;
    lg_planar_copy_kernel<T><<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, s>>>(M, src, count);
  } else if (cudaMemcpyAsync(M, src.a, count * sizeof(T), cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
    return FX_ERR_CUDA;
  }
  return cudaGetLastError() == cudaSuccess ? FX_OK : FX_ERR_CUDA;
}

// The trailing update M -= C P over rows [lo, n) x columns [lo, n) (Gauss-Jordan: lo = 0)
// of cnt matrices: the tcgen05 3xTF32 kernel for float32 / complex64 under prec tf32x3
// (the default of those dtypes), the DMMA kernel for complex128, and the FMA-tiled kernel
// for float64 and for float32 / complex64 under prec ieee.
template <typename T, bool SKEW>
int lg_update(cudaStream_t s, const LgArgs<T>& A, int lo, int cnt, int prec) {
  const int n = A.n;
  if (lo >= n) return FX_OK;
  if constexpr (std::is_same<T, float>::value || std::is_same<T, c64_t>::value) {
    if (prec != FX_PREC_IEEE) {
      const size_t smem = lg_tc_smem<T>();
      void* k = (void*)&lg_tc_update_kernel<T, SKEW>;
      if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return FX_ERR_CUDA;
      LgArgs<T> arg = A;
      int r_lo = lo, c_lo = lo;
      void* args[] = {&arg, &r_lo, &c_lo};
      const dim3 grid((unsigned)((n - lo + 127) / 128), (unsigned)cnt);
      return cudaLaunchKernel(k, grid, dim3(128), args, smem, s) == cudaSuccess ? FX_OK : FX_ERR_CUDA;
    }
  }
  if constexpr (std::is_same<T, c128_t>::value) {
    // complex128: fp64 tensor cores (DMMA), IEEE fp64 FMA arithmetic. (float64 keeps the
    // DFMA tile kernel below: on B200 the fp64 tensor and vector peaks are equal, and that
    // kernel measured faster for the real LU update, 164 vs 134 matrices/s on C5a.)
    constexpr int TC = LgDm<T>::TC;
    const size_t smem = lg_dm_smem<T>();
    void* k = (void*)&lg_dmma_update_kernel<T, SKEW>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return FX_ERR_CUDA;
    LgArgs<T> arg = A;
    int r_lo = lo, c_lo = lo;
    void* args[] = {&arg, &r_lo, &c_lo};
    // one CTA per run of kLgDmTiles column tiles of a 128-row strip
    const int tiles = (n - lo + TC - 1) / TC;
    const dim3 grid((unsigned)((tiles + kLgDmTiles - 1) / kLgDmTiles), (unsigned)((n - lo + 127) / 128), (unsigned)cnt);
    return cudaLaunchKernel(k, grid, dim3(256), args, smem, s) == cudaSuccess ? FX_OK : FX_ERR_CUDA;
  }
  // the largest shared-memory carveout, so that four blocks' tiles fit beside each other
  if (cudaFuncSetAttribute(lg_update_kernel<T, SKEW>, cudaFuncAttributePreferredSharedMemoryCarveout, 100) !=
      cudaSuccess)
    return FX_ERR_CUDA;
  lg_update_kernel<T, SKEW><<<dim3((n - lo + 63) / 64, (n - lo + 63) / 64, cnt), 256, 0, s>>>(A, lo, lo);
  return cudaGetLastError() == cudaSuccess ? FX_OK : FX_ERR_CUDA;
}

constexpr int kLgSliceBlocks = 4;  // a slice holds at most SMs x 4 matrices

template <typename T>
struct LgLayout {
  size_t M, C, P, LU, piv, ipiv, cand, perm, flag, total;
  LgLayout(int64_t bs, int n) {
    constexpr int NB = LgCfg<T>::NB;
    const int nchunk = (n + kLgChunk - 1) / kLgChunk;
    size_t o = 0;
    M = o;    o = align256(o + (size_t)bs * n * n * sizeof(T));
    C = o;    o = align256(o + (size_t)bs * n * NB * sizeof(T));
    P = o;    o = align256(o + (size_t)bs * NB * n * sizeof(T));
    LU = o;   o = align256(o + (size_t)bs * 3 * NB * NB * sizeof(T));
    piv = o;  o = align256(o + (size_t)bs * n * sizeof(T));
    ipiv = o; o = align256(o + (size_t)bs * n * sizeof(int));
    cand = o; o = align256(o + (size_t)bs * nchunk * NB * sizeof(int));
    perm = o; o = align256(o + (size_t)bs * n * sizeof(int));
    flag = o; o = align256(o + (size_t)bs * sizeof(int));
    total = o;
  }
};

constexpr size_t kLgSliceBytes = (size_t)8 << 30;  // workspace aimed at per slice (8 GiB)

// Matrices per slice: enough to fill the GPU (SMs x 4), no more than the batch, and the
// workspace kept near kLgSliceBytes for large n (at least one matrix).
template <typename T>
int64_t lg_slice(int64_t batch, int n) {
  const DevInfo* D = dev_info();
  int64_t cap = (int64_t)(D ? D->sms : 148) * kLgSliceBlocks;
  const int64_t by_mem = (int64_t)(kLgSliceBytes / LgLayout<T>(1, n).total);
  if (by_mem < cap) cap = by_mem < 1 ? 1 : by_mem;
  return batch < cap ? batch : cap;
}

template <typename T>
size_t lg_ws_bytes(int64_t batch, int n) {
  return LgLayout<T>(lg_slice<T>(batch, n), n).total;
}

template <typename T>
int run_large_lu(cudaStream_t s, Job<T> J, void* ws, size_t wsb, bool grad, bool pf_grad) {
  constexpr int NB = LgCfg<T>::NB;
  const int n = J.n;
  if (!ws) return FX_ERR_WORKSPACE;
  int64_t bs = lg_slice<T>(J.B, n);
  while (bs > 1 && LgLayout<T>(bs, n).total > wsb) bs = bs / 2;
  const LgLayout<T> Lw(bs, n);
  if (Lw.total > wsb) return FX_ERR_WORKSPACE;
  unsigned char* w = static_cast<unsigned char*>(ws);
  LgArgs<T> A{};
  A.M = reinterpret_cast<T*>(w + Lw.M);
  A.C = reinterpret_cast<T*>(w + Lw.C);
  A.P = reinterpret_cast<T*>(w + Lw.P);
  A.LU11 = reinterpret_cast<T*>(w + Lw.LU);
  A.piv = reinterpret_cast<T*>(w + Lw.piv);
  A.ipiv = reinterpret_cast<int*>(w + Lw.ipiv);
  A.cand = reinterpret_cast<int*>(w + Lw.cand);
  A.perm = reinterpret_cast<int*>(w + Lw.perm);
  A.flag = reinterpret_cast<int*>(w + Lw.flag);
  A.n = n;
  A.grad = grad ? 1 : 0;
  A.primal = pf_grad ? 0 : 1;
  A.gscale = pf_grad ? typename Sc<T>::R(0.5) : typename Sc<T>::R(1);
  A.zsign = pf_grad ? J.sign : nullptr;
  A.wait_polls = J.wait_polls;
  const size_t leaf_smem = kLgChunk * sizeof(int) + lg_gepp_smem<T>();
  const size_t tree_smem = lg_tree_smem<T>((n + kLgChunk - 1) / kLgChunk);
  void* tree_k = (void*)&lg_tree_kernel<T>;
  if (tree_smem > 48 * 1024 &&
      cudaFuncSetAttribute(tree_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (dev_info() ? dev_info()->smem_optin : (int)tree_smem)) != cudaSuccess)
    return FX_ERR_CUDA;
  for (int64_t b0 = 0; b0 < J.B; b0 += bs) {
    const int cnt = (int)(J.B - b0 < bs ? J.B - b0 : bs);
    if (lg_copy_in<T>(s, A.M, J, b0, cnt, n, pf_grad && J.skew)) return FX_ERR_CUDA;
    for (int k0 = 0; k0 < n; k0 += NB) {
      A.k0 = k0;
      A.kw = n - k0 < NB ? n - k0 : NB;
      A.nchunk = (n - k0 + kLgChunk - 1) / kLgChunk;
      if (A.nchunk > 1) lg_leaf_kernel<T><<<dim3(A.nchunk, cnt), kLgChunk, leaf_smem, s>>>(A);
      lg_tree_kernel<T><<<cnt, kLgChunk, tree_smem, s>>>(A);
      const int c_lo = grad ? 0 : k0;
      lg_swap_kernel<T><<<dim3((n - c_lo + 255) / 256, cnt), 256, 0, s>>>(A, c_lo);
      const int r_lo = grad ? 0 : k0;
      if (grad) {
        lg_coef_kernel<T, true><<<dim3((n - r_lo + 255) / 256, cnt), 256, 0, s>>>(A, r_lo);
      } else {
        lg_coef_kernel<T, false><<<dim3((n - r_lo + 255) / 256, cnt), 256, 0, s>>>(A, r_lo);
      }
      const int u_lo = grad ? 0 : k0 + A.kw;
      if (int e = lg_update<T, false>(s, A, u_lo, cnt, J.prec)) return e;
    }
    lg_finish_kernel<T><<<cnt, 32, 0, s>>>(A, J, b0, grad ? 1 : 0);
    if (grad) {
      lg_check_kernel<T><<<dim3(16, cnt), 256, 0, s>>>(A);
      lg_grad_kernel<T><<<dim3((n + 31) / 32, (n + 31) / 32, cnt), 256, 0, s>>>(A, J, b0);
    }
    if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
  }
  return FX_OK;
}

// Cluster launch of the split panel: CL blocks of ROWS threads per matrix, NP pairs.
template <typename T, int CL, int ROWS, int NP>
int launch_pfl_cl(cudaStream_t s, const PflArgs<T>& A, int cnt) {
  const size_t smem = pfl_panel_cl_smem<T, ROWS, NP>();
  void* k = (void*)&pfl_panel_cl_kernel<T, CL, ROWS, NP>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FX_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(CL * cnt));
  cfg.blockDim = dim3(ROWS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CL;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  PflArgs<T> arg = A;
  void* args[] = {&arg};
  return cudaLaunchKernelExC(&cfg, k, args) == cudaSuccess ? FX_OK : FX_ERR_CUDA;
}

// Large-n Parlett-Reid forward (kSmallMax < n <= kPflMaxN, n even): the panel loop of
// large_pf.cuh over slices of the batch, on the large-LU workspace layout.
template <typename T>
int run_large_pf(cudaStream_t s, Job<T> J, void* ws, size_t wsb) {
  constexpr int NP = PflCfg<T>::NP;
  const int n = J.n;
  if (!ws) return FX_ERR_WORKSPACE;
  int64_t bs = lg_slice<T>(J.B, n);
  while (bs > 1 && LgLayout<T>(bs, n).total > wsb) bs = bs / 2;
  const LgLayout<T> Lw(bs, n);
  if (Lw.total > wsb) return FX_ERR_WORKSPACE;
  unsigned char* w = static_cast<unsigned char*>(ws);
  PflArgs<T> A{};
  A.M = reinterpret_cast<T*>(w + Lw.M);
  A.C = reinterpret_cast<T*>(w + Lw.C);
  A.P = reinterpret_cast<T*>(w + Lw.P);
  A.dvec = reinterpret_cast<T*>(w + Lw.piv);
  A.ipiv = reinterpret_cast<int*>(w + Lw.ipiv);
  A.n = n;
  LgArgs<T> U{};
  U.M = A.M;
  U.C = A.C;
  U.P = A.P;
  U.n = n;
  U.wait_polls = J.wait_polls;
  // n <= 512: 512-row panel blocks with twice the pairs (a wider, less memory-bound update);
  // complex128 also takes 8-pair panels on 512-row cluster blocks while n - k0 <= 4096
  const bool small = n <= 512;
  constexpr int NPS = PflCfg<T>::NP_SMALL;
  using Wd = PflWide<T>;
  const size_t psmem = small ? pfl_panel_smem<T, NPS, 512>() : pfl_panel_smem<T, NP, kPflRows>();
  void* pk = small ? (void*)&pfl_panel_kernel<T, NPS, 512> : (void*)&pfl_panel_kernel<T, NP, kPflRows>;
  if (cudaFuncSetAttribute(pk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem) != cudaSuccess)
    return FX_ERR_CUDA;
  if (Wd::on) {
    void* wk = (void*)&pfl_panel_kernel<T, NPS, 512>;
    if (cudaFuncSetAttribute(wk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pfl_panel_smem<T, NPS, 512>()) !=
        cudaSuccess)
      return FX_ERR_CUDA;
  }
  for (int64_t b0 = 0; b0 < J.B; b0 += bs) {
    const int cnt = (int)(J.B - b0 < bs ? J.B - b0 : bs);
    if (lg_copy_in<T>(s, A.M, J, b0, cnt, n, J.skew)) return FX_ERR_CUDA;
    for (int k0 = 0; k0 < n;) {
      const int m = n - k0;
      const bool wide = Wd::on && !small && m <= Wd::MAXM;
      const int np_max = small ? NPS : (wide ? Wd::NP : NP);
      A.k0 = k0;
      A.np = m / 2 < np_max ? m / 2 : np_max;
      if (small || (wide && m <= 512)) {
        pfl_panel_kernel<T, NPS, 512><<<cnt, 512, pfl_panel_smem<T, NPS, 512>(), s>>>(A);
      } else if (wide) {
        int e = FX_ERR_SHAPE;
        if constexpr (PflWide<T>::on) {
          switch ((m + Wd::ROWS - 1) / Wd::ROWS) {
            case 2: e = launch_pfl_cl<T, 2, Wd::ROWS, Wd::NP>(s, A, cnt); break;
            case 3: e = launch_pfl_cl<T, 3, Wd::ROWS, Wd::NP>(s, A, cnt); break;
            case 4: e = launch_pfl_cl<T, 4, Wd::ROWS, Wd::NP>(s, A, cnt); break;
            case 5: e = launch_pfl_cl<T, 5, Wd::ROWS, Wd::NP>(s, A, cnt); break;
            case 6: e = launch_pfl_cl<T, 6, Wd::ROWS, Wd::NP>(s, A, cnt); break;
            case 7: e = launch_pfl_cl<T, 7, Wd::ROWS, Wd::NP>(s, A, cnt); break;
            case 8: e = launch_pfl_cl<T, 8, Wd::ROWS, Wd::NP>(s, A, cnt); break;
          }
        }
        if (e) return e;
      } else if (m <= kPflRows) {
        pfl_panel_kernel<T, NP, kPflRows><<<cnt, kPflRows, psmem, s>>>(A);
      } else {
        int e = FX_ERR_SHAPE;
        switch ((m + kPflRows - 1) / kPflRows) {
          case 2: e = launch_pfl_cl<T, 2, kPflRows, NP>(s, A, cnt); break;
          case 3: e = launch_pfl_cl<T, 3, kPflRows, NP>(s, A, cnt); break;
          case 4: e = launch_pfl_cl<T, 4, kPflRows, NP>(s, A, cnt); break;
          case 5: e = launch_pfl_cl<T, 5, kPflRows, NP>(s, A, cnt); break;
          case 6: e = launch_pfl_cl<T, 6, kPflRows, NP>(s, A, cnt); break;
          case 7: e = launch_pfl_cl<T, 7, kPflRows, NP>(s, A, cnt); break;
          case 8: e = launch_pfl_cl<T, 8, kPflRows, NP>(s, A, cnt); break;
        }
        if (e) return e;
      }
      pfl_swap_rows_kernel<T><<<dim3((n - k0 + 255) / 256, cnt), 256, 0, s>>>(A);
      pfl_swap_cols_kernel<T><<<dim3((n - k0 + 255) / 256, cnt), 256, 0, s>>>(A);
      const int lo = k0 + 2 * A.np;
      if (lo < n) {
        U.k0 = k0;
        U.kw = 2 * A.np;
        if (int e = lg_update<T, true>(s, U, lo, cnt, J.prec)) return e;
      }
      k0 = lo;
    }
    pfl_finish_kernel<T><<<cnt, 32, 0, s>>>(A, J, b0);
    if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
  }
  return FX_OK;
}

}  // namespace fxh
