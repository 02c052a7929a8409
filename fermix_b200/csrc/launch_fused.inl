// Register-panel (small.cuh) and generic one-block-per-matrix (fused_lu.cuh,
// fused_pf.cuh) kernels: launch geometry and launch. Included by launch_fused_real.cu and
// launch_fused_complex.cu, which instantiate it for their dtypes.
#pragma once
#include "dispatch.cuh"
#include "small.cuh"

namespace fxh {

inline int threads_for(int n) { return n <= 24 ? 32 : (n <= 64 ? 128 : 256); }

inline int rows_per_lane(int n) { return n <= 32 ? 1 : (n <= 64 ? 2 : (n <= 128 ? 4 : 8)); }

template <typename T, bool PF>
void* small_kernel_ptr(int rs) {
  switch (rs) {
    case 1:
      return PF ? (void*)&pf_small_kernel<T, 1> : (void*)&lu_small_kernel<T, 1>;
    case 2:
      return PF ? (void*)&pf_small_kernel<T, 2> : (void*)&lu_small_kernel<T, 2>;
    case 4:
      return PF ? (void*)&pf_small_kernel<T, 4> : (void*)&lu_small_kernel<T, 4>;
    default:
      return PF ? (void*)&pf_small_kernel<T, 8> : (void*)&lu_small_kernel<T, 8>;
  }
}

// Buffers per matrix: pf uses one in-place buffer for forward and gradient; LU needs a
// second one for the inverse.
template <typename T, bool PF>
int plan_fused(int64_t batch, int n, int mode, Plan& P) {
  const DevInfo* D = dev_info();
  if (!D) return FX_ERR_DEVICE;
  const bool small = n <= kSmallMax;
  const int nbuf = (PF && small) ? 1 : (mode == MODE_FWD ? 1 : 2);
  P.threads = threads_for(n);
  const int ld_s = (n % 2 == 0) ? n + 1 : n;  // odd stride: conflict-free column access
  auto bytes = [&](int ld, bool in_smem) -> size_t {
    if (small) return PF ? Small<T>::bytes(n, ld, in_smem) : LuSmall<T>::bytes(n, ld, nbuf, in_smem);
    return SmemLayout<T>::bytes(n, ld, nbuf, in_smem);
  };
  const size_t full = bytes(ld_s, true);
  P.in_smem = full <= (size_t)D->smem_optin;
  P.ld = P.in_smem ? ld_s : n;
  P.smem = P.in_smem ? full : bytes(n, false);
  P.slot = P.in_smem ? 0 : (size_t)nbuf * n * n * sizeof(T);
  if (small)
    P.kernel = small_kernel_ptr<T, PF>(rows_per_lane(n));
  else
    P.kernel = PF ? (void*)&pf_fused_kernel<T> : (void*)&lu_fused_kernel<T>;
  // the device's opt-in limit, the same value on every call: one kernel serves a range of
  // n, and a per-call size could be lowered by a concurrent call between set and launch
  if (cudaFuncSetAttribute(P.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, D->smem_optin) != cudaSuccess)
    return FX_ERR_CUDA;
  // shared memory over L1: these kernels keep their matrices in shared memory
  if (cudaFuncSetAttribute(P.kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
    return FX_ERR_CUDA;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, P.kernel, P.threads, P.smem) != cudaSuccess)
    return FX_ERR_CUDA;
  if (occ < 1) occ = 1;
  P.grid = batch < (int64_t)D->sms * occ ? batch : (int64_t)D->sms * occ;
  return FX_OK;
}

template <typename T, bool PF>
int launch_fused(cudaStream_t s, Job<T> J, void* ws, size_t ws_bytes) {
  Plan P;
  int e = plan_fused<T, PF>(J.B, J.n, J.mode, P);
  if (e) return e;
  J.ld = P.ld;
  J.in_smem = P.in_smem;
  J.ws = nullptr;
  int64_t grid = P.grid;
  if (!P.in_smem) {
    if (!ws) return FX_ERR_WORKSPACE;
    int64_t slots = (int64_t)(ws_bytes / P.slot);
    if (slots < 1) return FX_ERR_WORKSPACE;
    if (grid > slots) grid = slots;
    J.ws = static_cast<T*>(ws);
  }
  if (grid < 1) return FX_OK;
  void* args[] = {&J};
  if (cudaLaunchKernel(P.kernel, dim3((unsigned)grid), dim3(P.threads), args, P.smem, s) != cudaSuccess)
    return FX_ERR_CUDA;
  return FX_OK;
}

}  // namespace fxh
