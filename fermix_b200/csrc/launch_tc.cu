// Tensor-memory (tcgen05) kernels: float32, slogpf n <= 128 and slogdet n <= 256 (prec tf32x3:
// tensor-core block updates; prec ieee: FMA block updates), forward and slogdet / slogpf
// gradient.
#include "dispatch.cuh"
#include "lu_tc.cuh"
#include "pf_tc.cuh"

namespace fxh {

// Tensor-memory slogpf (float32, 8 <= n <= 128, forward or slogpf gradient): one 128-thread
// block per matrix, the matrix resident in TMEM (128 of the SM's 512 columns); the block
// updates run on the tensor cores under tf32x3 and as IEEE FMAs under prec ieee. The
// shared-memory request is padded so that exactly four blocks share an SM (four blocks use
// all 512 TMEM columns; a fifth would wait in tcgen05.alloc).
constexpr size_t kTcSmem = 50 * 1024;
static_assert(sizeof(PfTcSmem) <= kTcSmem, "PfTcSmem too large");

int launch_pf_tc(cudaStream_t s, Job<float> J) {
  const DevInfo* D = dev_info();
  if (!D) return FX_ERR_DEVICE;
  const bool ieee = J.prec == FX_PREC_IEEE;
  void* k = J.mode == MODE_FWD ? (ieee ? (void*)&pf_tc_kernel<false, true> : (void*)&pf_tc_kernel<false, false>)
                               : (ieee ? (void*)&pf_tc_kernel<true, true> : (void*)&pf_tc_kernel<true, false>);
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem) != cudaSuccess)
    return FX_ERR_CUDA;
  if (cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
    return FX_ERR_CUDA;
  // four 128-thread blocks per SM: 4 x 51 KB shared memory, 4 x 128 TMEM columns
  const int64_t cap = (int64_t)D->sms * 4;
  const int64_t grid = J.B < cap ? J.B : cap;
  if (grid < 1) return FX_OK;
  void* args[] = {&J};
  if (cudaLaunchKernel(k, dim3((unsigned)grid), dim3(128), args, kTcSmem, s) != cudaSuccess) return FX_ERR_CUDA;
  return FX_OK;
}

// Tensor-core slogdet (float32, prec tf32x3, 8 <= n <= 256, forward or slogdet gradient):
// n <= 128 as the Pfaffian kernel above (four 128-thread blocks per SM); 129 <= n <= 256
// one 256-thread block per SM holding the whole matrix in the SM's 512 TMEM columns, its
// shared-memory request above half the SM so that no second block (a tcgen05.alloc
// waiter) is placed beside it.
constexpr size_t kLuTcSmem = 56 * 1024;  // four blocks per SM: 4 x (56 KB + 1 KB reserved) = 228 KB
static_assert(sizeof(LuTcSmemT<128>) <= kLuTcSmem, "LuTcSmem too large");
constexpr size_t kLuTc256Smem = 120 * 1024;
static_assert(sizeof(LuTcSmemT<256>) <= kLuTc256Smem, "LuTcSmemT<256> too large");

int launch_lu_tc(cudaStream_t s, Job<float> J) {
  const DevInfo* D = dev_info();
  if (!D) return FX_ERR_DEVICE;
  const bool big = J.n > kTcN, fwd = J.mode == MODE_FWD;
  void* k;
  if (J.prec == FX_PREC_IEEE)
    k = big ? (fwd ? (void*)&lu_tc_kernel<256, false, true> : (void*)&lu_tc_kernel<256, true, true>)
            : (fwd ? (void*)&lu_tc_kernel<128, false, true> : (void*)&lu_tc_kernel<128, true, true>);
  else
    k = big ? (fwd ? (void*)&lu_tc_kernel<256, false> : (void*)&lu_tc_kernel<256, true>)
            : (fwd ? (void*)&lu_tc_kernel<128, false> : (void*)&lu_tc_kernel<128, true>);
  const size_t smem = big ? kLuTc256Smem : kLuTcSmem;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FX_ERR_CUDA;
  if (cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
    return FX_ERR_CUDA;
  const int64_t cap = (int64_t)D->sms * (big ? 1 : 4);
  const int64_t grid = J.B < cap ? J.B : cap;
  if (grid < 1) return FX_OK;
  void* args[] = {&J};
  if (cudaLaunchKernel(k, dim3((unsigned)grid), dim3(big ? 256 : 128), args, smem, s) != cudaSuccess)
    return FX_ERR_CUDA;
  return FX_OK;
}

int tc_status(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, umma::fx_status_word, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(umma::fx_status_word, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

}  // namespace fxh

extern "C" {
#ifdef FX_PHASE_TIMERS
// profiling builds only: copy out / reset the per-phase cycle counters of the
// tensor-memory kernels (each translation unit has its own counter array)
int fermix_debug_phase_cycles(unsigned long long* out, int reset) {
  if (cudaMemcpyFromSymbol(out, fx::fx_phase_cycles, sizeof(unsigned long long) * 16) != cudaSuccess) return 1;
  if (reset) {
    unsigned long long z[16] = {0};
    if (cudaMemcpyToSymbol(fx::fx_phase_cycles, z, sizeof(z)) != cudaSuccess) return 1;
  }
  return 0;
}
#endif
}  // extern "C"
