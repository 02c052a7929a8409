// extern "C" entry points of libfermix_b200.so (declared in include/fermix_b200.h).
//
// Dispatch (replacing the reference's per-GPU TUNES table, src/fermix/_common.py:17-378):
//   det n <= 4, pf n <= 6      -> the closed forms (poly.cuh), one thread per matrix
//   pf with odd n              -> (0, -inf), zero gradient
//   otherwise                  -> the fused one-block-per-matrix kernels (fused_lu.cuh,
//                                 fused_pf.cuh): work buffers in shared memory when
//                                 they fit (227 KB per block on B200), else in the
//                                 caller's workspace (one slot per resident block).
// The only process state is a once-initialised per-device attribute cache.
#include <cuda_runtime.h>

#include <mutex>
#include <type_traits>

#include "fermix_b200.h"
#include "fused_pf.cuh"
#include "poly.cuh"
#include "small.cuh"
#include "pf_tc.cuh"
#include "lu_tc.cuh"
#include "large_lu.cuh"
#include "large_pf.cuh"
#include "update.cuh"

namespace {

using namespace fx;

constexpr int kMaxDevices = 64;

struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
  int ok = 0;
};

DevInfo g_dev[kMaxDevices];
std::once_flag g_once[kMaxDevices];

const DevInfo* dev_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(g_once[dev], [dev]() {
    DevInfo d;
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess)
      d.ok = 1;
    g_dev[dev] = d;
  });
  return g_dev[dev].ok ? &g_dev[dev] : nullptr;
}

int validate(int dtype, int prec, int64_t batch, int64_t n) {
  if (dtype < FX_F32 || dtype > FX_C128) return FX_ERR_DTYPE;
  if (batch < 0 || n < 0 || n > 46000) return FX_ERR_SHAPE;
  return fermix_check_prec(dtype, prec);
}

int threads_for(int n) { return n <= 24 ? 32 : (n <= 64 ? 128 : 256); }

// Launch geometry of one fused call (shared by the launch and the workspace query).
struct Plan {
  int threads = 0, ld = 0, in_smem = 0;
  size_t smem = 0, slot = 0;
  int64_t grid = 0;
  void* kernel = nullptr;
};

constexpr int kSmallMax = 256;  // register-panel kernels: ceil(n / 32) <= 8 rows per lane

int rows_per_lane(int n) { return n <= 32 ? 1 : (n <= 64 ? 2 : (n <= 128 ? 4 : 8)); }

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
  if (cudaFuncSetAttribute(P.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P.smem) != cudaSuccess)
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

// Tensor-core slogpf (float32, prec tf32x3, 8 <= n <= 128, forward or slogpf gradient):
// one 128-thread block per matrix, the matrix resident in TMEM (128 of the SM's 512
// columns). The shared-memory request is padded so that exactly four blocks share an SM
// (four blocks use all 512 TMEM columns; a fifth would wait in tcgen05.alloc).
constexpr size_t kTcSmem = 50 * 1024;
static_assert(sizeof(PfTcSmem) <= kTcSmem, "PfTcSmem too large");

bool use_pf_tc(int dtype_is_f32, int prec, int n, int mode) {
  return dtype_is_f32 && prec != FX_PREC_IEEE && n >= 8 && n <= kTcN && (mode == MODE_FWD || mode == MODE_SLOG_GRAD);
}

int launch_pf_tc(cudaStream_t s, Job<float> J) {
  const DevInfo* D = dev_info();
  if (!D) return FX_ERR_DEVICE;
  void* k = J.mode == MODE_FWD ? (void*)&pf_tc_kernel<false> : (void*)&pf_tc_kernel<true>;
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

bool use_lu_tc(int dtype_is_f32, int prec, int n, int mode) {
  return dtype_is_f32 && prec != FX_PREC_IEEE && n >= 8 && n <= 2 * kTcN &&
         (mode == MODE_FWD || mode == MODE_SLOG_GRAD);
}

int launch_lu_tc(cudaStream_t s, Job<float> J) {
  const DevInfo* D = dev_info();
  if (!D) return FX_ERR_DEVICE;
  const bool big = J.n > kTcN;
  void* k = big ? (J.mode == MODE_FWD ? (void*)&lu_tc_kernel<256, false> : (void*)&lu_tc_kernel<256, true>)
                : (J.mode == MODE_FWD ? (void*)&lu_tc_kernel<128, false> : (void*)&lu_tc_kernel<128, true>);
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

template <typename T>
int launch_poly(cudaStream_t s, const Job<T>& J, int is_pf) {
  const int th = 128;
  const int64_t blocks = (J.B + th - 1) / th;
  poly_kernel<T><<<(unsigned)blocks, th, 0, s>>>(J, is_pf);
  return cudaGetLastError() == cudaSuccess ? FX_OK : FX_ERR_CUDA;
}

template <typename T>
Job<T> make_job(int64_t batch, int64_t n, const void* a, const void* coef, int conj_out, int skew, int mode,
                void* sign, void* logabs, void* value, void* grad) {
  Job<T> J{};
  J.a = static_cast<const T*>(a);
  J.sign = static_cast<T*>(sign);
  J.logabs = static_cast<typename Sc<T>::R*>(logabs);
  J.g = static_cast<T*>(grad);
  J.value = static_cast<T*>(value);
  J.coef = static_cast<const T*>(coef);
  J.conj_out = conj_out;
  J.skew = skew;
  J.B = batch;
  J.n = (int)n;
  J.mode = mode;
  return J;
}

// ---------------------------------------------------------------- large-n LU engine
// n > kSmallMax, slogdet forward and gradient: the panel loop of large_lu.cuh over slices
// of the batch. Workspace per matrix: the matrix itself, the panel coefficients and
// pivot-row snapshot, L11 / U11, pivots and index arrays; each array 256-byte aligned.
constexpr int kLgSliceBlocks = 4;  // a slice holds at most SMs x 4 matrices

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

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

// primal: write (sign, logabs, value); pf_grad: the input is skew-symmetrised when J.skew,
// the gradient is S^-T / 2 and zero where J.sign (the Pfaffian forward's) is zero.
template <typename T>
int run_large_lu(cudaStream_t s, Job<T> J, void* ws, size_t wsb, bool grad, bool pf_grad = false) {
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
  const size_t leaf_smem = kLgChunk * sizeof(int) + lg_gepp_smem<T>();
  const size_t tree_smem = lg_tree_smem<T>((n + kLgChunk - 1) / kLgChunk);
  void* tree_k = (void*)&lg_tree_kernel<T>;
  if (tree_smem > 48 * 1024 &&
      cudaFuncSetAttribute(tree_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tree_smem) != cudaSuccess)
    return FX_ERR_CUDA;
  for (int64_t b0 = 0; b0 < J.B; b0 += bs) {
    const int cnt = (int)(J.B - b0 < bs ? J.B - b0 : bs);
    if (pf_grad && J.skew) {
      lg_skew_copy_kernel<T><<<dim3((n + 31) / 32, (n + 31) / 32, cnt), 256, 0, s>>>(A.M, J.a + b0 * (int64_t)n * n, n);
    } else if (cudaMemcpyAsync(A.M, J.a + b0 * (int64_t)n * n, (size_t)cnt * n * n * sizeof(T),
                               cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
      return FX_ERR_CUDA;
    }
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
      if (u_lo < n) lg_update_kernel<T><<<dim3((n - u_lo + 63) / 64, (n - u_lo + 63) / 64, cnt), 256, 0, s>>>(A, u_lo, u_lo);
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

// Cluster launch of the split panel: CL blocks of 1024 threads per matrix.
template <typename T, int CL>
int launch_pfl_cl(cudaStream_t s, const PflArgs<T>& A, int cnt) {
  const size_t smem = pfl_panel_cl_smem<T>();
  void* k = (void*)&pfl_panel_cl_kernel<T, CL>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FX_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(CL * cnt));
  cfg.blockDim = dim3(kPflRows);
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
  // n <= 512: 512-row panel blocks with twice the pairs (a wider, less memory-bound update)
  const bool small = n <= 512;
  constexpr int NPS = PflCfg<T>::NP_SMALL;
  const int np_max = small ? NPS : NP;
  const size_t psmem = small ? pfl_panel_smem<T, NPS, 512>() : pfl_panel_smem<T, NP, kPflRows>();
  void* pk = small ? (void*)&pfl_panel_kernel<T, NPS, 512> : (void*)&pfl_panel_kernel<T, NP, kPflRows>;
  if (cudaFuncSetAttribute(pk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem) != cudaSuccess)
    return FX_ERR_CUDA;
  for (int64_t b0 = 0; b0 < J.B; b0 += bs) {
    const int cnt = (int)(J.B - b0 < bs ? J.B - b0 : bs);
    if (J.skew) {
      lg_skew_copy_kernel<T><<<dim3((n + 31) / 32, (n + 31) / 32, cnt), 256, 0, s>>>(A.M, J.a + b0 * (int64_t)n * n, n);
    } else if (cudaMemcpyAsync(A.M, J.a + b0 * (int64_t)n * n, (size_t)cnt * n * n * sizeof(T),
                               cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
      return FX_ERR_CUDA;
    }
    for (int k0 = 0; k0 < n; k0 += 2 * np_max) {
      A.k0 = k0;
      A.np = (n - k0) / 2 < np_max ? (n - k0) / 2 : np_max;
      const int m = n - k0;
      if (small) {
        pfl_panel_kernel<T, NPS, 512><<<cnt, 512, psmem, s>>>(A);
      } else if (m <= kPflRows) {
        pfl_panel_kernel<T, NP, kPflRows><<<cnt, kPflRows, psmem, s>>>(A);
      } else {
        int e = FX_ERR_SHAPE;
        switch ((m + kPflRows - 1) / kPflRows) {
          case 2: e = launch_pfl_cl<T, 2>(s, A, cnt); break;
          case 3: e = launch_pfl_cl<T, 3>(s, A, cnt); break;
          case 4: e = launch_pfl_cl<T, 4>(s, A, cnt); break;
          case 5: e = launch_pfl_cl<T, 5>(s, A, cnt); break;
          case 6: e = launch_pfl_cl<T, 6>(s, A, cnt); break;
          case 7: e = launch_pfl_cl<T, 7>(s, A, cnt); break;
          case 8: e = launch_pfl_cl<T, 8>(s, A, cnt); break;
        }
        if (e) return e;
      }
      pfl_swap_rows_kernel<T><<<dim3((n - k0 + 255) / 256, cnt), 256, 0, s>>>(A);
      pfl_swap_cols_kernel<T><<<dim3((n - k0 + 255) / 256, cnt), 256, 0, s>>>(A);
      const int lo = k0 + 2 * A.np;
      if (lo < n) {
        U.k0 = k0;
        U.kw = 2 * A.np;
        lg_update_kernel<T, true><<<dim3((n - lo + 63) / 64, (n - lo + 63) / 64, cnt), 256, 0, s>>>(U, lo, lo);
      }
    }
    pfl_finish_kernel<T><<<cnt, 32, 0, s>>>(A, J, b0);
    if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
  }
  return FX_OK;
}

template <typename T>
int run_det(cudaStream_t s, int prec, int64_t batch, int64_t n, const void* a, const void* coef, int conj_out,
            int mode, void* sign, void* logabs, void* value, void* grad, void* ws, size_t wsb) {
  Job<T> J = make_job<T>(batch, n, a, coef, conj_out, 0, mode, sign, logabs, value, grad);
  if (n <= DET_POLY_MAX) return launch_poly<T>(s, J, 0);
  if constexpr (std::is_same<T, float>::value) {
    if (use_lu_tc(1, prec, (int)n, mode)) return launch_lu_tc(s, J);
    if (mode == MODE_VALUE_GRAD && use_lu_tc(1, prec, (int)n, MODE_FWD)) {
      // the adjugate comes from the register-panel kernel; (sign, logabs, value) are
      // rewritten by the tensor-core forward (same stream) to equal fermix_slogdet's bits
      int e = launch_fused<T, false>(s, J, ws, wsb);
      if (e) return e;
      Job<T> F = J;
      F.mode = MODE_FWD;
      F.g = nullptr;
      return launch_lu_tc(s, F);
    }
  }
  if (n > kSmallMax) {
    if (mode == MODE_FWD || mode == MODE_SLOG_GRAD) return run_large_lu<T>(s, J, ws, wsb, mode == MODE_SLOG_GRAD);
    // the det adjugate comes from the generic kernel; (sign, logabs, value) are rewritten
    // by the large-n forward (same stream, same workspace) to equal fermix_slogdet's bits
    int e = launch_fused<T, false>(s, J, ws, wsb);
    if (e) return e;
    Job<T> F = J;
    F.mode = MODE_FWD;
    F.g = nullptr;
    return run_large_lu<T>(s, F, ws, wsb, false);
  }
  return launch_fused<T, false>(s, J, ws, wsb);
}

template <typename T>
int run_pf(cudaStream_t s, int prec, int64_t batch, int64_t n, int skew, const void* a, const void* coef, int conj_out,
           int mode, void* sign, void* logabs, void* value, void* grad, void* ws, size_t wsb) {
  Job<T> J = make_job<T>(batch, n, a, coef, conj_out, skew, mode, sign, logabs, value, grad);
  if (n % 2 == 1) {
    if (grad && batch * n * n > 0 &&
        cudaMemsetAsync(grad, 0, (size_t)batch * n * n * sizeof(T), s) != cudaSuccess)
      return FX_ERR_CUDA;
    const int th = 128;
    pf_odd_kernel<T><<<(unsigned)((batch + th - 1) / th), th, 0, s>>>(J);
    return cudaGetLastError() == cudaSuccess ? FX_OK : FX_ERR_CUDA;
  }
  if (n <= PF_POLY_MAX) return launch_poly<T>(s, J, 1);
  if constexpr (std::is_same<T, float>::value) {
    if (use_pf_tc(1, prec, (int)n, mode)) return launch_pf_tc(s, J);
    if (mode == MODE_VALUE_GRAD && use_pf_tc(1, prec, (int)n, MODE_FWD)) {
      // the Pfaffian adjugate comes from the register-panel kernel; the primal it returns
      // must be the forward's own bits, so the tensor-core forward rewrites
      // (sign, logabs, value) after it (same stream)
      int e = launch_fused<T, true>(s, J, ws, wsb);
      if (e) return e;
      Job<T> F = J;
      F.mode = MODE_FWD;
      F.g = nullptr;
      return launch_pf_tc(s, F);
    }
  }
  if (n > kSmallMax) {
    // large n: the blocked Parlett-Reid forward (n <= kPflMaxN; the generic kernel above),
    // the gradient S^-T / 2 from the Gauss-Jordan engine, the Pfaffian adjugate from the
    // generic kernel with (sign, logabs, value) rewritten by the forward -- one after the
    // other on the same stream and workspace
    Job<T> F = J;
    F.mode = MODE_FWD;
    F.g = nullptr;
    auto forward = [&]() { return n <= kPflMaxN ? run_large_pf<T>(s, F, ws, wsb) : launch_fused<T, true>(s, F, ws, wsb); };
    if (mode == MODE_FWD) return forward();
    if (mode == MODE_SLOG_GRAD) {
      int e = forward();
      if (e) return e;
      return run_large_lu<T>(s, J, ws, wsb, true, true);
    }
    int e = launch_fused<T, true>(s, J, ws, wsb);
    if (e) return e;
    return n <= kPflMaxN ? run_large_pf<T>(s, F, ws, wsb) : FX_OK;
  }
  return launch_fused<T, true>(s, J, ws, wsb);
}

template <typename F>
int by_dtype(int dtype, F&& f) {
  switch (dtype) {
    case FX_F32:
      return f(float());
    case FX_F64:
      return f(double());
    case FX_C64:
      return f(c64_t());
    case FX_C128:
      return f(c128_t());
  }
  return FX_ERR_DTYPE;
}

template <typename T>
size_t ws_bytes_t(int op, int64_t batch, int64_t n, int grad) {
  const int mode = grad ? MODE_SLOG_GRAD : MODE_FWD;
  if (op == FX_OP_SLOGDET && n <= DET_POLY_MAX) return 0;
  if (op == FX_OP_SLOGPF && (n % 2 == 1 || n <= PF_POLY_MAX)) return 0;
  if (op == FX_OP_SLOGPF && std::is_same<T, float>::value && n <= kTcN) return 0;  // TMEM / shared memory only
  Plan P;
  int e = op == FX_OP_SLOGPF ? plan_fused<T, true>(batch, (int)n, mode, P) : plan_fused<T, false>(batch, (int)n, mode, P);
  const size_t generic = (e || P.in_smem) ? 0 : (size_t)P.grid * P.slot;
  if (n > kSmallMax && (op == FX_OP_SLOGDET || grad || n <= kPflMaxN)) {
    // the large-n engine (the det adjugate and the Pfaffian gradient also run the generic
    // kernel, one after the other on the same workspace)
    const size_t lg = lg_ws_bytes<T>(batch, (int)n);
    Plan F;
    const size_t fwd = (op == FX_OP_SLOGPF && plan_fused<T, true>(batch, (int)n, MODE_FWD, F) == FX_OK && !F.in_smem)
                           ? (size_t)F.grid * F.slot
                           : 0;
    size_t m = lg > generic ? lg : generic;
    return m > fwd ? m : fwd;
  }
  return generic;
}

// ---------------------------------------------------------------- gathered slogdet
// Matrix b = rows occ[b, 0 .. n) of phi (phi_rows x phi_ld, row-major), columns 0 .. n.
template <typename T>
__global__ void __launch_bounds__(256) gather_rows_kernel(T* M, const T* phi, int64_t ld, int64_t rows,
                                                          const int* idx, int n) {
  typedef typename Sc<T>::R R;
  const int64_t b = blockIdx.y;
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (int64_t)n * n) return;
  const int i = (int)(e / n), j = (int)(e % n);
  const int r = idx[b * n + i];
  T v = s_zero<T>();
  if (r >= 0 && (int64_t)r < rows) {
    v = phi[(int64_t)r * ld + j];
  } else {
    const R q = R(NAN);
    if constexpr (Sc<T>::cx) v = {q, q};
    else v = q;
  }
  M[b * (int64_t)n * n + e] = v;
}

// the tensor-memory LU reads the rows itself; otherwise the batch is gathered into the
// front of the workspace and the regular path runs on it (its workspace behind)
template <typename T>
bool gather_direct(int prec, int64_t n, int mode) {
  return std::is_same<T, float>::value && use_lu_tc(1, prec, (int)n, mode);
}

template <typename T>
size_t gather_ws_bytes(int prec, int64_t batch, int64_t n, int grad) {
  const int mode = grad ? MODE_SLOG_GRAD : MODE_FWD;
  if (gather_direct<T>(prec, n, mode)) return 0;
  return align256((size_t)batch * n * n * sizeof(T)) + ws_bytes_t<T>(FX_OP_SLOGDET, batch, n, grad);
}

template <typename T>
int run_gather(cudaStream_t s, int prec, int64_t batch, int64_t n, const void* phi, int64_t rows, int64_t ld,
               const int* occ, const void* coef, int conj_out, void* sign, void* logabs, void* value, void* grad,
               void* ws, size_t wsb) {
  const int mode = grad ? MODE_SLOG_GRAD : MODE_FWD;
  if (gather_direct<T>(prec, n, mode)) {
    Job<T> J = make_job<T>(batch, n, nullptr, coef, conj_out, 0, mode, sign, logabs, value, grad);
    J.gidx = occ;
    J.gbase = static_cast<const T*>(phi);
    J.gld = ld;
    J.grows = rows;
    if constexpr (std::is_same<T, float>::value) return launch_lu_tc(s, J);
    return FX_ERR_DTYPE;
  }
  const size_t mat = align256((size_t)batch * n * n * sizeof(T));
  if (!ws || wsb < mat) return FX_ERR_WORKSPACE;
  T* M = static_cast<T*>(ws);
  if (n > 0) {
    gather_rows_kernel<T><<<dim3((unsigned)((n * n + 255) / 256), (unsigned)batch), 256, 0, s>>>(
        M, static_cast<const T*>(phi), ld, rows, occ, (int)n);
    if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
  }
  return run_det<T>(s, prec, batch, n, M, coef, conj_out, mode, sign, logabs, value, grad,
                    static_cast<unsigned char*>(ws) + mat, wsb - mat);
}

// ---------------------------------------------------------------- rank-k row updates
// Workspace of fermix_slogdet_update: the per-matrix action (B ints), then H (B x k x n).
template <typename T>
size_t upd_ws_bytes(int64_t batch, int64_t n, int64_t k) {
  return align256((size_t)batch * sizeof(int)) + align256((size_t)batch * k * n * sizeof(T));
}

int upd_validate(int dtype, int64_t batch, int64_t n, int64_t k) {
  int e = validate(dtype, FX_PREC_DEFAULT, batch, n);
  if (e) return e;
  if (k < 0 || k > kUpdMaxK || k > n) return FX_ERR_SHAPE;
  return FX_OK;
}

// ratio only (apply == false) or ratio plus the in-place update of G
template <typename T>
int run_update(cudaStream_t s, int64_t batch, int64_t n, int64_t k, void* g, const void* u, const int* idx,
               const unsigned char* accept, void* sign, void* logabs, void* ws, size_t wsb, bool apply) {
  const DevInfo* D = dev_info();
  if (!D) return FX_ERR_DEVICE;
  UpdArgs<T> A;
  A.g = static_cast<T*>(g);
  A.u = static_cast<const T*>(u);
  A.idx = idx;
  A.accept = accept;
  A.sign = static_cast<T*>(sign);
  A.logabs = static_cast<typename Sc<T>::R*>(logabs);
  A.h = nullptr;
  A.act = nullptr;
  A.B = batch;
  A.n = (int)n;
  A.k = (int)k;
  if (apply) {
    if (!ws || wsb < upd_ws_bytes<T>(batch, n, k)) return FX_ERR_WORKSPACE;
    A.act = static_cast<int*>(ws);
    A.h = reinterpret_cast<T*>(static_cast<unsigned char*>(ws) + align256((size_t)batch * sizeof(int)));
  }
  const int64_t pcap = (int64_t)D->sms * 8;
  if (k == 1) {
    const int64_t need = (batch + kUpdRowThreads / 32 - 1) / (kUpdRowThreads / 32);
    upd_prep1_kernel<T><<<(unsigned)(need < pcap ? need : pcap), kUpdRowThreads, 0, s>>>(A);
  } else {
    upd_prep_kernel<T><<<(unsigned)(batch < pcap ? batch : pcap), kUpdPrepThreads, 0, s>>>(A);
  }
  if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
  if (apply && k > 0) {
    const int64_t wpb = kUpdRowThreads / 32, rcap = (int64_t)D->sms * 8;
    const size_t rowb = (size_t)n * sizeof(T);
    const bool vec = rowb % 16 == 0 && rowb <= 8 * 512 &&
                     ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(u)) & 15) == 0;
    const size_t blk_smem = 2 * (size_t)k * rowb;
    if (vec && k > 1 && blk_smem <= (size_t)kUpdBlkSmem) {
      // U and H of a matrix in shared memory, one block per matrix at a time
      const int ch = rowb <= 512 ? 1 : rowb <= 1024 ? 2 : rowb <= 2048 ? 4 : 8;
      const bool big = k > 4;
      void* kern = nullptr;
      if (big) {
        kern = ch == 1 ? (sizeof(T) >= 8 ? (void*)&upd_rows_blk_kernel<T, 1, 1, kUpdMaxK>
                                         : (void*)&upd_rows_blk_kernel<T, 1, 2, kUpdMaxK>)
             : ch == 2 ? (void*)&upd_rows_blk_kernel<T, 2, 1, kUpdMaxK>
             : ch == 4 ? (void*)&upd_rows_blk_kernel<T, 4, 1, kUpdMaxK>
                       : (void*)&upd_rows_blk_kernel<T, 8, 1, kUpdMaxK>;
      } else {
        kern = ch == 1 ? (void*)&upd_rows_blk_kernel<T, 1, 2, 4>
             : ch == 2 ? (void*)&upd_rows_blk_kernel<T, 2, 2, 4>
             : ch == 4 ? (void*)&upd_rows_blk_kernel<T, 4, 1, 4>
                       : (void*)&upd_rows_blk_kernel<T, 8, 1, 4>;
      }
      if (blk_smem > 48 * 1024 &&
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kUpdBlkSmem) != cudaSuccess)
        return FX_ERR_CUDA;
      const int64_t cap = (int64_t)D->sms * 4;
      const unsigned grid = (unsigned)(batch < cap ? batch : cap);
      void* args[] = {&A};
      if (cudaLaunchKernel(kern, dim3(grid), dim3(kUpdRowThreads), args, blk_smem, s) != cudaSuccess)
        return FX_ERR_CUDA;
    } else if (vec) {
      // pieces per lane, and rows per warp: 4 KB of G in flight per warp where k <= 4
      const int ch = rowb <= 512 ? 1 : rowb <= 1024 ? 2 : rowb <= 2048 ? 4 : 8;
      const bool k4 = k > 1 && k <= 4;
      int rw = k > 4 ? 1 : ch == 1 ? 4 : ch == 2 ? 2 : ch == 4 ? 2 : 1;
      if (k4 && ch == 1 && sizeof(T) >= 8) rw = 2;   // register budget of 4 coefficients per row
      if (k4 && ch == 4 && sizeof(T) == 16) rw = 1;
      const int64_t need = (batch * ((n + rw - 1) / rw) + wpb - 1) / wpb;
      const unsigned grid = (unsigned)(need < rcap ? need : rcap);
      void* kern = nullptr;
      if (k == 1) {
        kern = ch == 1 ? (void*)&upd_rows_vec_kernel<T, 1, 4, 1>
             : ch == 2 ? (void*)&upd_rows_vec_kernel<T, 2, 2, 1>
             : ch == 4 ? (void*)&upd_rows_vec_kernel<T, 4, 2, 1>
                       : (void*)&upd_rows_vec_kernel<T, 8, 1, 1>;
      } else if (k <= 4) {
        kern = ch == 1 ? (rw == 4 ? (void*)&upd_rows_vec_kernel<T, 1, 4, 4> : (void*)&upd_rows_vec_kernel<T, 1, 2, 4>)
             : ch == 2 ? (void*)&upd_rows_vec_kernel<T, 2, 2, 4>
             : ch == 4 ? (rw == 2 ? (void*)&upd_rows_vec_kernel<T, 4, 2, 4> : (void*)&upd_rows_vec_kernel<T, 4, 1, 4>)
                       : (void*)&upd_rows_vec_kernel<T, 8, 1, 4>;
      } else {
        kern = ch == 1 ? (void*)&upd_rows_vec_kernel<T, 1, 1, kUpdMaxK>
             : ch == 2 ? (void*)&upd_rows_vec_kernel<T, 2, 1, kUpdMaxK>
             : ch == 4 ? (void*)&upd_rows_vec_kernel<T, 4, 1, kUpdMaxK>
                       : (void*)&upd_rows_vec_kernel<T, 8, 1, kUpdMaxK>;
      }
      void* args[] = {&A};
      if (cudaLaunchKernel(kern, dim3(grid), dim3(kUpdRowThreads), args, 0, s) != cudaSuccess) return FX_ERR_CUDA;
    } else {
      const int64_t need = (batch * n + wpb - 1) / wpb;
      upd_rows_kernel<T><<<(unsigned)(need < rcap ? need : rcap), kUpdRowThreads, 0, s>>>(A);
      if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
    }
  }
  return FX_OK;
}

template <typename T>
size_t pfm_ws_bytes(int64_t batch, int64_t n) {
  return align256((size_t)batch * sizeof(int)) + align256((size_t)batch * sizeof(T)) +
         2 * align256((size_t)batch * n * sizeof(T));
}

// Pfaffian one-index move: ratio only (apply == false) or ratio plus the in-place update
template <typename T>
int run_pf_move(cudaStream_t s, int64_t batch, int64_t n, void* g, const void* u, const int* idx,
                const unsigned char* accept, void* sign, void* logabs, void* ws, size_t wsb, bool apply) {
  const DevInfo* D = dev_info();
  if (!D) return FX_ERR_DEVICE;
  PfMoveArgs<T> A;
  A.g = static_cast<T*>(g);
  A.u = static_cast<const T*>(u);
  A.idx = idx;
  A.accept = accept;
  A.sign = static_cast<T*>(sign);
  A.logabs = static_cast<typename Sc<T>::R*>(logabs);
  A.h = A.v = A.rho = nullptr;
  A.act = nullptr;
  A.B = batch;
  A.n = (int)n;
  if (apply) {
    if (!ws || wsb < pfm_ws_bytes<T>(batch, n)) return FX_ERR_WORKSPACE;
    unsigned char* p = static_cast<unsigned char*>(ws);
    A.act = reinterpret_cast<int*>(p);
    p += align256((size_t)batch * sizeof(int));
    A.rho = reinterpret_cast<T*>(p);
    p += align256((size_t)batch * sizeof(T));
    A.h = reinterpret_cast<T*>(p);
    p += align256((size_t)batch * n * sizeof(T));
    A.v = reinterpret_cast<T*>(p);
  }
  if (apply && n * n * (int64_t)sizeof(T) <= kPfmSmemMax && (n * sizeof(T)) % 16 == 0 &&
      (reinterpret_cast<uintptr_t>(g) & 15) == 0) {
    // G fits one block's shared memory: the whole move in one launch (the workspace is unused)
    const size_t sm = pfm_smem_bytes((int)n, sizeof(T));
    if (cudaFuncSetAttribute(pfm_smem_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) !=
        cudaSuccess)
      return FX_ERR_CUDA;
    const int64_t cap = (int64_t)D->sms * 3;
    pfm_smem_kernel<T><<<(unsigned)(batch < cap ? batch : cap), kPfmThreads, sm, s>>>(A);
    return cudaGetLastError() == cudaSuccess ? FX_OK : FX_ERR_CUDA;
  }
  const int64_t wpb = kUpdRowThreads / 32, cap = (int64_t)D->sms * 8;
  const int64_t gp = (batch + wpb - 1) / wpb;
  pfm_prep_kernel<T><<<(unsigned)(gp < cap ? gp : cap), kUpdRowThreads, 0, s>>>(A);
  if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
  if (apply) {
    const size_t rowb = (size_t)n * sizeof(T);
    const bool vec = rowb % 16 == 0 && rowb <= 8 * 512 &&
                     ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(u)) & 15) == 0;
    if (vec) {
      const int ch = rowb <= 512 ? 1 : rowb <= 1024 ? 2 : rowb <= 2048 ? 4 : 8;
      const int rw = ch == 1 ? 4 : ch == 8 ? 1 : 2;
      const int64_t need = (batch * ((n + rw - 1) / rw) + wpb - 1) / wpb;
      const unsigned grid = (unsigned)(need < cap ? need : cap);
      void* kv = ch == 1 ? (void*)&pfm_v_vec_kernel<T, 1, 4> : ch == 2 ? (void*)&pfm_v_vec_kernel<T, 2, 2>
               : ch == 4 ? (void*)&pfm_v_vec_kernel<T, 4, 2> : (void*)&pfm_v_vec_kernel<T, 8, 1>;
      void* kr = ch == 1 ? (void*)&pfm_rows_vec_kernel<T, 1, 4> : ch == 2 ? (void*)&pfm_rows_vec_kernel<T, 2, 2>
               : ch == 4 ? (void*)&pfm_rows_vec_kernel<T, 4, 2> : (void*)&pfm_rows_vec_kernel<T, 8, 1>;
      void* args[] = {&A};
      if (cudaLaunchKernel(kv, dim3(grid), dim3(kUpdRowThreads), args, 0, s) != cudaSuccess) return FX_ERR_CUDA;
      if (cudaLaunchKernel(kr, dim3(grid), dim3(kUpdRowThreads), args, 0, s) != cudaSuccess) return FX_ERR_CUDA;
      return FX_OK;
    }
    const int64_t gr = (batch * n + wpb - 1) / wpb;
    pfm_v_kernel<T><<<(unsigned)(gr < cap ? gr : cap), kUpdRowThreads, 0, s>>>(A);
    if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
    pfm_rows_kernel<T><<<(unsigned)(gr < cap ? gr : cap), kUpdRowThreads, 0, s>>>(A);
    if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
  }
  return FX_OK;
}

}  // namespace

extern "C" {

int fermix_check_prec(int dtype, int prec) {
  if (prec != FX_PREC_DEFAULT && prec != FX_PREC_TF32X3 && prec != FX_PREC_IEEE) return FX_ERR_PREC;
  if (prec == FX_PREC_TF32X3 && (dtype == FX_F64 || dtype == FX_C128)) return FX_ERR_PREC;
  return FX_OK;
}

int fermix_slogdet(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* a, void* sign,
                   void* logabs, void* value, void* workspace, size_t workspace_bytes) {
  int e = validate(dtype, prec, batch, n);
  if (e) return e;
  if (batch == 0) return FX_OK;
  if ((!a && n > 0) || !sign || !logabs) return FX_ERR_NULL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_det<T>(s, prec, batch, n, a, nullptr, 0, MODE_FWD, sign, logabs, value, nullptr, workspace,
                      workspace_bytes);
  });
}

int fermix_slogdet_grad(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* a,
                        const void* coef, int conj_out, int adjugate, void* sign, void* logabs, void* value,
                        void* grad, void* workspace, size_t workspace_bytes) {
  int e = validate(dtype, prec, batch, n);
  if (e) return e;
  if (batch == 0) return FX_OK;
  if ((!a && n > 0) || !sign || !logabs || (!grad && n > 0)) return FX_ERR_NULL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int mode = adjugate ? MODE_VALUE_GRAD : MODE_SLOG_GRAD;
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_det<T>(s, prec, batch, n, a, coef, conj_out, mode, sign, logabs, value, grad, workspace, workspace_bytes);
  });
}

int fermix_slogpf(void* stream, int dtype, int prec, int64_t batch, int64_t n, int skew_symmetrize, const void* a,
                  void* sign, void* logabs, void* value, void* workspace, size_t workspace_bytes) {
  int e = validate(dtype, prec, batch, n);
  if (e) return e;
  if (batch == 0) return FX_OK;
  if ((!a && n > 0) || !sign || !logabs) return FX_ERR_NULL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_pf<T>(s, prec, batch, n, skew_symmetrize, a, nullptr, 0, MODE_FWD, sign, logabs, value, nullptr,
                     workspace, workspace_bytes);
  });
}

int fermix_slogpf_grad(void* stream, int dtype, int prec, int64_t batch, int64_t n, int skew_symmetrize,
                       const void* a, const void* coef, int conj_out, int adjugate, void* sign, void* logabs,
                       void* value, void* grad, void* workspace, size_t workspace_bytes) {
  int e = validate(dtype, prec, batch, n);
  if (e) return e;
  if (batch == 0) return FX_OK;
  if ((!a && n > 0) || !sign || !logabs || (!grad && n > 0)) return FX_ERR_NULL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int mode = adjugate ? MODE_VALUE_GRAD : MODE_SLOG_GRAD;
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_pf<T>(s, prec, batch, n, skew_symmetrize, a, coef, conj_out, mode, sign, logabs, value, grad,
                     workspace, workspace_bytes);
  });
}

int fermix_slogdet_gather(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* phi,
                          int64_t phi_rows, int64_t phi_ld, const int* occ, const void* coef, int conj_out,
                          void* sign, void* logabs, void* value, void* grad, void* workspace,
                          size_t workspace_bytes) {
  int e = validate(dtype, prec, batch, n);
  if (e) return e;
  if (phi_rows < 0 || phi_ld < n) return FX_ERR_SHAPE;
  if (batch == 0) return FX_OK;
  if ((n > 0 && (!phi || !occ)) || !sign || !logabs) return FX_ERR_NULL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_gather<T>(s, prec, batch, n, phi, phi_rows, phi_ld, occ, coef, conj_out, sign, logabs, value, grad,
                         workspace, workspace_bytes);
  });
}

size_t fermix_slogdet_gather_workspace_bytes(int dtype, int prec, int64_t batch, int64_t n, int grad) {
  if (validate(dtype, prec, batch, n) || batch == 0) return 0;
  return (size_t)by_dtype(dtype, [&](auto t) -> int {
    using T = decltype(t);
    return (int)((gather_ws_bytes<T>(prec, batch, n, grad) + 255) / 256);
  }) * 256;
}

size_t fermix_workspace_bytes(int op, int dtype, int64_t batch, int64_t n, int grad) {
  if (validate(dtype, FX_PREC_DEFAULT, batch, n) || batch == 0) return 0;
  return (size_t)by_dtype(dtype, [&](auto t) -> int {
    using T = decltype(t);
    size_t b = ws_bytes_t<T>(op, batch, n, grad);
    // returned through an int-typed dispatcher: report in 256-byte units
    return (int)((b + 255) / 256);
  }) * 256;
}

const char* fermix_strerror(int code) {
  switch (code) {
    case FX_OK:
      return "ok";
    case FX_ERR_DTYPE:
      return "unsupported dtype (float32, float64, complex64 and complex128 are supported)";
    case FX_ERR_SHAPE:
      return "bad shape: batch and n must be >= 0 and n <= 46000";
    case FX_ERR_PREC:
      return "prec must be 'tf32x3' or 'ieee'; 'tf32x3' applies to float32 / complex64 only";
    case FX_ERR_WORKSPACE:
      return "workspace missing or smaller than one matrix slot (see fermix_workspace_bytes)";
    case FX_ERR_NULL:
      return "a required pointer is NULL";
    case FX_ERR_CUDA:
      return "CUDA launch or attribute call failed";
    case FX_ERR_DEVICE:
      return "no usable CUDA device";
  }
  return "unknown error code";
}

int fermix_version(void) { return 100; }

int fermix_slogpf_ratio(void* stream, int dtype, int64_t batch, int64_t n, const void* g, const void* row,
                        const int* idx, void* sign, void* logabs) {
  int e = validate(dtype, FX_PREC_DEFAULT, batch, n);
  if (e) return e;
  if (n < 2) return FX_ERR_SHAPE;
  if (batch == 0) return FX_OK;
  if (!g || !row || !idx || !sign || !logabs) return FX_ERR_NULL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_pf_move<T>(s, batch, n, const_cast<void*>(g), row, idx, nullptr, sign, logabs, nullptr, 0, false);
  });
}

int fermix_slogpf_update(void* stream, int dtype, int64_t batch, int64_t n, void* g, const void* row, const int* idx,
                         const unsigned char* accept, void* sign, void* logabs, void* workspace,
                         size_t workspace_bytes) {
  int e = validate(dtype, FX_PREC_DEFAULT, batch, n);
  if (e) return e;
  if (n < 2) return FX_ERR_SHAPE;
  if (batch == 0) return FX_OK;
  if (!g || !row || !idx || !sign || !logabs) return FX_ERR_NULL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_pf_move<T>(s, batch, n, g, row, idx, accept, sign, logabs, workspace, workspace_bytes, true);
  });
}

size_t fermix_slogpf_update_workspace_bytes(int dtype, int64_t batch, int64_t n) {
  if (validate(dtype, FX_PREC_DEFAULT, batch, n) || batch == 0 || n < 2) return 0;
  return (size_t)by_dtype(dtype, [&](auto t) -> int {
    using T = decltype(t);
    return (int)((pfm_ws_bytes<T>(batch, n) + 255) / 256);
  }) * 256;
}

int fermix_slogdet_ratio(void* stream, int dtype, int64_t batch, int64_t n, int64_t k, const void* g,
                         const void* rows, const int* idx, void* sign, void* logabs) {
  int e = upd_validate(dtype, batch, n, k);
  if (e) return e;
  if (batch == 0) return FX_OK;
  if ((k > 0 && (!g || !rows || !idx)) || !sign || !logabs) return FX_ERR_NULL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_update<T>(s, batch, n, k, const_cast<void*>(g), rows, idx, nullptr, sign, logabs, nullptr, 0,
                         false);
  });
}

int fermix_slogdet_update(void* stream, int dtype, int64_t batch, int64_t n, int64_t k, void* g, const void* rows,
                          const int* idx, const unsigned char* accept, void* sign, void* logabs, void* workspace,
                          size_t workspace_bytes) {
  int e = upd_validate(dtype, batch, n, k);
  if (e) return e;
  if (batch == 0) return FX_OK;
  if ((k > 0 && (!g || !rows || !idx)) || !sign || !logabs) return FX_ERR_NULL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_update<T>(s, batch, n, k, g, rows, idx, accept, sign, logabs, workspace, workspace_bytes, true);
  });
}

size_t fermix_slogdet_update_workspace_bytes(int dtype, int64_t batch, int64_t n, int64_t k) {
  if (upd_validate(dtype, batch, n, k) || batch == 0) return 0;
  return (size_t)by_dtype(dtype, [&](auto t) -> int {
    using T = decltype(t);
    return (int)((upd_ws_bytes<T>(batch, n, k) + 255) / 256);
  }) * 256;
}

}  // extern "C"

// ---------------------------------------------------------------- static-scratch variant
// fermix_slogdet_grad_static: fermix_slogdet_grad whose LU kernels take their matrix
// slots (factor + inverse, 2 n^2 elements per resident block, used only when a matrix
// does not fit in one block's shared memory) from the fixed device array below instead
// of a caller workspace. It is for callers that cannot allocate device memory when they
// call: a host framework whose allocator owns all device memory and hands the op no
// scratch operand, or a latency-bound loop where cudaMalloc / cudaFree would synchronise
// the device. Nothing in the slots has to start at zero: the kernels write every element
// of a slot (the matrix load, then the column-by-column inverse) before reading it, so
// the array is never cleared. The array is shared by every call on a device: two calls
// in flight at once on one device (different streams or host threads) race on it and
// must be serialised by the caller (one stream, or an event between them).
static __device__ __align__(256) unsigned char fx_static_scratch[FX_STATIC_SCRATCH_BYTES];

namespace {

void* g_scratch_ptr[kMaxDevices];
std::once_flag g_scratch_once[kMaxDevices];

// Device address of fx_static_scratch on the current device, looked up once per device
// with that device current (nullptr if the lookup failed). The lookup may load this
// module on the device, so the first call on each device belongs before any stream
// capture.
void* static_scratch() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(g_scratch_once[dev], [dev]() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, fx_static_scratch) == cudaSuccess) {
      g_scratch_ptr[dev] = p;
    } else {
      g_scratch_ptr[dev] = nullptr;
      (void)cudaGetLastError();  // clear the error state so later calls report their own errors
    }
  });
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" {

int fermix_slogdet_grad_static(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* a,
                               const void* coef, int conj_out, int adjugate, void* sign, void* logabs, void* value,
                               void* grad) {
  int e = validate(dtype, prec, batch, n);
  if (e) return e;
  if (batch == 0) return FX_OK;
  if ((!a && n > 0) || !sign || !logabs || (!grad && n > 0)) return FX_ERR_NULL;
  // one matrix slot must fit: the workspace a single-member batch needs is one slot
  const size_t slot = fermix_workspace_bytes(FX_OP_SLOGDET, dtype, 1, n, 1);
  if (slot > (size_t)FX_STATIC_SCRATCH_BYTES) return FX_ERR_WORKSPACE;
  void* scratch = static_scratch();
  if (!scratch) return FX_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int mode = adjugate ? MODE_VALUE_GRAD : MODE_SLOG_GRAD;
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_det<T>(s, prec, batch, n, a, coef, conj_out, mode, sign, logabs, value, grad, scratch,
                      (size_t)FX_STATIC_SCRATCH_BYTES);
  });
}

#ifdef FX_PHASE_TIMERS
// profiling builds only: copy out / reset the per-phase cycle counters
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
