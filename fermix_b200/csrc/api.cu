// extern "C" entry points of libfermix_b200.so (declared in include/fermix_b200.h).
//
// Dispatch (replacing the reference's per-GPU TUNES table, src/fermix/_common.py:17-378):
//   det n <= 4, pf n <= 6      -> the closed forms (poly.cuh), one thread per matrix
//   pf with odd n              -> (0, -inf), zero gradient
//   otherwise                  -> the fused one-block-per-matrix kernels (fused_lu.cuh,
//                                 fused_pf.cuh): work buffers in shared memory when
//                                 they fit (227 KB per block on B200), else in the
//                                 caller's workspace (one slot per resident block).
// Process state: a once-initialised per-device attribute cache, the bounded-wait limit
// (fermix_set_wait_polls) and the device address of the static scratch array.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <type_traits>

#include "dispatch.cuh"

namespace fxh {

static DevInfo g_dev[kMaxDevices];
static std::once_flag g_once[kMaxDevices];

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

static std::atomic<uint32_t> g_wait_polls{FX_WAIT_POLLS_DEFAULT};

uint32_t wait_polls() { return g_wait_polls.load(std::memory_order_relaxed); }

}  // namespace fxh

namespace {

using namespace fxh;

static_assert(FX_ERR_TIMEOUT == 8, "the kernels record FX_ERR_TIMEOUT as 8");

// The kernels cut the workspace into 256-byte aligned arrays and read some of them as
// 16-byte pieces. A caller's workspace of any alignment is therefore moved up to the next
// 256-byte boundary here; the *_workspace_bytes queries include those 256 bytes.
constexpr size_t kWsSlack = 256;

void align_workspace(void*& ws, size_t& wsb) {
  if (!ws) {
    wsb = 0;
    return;
  }
  const uintptr_t p = reinterpret_cast<uintptr_t>(ws);
  const size_t skip = (size_t)(((p + 255) & ~(uintptr_t)255) - p);
  if (wsb <= skip) {
    ws = nullptr;
    wsb = 0;
    return;
  }
  ws = reinterpret_cast<void*>(p + skip);
  wsb -= skip;
}

size_t with_slack(size_t bytes) { return bytes ? bytes + kWsSlack : 0; }

template <typename T>
int launch_poly(cudaStream_t s, const Job<T>& J, int is_pf) {
  const int th = 128;
  const int64_t blocks = (J.B + th - 1) / th;
  poly_kernel<T><<<(unsigned)blocks, th, 0, s>>>(J, is_pf);
  return cudaGetLastError() == cudaSuccess ? FX_OK : FX_ERR_CUDA;
}

// Split real / imaginary planes of a complex call's input and gradient (the blocked
// engines read and write them directly).
template <typename T>
struct Planes {
  typedef typename Sc<T>::R R;
  const R* a_re;
  const R* a_im;
  R* g_re;
  R* g_im;
};

template <typename T>
void set_planes(Job<T>& J, const Planes<T>* pl) {
  if (!pl) return;
  J.a_re = pl->a_re;
  J.a_im = pl->a_im;
  J.g_re = pl->g_re;
  J.g_im = pl->g_im;
}

template <typename T>
int run_det(cudaStream_t s, int prec, int64_t batch, int64_t n, const void* a, const void* coef, int conj_out,
            int mode, void* sign, void* logabs, void* value, void* grad, void* ws, size_t wsb,
            const Planes<T>* pl = nullptr) {
  Job<T> J = make_job<T>(batch, n, a, coef, conj_out, 0, mode, sign, logabs, value, grad);
  J.prec = prec;
  set_planes(J, pl);
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
           int mode, void* sign, void* logabs, void* value, void* grad, void* ws, size_t wsb,
           const Planes<T>* pl = nullptr) {
  Job<T> J = make_job<T>(batch, n, a, coef, conj_out, skew, mode, sign, logabs, value, grad);
  J.prec = prec;
  set_planes(J, pl);
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

// ---------------------------------------------------------------- split planes
// Complex calls whose input and gradient are split real / imaginary planes (the layout of
// the reference's Field.split / join, src/fermix/_field.py:246-256). The blocked engines
// (n > 256: slogdet / slogpf forward and slog gradient) read and write the planes in their
// copy-in and gradient kernels, so the planar call moves the same bytes as the interleaved
// one. Every other case goes through the workspace in chunks: the chunk is interleaved,
// the interleaved path runs on it, and its gradient is split back into planes.
template <typename T>
__global__ void __launch_bounds__(256) interleave_kernel(T* out, const typename Sc<T>::R* re,
                                                         const typename Sc<T>::R* im, size_t count) {
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < count; e += (size_t)gridDim.x * blockDim.x)
    out[e] = T{re[e], im[e]};
}

template <typename T>
__global__ void __launch_bounds__(256) split_kernel(typename Sc<T>::R* re, typename Sc<T>::R* im, const T* in,
                                                    size_t count) {
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < count; e += (size_t)gridDim.x * blockDim.x) {
    const T v = in[e];
    re[e] = v.re;
    im[e] = v.im;
  }
}

inline unsigned elementwise_grid(size_t count) {
  const size_t blocks = (count + 255) / 256;
  return (unsigned)(blocks < 148 * 16 ? blocks : 148 * 16);
}

bool planar_native(bool pf, int64_t n, int mode) {
  if (n <= kSmallMax || (mode != MODE_FWD && mode != MODE_SLOG_GRAD)) return false;
  return !pf || (n % 2 == 0 && n <= kPflMaxN);
}

// matrices per chunk of the converting route: the whole batch up to about 1 GiB per plane copy
template <typename T>
int64_t planar_chunk(int64_t batch, int64_t n) {
  const size_t per = (size_t)n * n * sizeof(T);
  int64_t c = per ? (int64_t)(((size_t)1 << 30) / per) : batch;
  if (c < 1) c = 1;
  return batch < c ? batch : c;
}

template <typename T>
size_t planar_ws_bytes(int op, int64_t batch, int64_t n, int grad) {
  const int mode = grad ? MODE_SLOG_GRAD : MODE_FWD;
  if (planar_native(op == FX_OP_SLOGPF, n, mode)) return ws_bytes_t<T>(op, batch, n, grad);
  const int64_t c = planar_chunk<T>(batch, n);
  const size_t m = align256((size_t)c * n * n * sizeof(T));
  return m * (grad ? 2 : 1) + ws_bytes_t<T>(op, c, n, grad);
}

template <typename T>
int run_planar(cudaStream_t s, bool pf, int prec, int64_t batch, int64_t n, int skew, const void* re, const void* im,
               const void* coef, int conj_out, int mode, void* sign, void* logabs, void* value, void* g_re,
               void* g_im, void* ws, size_t wsb) {
  typedef typename Sc<T>::R R;
  Planes<T> pl{static_cast<const R*>(re), static_cast<const R*>(im), static_cast<R*>(g_re), static_cast<R*>(g_im)};
  if (planar_native(pf, n, mode)) {
    return pf ? run_pf<T>(s, prec, batch, n, skew, nullptr, coef, conj_out, mode, sign, logabs, value, nullptr, ws, wsb,
                          &pl)
              : run_det<T>(s, prec, batch, n, nullptr, coef, conj_out, mode, sign, logabs, value, nullptr, ws, wsb,
                           &pl);
  }
  const bool grad = mode != MODE_FWD;
  const int64_t c = planar_chunk<T>(batch, n);
  const size_t m = align256((size_t)c * n * n * sizeof(T));
  const size_t need = m * (grad ? 2 : 1);
  if (n > 0 && (!ws || wsb < need)) return FX_ERR_WORKSPACE;
  unsigned char* w = static_cast<unsigned char*>(ws);
  T* A = reinterpret_cast<T*>(w);
  T* G = grad ? reinterpret_cast<T*>(w + m) : nullptr;
  void* rest = n > 0 ? w + need : ws;
  const size_t rest_b = n > 0 ? wsb - need : wsb;
  const size_t nn = (size_t)n * n;
  for (int64_t b0 = 0; b0 < batch; b0 += c) {
    const int64_t cnt = batch - b0 < c ? batch - b0 : c;
    const size_t count = (size_t)cnt * nn;
    if (count) {
      interleave_kernel<T><<<elementwise_grid(count), 256, 0, s>>>(A, pl.a_re + b0 * nn, pl.a_im + b0 * nn, count);
      if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
    }
    T* sg = static_cast<T*>(sign) + b0;
    R* la = static_cast<R*>(logabs) + b0;
    T* val = value ? static_cast<T*>(value) + b0 : nullptr;
    const T* cf = coef ? static_cast<const T*>(coef) + b0 : nullptr;
    const int e = pf ? run_pf<T>(s, prec, cnt, n, skew, A, cf, conj_out, mode, sg, la, val, G, rest, rest_b)
                     : run_det<T>(s, prec, cnt, n, A, cf, conj_out, mode, sg, la, val, G, rest, rest_b);
    if (e) return e;
    if (grad && count) {
      split_kernel<T><<<elementwise_grid(count), 256, 0, s>>>(pl.g_re + b0 * nn, pl.g_im + b0 * nn, G, count);
      if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
    }
  }
  return FX_OK;
}

// complex dtypes only
template <typename F>
int by_complex(int dtype, F&& f) {
  switch (dtype) {
    case FX_C64:
      return f(c64_t());
    case FX_C128:
      return f(c128_t());
  }
  return FX_ERR_DTYPE;
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
    J.prec = prec;  // the tensor-memory LU's update kind (tensor cores or IEEE FMAs)
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
  align_workspace(workspace, workspace_bytes);
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
  align_workspace(workspace, workspace_bytes);
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
  align_workspace(workspace, workspace_bytes);
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
  align_workspace(workspace, workspace_bytes);
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
  align_workspace(workspace, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_gather<T>(s, prec, batch, n, phi, phi_rows, phi_ld, occ, coef, conj_out, sign, logabs, value, grad,
                         workspace, workspace_bytes);
  });
}

int fermix_slogdet_planar(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* a_re,
                          const void* a_im, void* sign, void* logabs, void* value, void* workspace,
                          size_t workspace_bytes) {
  int e = validate(dtype, prec, batch, n);
  if (e) return e;
  if (dtype != FX_C64 && dtype != FX_C128) return FX_ERR_DTYPE;
  if (batch == 0) return FX_OK;
  if ((n > 0 && (!a_re || !a_im)) || !sign || !logabs) return FX_ERR_NULL;
  align_workspace(workspace, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_complex(dtype, [&](auto t) {
    using T = decltype(t);
    return run_planar<T>(s, false, prec, batch, n, 0, a_re, a_im, nullptr, 0, MODE_FWD, sign, logabs, value, nullptr,
                         nullptr, workspace, workspace_bytes);
  });
}

int fermix_slogdet_grad_planar(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* a_re,
                               const void* a_im, const void* coef, int conj_out, int adjugate, void* sign,
                               void* logabs, void* value, void* grad_re, void* grad_im, void* workspace,
                               size_t workspace_bytes) {
  int e = validate(dtype, prec, batch, n);
  if (e) return e;
  if (dtype != FX_C64 && dtype != FX_C128) return FX_ERR_DTYPE;
  if (batch == 0) return FX_OK;
  if ((n > 0 && (!a_re || !a_im || !grad_re || !grad_im)) || !sign || !logabs) return FX_ERR_NULL;
  align_workspace(workspace, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int mode = adjugate ? MODE_VALUE_GRAD : MODE_SLOG_GRAD;
  return by_complex(dtype, [&](auto t) {
    using T = decltype(t);
    return run_planar<T>(s, false, prec, batch, n, 0, a_re, a_im, coef, conj_out, mode, sign, logabs, value, grad_re,
                         grad_im, workspace, workspace_bytes);
  });
}

int fermix_slogpf_planar(void* stream, int dtype, int prec, int64_t batch, int64_t n, int skew_symmetrize,
                         const void* a_re, const void* a_im, void* sign, void* logabs, void* value, void* workspace,
                         size_t workspace_bytes) {
  int e = validate(dtype, prec, batch, n);
  if (e) return e;
  if (dtype != FX_C64 && dtype != FX_C128) return FX_ERR_DTYPE;
  if (batch == 0) return FX_OK;
  if ((n > 0 && (!a_re || !a_im)) || !sign || !logabs) return FX_ERR_NULL;
  align_workspace(workspace, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_complex(dtype, [&](auto t) {
    using T = decltype(t);
    return run_planar<T>(s, true, prec, batch, n, skew_symmetrize, a_re, a_im, nullptr, 0, MODE_FWD, sign, logabs,
                         value, nullptr, nullptr, workspace, workspace_bytes);
  });
}

int fermix_slogpf_grad_planar(void* stream, int dtype, int prec, int64_t batch, int64_t n, int skew_symmetrize,
                              const void* a_re, const void* a_im, const void* coef, int conj_out, int adjugate,
                              void* sign, void* logabs, void* value, void* grad_re, void* grad_im, void* workspace,
                              size_t workspace_bytes) {
  int e = validate(dtype, prec, batch, n);
  if (e) return e;
  if (dtype != FX_C64 && dtype != FX_C128) return FX_ERR_DTYPE;
  if (batch == 0) return FX_OK;
  if ((n > 0 && (!a_re || !a_im || !grad_re || !grad_im)) || !sign || !logabs) return FX_ERR_NULL;
  align_workspace(workspace, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int mode = adjugate ? MODE_VALUE_GRAD : MODE_SLOG_GRAD;
  return by_complex(dtype, [&](auto t) {
    using T = decltype(t);
    return run_planar<T>(s, true, prec, batch, n, skew_symmetrize, a_re, a_im, coef, conj_out, mode, sign, logabs,
                         value, grad_re, grad_im, workspace, workspace_bytes);
  });
}

size_t fermix_workspace_bytes_planar(int op, int dtype, int64_t batch, int64_t n, int grad) {
  if (validate(dtype, FX_PREC_DEFAULT, batch, n) || batch == 0) return 0;
  if (dtype != FX_C64 && dtype != FX_C128) return 0;
  const size_t units = (size_t)by_complex(dtype, [&](auto t) -> int {
    using T = decltype(t);
    return (int)((planar_ws_bytes<T>(op, batch, n, grad) + 255) / 256);
  });
  return with_slack(units * 256);
}

size_t fermix_slogdet_gather_workspace_bytes(int dtype, int prec, int64_t batch, int64_t n, int grad) {
  if (validate(dtype, prec, batch, n) || batch == 0) return 0;
  return with_slack((size_t)by_dtype(dtype, [&](auto t) -> int {
    using T = decltype(t);
    return (int)((gather_ws_bytes<T>(prec, batch, n, grad) + 255) / 256);
  }) * 256);
}

size_t fermix_workspace_bytes(int op, int dtype, int64_t batch, int64_t n, int grad) {
  if (validate(dtype, FX_PREC_DEFAULT, batch, n) || batch == 0) return 0;
  // returned through an int-typed dispatcher: counted in 256-byte units
  const size_t units = (size_t)by_dtype(dtype, [&](auto t) -> int {
    using T = decltype(t);
    return (int)((ws_bytes_t<T>(op, batch, n, grad) + 255) / 256);
  });
  return with_slack(units * 256);
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
    case FX_ERR_TIMEOUT:
      return "a bounded wait inside a kernel gave up; the affected members' outputs are NaN";
  }
  return "unknown error code";
}

int fermix_version(void) { return 200; }

unsigned fermix_set_wait_polls(unsigned polls) { return g_wait_polls.exchange(polls); }

int fermix_device_status(int clear) {
  if (!dev_info()) return FX_ERR_DEVICE;
  if (cudaDeviceSynchronize() != cudaSuccess) return FX_ERR_CUDA;
  const int a = tc_status(clear), b = update_status(clear);
  if (a < 0 || b < 0) return FX_ERR_CUDA;
  return a ? a : b;
}

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
  align_workspace(workspace, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_pf_move<T>(s, batch, n, g, row, idx, accept, sign, logabs, workspace, workspace_bytes, true);
  });
}

size_t fermix_slogpf_update_workspace_bytes(int dtype, int64_t batch, int64_t n) {
  if (validate(dtype, FX_PREC_DEFAULT, batch, n) || batch == 0 || n < 2) return 0;
  return with_slack((size_t)by_dtype(dtype, [&](auto t) -> int {
    using T = decltype(t);
    return (int)((pfm_ws_bytes<T>(batch, n) + 255) / 256);
  }) * 256);
}

int fermix_slogpf_ratio_k(void* stream, int dtype, int64_t batch, int64_t n, int64_t k, const void* g,
                          const void* rows, const int* idx, void* sign, void* logabs, void* workspace,
                          size_t workspace_bytes) {
  int e = upd_validate(dtype, batch, n, k);
  if (e) return e;
  if (n < 2) return FX_ERR_SHAPE;
  if (batch == 0) return FX_OK;
  if ((k > 0 && (!g || !rows || !idx)) || !sign || !logabs) return FX_ERR_NULL;
  align_workspace(workspace, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_pf_move_k<T>(s, batch, n, k, const_cast<void*>(g), rows, idx, nullptr, sign, logabs, workspace,
                            workspace_bytes, false);
  });
}

int fermix_slogpf_update_k(void* stream, int dtype, int64_t batch, int64_t n, int64_t k, void* g, const void* rows,
                           const int* idx, const unsigned char* accept, void* sign, void* logabs, void* workspace,
                           size_t workspace_bytes) {
  int e = upd_validate(dtype, batch, n, k);
  if (e) return e;
  if (n < 2) return FX_ERR_SHAPE;
  if (batch == 0) return FX_OK;
  if ((k > 0 && (!g || !rows || !idx)) || !sign || !logabs) return FX_ERR_NULL;
  align_workspace(workspace, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_pf_move_k<T>(s, batch, n, k, g, rows, idx, accept, sign, logabs, workspace, workspace_bytes, true);
  });
}

size_t fermix_slogpf_move_k_workspace_bytes(int dtype, int64_t batch, int64_t n, int64_t k) {
  if (upd_validate(dtype, batch, n, k) || batch == 0 || n < 2) return 0;
  return with_slack((size_t)by_dtype(dtype, [&](auto t) -> int {
    using T = decltype(t);
    return (int)((pfk_ws_bytes<T>(batch, n, k) + 255) / 256);
  }) * 256);
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
  align_workspace(workspace, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return run_update<T>(s, batch, n, k, g, rows, idx, accept, sign, logabs, workspace, workspace_bytes, true);
  });
}

size_t fermix_slogdet_update_workspace_bytes(int dtype, int64_t batch, int64_t n, int64_t k) {
  if (upd_validate(dtype, batch, n, k) || batch == 0) return 0;
  return with_slack((size_t)by_dtype(dtype, [&](auto t) -> int {
    using T = decltype(t);
    return (int)((upd_ws_bytes<T>(batch, n, k) + 255) / 256);
  }) * 256);
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

std::atomic<void*> g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mu;

// Device address of fx_static_scratch on the current device, looked up with that device
// current on the first call that succeeds (nullptr if the lookup failed). Only a
// successful lookup is kept: a failed one is tried again on the next call. The lookup may
// load this module on the device, so the first call on each device belongs before any
// stream capture.
void* static_scratch() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  void* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p) return p;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p) return p;
  // an error the caller had already left pending is not ours to clear
  const bool clean = cudaPeekAtLastError() == cudaSuccess;
  if (cudaGetSymbolAddress(&p, fx_static_scratch) != cudaSuccess) {
    if (clean) (void)cudaGetLastError();  // clear only the error this lookup set
    return nullptr;
  }
  g_scratch_ptr[dev].store(p, std::memory_order_release);
  return p;
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
  size_t slot = fermix_workspace_bytes(FX_OP_SLOGDET, dtype, 1, n, 1);
  if (slot) slot -= kWsSlack;  // the array is 256-byte aligned: no alignment slack needed
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


}  // extern "C"
