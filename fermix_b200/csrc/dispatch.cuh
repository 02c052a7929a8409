// Host-side launch layer shared by the translation units of libfermix_b200.so.
//
// The library is compiled as several .cu files in parallel, one per kernel family:
//   api.cu            extern "C" entry points, argument checks, dtype / size dispatch
//   launch_fused_*.cu register-panel and generic one-block-per-matrix kernels (n <= 256,
//                     the adjugates), real and complex dtypes
//   launch_tc.cu      tensor-memory (tcgen05) kernels, float32 tf32x3
//   launch_large_*.cu blocked LU / Parlett-Reid engines for n > 256
//   launch_update.cu  rank-k determinant and one-index Pfaffian moves
// Each launcher below is a template defined in one of those files and explicitly
// instantiated there for the four dtypes; the kernel templates themselves are only
// instantiated in the file that launches them.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "fermix_b200.h"
#include "large_pf.cuh"
#include "poly.cuh"
#include "tc_common.cuh"
#include "update.cuh"

namespace fxh {

using namespace fx;

constexpr int kMaxDevices = 64;

struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
  int ok = 0;
};

// Attributes of the current device, read once per device (nullptr without a device).
const DevInfo* dev_info();

int validate(int dtype, int prec, int64_t batch, int64_t n);

// Polls of each bounded wait for launches issued now (fermix_set_wait_polls).
uint32_t wait_polls();

// Status word of one translation unit's kernels on the current device (0 or an FX_ERR_*
// code), reset to 0 when clear; -1 if it cannot be read. Defined in launch_tc.cu and
// launch_update.cu, the files whose kernels have bounded waits.
int tc_status(int clear);
int update_status(int clear);

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

constexpr int kSmallMax = 256;  // register-panel kernels: ceil(n / 32) <= 8 rows per lane

// Launch geometry of one fused call (shared by the launch and the workspace query).
struct Plan {
  int threads = 0, ld = 0, in_smem = 0;
  size_t smem = 0, slot = 0;
  int64_t grid = 0;
  void* kernel = nullptr;
};

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
  J.wait_polls = wait_polls();
  return J;
}

// ---- launch_fused_*.cu
template <typename T, bool PF>
int plan_fused(int64_t batch, int n, int mode, Plan& P);
template <typename T, bool PF>
int launch_fused(cudaStream_t s, Job<T> J, void* ws, size_t ws_bytes);

// ---- launch_tc.cu
inline bool use_pf_tc(int dtype_is_f32, int prec, int n, int mode) {
  (void)prec;  // tf32x3 and ieee both (tensor-core or FMA block updates)
  return dtype_is_f32 && n >= 8 && n <= kTcN && (mode == MODE_FWD || mode == MODE_SLOG_GRAD);
}
inline bool use_lu_tc(int dtype_is_f32, int prec, int n, int mode) {
  (void)prec;  // tf32x3 and ieee both (tensor-core or FMA block updates)
  return dtype_is_f32 && n >= 8 && n <= 2 * kTcN &&
         (mode == MODE_FWD || mode == MODE_SLOG_GRAD);
}
int launch_pf_tc(cudaStream_t s, Job<float> J);
int launch_lu_tc(cudaStream_t s, Job<float> J);

// ---- launch_large_*.cu
template <typename T>
size_t lg_ws_bytes(int64_t batch, int n);
// primal: write (sign, logabs, value); pf_grad: the input is skew-symmetrised when J.skew,
// the gradient is S^-T / 2 and zero where J.sign (the Pfaffian forward's) is zero.
template <typename T>
int run_large_lu(cudaStream_t s, Job<T> J, void* ws, size_t wsb, bool grad, bool pf_grad = false);
template <typename T>
int run_large_pf(cudaStream_t s, Job<T> J, void* ws, size_t wsb);

// ---- launch_update.cu
int upd_validate(int dtype, int64_t batch, int64_t n, int64_t k);
template <typename T>
size_t upd_ws_bytes(int64_t batch, int64_t n, int64_t k);
template <typename T>
int run_update(cudaStream_t s, int64_t batch, int64_t n, int64_t k, void* g, const void* u, const int* idx,
               const unsigned char* accept, void* sign, void* logabs, void* ws, size_t wsb, bool apply);
template <typename T>
size_t pfm_ws_bytes(int64_t batch, int64_t n);
template <typename T>
int run_pf_move(cudaStream_t s, int64_t batch, int64_t n, void* g, const void* u, const int* idx,
                const unsigned char* accept, void* sign, void* logabs, void* ws, size_t wsb, bool apply);

template <typename T>
size_t pfk_ws_bytes(int64_t batch, int64_t n, int64_t k);
template <typename T>
int run_pf_move_k(cudaStream_t s, int64_t batch, int64_t n, int64_t k, void* g, const void* u, const int* idx,
                  const unsigned char* accept, void* sign, void* logabs, void* ws, size_t wsb, bool apply);

}  // namespace fxh

// Explicit instantiation of a launcher template for the four dtypes.
#define FXH_FOR_REAL(M) M(float) M(double)
#define FXH_FOR_COMPLEX(M) M(fx::c64_t) M(fx::c128_t)
