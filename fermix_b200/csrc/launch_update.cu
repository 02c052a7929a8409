// Rank-k determinant moves and one-index Pfaffian moves (update.cuh): workspace layout
// and launches.
#include "dispatch.cuh"
#include "update.cuh"
#include "update_pfk.cuh"

namespace fxh {

int upd_validate(int dtype, int64_t batch, int64_t n, int64_t k) {
  int e = validate(dtype, FX_PREC_DEFAULT, batch, n);
  if (e) return e;
  if (k < 0 || k > kUpdMaxK || k > n) return FX_ERR_SHAPE;
  return FX_OK;
}

// ---------------------------------------------------------------- rank-k row updates
// Workspace of fermix_slogdet_update: the per-matrix action (B ints), then H (B x k x n).
template <typename T>
size_t upd_ws_bytes(int64_t batch, int64_t n, int64_t k) {
  return align256((size_t)batch * sizeof(int)) + align256((size_t)batch * k * n * sizeof(T));
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
  A.wait_polls = wait_polls();
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
    // the limit is one constant bound for every n this path takes (n^2 s <= kPfmSmemMax), so
    // concurrent calls with different n on other host threads all write the same value
    if (cudaFuncSetAttribute(pfm_smem_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(kPfmSmemMax + 4096)) !=
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

// Workspace of the k-index Pfaffian move: the action (B ints), 1 / rho (B x k), then V, g_t
// and y_t (B x k x n each).
template <typename T>
size_t pfk_ws_bytes(int64_t batch, int64_t n, int64_t k) {
  return align256((size_t)batch * sizeof(int)) + align256((size_t)batch * k * sizeof(T)) +
         3 * align256((size_t)batch * k * n * sizeof(T));
}

// k-index Pfaffian move: ratio only (apply == false) or ratio plus the in-place update
template <typename T>
int run_pf_move_k(cudaStream_t s, int64_t batch, int64_t n, int64_t k, void* g, const void* u, const int* idx,
                  const unsigned char* accept, void* sign, void* logabs, void* ws, size_t wsb, bool apply) {
  const DevInfo* D = dev_info();
  if (!D) return FX_ERR_DEVICE;
  if (!ws || wsb < pfk_ws_bytes<T>(batch, n, k)) return FX_ERR_WORKSPACE;
  PfkArgs<T> A;
  A.g = static_cast<T*>(g);
  A.u = static_cast<const T*>(u);
  A.idx = idx;
  A.accept = accept;
  A.sign = static_cast<T*>(sign);
  A.logabs = static_cast<typename Sc<T>::R*>(logabs);
  A.B = batch;
  A.n = (int)n;
  A.k = (int)k;
  unsigned char* p = static_cast<unsigned char*>(ws);
  A.act = reinterpret_cast<int*>(p);
  p += align256((size_t)batch * sizeof(int));
  A.rinv = reinterpret_cast<T*>(p);
  p += align256((size_t)batch * k * sizeof(T));
  A.v = reinterpret_cast<T*>(p);
  p += align256((size_t)batch * k * n * sizeof(T));
  A.gv = reinterpret_cast<T*>(p);
  p += align256((size_t)batch * k * n * sizeof(T));
  A.yv = reinterpret_cast<T*>(p);
  const int64_t wpb = kUpdRowThreads / 32, cap = (int64_t)D->sms * 8;
  const int64_t gr = (batch * n + wpb - 1) / wpb;
  const unsigned grid = (unsigned)(gr < 2 * cap ? gr : 2 * cap);  // two 256-thread blocks per SM, 8 waves
  void* kv = k <= 2 ? (void*)&pfk_v_kernel<T, 2> : k <= 4 ? (void*)&pfk_v_kernel<T, 4>
           : k <= 8 ? (void*)&pfk_v_kernel<T, 8> : (void*)&pfk_v_kernel<T, 16>;
  void* kr = k <= 2 ? (void*)&pfk_rows_kernel<T, 2> : k <= 4 ? (void*)&pfk_rows_kernel<T, 4>
           : k <= 8 ? (void*)&pfk_rows_kernel<T, 8> : (void*)&pfk_rows_kernel<T, 16>;
  void* args[] = {&A};
  if (cudaLaunchKernel(kv, dim3(grid), dim3(kUpdRowThreads), args, 0, s) != cudaSuccess) return FX_ERR_CUDA;
  const int64_t pcap = (int64_t)D->sms * 8;
  pfk_prep_kernel<T><<<(unsigned)(batch < pcap ? batch : pcap), kPfkPrepThreads, 0, s>>>(A);
  if (cudaGetLastError() != cudaSuccess) return FX_ERR_CUDA;
  if (apply && cudaLaunchKernel(kr, dim3(grid), dim3(kUpdRowThreads), args, 0, s) != cudaSuccess)
    return FX_ERR_CUDA;
  return FX_OK;
}

int update_status(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, umma::fx_status_word, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(umma::fx_status_word, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

#define FXH_INST(T)                                                                                       \
  template size_t upd_ws_bytes<T>(int64_t, int64_t, int64_t);                                             \
  template int run_update<T>(cudaStream_t, int64_t, int64_t, int64_t, void*, const void*, const int*,     \
                             const unsigned char*, void*, void*, void*, size_t, bool);                    \
  template size_t pfm_ws_bytes<T>(int64_t, int64_t);                                                      \
  template int run_pf_move<T>(cudaStream_t, int64_t, int64_t, void*, const void*, const int*,             \
                              const unsigned char*, void*, void*, void*, size_t, bool);                   \
  template size_t pfk_ws_bytes<T>(int64_t, int64_t, int64_t);                                             \
  template int run_pf_move_k<T>(cudaStream_t, int64_t, int64_t, int64_t, void*, const void*, const int*,  \
                                const unsigned char*, void*, void*, void*, size_t, bool);
FXH_FOR_REAL(FXH_INST)
FXH_FOR_COMPLEX(FXH_INST)

}  // namespace fxh
