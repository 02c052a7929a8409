// Shared pieces of the tensor-memory resident float32 kernels (pf_tc.cuh, lu_tc.cuh):
// one 128-thread block per matrix, thread x owns row x = TMEM lane x, the n x n matrix
// (n <= 128) occupies 128 TMEM columns for the whole call.
#pragma once
#include <stdint.h>

#include "umma.cuh"

namespace fx {

constexpr int kTcN = 128;                     // TMEM lanes / columns of the matrix
constexpr uint32_t kTcSlab = kTcN * 8 * 4;    // bytes of one K = 8 operand slab (128 rows)
constexpr uint32_t kTcWaitIters = 1u << 26;   // bounded MMA completion wait

__device__ __forceinline__ void tc_sync() {
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
}

// Order key of a pivot candidate for redux.sync: 0 = not a candidate, 1 = NaN (a
// candidate only when every candidate is NaN), else |v| ordered as its bit pattern,
// shifted above 1.
__device__ __forceinline__ unsigned piv_key(float v, bool live) {
  if (!live) return 0u;
  if (v != v) return 1u;
  return __float_as_uint(fabsf(v)) + 2u;
}

// Start pulling an n x n float32 matrix into L2 (bulk prefetch, 16 KB pieces). Skipped
// unless the address and size are 16-byte multiples, as the instruction requires.
__device__ __forceinline__ void tc_prefetch_l2(const float* p, int n) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t bytes = (uint32_t)n * (uint32_t)n * 4u;
  if ((a & 15) || (bytes & 15)) return;
  for (uint32_t off = 0; off < bytes; off += 16384u) {
    const uint32_t sz = bytes - off < 16384u ? bytes - off : 16384u;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a + off), "r"(sz) : "memory");
  }
}

// Row x of S = (skew ? (A - A^T) / 2 : A) into TMEM lane x (trow = this warp's lane
// base), zero outside n x n; A is n x n row-major at src. 32 columns at a time: the row
// part as 16-byte loads when every row starts on a 16-byte boundary (scalar otherwise;
// the 32 rows a warp touches stay in L1 across the column blocks), the transposed part
// as one coalesced 128-byte load per column (lanes read consecutive entries of a row).
// NC: TMEM columns to fill (the block's matrix width, 128 or 256).
template <int NC = kTcN>
__device__ __forceinline__ void tc_load_matrix(const float* __restrict__ src, int n, bool skew, uint32_t trow,
                                               int x) {
  const bool vec = ((reinterpret_cast<uintptr_t>(src) | ((uintptr_t)n * 4u)) & 15u) == 0;
#pragma unroll 1
  for (int c0 = 0; c0 < NC; c0 += 32) {
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = 0.f;
    if (x < n && c0 < n) {
      const float* row = src + (size_t)x * n + c0;
      if (vec) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (c0 + 4 * q < n) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(row) + q);
            v[4 * q] = t.x;
            v[4 * q + 1] = t.y;
            v[4 * q + 2] = t.z;
            v[4 * q + 3] = t.w;
          }
        }
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k)
          if (c0 + k < n) v[k] = __ldg(row + k);
      }
      if (skew) {
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float t = (c0 + k < n) ? __ldg(src + (size_t)(c0 + k) * n + x) : 0.f;
          v[k] = (v[k] - t) * 0.5f;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = __float_as_uint(v[8 * q + j]);
      umma::tmem_st8(trow + c0 + 8 * q, w);
    }
  }
  umma::tmem_wait_st();
}

// As tc_load_matrix (no skew) with row x taken from base[idx[x] * ld ..] (a gathered row of
// a shared matrix, typically L2-resident); an index outside [0, rows) fills the row with NaN.
template <int NC = kTcN>
__device__ __forceinline__ void tc_load_gathered(const float* __restrict__ base, int64_t ld, int64_t rows,
                                                 const int* __restrict__ idx, int n, uint32_t trow, int x) {
  const bool vec = ((reinterpret_cast<uintptr_t>(base) | ((uintptr_t)ld * 4u)) & 15u) == 0;
  int r = -1;
  if (x < n) r = __ldg(idx + x);
  const bool ok = r >= 0 && (int64_t)r < rows;
  const float* row = base + (ok ? (int64_t)r * ld : 0);
#pragma unroll 1
  for (int c0 = 0; c0 < NC; c0 += 32) {
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = 0.f;
    if (x < n && c0 < n) {
      if (!ok) {
#pragma unroll
        for (int k = 0; k < 32; ++k)
          if (c0 + k < n) v[k] = __int_as_float(0x7fc00000);
      } else if (vec) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (c0 + 4 * q < n) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(row + c0) + q);
            v[4 * q] = t.x;
            v[4 * q + 1] = t.y;
            v[4 * q + 2] = t.z;
            v[4 * q + 3] = t.w;
          }
        }
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k)
          if (c0 + k < n) v[k] = __ldg(row + c0 + k);
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = __float_as_uint(v[8 * q + j]);
      umma::tmem_st8(trow + c0 + 8 * q, w);
    }
  }
  umma::tmem_wait_st();
}

// dst[x * n + c] = f * TMEM[x][c] for c < n (zero when zero_out), thread x = row x; each
// warp writes its own 32 rows, 32 columns at a time (16-byte stores when aligned).
__device__ __forceinline__ void tc_store_rows(float* __restrict__ dst, int n, float f, bool zero_out,
                                              uint32_t trow, int x) {
  const bool vec = ((reinterpret_cast<uintptr_t>(dst) | ((uintptr_t)n * 4u)) & 15u) == 0;
#pragma unroll 1
  for (int c0 = 0; c0 < n; c0 += 32) {
    uint32_t w[32];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t t[8];
      umma::tmem_ld8(trow + c0 + 8 * q, t);
#pragma unroll
      for (int j = 0; j < 8; ++j) w[8 * q + j] = t[j];
    }
    umma::tmem_wait_ld();
    if (x < n) {
      float* row = dst + (size_t)x * n + c0;
      float v[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = zero_out ? 0.f : f * __uint_as_float(w[k]);
      if (vec) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (c0 + 4 * q < n)
            reinterpret_cast<float4*>(row)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k)
          if (c0 + k < n) row[k] = v[k];
      }
    }
  }
}

// As tc_store_rows for a 16-byte aligned dst and n % 4 == 0, through this warp's 32 x 36 float
// block of shared memory (wsm): each lane parks its 32 values of a column chunk as 16-byte
// stores (conflict-free quarter-warps), then every warp store writes 4 whole 128-byte row
// pieces instead of 32 separate 16-byte pieces of 32 rows (fewer L2 write transactions;
// measured faster for the gradient kernels).
__device__ __forceinline__ void tc_store_rows_staged(float* __restrict__ dst, int n, float f, bool zero_out,
                                                     uint32_t trow, int x, float* __restrict__ wsm) {
  const int lane = x & 31, r0 = x - lane;
#pragma unroll 1
  for (int c0 = 0; c0 < n; c0 += 32) {
    uint32_t w[32];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t t[8];
      umma::tmem_ld8(trow + c0 + 8 * q, t);
#pragma unroll
      for (int j = 0; j < 8; ++j) w[8 * q + j] = t[j];
    }
    umma::tmem_wait_ld();
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = zero_out ? 0.f : f * __uint_as_float(w[4 * q + e]);
      *reinterpret_cast<float4*>(wsm + lane * 36 + 4 * q) = make_float4(v[0], v[1], v[2], v[3]);
    }
    __syncwarp();
    const int cq = 4 * (lane & 7);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = 4 * i + (lane >> 3);
      if (r0 + rr < n && c0 + cq < n)
        *reinterpret_cast<float4*>(dst + (size_t)(r0 + rr) * n + c0 + cq) =
            *reinterpret_cast<const float4*>(wsm + rr * 36 + cq);
    }
    __syncwarp();
  }
}

}  // namespace fx
