// Self-test of the tensor-core building blocks (umma.cuh) on the running GPU: one
// 128 x 128 x 16 update D = C +- A B^T in TMEM with the 3xTF32 split, read back to
// global memory. Used by the GPU tests to pin the descriptor and TMEM conventions
// before the TMEM-resident kernels rely on them.
#include <cuda_runtime.h>

#include "fermix_b200.h"
#include "umma.cuh"

namespace {

using namespace fx::umma;

constexpr int kM = 128, kN = 128, kK = 16;
constexpr uint32_t kSlab = kM * 8 * 4;  // bytes of one K = 8 slab of a 128-row operand

__global__ void __launch_bounds__(128) umma_selftest_kernel(const float* A, const float* B, const float* C, float* D,
                                                            int negate, int accumulate, uint4 dis, int* status) {
  __shared__ __align__(1024) float sAhi[kM * kK], sAlo[kM * kK], sBhi[kN * kK], sBlo[kN * kK];
  __shared__ uint32_t tslot;
  __shared__ __align__(8) uint64_t mbar;
  const int tid = threadIdx.x, warp = tid >> 5;
  if (warp == 0) {
    tmem_alloc(&tslot, 128);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&mbar, 1);
    fence_mbar_init();
  }
  // operands, split into TF32 hi / lo parts, in the K-major interleaved layout
  {
    const int r = tid;
    for (int k = 0; k < kK; ++k) {
      const uint32_t off = kmajor_offset(r, k, kSlab) / 4;
      float a = A[r * kK + k], ah = tf32_round(a);
      sAhi[off] = ah;
      sAlo[off] = tf32_round(a - ah);
      float b = B[r * kK + k], bh = tf32_round(b);
      sBhi[off] = bh;
      sBlo[off] = tf32_round(b - bh);
    }
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = tslot;
  const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);
  for (int c = 0; c < kN; ++c) tmem_st1(trow + c, __float_as_uint(C[tid * kN + c]));
  tmem_wait_st();
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (tid == 0) {
    const uint32_t idesc = idesc_tf32(kM, kN, negate != 0);
    const uint32_t m4[4] = {dis.x, dis.y, dis.z, dis.w};
    for (int s = 0; s < kK / 8; ++s) {
      const uint64_t ahi = smem_desc_kmajor(smem_u32(sAhi) + s * kSlab, 128, 256);
      const uint64_t alo = smem_desc_kmajor(smem_u32(sAlo) + s * kSlab, 128, 256);
      const uint64_t bhi = smem_desc_kmajor(smem_u32(sBhi) + s * kSlab, 128, 256);
      const uint64_t blo = smem_desc_kmajor(smem_u32(sBlo) + s * kSlab, 128, 256);
      mma_tf32_masked(tbase, ahi, bhi, idesc, accumulate != 0 || s > 0, m4);
      mma_tf32_masked(tbase, ahi, blo, idesc, true, m4);
      mma_tf32_masked(tbase, alo, bhi, idesc, true, m4);
    }
    mma_commit(&mbar);
  }
  __syncwarp();
  const bool ok = mbar_wait(&mbar, 0, 1u << 24);
  fence_after_sync();
  for (int c = 0; c < kN; c += 8) {
    uint32_t v[8];
    tmem_ld8(trow + c, v);
    tmem_wait_ld();
    for (int j = 0; j < 8; ++j) D[tid * kN + c + j] = __uint_as_float(v[j]);
  }
  if (!ok) atomicOr(status, 1);
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 128);
}

}  // namespace

extern "C" int fermix_selftest_umma(void* stream, const float* a, const float* b, const float* c, float* d, int negate,
                                    int accumulate, const unsigned* disable_lanes, int* status) {
  if (!a || !b || !c || !d || !status) return FX_ERR_NULL;
  uint4 dis = make_uint4(0, 0, 0, 0);
  if (disable_lanes) dis = make_uint4(disable_lanes[0], disable_lanes[1], disable_lanes[2], disable_lanes[3]);
  umma_selftest_kernel<<<1, 128, 0, static_cast<cudaStream_t>(stream)>>>(a, b, c, d, negate, accumulate, dis, status);
  return cudaGetLastError() == cudaSuccess ? FX_OK : FX_ERR_CUDA;
}

// FMA-pipe throughput probe: every thread runs 8 independent FMA chains of `iters` steps
// (16 flops per step and thread), so the issue of the FP32 / FP64 FMA pipe, not latency,
// bounds it. The chains' sum goes to out so that nothing is optimised away.
namespace {

template <typename R>
__global__ void __launch_bounds__(256) fma_rate_kernel(int iters, R seed, R* out) {
  R x[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) x[c] = seed + (R)(threadIdx.x + c);
  const R m = (R)0.999999, k = (R)1e-7;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int c = 0; c < 8; ++c) x[c] = fma(x[c], m, k);
  }
  R s = 0;
#pragma unroll
  for (int c = 0; c < 8; ++c) s += x[c];
  if (s == (R)-1.2345) out[blockIdx.x] = s;  // never true for these inputs
}

}  // namespace

extern "C" int fermix_selftest_fma_rate(void* stream, int dtype, int blocks, int iters, void* out) {
  if (!out) return FX_ERR_NULL;
  if (blocks < 1 || iters < 1) return FX_ERR_SHAPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == FX_F32)
    fma_rate_kernel<float><<<blocks, 256, 0, s>>>(iters, 1.0f, static_cast<float*>(out));
  else if (dtype == FX_F64)
    fma_rate_kernel<double><<<blocks, 256, 0, s>>>(iters, 1.0, static_cast<double*>(out));
  else
    return FX_ERR_DTYPE;
  return cudaGetLastError() == cudaSuccess ? FX_OK : FX_ERR_CUDA;
}
