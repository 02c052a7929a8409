// Thin wrappers over the sm_100a tensor-core (tcgen05) and tensor-memory instructions
// used by the TMEM-resident kernels: TMEM allocation, 32-lane TMEM loads / stores,
// shared-memory operand descriptors (K-major, no swizzle), the kind::tf32 instruction
// descriptor, the MMA itself, its commit to an mbarrier, and a bounded mbarrier wait.
//
// Operand layout in shared memory (K-major, SWIZZLE_NONE, the "interleaved" canonical
// layout): 8-row x 16-byte core matrices; element (r, k) of a K = 8 slab lives at
//   (r / 8) * SBO + (k / 4) * LBO + (r % 8) * 16 + (k % 4) * 4   bytes,
// with LBO = 128 (the two K-halves of a row group are adjacent) and SBO = 256.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fx {
namespace umma {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- TMEM allocation
// One full warp: allocates ncols (power of two >= 32) columns of all 128 lanes and writes
// the base TMEM address to *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// ---------------------------------------------------------------- TMEM <-> registers
// 32x32b shape: thread t of the warp reads / writes lane (lane_base + t) of the given
// column(s). taddr = base | (lane_base << 16) | column.
__device__ __forceinline__ uint32_t tmem_ld1(uint32_t taddr) {
  uint32_t v;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v) : "r"(taddr));
  return v;
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v));
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// generic-proxy shared-memory writes -> visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor, K-major, no swizzle (version 1 for sm_100).
__device__ __forceinline__ uint64_t smem_desc_kmajor(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // version
  // base_offset = 0, lbo_mode = 0, layout type 0 = SWIZZLE_NONE
  return d;
}

// kind::tf32 instruction descriptor: F32 accumulator, TF32 A and B, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, bool negate_a) {
  return (1u << 4)                        // D format F32
         | (2u << 7)                      // A format TF32
         | (2u << 10)                     // B format TF32
         | ((negate_a ? 1u : 0u) << 13)   // negate A
         | ((uint32_t)(N >> 3) << 17)     // N / 8
         | ((uint32_t)(M >> 4) << 24);    // M / 16
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(0u));
}

// The same with output lanes disabled: bit l of dis[w] keeps TMEM lane 32 w + l of D
// unwritten.
__device__ __forceinline__ void mma_tf32_masked(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                bool accumulate, const uint32_t (&dis)[4]) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(dis[0]), "r"(dis[1]), "r"(dis[2]),
      "r"(dis[3]));
}

// Arrive on the mbarrier once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(mbar))
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(mbar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// The executing thread's arrival on the mbarrier, announcing tx_bytes of async copies
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* mbar, uint32_t tx_bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(mbar)), "r"(tx_bytes)
               : "memory");
}

// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global to
// this CTA's shared memory, completing `bytes` transactions on the mbarrier
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(mbar))
      : "memory");
}

// Status word of the kernels in one translation unit (each .cu file that includes this
// header has its own copy, read back by that file's status function): 0, or the first
// error code a kernel recorded (8 = FX_ERR_TIMEOUT, a bounded wait that gave up).
static __device__ int fx_status_word;

__device__ __forceinline__ void record_status(int code) { atomicCAS(&fx_status_word, 0, code); }

// Wait for the phase with the given parity to complete; gives up after max_iters polls
// and returns false (the caller records an error instead of hanging). max_iters == 0
// gives up at once.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity, uint32_t max_iters) {
  const uint32_t a = smem_u32(mbar);
  for (uint32_t it = 0; it < max_iters; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// Round an f32 to TF32 (nearest, ties away; the low 13 mantissa bits become zero).
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Byte offset of element (r, k) in a K-major no-swizzle operand made of K = 8 slabs
// (slab_bytes apart): LBO = 128, SBO = 256.
__host__ __device__ __forceinline__ uint32_t kmajor_offset(int r, int k, uint32_t slab_bytes) {
  const int slab = k >> 3, kk = k & 7;
  return (uint32_t)slab * slab_bytes + (uint32_t)(r >> 3) * 256u + (uint32_t)(kk >> 2) * 128u +
         (uint32_t)(r & 7) * 16u + (uint32_t)(kk & 3) * 4u;
}

}  // namespace umma
}  // namespace fx
