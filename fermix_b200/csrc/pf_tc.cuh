// Tensor-memory resident Parlett-Reid "sweep" for float32 slogpf, 8 <= n <= 128,
// prec = "tf32x3": forward (sign, logabs) and, in the same pass, S^-1 for the gradient.
//
// Reference behaviour: the pair steps and pivoting of src/fermix/_fallback.py:266-300
// (pivot = largest corrected entry of column a among the unassigned rows, d = S[a, p]),
// blocked as in src/fermix/_pf.py:516-570, with the tf32x3 block updates of
// src/fermix/_field.py:173-190 (3 TF32 products per update); the gradient is S^-T / 2 of
// src/fermix/_diff.py:139-154, zero for an exactly singular S (_pfinv.py:263-268).
//
// Design (B200). The 128 x 128 matrix lives in tensor memory (TMEM lane i = row i, one
// 32-bit column per matrix column) for the whole call; thread i of the 128-thread block
// owns row i. Each panel of up to 8 pairs is found by the pair steps on corrected
// columns (one TMEM column read per step and thread), then the whole matrix gets the
// rank-16 block-sweep update D -= W B^T as six tcgen05.mma kind::tf32 instructions
// (K = 16, hi / lo split) issued by one thread, accumulating in TMEM. In gradient mode the
// panel's pivot rows and columns are then replaced by the block-sweep values
//   A'_XP = A_XP A_PP^-1,  A'_PX = -+A'_XP^T,  A'_PP = -A_PP^-1,
// so that after the last panel TMEM holds -S^-1 (sweeping every index inverts the
// matrix); the forward-only mode skips the replacement and its (sign, logabs) are
// bit-identical (the unswept part evolves identically). Row-derived operand values come
// from the column values by the sweep's sign pattern: skew inside the unswept and inside
// the swept index sets, symmetric across them.
#pragma once
#include "fused_lu.cuh"
#include "tc_common.cuh"

namespace fx {

struct PfTcSmem {
  float u[8][kTcN];  // u_t[x] = col_p[x] / d_t of the panel's pairs (broadcast reads)
  float v[8][kTcN];  // v_t[x] = -col_a[x] / d_t
  float whi[kTcN * 16], wlo[kTcN * 16];  // MMA A operand (K-major, interleaved), TF32 hi / lo
  float bhi[kTcN * 16], blo[kTcN * 16];  // MMA B operand
  __align__(16) float app[16][20];       // A_PP of the panel, then A_PP^-1 (16-byte rows)
  uint4 pcand[4];                        // per-warp pivot candidates: key, row, -, value bits
  int cand_f[4];                         // scratch (the singular flag at the end)
  int at[kTcN], pof[kTcN];               // position -> row, row -> position (virtual pivoting)
  int pidx[16];                          // the panel's pivot rows a_0, p_0, a_1, p_1, ...
  unsigned char isP[kTcN];
  float dvec[kTcN / 2];
  uint32_t tslot;
  uint32_t dis[4];  // MMA output-lane mask: lanes that are not pivot rows
  int parity, bad;
  uint64_t mbar;
};

// Inverse of the m x m (m = 2 np <= 16) pivot block in S.app by sequential 2 x 2 pair
// sweeps (pairs (2q, 2q+1)); warp 0, lane k owns row k. Result: S.app = A_PP^-1.
__device__ void tc_block_inverse(PfTcSmem& S, int np) {
  const int lane = threadIdx.x & 31;
  const int m = 2 * np;
  float r[16];
#pragma unroll
  for (int y = 0; y < 16; ++y) r[y] = (lane < m && y < m) ? S.app[lane][y] : 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    if (q < np) {
      const int i = 2 * q, j = i + 1;
      float ri[16], rj[16];
#pragma unroll
      for (int y = 0; y < 16; ++y) {
        ri[y] = __shfl_sync(0xffffffffu, r[y], i);
        rj[y] = __shfl_sync(0xffffffffu, r[y], j);
      }
      const float d00 = ri[i], d01 = ri[j], d10 = rj[i], d11 = rj[j];
      const float det = d00 * d11 - d01 * d10;
      const float id = det == 0.f ? 0.f : __fdiv_rn(1.f, det);
      const float e00 = d11 * id, e01 = -d01 * id, e10 = -d10 * id, e11 = d00 * id;
      if (lane == i || lane == j) {
        const float f0 = lane == i ? e00 : e10, f1 = lane == i ? e01 : e11;
#pragma unroll
        for (int y = 0; y < 16; ++y)
          if (y != i && y != j) r[y] = fmaf(f0, ri[y], f1 * rj[y]);
        r[i] = -f0;
        r[j] = -f1;
      } else if (lane < m) {
        const float xi = r[i], xj = r[j];
        const float ci = fmaf(xi, e00, xj * e10), cj = fmaf(xi, e01, xj * e11);
#pragma unroll
        for (int y = 0; y < 16; ++y)
          if (y != i && y != j) r[y] = fmaf(-ci, ri[y], fmaf(-cj, rj[y], r[y]));
        r[i] = ci;
        r[j] = cj;
      }
    }
  }
  __syncwarp();
  if (lane < m) {
#pragma unroll
    for (int y = 0; y < 16; ++y)
      if (y < m) S.app[lane][y] = -r[y];  // the sweep leaves -A_PP^-1
  }
}

template <bool GRAD>
__global__ void __launch_bounds__(128) pf_tc_kernel(Job<float> J) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PfTcSmem& S = *reinterpret_cast<PfTcSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = J.n;
  const int x = tid;  // this thread's row / TMEM lane
  if (warp == 0) {
    umma::tmem_alloc(&S.tslot, kTcN);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    umma::mbar_init(&S.mbar, 1);
    umma::fence_mbar_init();
  }
  tc_sync();
#ifdef FX_PHASE_TIMERS
  if (blockIdx.x == 0 && tid == 0) fx_phase_cycles[15] = gridDim.x;
#endif
  const uint32_t tbase = S.tslot;
  const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);
  uint32_t phase = 0;

  for (int64_t b = blockIdx.x; b < J.B; b += gridDim.x) {
    FX_TIC(tq);
    // ---- the (skew-symmetrised) matrix into TMEM, zero outside n x n; the block's
    // next matrix starts streaming into L2 meanwhile
    const float* src = J.a + b * (int64_t)n * n;
    if (tid == 0 && b + gridDim.x < J.B) tc_prefetch_l2(src + (int64_t)gridDim.x * n * n, n);
    tc_load_matrix(src, n, J.skew != 0, trow, x);
    S.at[x] = x;
    S.pof[x] = x;
    S.isP[x] = 0;
    if (tid == 0) {
      S.parity = 0;
      S.bad = 0;
    }
    bool live = x < n;
    tc_sync();
    FX_TOC(tq, 8);

    const int npairs = n / 2;
    for (int g0 = 0; g0 < npairs; g0 += 8) {
      const int np = min(8, npairs - g0);
      const bool swept_before = !live && x < n;
      float ur[8], vr[8], dr[8], s0[16];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        ur[t] = vr[t] = dr[t] = 0.f;
        s0[2 * t] = s0[2 * t + 1] = 0.f;
      }
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        if (s < np) {
          const int c = 2 * (g0 + s);
          const int a = S.at[c];
          if (x == a) live = false;
          // column a of the current matrix: stale TMEM value plus this panel's corrections
          float colA = __uint_as_float(umma::tmem_ld1(trow + a));
          umma::tmem_wait_ld();
          s0[2 * s] = colA;
#pragma unroll
          for (int t = 0; t < 8; ++t)
            if (t < s) {
              const float r1 = dr[t] * S.v[t][a], r2 = -dr[t] * S.u[t][a];
              colA = fmaf(-ur[t], r1, colA);
              colA = fmaf(-vr[t], r2, colA);
            }
          // pivot: largest |colA| over the unassigned rows (first occurrence): per warp two
          // redux.sync on the packed key, then the four warps' candidates
          const unsigned key = piv_key(colA, live);
          const unsigned km = __reduce_max_sync(0xffffffffu, key);
          const int wi = __reduce_min_sync(0xffffffffu, key == km ? x : 0x7fffffff);
          if (x == wi) S.pcand[warp] = make_uint4(km, (unsigned)wi, 0u, __float_as_uint(colA));
          __syncthreads();
          uint4 hd[4];
#pragma unroll
          for (int w = 0; w < 4; ++w) hd[w] = S.pcand[w];
          unsigned bk = hd[0].x, bp = hd[0].y, bvb = hd[0].w;
#pragma unroll
          for (int w = 1; w < 4; ++w)
            if (hd[w].x > bk || (hd[w].x == bk && hd[w].y < bp)) {
              bk = hd[w].x;
              bp = hd[w].y;
              bvb = hd[w].w;
            }
          const int p = (int)bp;
          const float d = -__uint_as_float(bvb);  // all candidates NaN: the first one, d = NaN
          const float inv = d == 0.f ? 0.f : __fdiv_rn(1.f, d);
          if (x == p) live = false;
          float colP = __uint_as_float(umma::tmem_ld1(trow + p));
          umma::tmem_wait_ld();
          s0[2 * s + 1] = colP;
#pragma unroll
          for (int t = 0; t < 8; ++t)
            if (t < s) {
              const float r1 = dr[t] * S.v[t][p], r2 = -dr[t] * S.u[t][p];
              colP = fmaf(-ur[t], r1, colP);
              colP = fmaf(-vr[t], r2, colP);
            }
          ur[s] = colP * inv;
          vr[s] = -colA * inv;
          dr[s] = d;
          S.u[s][x] = ur[s];
          S.v[s][x] = vr[s];
          if (tid == 0) {
            const int q = S.pof[p];
            if (q != c + 1) {
              const int y = S.at[c + 1];
              S.at[c + 1] = p;
              S.at[q] = y;
              S.pof[p] = c + 1;
              S.pof[y] = q;
              S.parity ^= 1;
            }
            S.dvec[g0 + s] = d;
            S.pidx[2 * s] = a;
            S.pidx[2 * s + 1] = p;
            S.isP[a] = 1;
            S.isP[p] = 1;
          }
          __syncthreads();
        }
      }
      FX_TOC(tq, 9);
      // ---- gradient mode: the pivot block A_PP (rows of the pivot threads) for its inverse,
      // and the output-lane mask of the pivot rows
      int kx = -1;
      if (GRAD) {
#pragma unroll
        for (int k = 0; k < 16; ++k)
          if (k < 2 * np && S.pidx[k] == x) kx = k;
        if (kx >= 0) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (j < 2 * np) S.app[kx][j] = s0[j];
        }
        const unsigned notP = __ballot_sync(0xffffffffu, kx < 0);
        if (lane == 0) S.dis[warp] = notP;
      }
      // ---- MMA operands: W[x] = (u_t, v_t), B[x] = sigma(x) d_t (v_t, -u_t), 16-byte stores
      {
        const float sig = swept_before ? -1.f : 1.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float wh[4], wl[4], zh[4], zl[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k = 4 * q + e, t = k >> 1;
            float w = 0.f, z = 0.f;
            if (t < np) {
              w = (k & 1) ? vr[t] : ur[t];
              z = (k & 1) ? -sig * dr[t] * ur[t] : sig * dr[t] * vr[t];
            }
            wh[e] = umma::tf32_round(w);
            wl[e] = umma::tf32_round(w - wh[e]);
            zh[e] = umma::tf32_round(z);
            zl[e] = umma::tf32_round(z - zh[e]);
          }
          const uint32_t off = umma::kmajor_offset(x, 4 * q, kTcSlab) / 4;
          *reinterpret_cast<float4*>(&S.whi[off]) = make_float4(wh[0], wh[1], wh[2], wh[3]);
          *reinterpret_cast<float4*>(&S.wlo[off]) = make_float4(wl[0], wl[1], wl[2], wl[3]);
          *reinterpret_cast<float4*>(&S.bhi[off]) = make_float4(zh[0], zh[1], zh[2], zh[3]);
          *reinterpret_cast<float4*>(&S.blo[off]) = make_float4(zl[0], zl[1], zl[2], zl[3]);
        }
      }
      umma::fence_proxy_async_smem();
      tc_sync();
      FX_TOC(tq, 10);
      if (tid == 0) {
        const uint32_t idesc = umma::idesc_tf32(kTcN, kTcN, true);  // D -= W B^T
#pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
          const uint64_t ah = umma::smem_desc_kmajor(umma::smem_u32(S.whi) + sl * kTcSlab, 128, 256);
          const uint64_t al = umma::smem_desc_kmajor(umma::smem_u32(S.wlo) + sl * kTcSlab, 128, 256);
          const uint64_t bh = umma::smem_desc_kmajor(umma::smem_u32(S.bhi) + sl * kTcSlab, 128, 256);
          const uint64_t bl = umma::smem_desc_kmajor(umma::smem_u32(S.blo) + sl * kTcSlab, 128, 256);
          umma::mma_tf32(tbase, ah, bh, idesc, true);
          umma::mma_tf32(tbase, ah, bl, idesc, true);
          umma::mma_tf32(tbase, al, bh, idesc, true);
        }
        umma::mma_commit(&S.mbar);
      }
      // gradient mode: warp 0 inverts A_PP while the tensor core runs the update
      if (GRAD && warp == 0) tc_block_inverse(S, np);
      __syncwarp();
      if (!umma::mbar_wait(&S.mbar, phase, kTcWaitIters)) S.bad = 1;
      phase ^= 1;
      umma::fence_after_sync();
      FX_TOC(tq, 11);

      if (GRAD) {
        // pivot rows / columns -> the block-sweep values (A = panel-start matrix):
        //   A'_XP = A_XP A_PP^-1, A'_PP = -A_PP^-1 (16 TMEM column stores per thread),
        //   A'_PY = A_PP^-1 A_PY = A_PP^-1 (tau(y) A_YP^T), tau = -1 unswept / +1 swept y,
        // the latter as a second MMA whose output lanes are only the pivot rows.
        __syncthreads();  // A_PP^-1 complete
        FX_TOC(tq, 1);
        float pv[16], a2[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) pv[j] = a2[j] = 0.f;
        if (kx >= 0) {
          const float4* r4 = reinterpret_cast<const float4*>(S.app[kx]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 v = r4[q];
            a2[4 * q] = v.x;
            a2[4 * q + 1] = v.y;
            a2[4 * q + 2] = v.z;
            a2[4 * q + 3] = v.w;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) pv[j] = -a2[j];
        } else {
          // s0 A_PP^-1: broadcast 16-byte row loads, 16 independent accumulators
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (i < 2 * np) {
              const float4* r4 = reinterpret_cast<const float4*>(S.app[i]);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float4 v = r4[q];
                pv[4 * q] = fmaf(s0[i], v.x, pv[4 * q]);
                pv[4 * q + 1] = fmaf(s0[i], v.y, pv[4 * q + 1]);
                pv[4 * q + 2] = fmaf(s0[i], v.z, pv[4 * q + 2]);
                pv[4 * q + 3] = fmaf(s0[i], v.w, pv[4 * q + 3]);
              }
            }
          }
        }
        const float tau = swept_before ? 1.f : -1.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float ah[4], al[4], bh[4], bl[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 4 * q + e;
            const bool on = j < 2 * np;
            if (!on) pv[j] = 0.f;
            const float av = on ? a2[j] : 0.f, bv = on ? tau * s0[j] : 0.f;
            ah[e] = umma::tf32_round(av);
            al[e] = umma::tf32_round(av - ah[e]);
            bh[e] = umma::tf32_round(bv);
            bl[e] = umma::tf32_round(bv - bh[e]);
          }
          const uint32_t off = umma::kmajor_offset(x, 4 * q, kTcSlab) / 4;
          *reinterpret_cast<float4*>(&S.whi[off]) = make_float4(ah[0], ah[1], ah[2], ah[3]);
          *reinterpret_cast<float4*>(&S.wlo[off]) = make_float4(al[0], al[1], al[2], al[3]);
          *reinterpret_cast<float4*>(&S.bhi[off]) = make_float4(bh[0], bh[1], bh[2], bh[3]);
          *reinterpret_cast<float4*>(&S.blo[off]) = make_float4(bl[0], bl[1], bl[2], bl[3]);
        }
        umma::fence_proxy_async_smem();
        tc_sync();
        FX_TOC(tq, 2);
        if (tid == 0) {
          const uint32_t idesc = umma::idesc_tf32(kTcN, kTcN, false);
          const uint32_t dis[4] = {S.dis[0], S.dis[1], S.dis[2], S.dis[3]};
#pragma unroll
          for (int sl = 0; sl < 2; ++sl) {
            const uint64_t ah = umma::smem_desc_kmajor(umma::smem_u32(S.whi) + sl * kTcSlab, 128, 256);
            const uint64_t al = umma::smem_desc_kmajor(umma::smem_u32(S.wlo) + sl * kTcSlab, 128, 256);
            const uint64_t bh = umma::smem_desc_kmajor(umma::smem_u32(S.bhi) + sl * kTcSlab, 128, 256);
            const uint64_t bl = umma::smem_desc_kmajor(umma::smem_u32(S.blo) + sl * kTcSlab, 128, 256);
            umma::mma_tf32_masked(tbase, ah, bh, idesc, sl > 0, dis);
            umma::mma_tf32_masked(tbase, ah, bl, idesc, true, dis);
            umma::mma_tf32_masked(tbase, al, bh, idesc, true, dis);
          }
          umma::mma_commit(&S.mbar);
        }
        __syncwarp();
        if (!umma::mbar_wait(&S.mbar, phase, kTcWaitIters)) S.bad = 1;
        phase ^= 1;
        umma::fence_after_sync();
        FX_TOC(tq, 3);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < 2 * np) umma::tmem_st1(trow + S.pidx[j], __float_as_uint(pv[j]));
        umma::tmem_wait_st();
        tc_sync();
        FX_TOC(tq, 4);
      }
      // the panel's pivots are swept now
      S.isP[x] = 0;
      __syncthreads();
      FX_TOC(tq, 12);
    }

    // ---- (sign, logabs) from the pivots, warp 0 in a fixed order
    if (warp == 0) {
      float sg = 1.f;
      KSum<float> ls;
      ls.init();
      int nz = 0;
      for (int k = lane; k < npairs; k += 32) {
        const float d = S.dvec[k];
        sg *= d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f);
        ls.add(logf(fabsf(d)));
        nz += d == 0.f;
      }
      float lsum = ls.value();
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        sg *= __shfl_xor_sync(0xffffffffu, sg, off);
        lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
        nz += __shfl_xor_sync(0xffffffffu, nz, off);
      }
      if (lane == 0) {
        if (S.parity) sg = -sg;
        if (nz) sg = 0.f;
        const float la = nz ? -INFINITY : lsum;
        J.sign[b] = S.bad ? __int_as_float(0x7fc00000) : sg;
        J.logabs[b] = S.bad ? __int_as_float(0x7fc00000) : la;
        if (J.value) J.value[b] = sg * expf(la);
        S.cand_f[0] = nz;  // reused below as the singular flag
      }
    }
    __syncthreads();
    if (GRAD) {
      // TMEM = -S^-1: gradient of sum(logabs) = -S^-1 / 2, scaled by coef
      const bool zero = S.cand_f[0] != 0 || S.bad;
      const float f = 0.5f * (J.coef ? J.coef[b] : 1.f);
      tc_store_rows(J.g + b * (int64_t)n * n, n, f, zero, trow, x);
    }
    tc_sync();
    FX_TOC(tq, 13);
  }
  if (warp == 0) umma::tmem_dealloc(tbase, kTcN);
}

}  // namespace fx
