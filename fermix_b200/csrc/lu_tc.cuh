// Tensor-memory resident Gauss-Jordan LU for float32 slogdet, 8 <= n <= 128,
// prec = "tf32x3": forward (sign, logabs) and, in the same pass, A^-1 for the gradient.
//
// Reference behaviour: LU with partial pivoting (largest |entry| of the current column
// among the rows not yet pivoted, first occurrence on ties) as in src/fermix/_lu.py:51-120
// (panel) and :153-217 (blocked trailing update), sign / log|det| from the pivots and the
// row permutation as in src/fermix/_lu.py:543-611; trailing updates with the tf32x3
// products of src/fermix/_field.py:173-190; gradient A^-T of _lu_parts
// (src/fermix/_inverse.py:502-531), zero for an exactly singular member.
//
// Design (B200). Thread x of the 128-thread block owns row x = TMEM lane x; the matrix
// stays in TMEM (128 columns) for the whole call and rows are never moved (virtual
// pivoting). Per panel of 16 columns:
//   1. every row reads its 16 panel entries into registers and the panel is factored
//      there: per column one warp argmax, one block barrier (each warp's candidate row
//      travels with its candidate value), then every other row eliminates;
//   2. with P the panel's pivot rows, K its columns and l_x row x's multipliers, the
//      block exchange of (P, K) is ONE rank-16 tensor-core update D -= C B^T:
//        C_x = l_x L11^-1            (x not in P; back substitution, so that a row equal
//                                     to pivot row P_s gets exactly e_s),
//        C_{P_j} = e_j + (A_PK^-1)_j (gradient mode; 0 in forward mode),
//        B_y = A_{P,y} (y not in K), B_{K_t} = -e_t,
//      after the K columns are preset to 0 (rows not in P) / -e_j (row P_j). Sweeping all
//      panels leaves TMEM[p_s][t] = (A^-1)[s][p_t], p_s the row pivoted at step s. The
//      forward-only mode skips the presets and the pivot-row coefficients; the rows not
//      yet pivoted evolve identically, so its (sign, logabs) are bit-identical.
// B is split three ways (hi + mid + lo == value exactly) and the update uses the
// products hi*hi + hi*mid + hi*lo + lo*hi: a row that duplicates a pivot row therefore
// cancels to exact zeros, and duplicated rows give an exactly zero pivot as in the
// sequential elimination.
#pragma once
#include "fused_lu.cuh"
#include "tc_common.cuh"

namespace fx {

struct __align__(16) LuTcCand {
  float absv;     // candidate |value| (-1: no candidate in this warp)
  int idx;        // candidate row
  unsigned live;  // ballot of this warp's rows not yet pivoted
  int pad;
  float row[16];  // the candidate's current panel entries
};

constexpr int kProwLd = kTcN + 4;  // staged pivot rows: 16-byte rows, conflict-free column reads

struct LuTcSmem {
  float chi[kTcN * 16], clo[kTcN * 16];                   // A operand C, K-major, TF32 hi / lo
  float bhi[kTcN * 16], bmid[kTcN * 16], blo[kTcN * 16];  // B operand, K-major, exact 3-way split
  float prow[16][kProwLd];                                // the panel's pivot rows (TMEM values)
  LuTcCand cand[2][4];                                    // per-warp candidates, by step parity
  float L11[16][17];                                      // panel multipliers of the pivot rows
  float U11[16][17];                                      // panel pivot rows (gradient mode)
  float dvec[kTcN];                                       // pivots
  int at[kTcN];                                           // pivot position -> row
  int wpar[4];                                            // per-warp parity of inversions
  uint32_t tslot;
  int bad;
  uint64_t mbar;
};

// value == hi + mid + lo exactly, each part a TF32 number (hi, mid round to nearest)
__device__ __forceinline__ void split3(float v, float& hi, float& mid, float& lo) {
  hi = umma::tf32_round(v);
  const float r = v - hi;
  mid = umma::tf32_round(r);
  lo = r - mid;
}

template <bool GRAD>
__global__ void __launch_bounds__(128) lu_tc_kernel(Job<float> J) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  LuTcSmem& S = *reinterpret_cast<LuTcSmem*>(smem_raw);
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
  const uint32_t tbase = S.tslot;
  const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);
  uint32_t phase = 0;

  for (int64_t b = blockIdx.x; b < J.B; b += gridDim.x) {
    const float* src = J.a + b * (int64_t)n * n;
    if (tid == 0 && b + gridDim.x < J.B) tc_prefetch_l2(src + (int64_t)gridDim.x * n * n, n);
    tc_load_matrix(src, n, false, trow, x);
    int mypos = x < n ? -1 : kTcN;  // pivot position of this row (-1: not yet pivoted)
    int myinv = 0;                  // rows of smaller index still unpivoted when this one was
    if (tid == 0) S.bad = 0;
    tc_sync();

    for (int k0 = 0; k0 < n; k0 += 16) {
      const int kw = min(16, n - k0);
      float pr[16], lr[16];
      {
        uint32_t t0[8], t1[8];
        umma::tmem_ld8(trow + k0, t0);
        umma::tmem_ld8(trow + k0 + 8, t1);
        umma::tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          pr[t] = __uint_as_float(t0[t]);
          pr[t + 8] = __uint_as_float(t1[t]);
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) lr[t] = 0.f;
      }
      // ---- panel factorisation in registers
#pragma unroll
      for (int s = 0; s < 16; ++s) {
        if (s < kw) {
          const bool live = mypos < 0;
          const float v = pr[s];
          float best = live ? (v != v ? -0.5f : fabsf(v)) : -1.f;  // NaN: live, never preferred
          int bi = live ? x : 0x7fffffff;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ob > best || (ob == best && oi < bi)) {
              best = ob;
              bi = oi;
            }
          }
          const unsigned lm = __ballot_sync(0xffffffffu, live);
          LuTcCand& mine = S.cand[s & 1][warp];
          if (x == bi) {
            mine.absv = best;
            mine.idx = bi;
            float4* r4 = reinterpret_cast<float4*>(mine.row);
#pragma unroll
            for (int q = 0; q < 4; ++q) r4[q] = make_float4(pr[4 * q], pr[4 * q + 1], pr[4 * q + 2], pr[4 * q + 3]);
          }
          if (lane == 0) {
            mine.live = lm;
            if (bi == 0x7fffffff) {
              mine.absv = -1.f;
              mine.idx = 0x7fffffff;
            }
          }
          __syncthreads();
          int pw = 0;
          float pb = S.cand[s & 1][0].absv;
          int p = S.cand[s & 1][0].idx;
#pragma unroll
          for (int w = 1; w < 4; ++w) {
            const float ob = S.cand[s & 1][w].absv;
            const int oi = S.cand[s & 1][w].idx;
            if (ob > pb || (ob == pb && oi < p)) {
              pb = ob;
              p = oi;
              pw = w;
            }
          }
          float ur[16];
          {
            const float4* r4 = reinterpret_cast<const float4*>(S.cand[s & 1][pw].row);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 t = r4[q];
              ur[4 * q] = t.x;
              ur[4 * q + 1] = t.y;
              ur[4 * q + 2] = t.z;
              ur[4 * q + 3] = t.w;
            }
          }
          const float piv = ur[s];
          if (x == p) {
            mypos = k0 + s;
            int cnt = __popc(S.cand[s & 1][warp].live & ((1u << lane) - 1u));
#pragma unroll
            for (int w = 0; w < 4; ++w)
              if (w < warp) cnt += __popc(S.cand[s & 1][w].live);
            myinv = cnt & 1;
            S.dvec[k0 + s] = piv;
            S.at[k0 + s] = x;
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              if (t < s) S.L11[s][t] = lr[t];
              if (GRAD && t >= s) S.U11[s][t] = pr[t];
            }
          } else if (x < n && mypos < k0) {
            // every row outside this panel's pivots eliminates (rows pivoted in earlier
            // panels too: gradient mode needs their multipliers)
            const float l = piv == 0.f ? 0.f : __fdiv_rn(v, piv);
            lr[s] = l;
#pragma unroll
            for (int t = 0; t < 16; ++t)
              if (t > s) pr[t] = fmaf(-l, ur[t], pr[t]);
          }
        }
      }
      __syncthreads();  // L11 / U11 / at complete
      const bool inP = mypos >= k0 && mypos < kTcN;
      // ---- the pivot rows' current TMEM values into prow (warps holding pivot rows)
      if (__ballot_sync(0xffffffffu, inP) != 0u) {
        const int tp = mypos - k0;
#pragma unroll 1
        for (int c0 = 0; c0 < kTcN; c0 += 32) {
          uint32_t w[32];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t t8[8];
            umma::tmem_ld8(trow + c0 + 8 * q, t8);
#pragma unroll
            for (int e = 0; e < 8; ++e) w[8 * q + e] = t8[e];
          }
          umma::tmem_wait_ld();
          if (inP) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *reinterpret_cast<float4*>(&S.prow[tp][c0 + 4 * q]) =
                  make_float4(__uint_as_float(w[4 * q]), __uint_as_float(w[4 * q + 1]), __uint_as_float(w[4 * q + 2]),
                              __uint_as_float(w[4 * q + 3]));
          }
        }
      }

      // ---- coefficients C_x (A operand), K-major, hi / lo
      float c[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) c[t] = 0.f;
      if (x < n) {
        if (inP) {
          if (GRAD) {
            // row j of A_PK^-1 = (e_j U11^-1) L11^-1, then + e_j
            const int j = mypos - k0;
            float w[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              float acc = (t == j) ? 1.f : 0.f;
#pragma unroll
              for (int r = 0; r < 16; ++r)
                if (r < t) acc = fmaf(-w[r], S.U11[r][t], acc);
              w[t] = (t < kw && t >= j) ? __fdiv_rn(acc, S.U11[t][t]) : 0.f;
            }
#pragma unroll
            for (int t = 15; t >= 0; --t) {
              float acc = w[t];
#pragma unroll
              for (int r = 0; r < 16; ++r)
                if (r > t && r < kw) acc = fmaf(-c[r], S.L11[r][t], acc);
              c[t] = t < kw ? acc : 0.f;
            }
#pragma unroll
            for (int t = 0; t < 16; ++t)
              if (t == j) c[t] += 1.f;
          }
        } else if (GRAD || mypos < 0) {
          // C_x L11 = l_x, by back substitution (increasing r inside each sum)
#pragma unroll
          for (int t = 15; t >= 0; --t) {
            float acc = lr[t];
#pragma unroll
            for (int r = 0; r < 16; ++r)
              if (r > t && r < kw) acc = fmaf(-c[r], S.L11[r][t], acc);
            c[t] = t < kw ? acc : 0.f;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t off = umma::kmajor_offset(x, 4 * q, kTcSlab) / 4;
        float h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          h[e] = umma::tf32_round(c[4 * q + e]);
          l[e] = umma::tf32_round(c[4 * q + e] - h[e]);
        }
        *reinterpret_cast<float4*>(&S.chi[off]) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4*>(&S.clo[off]) = make_float4(l[0], l[1], l[2], l[3]);
      }
      __syncthreads();  // staged pivot rows complete
      // ---- B operand (K-major): column y = x of the pivot rows, -e_t on the panel columns
      {
        const int y = x;
        float v[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          v[t] = t < kw ? S.prow[t][y] : 0.f;
          if (y >= k0 && y < k0 + kw) v[t] = (t < kw && y - k0 == t) ? -1.f : 0.f;
          if (y >= n) v[t] = 0.f;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t off = umma::kmajor_offset(y, 4 * q, kTcSlab) / 4;
          float h[4], m[4], l[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) split3(v[4 * q + e], h[e], m[e], l[e]);
          *reinterpret_cast<float4*>(&S.bhi[off]) = make_float4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<float4*>(&S.bmid[off]) = make_float4(m[0], m[1], m[2], m[3]);
          *reinterpret_cast<float4*>(&S.blo[off]) = make_float4(l[0], l[1], l[2], l[3]);
        }
      }
      if (GRAD) {
        // the panel columns become the exchanged block: preset 0 (rows outside P) or
        // -e_j (pivot row P_j), the update then adds C
        uint32_t z0[8], z1[8];
        const int j = inP ? mypos - k0 : -1;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          z0[t] = __float_as_uint(t == j ? -1.f : 0.f);
          z1[t] = __float_as_uint(t + 8 == j ? -1.f : 0.f);
        }
        umma::tmem_st8(trow + k0, z0);
        umma::tmem_st8(trow + k0 + 8, z1);
        umma::tmem_wait_st();
      }
      umma::fence_proxy_async_smem();
      tc_sync();
      if (tid == 0) {
        const uint32_t idesc = umma::idesc_tf32(kTcN, kTcN, true);  // D -= C B^T
#pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
          const uint64_t ah = umma::smem_desc_kmajor(umma::smem_u32(S.chi) + sl * kTcSlab, 128, 256);
          const uint64_t al = umma::smem_desc_kmajor(umma::smem_u32(S.clo) + sl * kTcSlab, 128, 256);
          const uint64_t bh = umma::smem_desc_kmajor(umma::smem_u32(S.bhi) + sl * kTcSlab, 128, 256);
          const uint64_t bm = umma::smem_desc_kmajor(umma::smem_u32(S.bmid) + sl * kTcSlab, 128, 256);
          const uint64_t bl = umma::smem_desc_kmajor(umma::smem_u32(S.blo) + sl * kTcSlab, 128, 256);
          umma::mma_tf32(tbase, ah, bh, idesc, true);
          umma::mma_tf32(tbase, ah, bm, idesc, true);
          umma::mma_tf32(tbase, ah, bl, idesc, true);
          umma::mma_tf32(tbase, al, bh, idesc, true);
        }
        umma::mma_commit(&S.mbar);
      }
      __syncwarp();
      if (!umma::mbar_wait(&S.mbar, phase, kTcWaitIters)) S.bad = 1;
      phase ^= 1;
      umma::fence_after_sync();
      __syncthreads();  // operand buffers free again
    }

    // ---- (sign, logabs): pivots in a fixed order (warp 0), permutation parity from the
    // per-row inversion counts
    {
      const unsigned pm = __ballot_sync(0xffffffffu, myinv != 0);
      if (lane == 0) S.wpar[warp] = __popc(pm) & 1;
    }
    __syncthreads();
    if (warp == 0) {
      float sg = 1.f;
      KSum<float> ls;
      ls.init();
      int nz = 0;
      for (int k = lane; k < n; k += 32) {
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
        if ((S.wpar[0] ^ S.wpar[1] ^ S.wpar[2] ^ S.wpar[3]) & 1) sg = -sg;
        if (nz) sg = 0.f;
        const float la = nz ? -INFINITY : lsum;
        J.sign[b] = S.bad ? __int_as_float(0x7fc00000) : sg;
        J.logabs[b] = S.bad ? __int_as_float(0x7fc00000) : la;
        if (J.value) J.value[b] = sg * expf(la);
        S.wpar[0] = nz;  // reused below as the singular flag
      }
    }
    __syncthreads();
    if (GRAD) {
      // TMEM[p_s][t] = (A^-1)[s][p_t] = grad[p_t][s]: row x writes column mypos of the
      // gradient at rows at[t] (each warp store covers one gradient row)
      const bool zero = S.wpar[0] != 0 || S.bad;
      const float f = J.coef ? J.coef[b] : 1.f;
      float* G = J.g + b * (int64_t)n * n;
#pragma unroll 1
      for (int c0 = 0; c0 < n; c0 += 32) {
        uint32_t w[32];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t t8[8];
          umma::tmem_ld8(trow + c0 + 8 * q, t8);
#pragma unroll
          for (int e = 0; e < 8; ++e) w[8 * q + e] = t8[e];
        }
        umma::tmem_wait_ld();
        if (x < n) {
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (c0 + k < n) G[(int64_t)S.at[c0 + k] * n + mypos] = zero ? 0.f : f * __uint_as_float(w[k]);
        }
      }
    }
    tc_sync();
  }
  if (warp == 0) umma::tmem_dealloc(tbase, kTcN);
}

}  // namespace fx
