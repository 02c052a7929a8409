// Tensor-memory resident Gauss-Jordan LU for float32 slogdet, 8 <= n <= 256: forward
// (sign, logabs) and, in the same pass, A^-1 for the gradient; prec = "tf32x3" (tensor-core
// block updates) or "ieee" (IEEE float32 FMA block updates, template flag IEEE).
//
// Reference behaviour: LU with partial pivoting (largest |entry| of the current column
// among the rows not yet pivoted, first occurrence on ties) as in src/fermix/_lu.py:51-120
// (panel) and :153-217 (blocked trailing update), sign / log|det| from the pivots and the
// row permutation as in src/fermix/_lu.py:543-611; trailing updates with the tf32x3
// products of src/fermix/_field.py:173-190; gradient A^-T of _lu_parts
// (src/fermix/_inverse.py:502-531), zero for an exactly singular member.
//
// Design (B200). Thread x of the NR-thread block owns row x; the matrix stays in TMEM for
// the whole call and rows are never moved (virtual pivoting). NR = 128: row x = lane x,
// 128 columns, four blocks per SM. NR = 256 (129 <= n <= 256): the matrix fills the SM's
// whole TMEM, row x in lane x % 128 at column offset 256 (x / 128), one block per SM and
// two M = 128, N = 256 MMAs per product. Per panel of 16 columns:
//   1. every row reads its 16 panel entries into registers and the panel is factored
//      there: per column a two-instruction warp argmax (redux.sync on a packed |value|
//      key, then on the row index), ONE block barrier (each warp's candidate row
//      travels with its key), then every other row eliminates;
//   2. with P the panel's pivot rows, K its columns and l_x row x's multipliers, the
//      block exchange of (P, K) is ONE rank-16 tensor-core update D -= C B^T:
//        C_x = l_x L11^-1            (x not in P; back substitution, so that a row equal
//                                     to pivot row P_s gets exactly e_s),
//        C_{P_j} = e_j + (A_PK^-1)_j (gradient mode; 0 in forward mode),
//        B_y = A_{P,y} (y not in K), B_{K_t} = -e_t,
//      after the K columns are preset to 0 (rows not in P) / -e_j (row P_j). Sweeping all
//      panels leaves TMEM[p_s][t] = (A^-1)[s][p_t], p_s the row pivoted at step s. The
//      forward-only mode skips the presets, the pivot-row coefficients and the rows
//      pivoted earlier; the rows not yet pivoted evolve identically, so its
//      (sign, logabs) are bit-identical.
// B is split three ways (hi + mid + lo == value exactly) and the update uses the
// products hi*hi + hi*mid + hi*lo + lo*hi: a row that duplicates a pivot row therefore
// cancels to exact zeros, and duplicated rows give an exactly zero pivot as in the
// sequential elimination.
#pragma once
#include "fused_lu.cuh"
#include "tc_common.cuh"

namespace fx {

template <int NR>
struct LuTcSmemT {
  static constexpr int NW = NR / 32;
  float chi[NR * 16], clo[NR * 16];                 // A operand C, K-major, TF32 hi / lo
  float bhi[NR * 16], bmid[NR * 16], blo[NR * 16];  // B operand, K-major, exact 3-way split
  // per-warp pivot candidates by step parity: packed order key (|value| key << 32 | ~row:
  // the largest key, then the smallest row, is the largest number), the reciprocal of the
  // candidate's pivot value and its panel entries
  __align__(16) unsigned long long ckey[2][NW];
  float cinv[2][NW];
  unsigned clm[16][NW];  // the warps' unpivoted rows at each pivot step of the panel
  __align__(16) float crow[2][NW][16];
  float prow[16][NR + 4];                           // the panel's pivot rows (16-byte rows, conflict-free columns)
  __align__(16) float L11[16][20];                  // multipliers of the pivot rows (strict lower part, 16-byte rows)
  float U11[16][17];                                // the pivot rows' panel entries (upper part)
  float Linv[16][17];                               // L11^-1 (gradient mode)
  float Uinv[16][17];                               // U11^-1 (gradient mode)
  __align__(16) float Ainv[16][20];                 // A_PK^-1 = U11^-1 L11^-1 (gradient mode, 16-byte rows)
  float dvec[NR];                                   // pivots
  int at[NR];                                       // pivot position -> row
  int wpar[NW];                                     // per-warp parity of the inversions
  uint32_t tslot;
  int bad, nz;
  uint64_t mbar;
};
using LuTcSmem = LuTcSmemT<128>;

// prec ieee: B's rows (16 values, 80-byte rows: conflict-free 16-byte stores) in the space of
// the tensor-core operands chi / clo, which that mode does not use
template <int NR>
__device__ __forceinline__ float (*lu_tc_brow(LuTcSmemT<NR>& S))[20] {
  static_assert(sizeof(float) * NR * 20 <= 2 * sizeof(S.chi), "brow fits chi + clo");
  return reinterpret_cast<float (*)[20]>(S.chi);
}

// value == hi + mid + lo exactly, each part a TF32 number (hi, mid round to nearest)
__device__ __forceinline__ void split3(float v, float& hi, float& mid, float& lo) {
  hi = umma::tf32_round(v);
  const float r = v - hi;
  mid = umma::tf32_round(r);
  lo = r - mid;
}


// prec ieee: D -= C B^T on this thread's TMEM row with IEEE float32 FMAs (one sequential chain
// per entry over the panel's 16 columns), C = this row's coefficients, B's rows (brow, 80-byte
// rows in the space of the tensor-core operands) broadcast from shared memory; 16 columns per
// TMEM round trip, from column c_lo on.
template <int NR>
__device__ __forceinline__ void lu_tc_fma_update(const float (*brow)[20], uint32_t trow, int n, int c_lo,
                                                 const float (&c)[16]) {
#pragma unroll 1
  for (int c0 = c_lo & ~15; c0 < n; c0 += 16) {
    uint32_t w0[8], w1[8];
    umma::tmem_ld8(trow + c0, w0);
    umma::tmem_ld8(trow + c0 + 8, w1);
    umma::tmem_wait_ld();
    float v[16];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[e] = __uint_as_float(w0[e]);
      v[e + 8] = __uint_as_float(w1[e]);
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      if (c0 + e < n) {
        const float4* b4 = reinterpret_cast<const float4*>(brow[c0 + e]);
        float acc = v[e];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 b = b4[q];
          acc = fmaf(-c[4 * q], b.x, acc);
          acc = fmaf(-c[4 * q + 1], b.y, acc);
          acc = fmaf(-c[4 * q + 2], b.z, acc);
          acc = fmaf(-c[4 * q + 3], b.w, acc);
        }
        v[e] = acc;
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      w0[e] = __float_as_uint(v[e]);
      w1[e] = __float_as_uint(v[e + 8]);
    }
    umma::tmem_st8(trow + c0, w0);
    umma::tmem_st8(trow + c0 + 8, w1);
  }
  umma::tmem_wait_st();
}

template <int NR, bool GRAD, bool IEEE = false>
__global__ void __launch_bounds__(NR, NR == 128 ? 4 : 1) lu_tc_kernel(Job<float> J) {
  constexpr int NW = NR / 32;
  constexpr uint32_t kCols = NR == 128 ? 128u : 512u;  // TMEM columns allocated
  constexpr uint32_t kSlab = NR * 8 * 4;                 // bytes of one K = 8 slab of an NR-row operand
  extern __shared__ __align__(16) unsigned char smem_raw[];
  LuTcSmemT<NR>& S = *reinterpret_cast<LuTcSmemT<NR>*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = J.n;
  const int x = tid;  // this thread's row
  if (warp == 0) {
    umma::tmem_alloc(&S.tslot, kCols);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    umma::mbar_init(&S.mbar, 1);
    umma::fence_mbar_init();
  }
  tc_sync();
  const uint32_t tbase = S.tslot;
  // this warp's 32 lanes; rows 128..255 sit 256 columns further right
  const uint32_t trow = tbase + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(warp >> 2) * 256u;
  uint32_t phase = 0;

  for (int64_t b = blockIdx.x; b < J.B; b += gridDim.x) {
    FX_TIC(tq);
    if (J.gidx) {
      tc_load_gathered<NR>(J.gbase, J.gld, J.grows, J.gidx + b * (int64_t)n, n, trow, x);
    } else {
      const float* src = J.a + b * (int64_t)n * n;
      // the forward streams the block's next matrix into L2 meanwhile; the gradient does not
      // (measured: the gradient writes evicted most prefetched lines before use, reading the
      // input twice from DRAM)
      if (!GRAD && tid == 0 && b + gridDim.x < J.B) tc_prefetch_l2(src + (int64_t)gridDim.x * n * n, n);
      tc_load_matrix<NR>(src, n, false, trow, x);
    }
    int mypos = x < n ? -1 : NR;  // pivot position of this row (-1: not yet pivoted)
    int myinv = 0;                  // parity of the inversions this row adds as a pivot
    if (tid == 0) S.bad = 0;
    tc_sync();
    FX_TOC(tq, 0);

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
      // ---- panel factorisation in registers, one block barrier per column
#pragma unroll
      for (int s = 0; s < 16; ++s) {
        if (s < kw) {
          const bool live = mypos < 0;
          const float v = pr[s];
          const unsigned key = piv_key(v, live);
          // every lane forms its reciprocal while the reductions run (only the winner's is kept)
          const float vinv = v == 0.f ? 0.f : __frcp_rn(v);
          const unsigned km = __reduce_max_sync(0xffffffffu, key);
          // the first lane holding the largest key: the smallest row
          const int wi = (warp << 5) + __ffs(__ballot_sync(0xffffffffu, key == km)) - 1;
          const unsigned lm = __ballot_sync(0xffffffffu, live);
          if (x == wi) {
            // this warp's candidate (key 0: the warp has no unpivoted row left)
            S.ckey[s & 1][warp] = ((unsigned long long)km << 32) | (unsigned)~wi;
            S.clm[s][warp] = lm;
            S.cinv[s & 1][warp] = vinv;
            float4* r4 = reinterpret_cast<float4*>(S.crow[s & 1][warp]);
#pragma unroll
            for (int q = 0; q < 4; ++q) r4[q] = make_float4(pr[4 * q], pr[4 * q + 1], pr[4 * q + 2], pr[4 * q + 3]);
          }
          __syncthreads();
          unsigned long long best;
          {
            const ulonglong2* k2 = reinterpret_cast<const ulonglong2*>(S.ckey[s & 1]);
            const ulonglong2 k01 = k2[0];
            best = k01.x > k01.y ? k01.x : k01.y;
#pragma unroll
            for (int w = 1; w < NW / 2; ++w) {
              const ulonglong2 kw2 = k2[w];
              const unsigned long long m = kw2.x > kw2.y ? kw2.x : kw2.y;
              best = m > best ? m : best;
            }
          }
          const int p = (int)~(unsigned)best;  // the pivot row, owned by warp p / 32
          const int pw = p >> 5;
          float ur[16];
          {
            const float4* r4 = reinterpret_cast<const float4*>(S.crow[s & 1][pw]);
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
          const float inv = S.cinv[s & 1][pw];
          if (x == p) {
            mypos = k0 + s;
            S.dvec[k0 + s] = piv;
            S.at[k0 + s] = x;
          } else if (x < n && (GRAD ? mypos < k0 : mypos < 0)) {
            // rows outside this panel's pivots eliminate (gradient mode: rows pivoted in
            // earlier panels too, for their multipliers); the multiplier is v times the
            // guarded reciprocal pivot as in the reference (src/fermix/_lu.py:170-173),
            // exactly +-1 for a row equal to +-(the pivot row's entry), so that duplicated
            // rows cancel to exact zeros
            const float l = piv == 0.f ? 0.f : (v == piv ? 1.f : (v == -piv ? -1.f : v * inv));
            lr[s] = l;
#pragma unroll
            for (int t = 0; t < 16; ++t)
              if (t > s) pr[t] = fmaf(-l, ur[t], pr[t]);
          }
        }
      }
      const bool inP = mypos >= k0 && mypos < k0 + kw;
      if (inP) {
        // a pivot row keeps its multipliers (L11 row, zero from the diagonal on) and its
        // remaining entries (U11 row), and counts the inversions it added: the rows of
        // smaller index still unpivoted at its step (the warps' ballots recorded then)
        const int j = mypos - k0;
        int cnt = __popc(S.clm[j][warp] & ((1u << lane) - 1u));
#pragma unroll
        for (int w = 0; w < NW; ++w)
          if (w < warp) cnt += __popc(S.clm[j][w]);
        myinv = cnt & 1;
        float4* l4 = reinterpret_cast<float4*>(S.L11[j]);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          l4[q] = make_float4(4 * q < j ? lr[4 * q] : 0.f, 4 * q + 1 < j ? lr[4 * q + 1] : 0.f,
                              4 * q + 2 < j ? lr[4 * q + 2] : 0.f, 4 * q + 3 < j ? lr[4 * q + 3] : 0.f);
        if (GRAD) {
#pragma unroll
          for (int t = 0; t < 16; ++t)
            if (t >= j) S.U11[j][t] = pr[t];
        }
      }
      __syncthreads();  // L11 / U11 / at complete
      FX_TOC(tq, 1);
      if (GRAD) {
        // L11^-1 by columns (warp 2) and U11^-1 by rows (warp 3), lanes < kw
        if (warp == 2 && lane < kw) {
          const int t = lane;
          float y[16];
#pragma unroll
          for (int r = 0; r < 16; ++r) {
            float acc = r == t ? 1.f : 0.f;
#pragma unroll
            for (int q = 0; q < 16; ++q)
              if (q < r) acc = fmaf(-S.L11[r][q], y[q], acc);
            y[r] = (r >= t && r < kw) ? acc : 0.f;
            S.Linv[r][t] = y[r];
          }
        } else if (warp == 3 && lane < kw) {
          const int j = lane;
          float w[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            float acc = t == j ? 1.f : 0.f;
#pragma unroll
            for (int r = 0; r < 16; ++r)
              if (r < t) acc = fmaf(-w[r], S.U11[r][t], acc);
            w[t] = (t >= j && t < kw) ? __fdiv_rn(acc, S.U11[t][t]) : 0.f;
            S.Uinv[j][t] = w[t];
          }
        }
      }
      // ---- the pivot rows' current TMEM values into prow (warps holding pivot rows;
      // forward mode: trailing columns only)
      if (__ballot_sync(0xffffffffu, inP) != 0u) {
        const int tp = mypos - k0;
#pragma unroll 1
        for (int c0 = GRAD ? 0 : ((k0 + kw) & ~31); c0 < NR; c0 += 32) {
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
      // ---- coefficients of the rows outside P: C_x L11 = l_x by back substitution
      // (increasing r inside each sum)
      float c[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) c[t] = 0.f;
      if (x < n && !inP && (GRAD || mypos < 0)) {
        // c = l L11^-1 column by column from the last: c[r] is final once the rows below
        // it are applied, then it is removed from the earlier entries with L11's row r
        // (16-byte broadcast reads)
#pragma unroll
        for (int t = 0; t < 16; ++t) c[t] = t < kw ? lr[t] : 0.f;
#pragma unroll
        for (int r = 15; r >= 1; --r) {
          if (r < kw) {
            const float cr = c[r];
            const float4* l4 = reinterpret_cast<const float4*>(S.L11[r]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (4 * q < r) {
                const float4 L = l4[q];
                const float lv[4] = {L.x, L.y, L.z, L.w};
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  if (4 * q + e < r) c[4 * q + e] = fmaf(-cr, lv[e], c[4 * q + e]);
              }
            }
          }
        }
      }
      FX_TOC(tq, 2);
      __syncthreads();  // prow, Linv, Uinv complete; the panel buffer is free
      if (GRAD) {
        // A_PK^-1 = U11^-1 L11^-1 by the whole block (256 entries), then each pivot row
        // reads its row and adds e_j
        for (int e = tid; e < 256; e += NR) {
          const int j = e >> 4, t = e & 15;
          float acc = 0.f;
#pragma unroll
          for (int r = 0; r < 16; ++r)
            if (r >= t && r < kw) acc = fmaf(S.Uinv[j][r], S.Linv[r][t], acc);
          S.Ainv[j][t] = (j < kw && t < kw) ? acc : 0.f;
        }
        __syncthreads();
        if (inP) {
          const int j = mypos - k0;
          const float4* r4 = reinterpret_cast<const float4*>(S.Ainv[j]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 v = r4[q];
            c[4 * q] = v.x;
            c[4 * q + 1] = v.y;
            c[4 * q + 2] = v.z;
            c[4 * q + 3] = v.w;
          }
#pragma unroll
          for (int t = 0; t < 16; ++t)
            if (t == j) c[t] += 1.f;
        }
      }
      if (!IEEE) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t off = umma::kmajor_offset(x, 4 * q, kSlab) / 4;
          float h[4], l[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            h[e] = umma::tf32_round(c[4 * q + e]);
            l[e] = umma::tf32_round(c[4 * q + e] - h[e]);
          }
          *reinterpret_cast<float4*>(&S.chi[off]) = make_float4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<float4*>(&S.clo[off]) = make_float4(l[0], l[1], l[2], l[3]);
        }
      }
      // ---- B operand (K-major): column y = x of the pivot rows, -e_t on the panel
      // columns (forward mode: the columns up to the panel's end stay zero)
      {
        const int y = x;
        const bool zero_col = y >= n || (!GRAD && y < k0 + kw);
        float v[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          v[t] = t < kw ? S.prow[t][y] : 0.f;
          if (y >= k0 && y < k0 + kw) v[t] = (t < kw && y - k0 == t) ? -1.f : 0.f;
          if (zero_col) v[t] = 0.f;
        }
        if (IEEE) {
          // row y of B for the FMA update, unsplit
          float4* b4 = reinterpret_cast<float4*>(lu_tc_brow<NR>(S)[y]);
#pragma unroll
          for (int q = 0; q < 4; ++q) b4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t off = umma::kmajor_offset(y, 4 * q, kSlab) / 4;
            float h[4], m[4], l[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) split3(v[4 * q + e], h[e], m[e], l[e]);
            *reinterpret_cast<float4*>(&S.bhi[off]) = make_float4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<float4*>(&S.bmid[off]) = make_float4(m[0], m[1], m[2], m[3]);
            *reinterpret_cast<float4*>(&S.blo[off]) = make_float4(l[0], l[1], l[2], l[3]);
          }
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
      FX_TOC(tq, 3);
      if (IEEE) {
        // the rows that the update changes: every row in gradient mode, the unpivoted ones in
        // the forward (whose coefficients of pivoted rows are zero); the forward's columns
        // before the panel's end stay as they are (B is zero there)
        if ((GRAD || k0 + kw < n) && __any_sync(0xffffffffu, x < n && (GRAD || mypos < 0)))
          lu_tc_fma_update<NR>(lu_tc_brow<NR>(S), trow, n, GRAD ? 0 : k0 + kw, c);
      } else if (GRAD || k0 + kw < n) {
        if (tid == 0) {
          const uint32_t idesc = umma::idesc_tf32(128, NR, true);  // D -= C B^T, M = 128, N = NR
#pragma unroll
          for (int h = 0; h < NR / 128; ++h) {  // row halves: rows 128 h .. 128 h + 127
#pragma unroll
            for (int sl = 0; sl < 2; ++sl) {
              const uint32_t ao = sl * kSlab + h * 4096u;
              const uint64_t ah = umma::smem_desc_kmajor(umma::smem_u32(S.chi) + ao, 128, 256);
              const uint64_t al = umma::smem_desc_kmajor(umma::smem_u32(S.clo) + ao, 128, 256);
              const uint64_t bh = umma::smem_desc_kmajor(umma::smem_u32(S.bhi) + sl * kSlab, 128, 256);
              const uint64_t bm = umma::smem_desc_kmajor(umma::smem_u32(S.bmid) + sl * kSlab, 128, 256);
              const uint64_t bl = umma::smem_desc_kmajor(umma::smem_u32(S.blo) + sl * kSlab, 128, 256);
              const uint32_t d = tbase + h * 256u;
              umma::mma_tf32(d, ah, bh, idesc, true);
              umma::mma_tf32(d, ah, bm, idesc, true);
              umma::mma_tf32(d, ah, bl, idesc, true);
              umma::mma_tf32(d, al, bh, idesc, true);
            }
          }
          umma::mma_commit(&S.mbar);
        }
        __syncwarp();
        if (!umma::mbar_wait(&S.mbar, phase, J.wait_polls)) {
          // give up on this member (NaN outputs, the status word records the timeout), but
          // wait once more, with the default limit, so that no MMA is still in flight when
          // the threads touch its operands, TMEM or the tensor memory allocation again
          S.bad = 1;
          (void)umma::mbar_wait(&S.mbar, phase, kTcWaitIters);
        }
        phase ^= 1;
        umma::fence_after_sync();
      }
      FX_TOC(tq, 4);
    }

    // ---- (sign, logabs): pivots in a fixed order (warp 0) and the permutation parity
    {
      const unsigned pm = __ballot_sync(0xffffffffu, myinv != 0);
      if (lane == 0) S.wpar[warp] = __popc(pm) & 1;
    }
    int par = 0;
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
        for (int w = 0; w < NW; ++w) par ^= S.wpar[w];
        if (par & 1) sg = -sg;
        if (nz) sg = 0.f;
        const float la = nz ? -INFINITY : lsum;
        J.sign[b] = S.bad ? __int_as_float(0x7fc00000) : sg;
        J.logabs[b] = S.bad ? __int_as_float(0x7fc00000) : la;
        if (J.value) J.value[b] = S.bad ? __int_as_float(0x7fc00000) : sg * expf(la);
        if (S.bad) umma::record_status(8);  // FX_ERR_TIMEOUT
        S.nz = nz;
      }
    }
    __syncthreads();
    if (GRAD) {
      // TMEM[p_s][t] = (A^-1)[s][p_t] = grad[p_t][s]: row x writes column pos(x) of the
      // gradient at rows at[t] (each warp store covers one gradient row)
      const bool zero = S.nz != 0 || S.bad;
      const float f = J.coef ? J.coef[b] : 1.f;
      float* G = J.g + b * (int64_t)n * n;
      if ((n & 3) == 0 && (reinterpret_cast<uintptr_t>(J.g) & 15) == 0) {
        // through shared memory (the free operand space): 32 gradient rows at a time are
        // assembled as gsm[k][pos] (row at[c0 + k]), then written as whole 16-byte pieces of
        // whole rows, so that the L2 receives whole sectors
        static_assert(offsetof(LuTcSmemT<NR>, blo) + sizeof(S.blo) == 5 * sizeof(S.chi) &&
                          sizeof(float) * 32 * (NR + 4) <= 5 * sizeof(S.chi),
                      "the gradient rows fit the operand space");
        float(*gsm)[NR + 4] = reinterpret_cast<float(*)[NR + 4]>(S.chi);
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
            for (int k = 0; k < 32; ++k) gsm[k][mypos] = zero ? 0.f : f * __uint_as_float(w[k]);
          }
          __syncthreads();
          for (int k = warp; k < 32 && c0 + k < n; k += NW) {
            float* grow = G + (int64_t)S.at[c0 + k] * n;
            for (int q = lane; 4 * q < n; q += 32)
              reinterpret_cast<float4*>(grow)[q] = *reinterpret_cast<const float4*>(&gsm[k][4 * q]);
          }
          __syncthreads();
        }
      } else {
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
    }
    tc_sync();
    FX_TOC(tq, 5);
  }
  if (warp == 0) umma::tmem_dealloc(tbase, kCols);
}

}  // namespace fx
