// Tensor-memory resident Parlett-Reid "sweep" for float32 slogpf, 8 <= n <= 128: forward
// (sign, logabs) and, in the same pass, S^-1 for the gradient; prec = "tf32x3" (tensor-core
// block updates) or "ieee" (IEEE float32 FMA block updates, template flag IEEE).
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
//   A'_XP = A_XP A_PP^-1,  A'_PY = sigma(y) A'_YP^T,  A'_PP = -A_PP^-1,
// so that after the last panel TMEM holds -S^-1 (sweeping every index inverts the
// matrix); the forward-only mode skips the replacement and its (sign, logabs) are
// bit-identical (the unswept part evolves identically). Row-derived operand values come
// from the column values by the sweep's sign pattern sigma: skew inside the unswept and
// inside the swept index sets, symmetric across them.
//
// The replacement needs no inverse of A_PP. The pair steps factor the panel as
// A_XP = W_X B_P^T with B = sigma W D_J (D_J = diag of the pairs' [[0, -d], [d, 0]]) and
// W_P (the pivot rows' multipliers) unit lower block-triangular, so
//   A'_XP = W_X Z,  A_PP^-1 = Z^T D_J^-T Z,  Z = W_P^-1:
// every thread solves z W_P = (its W row, or e_k on pivot row k) while the tensor core
// runs the update, the pivot rows' new rows are the other rows' z transposed through
// shared memory, and their pivot block is formed from the pivot rows' Z.
//
// Memory. With skew_symmetrize the matrix arrives through shared memory in 32-row chunks
// (bulk copies, read once); the gradient leaves through per-warp shared-memory blocks as
// whole 128-byte row pieces. Nothing is prefetched into L2 ahead of the block's next matrix:
// the gradient writes evicted such lines before use, and the input was read twice.
#pragma once
#include "fused_lu.cuh"
#include "tc_common.cuh"

namespace fx {

struct PfTcSmem {
  // uv[t][x] = (-d_t u_t[x], d_t v_t[x]) of the panel's pairs, with u_t = col_p / d_t and
  // v_t = -col_a / d_t (one 8-byte broadcast read per earlier pair in the later pair steps'
  // corrections); in gradient mode the same 8 KB are reused after the pair steps as
  // tcol[16][kTcN], the other rows' new pivot-column values sigma(x) z_j(x) read back along
  // the pivot rows
  __align__(16) float2 uv[8][kTcN];
  float whi[kTcN * 16], wlo[kTcN * 16];  // MMA A operand (K-major, interleaved), TF32 hi / lo
  float bhi[kTcN * 16], blo[kTcN * 16];  // MMA B operand
  __align__(16) float wp[16][20];        // W_P: the pivot rows' multipliers (16-byte rows)
  __align__(16) float zp[16][20];        // Z = W_P^-1, row k from pivot row k
  __align__(16) float ppm[16][20];       // A'_PP = -A_PP^-1, formed by the whole block
  // per-warp pivot candidates: packed order key (|value| key << 32 | ~row: the largest key,
  // then the smallest row, is the largest number) and the record (position, value bits,
  // reciprocal pivot bits) of the warp's candidate
  __align__(16) unsigned long long pkey[4];
  uint4 prec[4];
  unsigned cmask[4];                     // prec ieee forward: the unswept rows (columns to update)
  int cand_f[4];                         // scratch (the singular flag at the end)
  int at[kTcN];                          // position -> row (virtual pivoting)
  int pidx[16];                          // the panel's pivot rows a_0, p_0, a_1, p_1, ...
  float dvec[kTcN / 2];
  uint32_t tslot;
  int bad;
  uint64_t mbar;
  uint64_t lbar[2];  // the staged load's two chunk buffers
};

static_assert(sizeof(PfTcSmem::uv) == sizeof(float) * 16 * kTcN, "uv holds tcol[16][kTcN]");

// prec ieee: B's rows (16 values, 80-byte rows: conflict-free 16-byte stores) in the space
// of the tensor-core operands whi / wlo, which that mode does not use
__device__ __forceinline__ float (*pf_tc_brow(PfTcSmem& S))[20] { return reinterpret_cast<float (*)[20]>(S.whi); }
static_assert(offsetof(PfTcSmem, wlo) == offsetof(PfTcSmem, whi) + sizeof(float) * kTcN * 16 &&
                  sizeof(float) * kTcN * 20 <= 2 * sizeof(float) * kTcN * 16,
              "brow fits whi + wlo");

// prec ieee: the rank-16 update D -= W B^T of this thread's TMEM row with IEEE float32 FMAs
// (one sequential chain per entry over the panel's pairs, u then v of each pair), W = this
// row's (u_t, v_t), B's rows broadcast from shared memory; 16 columns per TMEM round trip.
// The forward updates only its unswept rows and columns (the rest is never read again).
template <bool GRAD>
__device__ __forceinline__ void pf_tc_fma_update(PfTcSmem& S, uint32_t trow, int n, int np, const float (&ur)[8],
                                                 const float (&vr)[8], bool live) {
  if (!GRAD && !__any_sync(0xffffffffu, live)) return;
  const float(*brow)[20] = pf_tc_brow(S);
#pragma unroll 1
  for (int c0 = 0; c0 < n; c0 += 16) {
    const unsigned cm = GRAD ? 0xffffu : (S.cmask[c0 >> 5] >> (c0 & 16)) & 0xffffu;
    if (cm == 0u) continue;
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
      if ((cm >> e) & 1u) {
        const float4* b4 = reinterpret_cast<const float4*>(brow[c0 + e]);
        float acc = v[e];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 b = b4[q];
          if (2 * q < np) {
            acc = fmaf(-ur[2 * q], b.x, acc);
            acc = fmaf(-vr[2 * q], b.y, acc);
          }
          if (2 * q + 1 < np) {
            acc = fmaf(-ur[2 * q + 1], b.z, acc);
            acc = fmaf(-vr[2 * q + 1], b.w, acc);
          }
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

// skew_symmetrize load through shared memory: 32-row chunks of A (528-byte rows, one bulk copy
// per row) in two buffers over the space of uv and the tensor-core operands (free between
// matrices). TMEM starts at zero; chunk c adds -A[32c + k][x] / 2 to every row's column block
// c (conflict-free column reads) and, on warp c, A[x][y] / 2 to its own rows (16-byte reads),
// so every entry is round(A[x][y] / 2 - A[y][x] / 2), the bits of (A[x][y] - A[y][x]) / 2.
// Needs n % 4 == 0 and a 16-byte aligned matrix (the rows are bulk copies).
constexpr int kTcStgLd = 132;  // staged row stride (floats): 16-byte rows, bank offset 4 per row
__device__ __forceinline__ float (*pf_tc_stage(PfTcSmem& S, int buf))[kTcStgLd] {
  return reinterpret_cast<float (*)[kTcStgLd]>(reinterpret_cast<unsigned char*>(&S.uv[0][0]) +
                                                (size_t)buf * 32 * kTcStgLd * sizeof(float));
}
static_assert(offsetof(PfTcSmem, whi) == sizeof(PfTcSmem::uv) && offsetof(PfTcSmem, blo) + sizeof(PfTcSmem::blo) ==
                  sizeof(PfTcSmem::uv) + 4 * sizeof(PfTcSmem::whi) &&
                  2 * 32 * kTcStgLd * sizeof(float) <= sizeof(PfTcSmem::uv) + 4 * sizeof(PfTcSmem::whi),
              "the staging buffers fit uv and the operands");

static_assert(4 * 32 * 36 * sizeof(float) <= sizeof(PfTcSmem::uv) + 4 * sizeof(PfTcSmem::whi),
              "the gradient store's per-warp blocks fit uv and the operands");

// warp 0: rows 32 c .. of the matrix into buffer c & 1 (lane l copies row 32 c + l)
__device__ __forceinline__ void pf_tc_stage_issue(PfTcSmem& S, const float* src, int n, int c, int lane) {
  const int rows = min(32, n - 32 * c);
  uint64_t* bar = &S.lbar[c & 1];
  umma::fence_proxy_async_smem();  // the buffer's earlier generic accesses before the copies
  if (lane == 0) umma::mbar_arrive_expect_tx(bar, (uint32_t)(rows * n * 4));
  __syncwarp();
  if (lane < rows) umma::bulk_g2s(pf_tc_stage(S, c & 1)[lane], src + (size_t)(32 * c + lane) * n, (uint32_t)n * 4u, bar);
}

// returns false when a chunk wait ran out (the member is then marked bad by the caller)
__device__ __forceinline__ bool pf_tc_load_skew_staged(PfTcSmem& S, const float* src, int n, uint32_t trow, int x,
                                                       int warp, int lane, uint32_t& lph, uint32_t polls) {
  const int nc = (n + 31) >> 5;
  if (warp == 0) {
    pf_tc_stage_issue(S, src, n, 0, lane);
    if (nc > 1) pf_tc_stage_issue(S, src, n, 1, lane);
  }
  {
    uint32_t z[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
    for (int c = 0; c < kTcN; c += 8) umma::tmem_st8(trow + c, z);
    umma::tmem_wait_st();
  }
  bool ok = true;
#pragma unroll 1
  for (int c = 0; c < nc; ++c) {
    const int bufi = c & 1;
    const uint32_t par = (lph >> bufi) & 1u;
    if (!umma::mbar_wait(&S.lbar[bufi], par, polls)) {
      ok = false;
      (void)umma::mbar_wait(&S.lbar[bufi], par, kTcWaitIters);  // no copy left in flight
    }
    lph ^= 1u << bufi;
    const float(*buf)[kTcStgLd] = pf_tc_stage(S, bufi);
    // every row: column block c -= A[32 c + k][x] / 2
    {
      uint32_t w[32];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t t8[8];
        umma::tmem_ld8(trow + 32 * c + 8 * q, t8);
#pragma unroll
        for (int e = 0; e < 8; ++e) w[8 * q + e] = t8[e];
      }
      umma::tmem_wait_ld();
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float cv = (x < n && 32 * c + k < n) ? buf[k][x] : 0.f;
        w[k] = __float_as_uint(fmaf(-0.5f, cv, __uint_as_float(w[k])));
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t t8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) t8[e] = w[8 * q + e];
        umma::tmem_st8(trow + 32 * c + 8 * q, t8);
      }
      umma::tmem_wait_st();
    }
    // warp c's own rows: += A[x][y] / 2
    if (warp == c) {
      const float* row = buf[x - 32 * c];
#pragma unroll 1
      for (int cb = 0; cb < kTcN; cb += 32) {
        uint32_t w[32];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t t8[8];
          umma::tmem_ld8(trow + cb + 8 * q, t8);
#pragma unroll
          for (int e = 0; e < 8; ++e) w[8 * q + e] = t8[e];
        }
        umma::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const bool in = x < n && cb + 4 * q < n;  // n % 4 == 0: whole 16-byte pieces
          const float4 r = in ? *reinterpret_cast<const float4*>(row + cb + 4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
          w[4 * q] = __float_as_uint(fmaf(0.5f, r.x, __uint_as_float(w[4 * q])));
          w[4 * q + 1] = __float_as_uint(fmaf(0.5f, r.y, __uint_as_float(w[4 * q + 1])));
          w[4 * q + 2] = __float_as_uint(fmaf(0.5f, r.z, __uint_as_float(w[4 * q + 2])));
          w[4 * q + 3] = __float_as_uint(fmaf(0.5f, r.w, __uint_as_float(w[4 * q + 3])));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t t8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) t8[e] = w[8 * q + e];
          umma::tmem_st8(trow + cb + 8 * q, t8);
        }
      }
      umma::tmem_wait_st();
    }
    __syncthreads();  // every thread is done with this buffer
    if (c + 2 < nc && warp == 0) pf_tc_stage_issue(S, src, n, c + 2, lane);
  }
  return ok;
}

template <bool GRAD, bool IEEE>
__global__ void __launch_bounds__(128, 4) pf_tc_kernel(Job<float> J) {
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
    umma::mbar_init(&S.lbar[0], 1);
    umma::mbar_init(&S.lbar[1], 1);
    umma::fence_mbar_init();
  }
  tc_sync();
#ifdef FX_PHASE_TIMERS
  if (blockIdx.x == 0 && tid == 0) fx_phase_cycles[15] = gridDim.x;
#endif
  const uint32_t tbase = S.tslot;
  const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);
  uint32_t phase = 0;
  uint32_t lph = 0u;  // the staged load's buffer phases (bit i: buffer i)
  // skew_symmetrize through the staged load when every row is a whole number of 16-byte pieces
  const bool staged = J.skew != 0 && (n & 3) == 0 && (reinterpret_cast<uintptr_t>(J.a) & 15) == 0;

  for (int64_t b = blockIdx.x; b < J.B; b += gridDim.x) {
    FX_TIC(tq);
    // ---- the (skew-symmetrised) matrix into TMEM, zero outside n x n. (No L2 prefetch of
    // the block's next matrix: measured, its lines were mostly evicted by the gradient
    // writes before use, reading the input twice from DRAM.)
    const float* src = J.a + b * (int64_t)n * n;
    if (tid == 0) S.bad = 0;
    if (staged) {
      __syncthreads();  // S.bad cleared before a chunk wait can set it
      if (!pf_tc_load_skew_staged(S, src, n, trow, x, warp, lane, lph, J.wait_polls) && lane == 0) S.bad = 1;
    } else {
      tc_load_matrix(src, n, J.skew != 0, trow, x);
    }
    S.at[x] = x;
    // virtual pivoting: each thread tracks its own row's position; every thread keeps the
    // interchange parity (all see the same pivots)
    int pos = x, par = 0;
    bool live = x < n;
    tc_sync();
    FX_TOC(tq, 8);

    const int npairs = n / 2;
    for (int g0 = 0; g0 < npairs; g0 += 8) {
      const int np = min(8, npairs - g0);
      const bool swept_before = !live && x < n;
      float ur[8], vr[8], dr[8], ir[8];  // ir[t] = 1 / d_t (0 for d_t = 0)
      int kx = -1;  // this row's slot among the panel's pivot rows (a_t -> 2 t, p_t -> 2 t + 1)
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        ur[t] = vr[t] = dr[t] = ir[t] = 0.f;
      }
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        if (s < np) {
          const int c = 2 * (g0 + s);
          const int a = S.at[c];
          if (x == a) live = false;
          // column a of the current matrix: stale TMEM value plus this panel's corrections
          float colA = __uint_as_float(umma::tmem_ld1(trow + a));
          {
            // this panel's corrections in two independent FMA chains (u and v terms)
            float cu = 0.f, cv = 0.f;
#pragma unroll
            for (int t = 0; t < 8; ++t)
              if (t < s) {
                const float2 w = S.uv[t][a];
                cu = fmaf(ur[t], w.y, cu);
                cv = fmaf(vr[t], w.x, cv);
              }
            umma::tmem_wait_ld();
            colA -= cu + cv;
          }
          // pivot: largest |colA| over the unassigned rows (first occurrence): per warp two
          // redux.sync on the packed key, then the largest of the four warps' packed keys
          const unsigned key = piv_key(colA, live);
          // every lane forms its reciprocal pivot 1 / (-colA) while the reductions run (only
          // the warp's candidate keeps it)
          const float pinv = colA == 0.f ? 0.f : __frcp_rn(-colA);
          const unsigned km = __reduce_max_sync(0xffffffffu, key);
          // the first lane holding the largest key: the smallest row
          const int wi = (warp << 5) + __ffs(__ballot_sync(0xffffffffu, key == km)) - 1;
          if (x == wi) {
            S.pkey[warp] = ((unsigned long long)km << 32) | (unsigned)~wi;
            S.prec[warp] = make_uint4((unsigned)pos, __float_as_uint(colA), __float_as_uint(pinv), 0u);
          }
          __syncthreads();
          int p;
          {
            const ulonglong2 k01 = *reinterpret_cast<const ulonglong2*>(&S.pkey[0]);
            const ulonglong2 k23 = *reinterpret_cast<const ulonglong2*>(&S.pkey[2]);
            const unsigned long long m01 = k01.x > k01.y ? k01.x : k01.y;
            const unsigned long long m23 = k23.x > k23.y ? k23.x : k23.y;
            p = (int)~(unsigned)(m01 > m23 ? m01 : m23);  // the pivot row (owned by warp p / 32)
          }
          const uint4 rec = S.prec[p >> 5];
          const int q = (int)rec.x;                 // the pivot row's position
          const float d = -__uint_as_float(rec.y);  // all candidates NaN: the first one, d = NaN
          const float inv = __uint_as_float(rec.z);
          if (x == p) live = false;
          float colP = __uint_as_float(umma::tmem_ld1(trow + p));
          {
            float cu = 0.f, cv = 0.f;
#pragma unroll
            for (int t = 0; t < 8; ++t)
              if (t < s) {
                const float2 w = S.uv[t][p];
                cu = fmaf(ur[t], w.y, cu);
                cv = fmaf(vr[t], w.x, cv);
              }
            umma::tmem_wait_ld();
            colP -= cu + cv;
          }
          ur[s] = colP * inv;
          vr[s] = -colA * inv;
          dr[s] = d;
          ir[s] = inv;
          // stored pre-multiplied by the pair pivot: the products every thread formed
          // for its corrections (d v_s and -d u_s), the same bits computed once
          S.uv[s][x] = make_float2(-d * ur[s], d * vr[s]);
          // the interchange of positions c + 1 and q, written by the two rows involved
          if (q != c + 1) {
            par ^= 1;
            if (x == p) {
              S.at[c + 1] = p;
              pos = c + 1;
            } else if (pos == c + 1) {
              S.at[q] = x;
              pos = q;
            }
          }
          if (x == p) {
            S.dvec[g0 + s] = d;
            S.pidx[2 * s + 1] = p;
            kx = 2 * s + 1;
          }
          if (x == a) {
            S.pidx[2 * s] = a;
            kx = 2 * s;
          }
          __syncthreads();
        }
      }
      FX_TOC(tq, 9);
      // ---- gradient mode: pivot row k publishes its row of W_P, the multipliers of the
      // earlier pairs (its own pair's identity block and the zero upper part are implied)
      if (GRAD) {
        if (kx >= 0) {
          const int kb = kx & ~1;
          float4* w4 = reinterpret_cast<float4*>(S.wp[kx]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float e[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int j = 4 * q + c;
              e[c] = j < kb ? ((j & 1) ? vr[j >> 1] : ur[j >> 1]) : 0.f;
            }
            w4[q] = make_float4(e[0], e[1], e[2], e[3]);
          }
        }
      }
      // the forward needs no update after the last panel
      const bool need_upd = GRAD || g0 + 8 < npairs;
      if (IEEE) {
        // ---- prec ieee: row y of B = sigma(y) d_t (v_t, -u_t) into brow[y] for the FMA
        // update below; the forward only updates the columns of the unswept rows
        if (need_upd) {
          const float sig = swept_before ? -1.f : 1.f;
          float4* b4 = reinterpret_cast<float4*>(pf_tc_brow(S)[x]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float e[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int k = 4 * q + c, t = k >> 1;
              e[c] = t < np ? ((k & 1) ? -sig * dr[t] * ur[t] : sig * dr[t] * vr[t]) : 0.f;
            }
            b4[q] = make_float4(e[0], e[1], e[2], e[3]);
          }
          if (!GRAD) {
            const unsigned lm = __ballot_sync(0xffffffffu, live);
            if (lane == 0) S.cmask[warp] = lm;
          }
        }
      } else if (need_upd) {
        // ---- MMA operands: W[x] = (u_t, v_t), B[x] = sigma(x) d_t (v_t, -u_t), 16-byte stores
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
        umma::fence_proxy_async_smem();
      }
      tc_sync();
      FX_TOC(tq, 10);
      if (!IEEE && need_upd && tid == 0) {
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
      // prec ieee: the FMA update now (the gradient's replacement values below only read
      // shared memory and this thread's registers)
      if (IEEE && need_upd) pf_tc_fma_update<GRAD>(S, trow, n, np, ur, vr, live);
      // gradient mode, while the tensor core runs the update: z W_P = rhs (rhs = this row's
      // W, or e_kx on pivot row kx), from the last row of W_P up
      float z[16];
      if (GRAD) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float wj = (j & 1) ? vr[j >> 1] : ur[j >> 1];
          z[j] = kx >= 0 ? (j == kx ? 1.f : 0.f) : (j < 2 * np ? wj : 0.f);
        }
#pragma unroll
        for (int m = 15; m >= 2; --m) {
          if (m < 2 * np) {
            const float zm = z[m];
            const float4* r4 = reinterpret_cast<const float4*>(S.wp[m]);
            const int mb = m & ~1;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (4 * q < mb) {
                const float4 v = r4[q];
                const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int c = 0; c < 4; ++c)
                  if (4 * q + c < mb) z[4 * q + c] = fmaf(-zm, vv[c], z[4 * q + c]);
              }
            }
          }
        }
        // the other rows' new pivot-column values, transposed through shared memory for the
        // pivot rows (A'_PY = sigma(y) A'_YP^T); pivot row kx keeps its row of Z
        float* tcol = reinterpret_cast<float*>(&S.uv[0][0]);
        if (kx < 0) {
          const float sg = swept_before ? -1.f : 1.f;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (j < 2 * np) tcol[j * kTcN + x] = sg * z[j];
        } else {
          float4* z4 = reinterpret_cast<float4*>(S.zp[kx]);
#pragma unroll
          for (int q = 0; q < 4; ++q) z4[q] = make_float4(z[4 * q], z[4 * q + 1], z[4 * q + 2], z[4 * q + 3]);
        }
        __syncthreads();
        // A'_PP = -(Z^T D_J^-T Z), entry (k, j) = sum_t (Z[2t][k] Z[2t+1][j] - Z[2t+1][k] Z[2t][j]) / d_t
        // (Z[j][k] = 0 for j < k), two entries of one row per thread
        {
          const int k = tid >> 3, j = 2 * (tid & 7);
          float p0 = 0.f, p1 = 0.f;
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            if (t < np && 2 * t + 1 >= k) {
              const float id = ir[t];
              const float za = S.zp[2 * t][k] * id, zb = S.zp[2 * t + 1][k] * id;
              const float2 a = *reinterpret_cast<const float2*>(&S.zp[2 * t][j]);
              const float2 c = *reinterpret_cast<const float2*>(&S.zp[2 * t + 1][j]);
              p0 = fmaf(za, c.x, fmaf(-zb, a.x, p0));
              p1 = fmaf(za, c.y, fmaf(-zb, a.y, p1));
            }
          }
          *reinterpret_cast<float2*>(&S.ppm[k][j]) = make_float2(p0, p1);
        }
        __syncthreads();
        if (kx >= 0) {
          // a pivot row's new pivot-column values are its row of A'_PP (z is no longer needed)
          const float4* r4 = reinterpret_cast<const float4*>(S.ppm[kx]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 v = r4[q];
            z[4 * q] = v.x;
            z[4 * q + 1] = v.y;
            z[4 * q + 2] = v.z;
            z[4 * q + 3] = v.w;
          }
        }
      }
      if (!IEEE && need_upd) {
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
      FX_TOC(tq, 11);

      if (GRAD) {
        // pivot rows: the whole row from the transposed values (a warp holding a pivot row
        // stores all its lanes, the other lanes write back their own row)
        if (__any_sync(0xffffffffu, kx >= 0)) {
          const float* trow_src = reinterpret_cast<const float*>(&S.uv[0][0]) + (kx >= 0 ? kx : 0) * kTcN;
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
            if (kx >= 0) {
              const float4* s4 = reinterpret_cast<const float4*>(trow_src + c0);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float4 v = s4[q];
                w[4 * q] = __float_as_uint(v.x);
                w[4 * q + 1] = __float_as_uint(v.y);
                w[4 * q + 2] = __float_as_uint(v.z);
                w[4 * q + 3] = __float_as_uint(v.w);
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t t8[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) t8[e] = w[8 * q + e];
              umma::tmem_st8(trow + c0 + 8 * q, t8);
            }
          }
          umma::tmem_wait_st();
        }
        FX_TOC(tq, 3);
        // pivot columns of every row: A'_XP = z, on the pivot rows A'_PP = -A_PP^-1
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < 2 * np) umma::tmem_st1(trow + S.pidx[j], __float_as_uint(z[j]));
        umma::tmem_wait_st();
        FX_TOC(tq, 4);
      }
      // the panel's pidx / at / dvec are read before the next panel's pair steps rewrite them;
      // TMEM stores complete before the next MMA (or the final read) on any thread
      tc_sync();
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
        if (par) sg = -sg;
        if (nz) sg = 0.f;
        const float la = nz ? -INFINITY : lsum;
        J.sign[b] = S.bad ? __int_as_float(0x7fc00000) : sg;
        J.logabs[b] = S.bad ? __int_as_float(0x7fc00000) : la;
        if (J.value) J.value[b] = S.bad ? __int_as_float(0x7fc00000) : sg * expf(la);
        if (S.bad) umma::record_status(8);  // FX_ERR_TIMEOUT
        S.cand_f[0] = nz;  // reused below as the singular flag
      }
    }
    __syncthreads();
    if (GRAD) {
      // TMEM = -S^-1: gradient of sum(logabs) = -S^-1 / 2, scaled by coef
      const bool zero = S.cand_f[0] != 0 || S.bad;
      const float f = 0.5f * (J.coef ? J.coef[b] : 1.f);
      float* G = J.g + b * (int64_t)n * n;
      if ((n & 3) == 0 && (reinterpret_cast<uintptr_t>(J.g) & 15) == 0)
        // whole-sector stores through a 32 x 36 block per warp in the (now free) uv / operand space
        tc_store_rows_staged(G, n, f, zero, trow, x, reinterpret_cast<float*>(&S.uv[0][0]) + warp * 32 * 36);
      else
        tc_store_rows(G, n, f, zero, trow, x);
    }
    tc_sync();
    FX_TOC(tq, 13);
  }
  if (warp == 0) umma::tmem_dealloc(tbase, kTcN);
}

}  // namespace fx
