// Tensor-core (tcgen05, kind::tf32) trailing update of the blocked engines for float32 and
// complex64 under prec = "tf32x3": M[x][y] -= sum_s C[x][s] P[s][y] over rows [r_lo, n) x
// columns [c_lo, n) minus the panel columns, the same update as lg_update_kernel
// (large_lu.cuh) with the products on the tensor cores.
//
// Reference behaviour: the blocked LU trailing GEMM _lu_gemm_kernel
// (src/fermix/_lu.py:334-393), the mirrored Parlett-Reid update _pf_update_kernel
// (src/fermix/_pf.py:287-382) and the Gauss-Jordan products of the inverse
// (src/fermix/_inverse.py:230-313), all computed there with dot(..., prec) and for tf32x3 as
// three TF32 products (src/fermix/_field.py:173-190).
//
// Design (B200). One 128-thread CTA per 128-row strip of one matrix; thread x owns row
// r0 + x = TMEM lane x. The strip's coefficients C (128 x NB) are split once into TF32
// hi + lo and written to shared memory in the K-major canonical layout; the CTA then walks
// the strip's column tiles (64 float32 / 32 complex64 storage columns). Per tile the pivot
// rows' snapshot P (NB x tile) is split three ways, hi + mid + lo == value exactly, and one
// thread issues the MMAs hi*hi + hi*mid + hi*lo + lo*hi into a 64-column TMEM accumulator
// (complex: [Cr | Ci] against [Pr | Pi] slabs, the Ci*Pi term with the descriptor's negate
// bit, the real part in TMEM columns 0-31 and the imaginary part in 32-63). The threads load
// their row of the M tile while the tensor core runs, then subtract the product.
//
// Exact cancellation: a row duplicating pivot row s has coefficients e_s exactly (the
// coefficient kernel's FMA chains), so its product is 1 * (hi + mid + lo) of P_s summed
// from zero, which is P_s exactly, and the row becomes exactly zero -- as in the FMA
// update, so exactly singular inputs still report (0, -inf).
//
// SKEW (Parlett-Reid): only entries below the diagonal are computed; M[y][x] = -M[x][y] is
// written beside them. Bounded wait: a completion wait that runs out records
// FX_ERR_TIMEOUT (8) in the status word, waits once more for the MMAs with the default
// limit, and writes NaN over the tile, so that the member's outputs become NaN.
#pragma once
#include "large_lu.cuh"
#include "tc_common.cuh"

namespace fx {

template <typename T>
struct LgTc;
template <>
struct LgTc<float> {
  static constexpr int K = 32;        // panel width NB (K of the product)
  static constexpr int TNC = 64;      // storage columns per tile (= TMEM columns)
  static constexpr int KS = K / 8;    // K = 8 slabs of A / B
};
template <>
struct LgTc<c64_t> {
  static constexpr int K = 64;        // [re | im] halves of the NB = 32 complex coefficients
  static constexpr int TNC = 32;      // complex columns per tile (re and im: 64 TMEM columns)
  static constexpr int KS = K / 8;
};

template <typename T>
struct LgTcSmem {
  static constexpr int K = LgTc<T>::K, TNC = LgTc<T>::TNC;
  float ahi[128 * K], alo[128 * K];                          // A = C: slabs of 128 rows x 8
  float bhi[2][TNC * K], bmid[2][TNC * K], blo[2][TNC * K];  // B = P^T, double-buffered
  uint64_t mbar[2];
  uint32_t tslot;
  int flag;
};

template <typename T>
constexpr size_t lg_tc_smem() {
  return sizeof(LgTcSmem<T>) + 16;
}

__host__ __device__ constexpr uint32_t idesc_tf32_nb(int M, int N, bool neg_a, bool neg_b) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((neg_a ? 1u : 0u) << 13) | ((neg_b ? 1u : 0u) << 14) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// The column tiles are pipelined two deep: while the epilogue of tile j runs (its M tile
// loaded, the product read from TMEM buffer j % 2 and subtracted), the operands of tile
// j + 1 are already in the other shared-memory buffer and its MMAs in flight into the other
// TMEM buffer.
template <typename T, bool SKEW>
__global__ void __launch_bounds__(128, 2) lg_tc_update_kernel(LgArgs<T> A, int r_lo, int c_lo) {
  typedef typename Sc<T>::R R;
  constexpr bool CX = Sc<T>::cx;
  constexpr int NB = LgCfg<T>::NB;
  constexpr int K = LgTc<T>::K, TNC = LgTc<T>::TNC, KS = LgTc<T>::KS;
  constexpr uint32_t ASLAB = 128 * 8 * 4, BSLAB = TNC * 8 * 4;  // bytes of one K = 8 slab
  constexpr int NF = CX ? 2 * TNC : TNC;                         // floats of a row segment (64)
  extern __shared__ __align__(16) unsigned char lgtc_raw[];
  LgTcSmem<T>& S = *reinterpret_cast<LgTcSmem<T>*>((reinterpret_cast<uintptr_t>(lgtc_raw) + 15) & ~(uintptr_t)15);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int b = blockIdx.y, n = A.n, k0 = A.k0, kw = A.kw;
  const int r0 = r_lo + blockIdx.x * 128;
  const int r = r0 + tid;
  const bool rv = r < n;
  T* Mb = A.M + (size_t)b * n * n;
  const T* Cb = A.C + (size_t)b * n * NB;
  const T* Pb = A.P + (size_t)b * NB * n;

  if (warp == 0) {
    umma::tmem_alloc(&S.tslot, 128);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    umma::mbar_init(&S.mbar[0], 1);
    umma::mbar_init(&S.mbar[1], 1);
    umma::fence_mbar_init();
    S.flag = 0;
  }
  // ---- A: this row's coefficients, TF32 hi / lo, K-major (complex: re in k < 32, im above)
  {
    R cre[NB], cim[NB];
    const T* cr = Cb + (size_t)(rv ? r : 0) * NB;
#pragma unroll
    for (int s = 0; s < NB; ++s) {
      T v = (rv && s < kw) ? cr[s] : s_zero<T>();
      if constexpr (CX) {
        cre[s] = v.re;
        cim[s] = v.im;
      } else {
        cre[s] = v;
        cim[s] = 0;
      }
    }
#pragma unroll
    for (int q = 0; q < K / 4; ++q) {
      float h[4], l[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int k = 4 * q + e;
        const float v = (float)(k < NB ? cre[k] : cim[k - NB]);
        h[e] = umma::tf32_round(v);
        l[e] = umma::tf32_round(v - h[e]);
      }
      const uint32_t off = umma::kmajor_offset(tid, 4 * q, ASLAB) / 4;
      *reinterpret_cast<float4*>(&S.ahi[off]) = make_float4(h[0], h[1], h[2], h[3]);
      *reinterpret_cast<float4*>(&S.alo[off]) = make_float4(l[0], l[1], l[2], l[3]);
    }
  }
  const int c_end = SKEW ? (r0 + 128 < n ? r0 + 128 : n) : n;  // SKEW: columns below the strip's last row
  const int ntile = c_end > c_lo ? (c_end - c_lo + TNC - 1) / TNC : 0;

  // B of tile j (row jj of B = tile column c_lo + j TNC + jj), split three ways, into buffer j % 2
  auto stage_b = [&](int j) {
    constexpr int PER = TNC * NB / 128;  // coefficients per thread
    const int jj = tid % TNC;
    const int s0 = (tid / TNC) * PER;
    const int c = c_lo + j * TNC + jj;
    const bool cv = c < n;
    float* bh = S.bhi[j & 1];
    float* bm = S.bmid[j & 1];
    float* bl = S.blo[j & 1];
#pragma unroll
    for (int q = 0; q < PER; q += 4) {
      float hr[4], mr[4], lr[4], hi_[4], mi_[4], li_[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int sidx = s0 + q + e;
        const T v = (cv && sidx < kw) ? Pb[(size_t)sidx * n + c] : s_zero<T>();
        float re, im = 0.f;
        if constexpr (CX) {
          re = v.re;
          im = v.im;
        } else {
          re = v;
        }
        float h = umma::tf32_round(re), rr = re - h, m = umma::tf32_round(rr);
        hr[e] = h;
        mr[e] = m;
        lr[e] = rr - m;
        h = umma::tf32_round(im);
        rr = im - h;
        m = umma::tf32_round(rr);
        hi_[e] = h;
        mi_[e] = m;
        li_[e] = rr - m;
      }
      const uint32_t off = umma::kmajor_offset(jj, s0 + q, BSLAB) / 4;
      *reinterpret_cast<float4*>(&bh[off]) = make_float4(hr[0], hr[1], hr[2], hr[3]);
      *reinterpret_cast<float4*>(&bm[off]) = make_float4(mr[0], mr[1], mr[2], mr[3]);
      *reinterpret_cast<float4*>(&bl[off]) = make_float4(lr[0], lr[1], lr[2], lr[3]);
      if constexpr (CX) {
        const uint32_t oi = umma::kmajor_offset(jj, NB + s0 + q, BSLAB) / 4;
        *reinterpret_cast<float4*>(&bh[oi]) = make_float4(hi_[0], hi_[1], hi_[2], hi_[3]);
        *reinterpret_cast<float4*>(&bm[oi]) = make_float4(mi_[0], mi_[1], mi_[2], mi_[3]);
        *reinterpret_cast<float4*>(&bl[oi]) = make_float4(li_[0], li_[1], li_[2], li_[3]);
      }
    }
  };
  // the MMAs of tile j into TMEM buffer j % 2 (columns 64 (j % 2) ..), one thread
  auto issue = [&](int j, uint32_t tbase) {
    const uint32_t a_hi = umma::smem_u32(S.ahi), a_lo = umma::smem_u32(S.alo);
    const uint32_t b_hi = umma::smem_u32(S.bhi[j & 1]), b_mid = umma::smem_u32(S.bmid[j & 1]),
                   b_lo = umma::smem_u32(S.blo[j & 1]);
    const uint32_t dbase = tbase + 64u * (uint32_t)(j & 1);
    bool first_re = true, first_im = true;
#pragma unroll
    for (int t = 0; t < (CX ? 4 : 1) * (KS / (CX ? 2 : 1)); ++t) {
      int as, bs, dcol;
      bool negate;
      if constexpr (CX) {
        const int h = KS / 2, part = t / h, sl = t % h;
        // part 0: re += Cr Pr; 1: re -= Ci Pi; 2: im += Cr Pi; 3: im += Ci Pr
        as = (part == 0 || part == 2) ? sl : h + sl;
        bs = (part == 0 || part == 3) ? sl : h + sl;
        negate = part == 1;
        dcol = part < 2 ? 0 : TNC;
      } else {
        as = bs = t;
        negate = false;
        dcol = 0;
      }
      const uint32_t idesc = idesc_tf32_nb(128, TNC, negate, false);
      const uint64_t ah = umma::smem_desc_kmajor(a_hi + as * ASLAB, 128, 256);
      const uint64_t al = umma::smem_desc_kmajor(a_lo + as * ASLAB, 128, 256);
      const uint64_t bh = umma::smem_desc_kmajor(b_hi + bs * BSLAB, 128, 256);
      const uint64_t bm = umma::smem_desc_kmajor(b_mid + bs * BSLAB, 128, 256);
      const uint64_t bl = umma::smem_desc_kmajor(b_lo + bs * BSLAB, 128, 256);
      bool& first = dcol == 0 ? first_re : first_im;
      const uint32_t d = dbase + dcol;
      umma::mma_tf32(d, ah, bh, idesc, !first);
      first = false;
      umma::mma_tf32(d, ah, bm, idesc, true);
      umma::mma_tf32(d, ah, bl, idesc, true);
      umma::mma_tf32(d, al, bh, idesc, true);
    }
    umma::mma_commit(&S.mbar[j & 1]);
  };

  if (ntile > 0) stage_b(0);
  umma::fence_proxy_async_smem();
  tc_sync();
  const uint32_t tbase = S.tslot;
  const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);
  if (ntile > 0 && tid == 0) issue(0, tbase);
  uint32_t ph0 = 0, ph1 = 0;
  const bool rowvec = ((n * sizeof(T)) % 16 == 0);

  for (int j = 0; j < ntile; ++j) {
    const int c0 = c_lo + j * TNC;
    if (j + 1 < ntile) {
      stage_b(j + 1);
      umma::fence_proxy_async_smem();
      tc_sync();
      if (tid == 0) issue(j + 1, tbase);
    }
    // ---- this row's M tile into registers while the tensor core runs
    float mv[NF];
    const bool full = c0 + TNC <= n && (c0 * sizeof(T)) % 16 == 0 && rowvec;
    {
      const T* row = Mb + (size_t)(rv ? r : 0) * n + c0;
      if (rv && full) {
#pragma unroll
        for (int q = 0; q < NF / 4; ++q) {
          const float4 t4 = reinterpret_cast<const float4*>(row)[q];
          mv[4 * q] = t4.x;
          mv[4 * q + 1] = t4.y;
          mv[4 * q + 2] = t4.z;
          mv[4 * q + 3] = t4.w;
        }
      } else {
#pragma unroll
        for (int jj = 0; jj < TNC; ++jj) {
          const T v = (rv && c0 + jj < n) ? row[jj] : s_zero<T>();
          if constexpr (CX) {
            mv[2 * jj] = v.re;
            mv[2 * jj + 1] = v.im;
          } else {
            mv[jj] = v;
          }
        }
      }
    }
    __syncwarp();
    {
      uint64_t* mb = &S.mbar[j & 1];
      const uint32_t ph = (j & 1) ? ph1 : ph0;
      if (!umma::mbar_wait(mb, ph, A.wait_polls)) {
        S.flag = 1;
        (void)umma::mbar_wait(mb, ph, kTcWaitIters);
      }
      if (j & 1) ph1 ^= 1;
      else ph0 ^= 1;
    }
    umma::fence_after_sync();
    // ---- M -= D, 32 TMEM columns at a time (complex: the real parts, then the imaginary)
    const uint32_t drow = trow + 64u * (uint32_t)(j & 1);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t t32[32];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t t8[8];
        umma::tmem_ld8(drow + 32 * h + 8 * q, t8);
#pragma unroll
        for (int e = 0; e < 8; ++e) t32[8 * q + e] = t8[e];
      }
      umma::tmem_wait_ld();
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        if constexpr (CX) mv[2 * jj + h] -= __uint_as_float(t32[jj]);
        else mv[32 * h + jj] -= __uint_as_float(t32[jj]);
      }
    }
    const bool bad = S.flag != 0;
    if (bad) {
      if (tid == 0) umma::record_status(8);  // FX_ERR_TIMEOUT
#pragma unroll
      for (int q = 0; q < NF; ++q) mv[q] = __int_as_float(0x7fc00000);
    }
    // clean segment: every column valid, outside the panel and (SKEW) below the diagonal
    const bool clean = rv && full && (c0 + TNC <= k0 || c0 >= k0 + kw) && (!SKEW || c0 + TNC - 1 < r);
    if (clean) {
      float4* row4 = reinterpret_cast<float4*>(Mb + (size_t)r * n + c0);
#pragma unroll
      for (int q = 0; q < NF / 4; ++q) row4[q] = make_float4(mv[4 * q], mv[4 * q + 1], mv[4 * q + 2], mv[4 * q + 3]);
    }
#pragma unroll
    for (int jj = 0; jj < TNC; ++jj) {
      const int c = c0 + jj;
      T v;
      if constexpr (CX) {
        v.re = mv[2 * jj];
        v.im = mv[2 * jj + 1];
      } else {
        v = mv[jj];
      }
      const bool ok = rv && c < n && (c < k0 || c >= k0 + kw) && (!SKEW || r > c);
      if (ok) {
        if (!clean) Mb[(size_t)r * n + c] = v;
        if (SKEW) Mb[(size_t)c * n + r] = neg(v);
      }
    }
    tc_sync();  // TMEM buffer j % 2 read before the MMAs of tile j + 2 overwrite it
  }
  if (warp == 0) umma::tmem_dealloc(tbase, 128);
}

// ---------------------------------------------------------------- float64 / complex128
// The same trailing update on the FP64 tensor cores (DMMA, mma.sync m8n8k4 f64) for the
// 64-bit dtypes, whose prec is always "ieee": every product and sum is an IEEE fp64
// fused multiply-add, as in the FMA kernel. A 256-thread CTA owns a 128-row strip and walks
// a run of kLgDmTiles column tiles of 64 columns (complex128: 32 complex columns) in it; its
// 8 warps (4 x 2) own 32 x 32 sub-tiles (complex: 32 x 16, real and imaginary
// accumulators). -C is staged in shared memory once per CTA; while one tile's products and
// stores run, the next tile's M entries (into a second register set) and P rows are already
// in flight, so the loads that bound a one-tile CTA overlap the rest. The accumulators start
// as the M tile and the coefficients are staged negated, so D = M + (-C) P is the update
// itself; a row duplicating pivot row s (coefficients e_s) ends as fma(-1, P_s, M) = 0
// exactly.
//
// m8n8k4 fragments (lane = 4 g + t): A element (g, t), B element (t, g), accumulator
// elements (g, 2 t) and (g, 2 t + 1). Shared-memory row strides are 4 (mod 16) doubles, so
// each half-warp's 16 doubles fall in distinct bank pairs.
__device__ __forceinline__ void dmma(double& d0, double& d1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
               : "+d"(d0), "+d"(d1)
               : "d"(a), "d"(b));
}

constexpr int kLgDmTiles = 4;  // column tiles per CTA

template <typename T>
struct LgDm;
template <>
struct LgDm<double> {
  static constexpr int NB = 32, TC = 64, WC = 32;  // K, tile columns, columns per warp
};
template <>
struct LgDm<c128_t> {
  static constexpr int NB = 16, TC = 32, WC = 16;
};

template <typename T>
struct LgDmSmem {
  static constexpr int NB = LgDm<T>::NB, TC = LgDm<T>::TC;
  static constexpr int SA = NB + 4, SB = TC + 4;  // strides, 4 (mod 16) doubles
  double ar[128 * SA];                            // -Re C (row-major)
  double ai[Sc<T>::cx ? 128 * SA : 1];            // -Im C
  double br[NB * SB];                             // Re P (k-major rows of the tile's columns)
  double bi[Sc<T>::cx ? NB * SB : 1];             // Im P
};

template <typename T>
constexpr size_t lg_dm_smem() {
  return sizeof(LgDmSmem<T>);
}

// The warp's M sub-tile at column offset c0 (zero outside n x n) into accumulator layout.
template <typename T, int MT, int NT>
__device__ __forceinline__ void lg_dm_load_m(const T* __restrict__ Mb, int n, int wr, int wc, int g, int t,
                                             double (&vr)[MT][NT][2], double (&vi)[Sc<T>::cx ? MT : 1][Sc<T>::cx ? NT : 1][2]) {
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int rr = wr + 8 * i + g, cc = wc + 8 * j + 2 * t + e;
        const T v = (rr < n && cc < n) ? Mb[(size_t)rr * n + cc] : s_zero<T>();
        if constexpr (Sc<T>::cx) {
          vr[i][j][e] = v.re;
          vi[i][j][e] = v.im;
        } else {
          vr[i][j][e] = v;
        }
      }
}

template <typename T, bool SKEW>
__global__ void __launch_bounds__(256, 1) lg_dmma_update_kernel(LgArgs<T> A, int r_lo, int c_lo) {
  constexpr bool CX = Sc<T>::cx;
  constexpr int NB = LgDm<T>::NB, TC = LgDm<T>::TC, WC = LgDm<T>::WC;
  constexpr int SA = LgDmSmem<T>::SA, SB = LgDmSmem<T>::SB;
  constexpr int MT = 4, NT = WC / 8;            // 8 x 8 accumulator tiles of a warp
  constexpr int PE = NB * TC / 256;             // P entries per thread and tile
  static_assert(NB * TC % 256 == 0, "P tile shared evenly");
  extern __shared__ __align__(16) unsigned char lgdm_raw[];
  LgDmSmem<T>& S = *reinterpret_cast<LgDmSmem<T>*>(lgdm_raw);
  const int b = blockIdx.z, n = A.n, k0 = A.k0, kw = A.kw;
  const int r0 = r_lo + blockIdx.y * 128;
  // this CTA's run of column tiles; the skew update keeps tiles that reach the lower triangle
  const int c_end = SKEW ? min(n, r0 + 128) : n;
  int c0 = c_lo + blockIdx.x * (kLgDmTiles * TC);
  if (c0 >= c_end) return;
  const int c_stop = min(c_end, c0 + kLgDmTiles * TC);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wr = r0 + (warp >> 1) * 32;
  T* Mb = A.M + (size_t)b * n * n;
  const T* Cb = A.C + (size_t)b * n * NB;
  const T* Pb = A.P + (size_t)b * NB * n;

  // ---- accumulators = the first M tile (re / im); its P rows and -C into shared memory
  double dr[MT][NT][2], di[CX ? MT : 1][CX ? NT : 1][2];
  lg_dm_load_m<T, MT, NT>(Mb, n, wr, c0 + (warp & 1) * WC, g, t, dr, di);
  for (int e = tid; e < 128 * NB; e += 256) {
    const int rr = e / NB, s = e % NB, r = r0 + rr;
    const T v = (r < n && s < kw) ? Cb[(size_t)r * NB + s] : s_zero<T>();
    if constexpr (CX) {
      S.ar[rr * SA + s] = -v.re;
      S.ai[rr * SA + s] = -v.im;
    } else {
      S.ar[rr * SA + s] = -v;
    }
  }
  T pv[PE];
#pragma unroll
  for (int q = 0; q < PE; ++q) {
    const int e = tid + 256 * q, s = e / TC, c = c0 + e % TC;
    pv[q] = (c < n && s < kw) ? Pb[(size_t)s * n + c] : s_zero<T>();
  }
  const int ar0 = (warp >> 1) * 32, bc0 = (warp & 1) * WC;
#pragma unroll 1
  for (;;) {
    // this tile's P rows into shared memory (the previous tile's readers are done)
#pragma unroll
    for (int q = 0; q < PE; ++q) {
      const int e = tid + 256 * q, s = e / TC, cc = e % TC;
      if constexpr (CX) {
        S.br[s * SB + cc] = pv[q].re;
        S.bi[s * SB + cc] = pv[q].im;
      } else {
        S.br[s * SB + cc] = pv[q];
      }
    }
    __syncthreads();
    // ---- the next tile's M entries and P rows start loading
    const int cn = c0 + TC;
    const bool more = cn < c_stop;
    double nr[MT][NT][2], ni[CX ? MT : 1][CX ? NT : 1][2];
    if (more) {
      lg_dm_load_m<T, MT, NT>(Mb, n, wr, cn + (warp & 1) * WC, g, t, nr, ni);
#pragma unroll
      for (int q = 0; q < PE; ++q) {
        const int e = tid + 256 * q, s = e / TC, c = cn + e % TC;
        pv[q] = (c < n && s < kw) ? Pb[(size_t)s * n + c] : s_zero<T>();
      }
    }
    // ---- D += (-C) P, K = 4 per step
#pragma unroll 1
    for (int k = 0; k < NB; k += 4) {
      double a_r[MT], a_i[CX ? MT : 1], b_r[NT], b_i[CX ? NT : 1];
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        a_r[i] = S.ar[(ar0 + 8 * i + g) * SA + k + t];
        if constexpr (CX) a_i[i] = S.ai[(ar0 + 8 * i + g) * SA + k + t];
      }
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        b_r[j] = S.br[(k + t) * SB + bc0 + 8 * j + g];
        if constexpr (CX) b_i[j] = S.bi[(k + t) * SB + bc0 + 8 * j + g];
      }
#pragma unroll
      for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          dmma(dr[i][j][0], dr[i][j][1], a_r[i], b_r[j]);
          if constexpr (CX) {
            // re += (-Cr) Pr - (-Ci) Pi; im += (-Cr) Pi + (-Ci) Pr
            dmma(dr[i][j][0], dr[i][j][1], -a_i[i], b_i[j]);
            dmma(di[i][j][0], di[i][j][1], a_r[i], b_i[j]);
            dmma(di[i][j][0], di[i][j][1], a_i[i], b_r[j]);
          }
        }
    }
    // ---- store the updated entries
    const int wc = c0 + bc0;
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int rr = wr + 8 * i + g, cc = wc + 8 * j + 2 * t + e;
          const bool ok = rr < n && cc < n && (cc < k0 || cc >= k0 + kw) && (!SKEW || rr > cc);
          if (ok) {
            T v;
            if constexpr (CX) {
              v.re = dr[i][j][e];
              v.im = di[i][j][e];
            } else {
              v = dr[i][j][e];
            }
            Mb[(size_t)rr * n + cc] = v;
            if (SKEW) Mb[(size_t)cc * n + rr] = neg(v);
          }
        }
    if (!more) break;
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          dr[i][j][e] = nr[i][j][e];
          if constexpr (CX) di[i][j][e] = ni[i][j][e];
        }
    c0 = cn;
    __syncthreads();  // every warp is done with this tile's P rows
  }
}

}  // namespace fx
