// INT8 Sol-Attn block-sparse forward on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Same unit and tile walk as the BF16 kernel (fwd_common.cuh, TileIter): first the
// 128-block chunks of pooled keys holding approximate blocks, then every routed block in
// ascending order. Arithmetic follows _forward_int8_ptr (_int8_fwd.py:190-372):
//   approximate tiles: bf16 q . kc^T (kc centred) on kind::f16, scores * s2; P = 2^(s - m)
//     in bf16 (TMEM) . vc on kind::f16 into the fp32 O accumulator; the row sum weighs
//     each pooled column by its block length (_int8_fwd.py:288-308).
//   exact tiles: acc = qi . ki^T on kind::i8 into int32 TMEM (_int8_fwd.py:329);
//     scores = fp32(acc) * (qs * s2 * ks) (:330), tokens >= T at -inf.
//     INT8 P.V (int8_pv, :336-353): bm = the block's row max, pe = 2^(s - bm),
//       beta = 2^(bm - m), l = l alpha + beta sum(pe), pi = trunc(min(pe*127 + 0.5, 127))
//       (int8 codes in shared memory), PV = pi . vi on kind::i8 into int32 TMEM, folded
//       by the softmax threads: O = O alpha + fp32(PV) * ((beta / 127) * vscale[d]) (vscale
//       applied in the epilogue, see below).
//     BF16 P.V: P = 2^(s - m) in bf16 (TMEM) . V (bf16) on kind::f16 into O.
// The online softmax keeps a per-row reference max m that is raised only when a tile
// exceeds it by more than 2^8 (then O and l are rescaled by alpha = 2^(m_old - m_new));
// the int8 codes are relative to each block's own max, so they do not depend on it.
//
// int32 -> fp32 conversions (scores and P.V) are exact: |acc| <= 127^2 * head_dim < 2^24.
// Folded int8 P.V products are accumulated in units of vscale[d] (fp32(PV) * beta / 127),
// the epilogue multiplies by vscale[d] (an approximate-tile contribution made before the
// first fold is divided by vscale[d] once).
//
// One CTA per unit, 256 threads: warps 0-3 softmax + fold + epilogue (thread = query row
// = TMEM lane), warp 4 TMA producer, warp 5 TMEM allocator + MMA issuer, warps 6-7 idle
// (they complete the second warpgroup, whose registers the softmax warps take). Two CTAs
// share an SM (256 TMEM columns and ~99 KB of shared memory each), so one CTA's
// tensor-core phases overlap the other's softmax.
//   TMEM   [0, 128)  S: scores (fp32 or int32), then bf16 P or the int32 P.V
//          [128, 128 + HD)  O (fp32)
//   smem   region Q (32 KB): bf16 q for the approximate tiles; then qi at +0 and the int8
//            P codes at +16 KB for the exact tiles (loaded once the last approximate
//            Q.K^T has read q), and the bf16 O staging at the end
//          region K (32 KB): kc chunk (approximate) or two 16 KB stages of ki
//          region V (32 KB): vc chunk (approximate), two 16 KB stages of vi (int8 P.V) or
//            one bf16 V tile (bf16 P.V)
//          key scales (a ring of 4 tiles), vscale, barriers
// Per tile the MMA issuer runs Q.K^T(j) once S is free, then P.V(j) once P(j) is written;
// the producer fills the other K / V stage meanwhile. Every wait is bounded.
#include "common.cuh"
#include "fwd_common.cuh"

namespace solb200 {

namespace {

// Descriptor of an operand with `rb`-byte rows (64 or 128) and the matching swizzle.
__device__ __forceinline__ uint64_t make_desc_rows(uint32_t addr, int rb, uint32_t lbo, uint32_t sbo) {
  uint64_t d = make_sw128_desc(addr, lbo, sbo);
  if (rb == 64) d = (d & ~((uint64_t)7 << 61)) | ((uint64_t)4 << 61);   // 64-byte swizzle
  return d;
}

// byte offset of 16-byte chunk `c` of row `r` in a swizzled tile with `rb`-byte rows
__device__ __forceinline__ uint32_t swz_off(int r, int c, int rb) {
  return rb == 128 ? (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)) : (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// four int8 codes (low bytes of c[0..3]) in one word, c[0] lowest
__device__ __forceinline__ uint32_t pack4(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3) {
  uint32_t a, b, w;
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(a) : "r"(c0), "r"(c1));
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(b) : "r"(c2), "r"(c3));
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(w) : "r"(a), "r"(b));
  return w;
}

// Maximum of n fp32 values held as bits in r[0..n).
template <int N>
__device__ __forceinline__ float max_n(const uint32_t (&r)[N]) {
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < N; i += 8) {
    m4[(i >> 3) & 3] = max3(m4[(i >> 3) & 3],
                            max3(__uint_as_float(r[i]), __uint_as_float(r[i + 1]), __uint_as_float(r[i + 2])),
                            max3(__uint_as_float(r[i + 3]), __uint_as_float(r[i + 4]),
                                 max3(__uint_as_float(r[i + 5]), __uint_as_float(r[i + 6]),
                                      __uint_as_float(r[i + 7]))));
  }
  return max3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
}

// Exact-tile scores of this row without the row factor: r[i] (int32 bits) <- fp32(acc_i) *
// ks_i, tokens at or past `valid` set to -inf when MASKED. The row factor qs * s2 (> 0, or
// 0 past T) multiplies the row max and enters the exponent's FMA; the reference multiplies
// acc by qs * s2 * ks at once (_int8_fwd.py:330): the two orders differ in the last bit.
template <int BLK, bool MASKED>
__device__ __forceinline__ void exact_scores(uint32_t (&r)[BLK], const float* __restrict__ ks, int valid) {
#pragma unroll
  for (int i = 0; i < BLK; i += 4) {
    const float4 k4 = *reinterpret_cast<const float4*>(ks + i);
    const float2 s01 = mul2(make_float2(__int2float_rn((int)r[i]), __int2float_rn((int)r[i + 1])),
                            make_float2(k4.x, k4.y));
    const float2 s23 = mul2(make_float2(__int2float_rn((int)r[i + 2]), __int2float_rn((int)r[i + 3])),
                            make_float2(k4.z, k4.w));
    r[i] = __float_as_uint(s01.x);
    r[i + 1] = __float_as_uint(s01.y);
    r[i + 2] = __float_as_uint(s23.x);
    r[i + 3] = __float_as_uint(s23.y);
  }
  if (MASKED) {
#pragma unroll
    for (int i = 0; i < BLK; ++i)
      if (i >= valid) r[i] = __float_as_uint(-INFINITY);
  }
}

// P = 2^(t * sc - m) as bf16 pairs written over r[0 .. BLK/2) (pair k = columns 2k, 2k+1);
// returns the row sum.
template <int BLK>
__device__ __forceinline__ float exp_bf16(uint32_t (&r)[BLK], float sc, float m) {
  const float2 nm = make_float2(-m, -m), scv = make_float2(sc, sc);
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int i = 0; i < BLK; i += 2) {
    const float2 x = fma2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), scv, nm);
    const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
    acc[(i >> 1) & 3] = add2(acc[(i >> 1) & 3], p);
    r[i >> 1] = pack_bf16x2(p.x, p.y);
  }
  const float2 a = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
  return a.x + a.y;
}

// INT8 P of this row (_int8_fwd.py:342-350): pe = 2^(s - bm) in [0, 1], code =
// trunc(min(pe*127 + 0.5, 127)) (read from the bits of RZ(w + 2^23), w = pe*127 + 0.5 <=
// 127.5, both steps rounded as the reference's), written to the swizzled K-major P tile
// in shared memory; returns sum(pe).
template <int BLK>
__device__ __forceinline__ float exp_codes(const uint32_t (&r)[BLK], float sc, float bm, uint8_t* sP, int row) {
  const float2 nbm = make_float2(-bm, -bm), k127 = make_float2(127.f, 127.f), scv = make_float2(sc, sc);
  const float2 half = make_float2(0.5f, 0.5f), big = make_float2(8388608.f, 8388608.f);
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int c = 0; c < BLK / 16; ++c) {
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t code[4];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = c * 16 + q * 4 + e * 2;
        const float2 x = fma2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), scv, nbm);
        const float2 pe = make_float2(fast_exp2(x.x), fast_exp2(x.y));
        acc[(q + e) & 3] = add2(acc[(q + e) & 3], pe);
        const float2 t = add_rz2(fma2(pe, k127, half), big);
        code[2 * e] = __float_as_uint(t.x);
        code[2 * e + 1] = __float_as_uint(t.y);
      }
      w[q] = pack4(code[0], code[1], code[2], code[3]);
    }
    *reinterpret_cast<uint4*>(sP + swz_off(row, c, BLK)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  const float2 a = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
  return a.x + a.y;
}

// O += fp32(PV) * f over this row's HD columns of O in TMEM (PV int32 in the S columns),
// O in units of vscale[d] (the epilogue multiplies by vscale[d]); with LIVE false,
// O = fp32(PV) * f.
template <int HD, bool LIVE>
__device__ __forceinline__ void fold_pv(uint32_t t_pv, uint32_t t_o, float f) {
  const float2 f2 = make_float2(f, f);
#pragma unroll 1
  for (int c = 0; c < HD / 32; ++c) {
    uint32_t pv[32], o[32];
    tmem_ld32(t_pv + c * 32, pv);
    if (LIVE) tmem_ld32(t_o + c * 32, o);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const float2 pf = make_float2(__int2float_rn((int)pv[i]), __int2float_rn((int)pv[i + 1]));
      const float2 v = LIVE ? fma2(pf, f2, make_float2(__uint_as_float(o[i]), __uint_as_float(o[i + 1])))
                            : mul2(pf, f2);
      o[i] = __float_as_uint(v.x);
      o[i + 1] = __float_as_uint(v.y);
    }
    tmem_st32(t_o + c * 32, o);
  }
}

// O[d] /= vscale[d] over this row's HD columns (O from true units to units of vscale[d]).
template <int HD>
__device__ __forceinline__ void to_vscale_units(uint32_t t_o, const float* __restrict__ vsc) {
#pragma unroll 1
  for (int c = 0; c < HD / 32; ++c) {
    uint32_t o[32];
    tmem_ld32(t_o + c * 32, o);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__fdiv_rn(__uint_as_float(o[i]), vsc[c * 32 + i]));
    tmem_st32(t_o + c * 32, o);
  }
  tmem_wait_st();
}

}  // namespace

template <int HD, int BLK>
__global__ void __launch_bounds__(256, 2)
sol_fwd_int8_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kc,
                    const __grid_constant__ CUtensorMap tm_vc, const __grid_constant__ CUtensorMap tm_o,
                    const __grid_constant__ CUtensorMap tm_qi, const __grid_constant__ CUtensorMap tm_ki,
                    const __grid_constant__ CUtensorMap tm_vi, const __grid_constant__ CUtensorMap tm_v,
                    const FwdParams p) {
  pdl_begin();
  static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
  static_assert(BLK == 64 || BLK == 128, "block 64 or 128");
  constexpr int NBOX = HD / 64;                  // 64-column (128-byte) bf16 boxes per row
  constexpr uint32_t BOX = 128 * 128;            // bf16 box: 128 rows x 128 bytes (16 KB apart)
  constexpr uint32_t REGION = 32768;
  constexpr uint32_t STAGE = REGION / 2;         // int8 tile stage (<= 128 rows x 128 bytes)
  constexpr int RB = HD;                         // bytes per int8 q / k / v row
  constexpr int PB = BLK;                        // bytes per int8 P row
  constexpr uint32_t IDESC_QK_APPROX = make_idesc(kFmtF32, kFmtBF16, kFmtBF16, 0, 0, 128, 128);
  constexpr uint32_t IDESC_PV_BF16 = make_idesc(kFmtF32, kFmtBF16, kFmtBF16, 0, 1, 128, HD);
  constexpr uint32_t IDESC_QK_I8 = make_idesc(kFmtS32, kFmtS8, kFmtS8, 0, 0, 128, BLK);
  constexpr uint32_t IDESC_PV_I8 = make_idesc(kFmtS32, kFmtS8, kFmtS8, 0, 1, 128, HD);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                    // bf16 q | (qi, int8 P) | O staging
  uint8_t* sQI = sQ;
  uint8_t* sP = sQ + STAGE;
  uint8_t* sK = sQ + REGION;
  uint8_t* sV = sK + REGION;
  float* sKS = reinterpret_cast<float*>(sV + REGION);       // [4][BLK] key scales, exact tile e at e % 4
  float* sVSC = sKS + 4 * BLK;                               // [HD]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sVSC + 128);
  uint64_t* bar_q = bars + 0;            // q (bf16) and vscale staged
  uint64_t* bar_qi = bars + 1;           // qi staged
  uint64_t* bar_kfull = bars + 2;        // [2]
  uint64_t* bar_vfull = bars + 4;        // [2]
  uint64_t* bar_kfree = bars + 6;        // [2] Q.K^T of the stage's tile complete
  uint64_t* bar_vfree = bars + 8;        // [2] P.V of the stage's tile complete
  uint64_t* bar_sfull = bars + 10;       // Q.K^T(j) complete: scores in TMEM
  uint64_t* bar_pfull = bars + 11;       // P(j) written (128 arrivals)
  uint64_t* bar_pvdone = bars + 12;      // P.V(j) complete
  uint64_t* bar_sfree = bars + 13;       // the softmax has read an int8 P.V out of S (128)
  uint64_t* bar_drain = bars + 14;
  uint64_t* bar_never = bars + 15;       // completed by nothing (the stall_unit test hook)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  int64_t* sTok = reinterpret_cast<int64_t*>(bars + 32);   // [128] output tokens (reordered calls)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const UnitInfo u = decode_unit(p, blockIdx.x);
  const int bh = u.b * p.H + u.h;
  const int tp = p.N * BLK;
  const bool pv8 = p.int8_pv != 0;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    mbar_init(bar_qi, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_kfull + i, 1);
      mbar_init(bar_vfull + i, 1);
      mbar_init(bar_kfree + i, 1);
      mbar_init(bar_vfree + i, 1);
    }
    mbar_init(bar_sfull, 1);
    mbar_init(bar_pfull, 128);
    mbar_init(bar_pvdone, 1);
    mbar_init(bar_sfree, 128);
    mbar_init(bar_drain, 1);
    mbar_init(bar_never, 1);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;
  const uint32_t tO = tmem + 128;

  // Stage of tile j in the K and V regions: approximate tiles fill a whole region
  // (stage 0); exact tile e = j - (approximate count) uses K stage e % 2, and V stage
  // e % 2 with int8 P.V (int8 vi tiles) or stage 0 with bf16 P.V (one bf16 V tile).
  auto vstage = [&](bool exact, int e) { return exact && pv8 ? (e & 1) : 0; };

  // Launched at 128 registers a thread: the producer / MMA warpgroup (warps 4-7, two of
  // them idle) keeps 40, the softmax warpgroup takes 216 (128 x 40 + 128 x 216 = 256 x 128;
  // measured best of 24-56 for the producer side: the softmax path spills at 168).
  if (warp >= 4) regs_decrease<40>();
  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_kc);
      tma_prefetch_desc(&tm_vc);
      tma_prefetch_desc(&tm_qi);
      tma_prefetch_desc(&tm_ki);
      tma_prefetch_desc(pv8 ? &tm_vi : &tm_v);
      mbar_arrive_expect_tx(bar_q, NBOX * BOX + (pv8 ? HD * 4 : 0));
      for (int i = 0; i < NBOX; ++i) tma_load_4d(sQ + i * BOX, &tm_q, bar_q, i * 64, u.h, u.qb * BLK, u.b);
      if (pv8) bulk_load(sVSC, p.vscale + (int64_t)bh * HD, HD * 4, bar_q);
      TileIter it(p, u);
      int kind, idx, e = -1, kn[2] = {0, 0}, vn[2] = {0, 0};
      bool ok = true, qi_issued = false;
      while (ok && it.next(kind, idx)) {
        const bool exact = kind == kTileExact;
        if (exact) ++e;
        const int ks_ = exact ? (e & 1) : 0, vs_ = vstage(exact, e);
        // K: the stage's previous tile must be done with it (its Q.K^T complete)
        if (kn[ks_] > 0 && !(ok = mbar_wait(bar_kfree + ks_, (kn[ks_] - 1) & 1, p.err, kErrWaitLoad, p.wait_ns)))
          break;
        if (exact && e == 0) {
          // qi replaces q in region Q once the last approximate Q.K^T has read q (covered
          // by the stage-0 wait above when there were approximate tiles)
          if (kn[0] == 0 && !(ok = mbar_wait(bar_q, 0, p.err, kErrWaitLoad, p.wait_ns))) break;
          mbar_arrive_expect_tx(bar_qi, 128 * RB);
          tma_load_4d(sQI, &tm_qi, bar_qi, 0, u.h, u.qb * BLK, u.b);
          qi_issued = true;
        }
        if (!exact) {
          mbar_arrive_expect_tx(bar_kfull, NBOX * BOX);
          for (int i = 0; i < NBOX; ++i) tma_load_4d(sK + i * BOX, &tm_kc, bar_kfull, i * 64, u.h, idx * 128, u.b);
        } else {
          mbar_arrive_expect_tx(bar_kfull + ks_, BLK * RB + BLK * 4);
          tma_load_4d(sK + ks_ * STAGE, &tm_ki, bar_kfull + ks_, 0, u.h, idx * BLK, u.b);
          bulk_load(sKS + (e & 3) * BLK, p.ks + (int64_t)bh * tp + (int64_t)idx * BLK, BLK * 4, bar_kfull + ks_);
        }
        ++kn[ks_];
        // V: the stage's previous tile must be done with it (its P.V complete)
        if (vn[vs_] > 0 && !(ok = mbar_wait(bar_vfree + vs_, (vn[vs_] - 1) & 1, p.err, kErrWaitLoad, p.wait_ns)))
          break;
        if (!exact) {
          mbar_arrive_expect_tx(bar_vfull, NBOX * BOX);
          for (int i = 0; i < NBOX; ++i) tma_load_4d(sV + i * BOX, &tm_vc, bar_vfull, i * 64, u.h, idx * 128, u.b);
        } else if (pv8) {
          mbar_arrive_expect_tx(bar_vfull + vs_, BLK * RB);
          tma_load_4d(sV + vs_ * STAGE, &tm_vi, bar_vfull + vs_, 0, u.h, idx * BLK, u.b);
        } else {
          mbar_arrive_expect_tx(bar_vfull, NBOX * BLK * 128);
          for (int i = 0; i < NBOX; ++i) tma_load_4d(sV + i * BOX, &tm_v, bar_vfull, i * 64, u.h, idx * BLK, u.b);
        }
        ++vn[vs_];
      }
      if (!ok) {
        // exit path: every issued copy must land before the CTA's shared memory goes away
        mbar_wait(bar_q, 0, p.err, kErrWaitDrain);
        if (qi_issued) mbar_wait(bar_qi, 0, nullptr, 0);
        for (int s = 0; s < 2; ++s) {
          if (kn[s] > 0) mbar_wait(bar_kfull + s, (kn[s] - 1) & 1, nullptr, 0);
          if (vn[s] > 0) mbar_wait(bar_vfull + s, (vn[s] - 1) & 1, nullptr, 0);
        }
      }
    }
  } else if (warp == 5) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t q_base = smem_u32(sQ), qi_base = smem_u32(sQI), p_base = smem_u32(sP);
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
      bool ok = mbar_wait(bar_q, 0, p.err, kErrWaitMma, p.wait_ns);
      if (ok && u.unit == p.stall_unit) ok = mbar_wait(bar_never, 0, p.err, kErrWaitMma, p.wait_ns);
      TileIter it(p, u);
      int kind, idx, j = 0, e = -1, kn[2] = {0, 0}, vn[2] = {0, 0}, nfold = 0;
      bool prev_fold = false;
      for (; ok && it.next(kind, idx); ++j) {
        const bool exact = kind == kTileExact;
        if (exact) ++e;
        const int ks_ = exact ? (e & 1) : 0, vs_ = vstage(exact, e);
        if (exact && e == 0 && !(ok = mbar_wait(bar_qi, 0, p.err, kErrWaitMma, p.wait_ns))) break;
        if (!(ok = mbar_wait(bar_kfull + ks_, kn[ks_] & 1, p.err, kErrWaitMma, p.wait_ns))) break;
        ++kn[ks_];
        // the S columns are free once the previous tile's P.V has read its bf16 P, or the
        // softmax has read its int8 P.V out of them
        if (j > 0) {
          ok = prev_fold ? mbar_wait(bar_sfree, (nfold - 1) & 1, p.err, kErrWaitMma, p.wait_ns)
                         : mbar_wait(bar_pvdone, (j - 1) & 1, p.err, kErrWaitMma, p.wait_ns);
          if (!ok) break;
        }
        tc_fence_after();
        if (!exact) {
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint32_t off = (k >> 2) * BOX + (k & 3) * 32;
            mma_bf16_ss(tS, make_sw128_desc(q_base + off, 16, 1024), make_sw128_desc(k_base + off, 16, 1024),
                        IDESC_QK_APPROX, k > 0);
          }
        } else {
          const uint32_t kb = k_base + ks_ * STAGE;
#pragma unroll
          for (int k = 0; k < RB / 32; ++k)
            mma_i8_ss(tS, make_desc_rows(qi_base + k * 32, RB, 16, 8 * RB), make_desc_rows(kb + k * 32, RB, 16, 8 * RB),
                      IDESC_QK_I8, k > 0);
        }
        tc_commit(bar_sfull);
        tc_commit(bar_kfree + ks_);
        if (!(ok = mbar_wait(bar_pfull, j & 1, p.err, kErrWaitMma, p.wait_ns))) break;
        if (!(ok = mbar_wait(bar_vfull + vs_, vn[vs_] & 1, p.err, kErrWaitMma, p.wait_ns))) break;
        ++vn[vs_];
        tc_fence_after();
        if (exact && pv8) {
          // PV = pi . vi (int32) into the S columns; the softmax threads fold it into O
          const uint32_t vb = v_base + vs_ * STAGE;
#pragma unroll
          for (int kk = 0; kk < BLK / 32; ++kk)
            mma_i8_ss(tS, make_desc_rows(p_base + kk * 32, PB, 16, 8 * PB), make_desc_rows(vb + kk * 32 * RB, RB, 0, 8 * RB),
                      IDESC_PV_I8, kk > 0);
          ++nfold;
          prev_fold = true;
        } else {
          const int keys = exact ? BLK : 128;
          for (int kk = 0; kk < keys / 16; ++kk)
            mma_bf16_ts(tO, tS + kk * 8, make_sw128_desc(v_base + kk * 2048, BOX, 1024), IDESC_PV_BF16,
                        (j > 0 || kk > 0) ? 1u : 0u);
          prev_fold = false;
        }
        tc_commit(bar_pvdone);
        tc_commit(bar_vfree + vs_);
      }
      // every MMA this thread issued has completed once bar_drain fires
      tc_commit(bar_drain);
      mbar_wait(bar_drain, 0, p.err, kErrWaitDrain);
    }
  } else if (warp < 4) {
    // ------------------------------------------- softmax, fold and epilogue (rows)
    regs_increase<216>();
    const int row = threadIdx.x;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    if (p.perm) prefetch_row_token<BLK>(p, u, row, sTok);
    const int qrow = u.qb * BLK + row;
    const float qs_log2 = (qrow < p.T ? __ldg(p.qs + (int64_t)bh * tp + qrow) : 0.f) * p.s2;
    float m_ref = -INFINITY, l_sum = 0.f;
    TileIter it(p, u);
    int j = 0, e = -1, kind, idx;
    bool ok = mbar_wait_warp(bar_q, 0, p.err, kErrWaitSoftmax, p.wait_ns);   // vscale is staged with q
    bool last_fold = false;
    bool o_scaled = false;   // O holds units of vscale[d] (int8 P.V folds; see fold_pv)
    for (; ok && it.next(kind, idx); ++j) {
      const bool exact = kind == kTileExact;
      if (exact) ++e;
      if (!(ok = mbar_wait_warp(bar_sfull, j & 1, p.err, kErrWaitSoftmax, p.wait_ns))) break;
      tc_fence_after();
      const uint32_t ts = tS + lane_base;
      const bool o_live = j > 0;
      if (!exact) {
        // ------------------------------------- approximate tile: bf16 P in TMEM
        uint32_t colmask[4];
        it.approx_bits(idx, colmask);
        const int tail_col = (p.N - 1 >= idx * 128 && p.N - 1 < idx * 128 + 128) ? p.N - 1 - idx * 128 : -1;
        softmax_tile<128, true, true, HD>(ts, tO + lane_base, colmask, p.s2, m_ref, l_sum, o_live, tail_col,
                                          (float)(p.T - (p.N - 1) * BLK), (float)BLK);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_pfull);
        last_fold = false;
        continue;
      }
      // ---------------------------------------------------------- exact tile
      uint32_t r[BLK];
#pragma unroll
      for (int c = 0; c < BLK / 32; ++c) tmem_ld32(ts + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
      tmem_wait_ld();
      const int valid = p.Tk - idx * BLK;
      const float* ks = sKS + (e & 3) * BLK;
      if (valid < BLK) exact_scores<BLK, true>(r, ks, valid);
      else exact_scores<BLK, false>(r, ks, valid);
      const float bm = max_n<BLK>(r) * qs_log2;   // the block's row max (log2 units)
      const float m_new = fmaxf(m_ref, bm);
      float alpha = 1.f;
      bool need = false;
      if (m_ref == -INFINITY) {
        m_ref = m_new;
      } else if (m_new > m_ref + 8.f) {
        alpha = fast_exp2(m_ref - m_new);
        m_ref = m_new;
        need = true;
      }
      // O holds every earlier tile's contribution (Q.K^T(j) complete implies P.V(j-1)
      // complete; int8 P.V tiles were folded by these threads)
      if (__any_sync(0xffffffffu, need) && o_live) {
        l_sum *= alpha;
        rescale_rows<HD>(tO + lane_base, alpha);
      }
      if (!pv8) {
        l_sum += exp_bf16<BLK>(r, qs_log2, m_ref);
#pragma unroll
        for (int c = 0; c < BLK / 32; ++c)
          tmem_st16(ts + c * 16, *reinterpret_cast<const uint32_t(*)[16]>(&r[c * 16]));
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_pfull);
        last_fold = false;
        continue;
      }
      // int8 P.V: codes to shared memory, then fold the tensor core's int32 product
      const float beta = fast_exp2(bm - m_ref);
      const float psum = exp_codes<BLK>(r, qs_log2, bm, sP, row);
      l_sum = l_sum + beta * psum;
      fence_proxy_async_smem();   // P (generic stores) -> tensor core (async proxy)
      tc_fence_before();
      mbar_arrive(bar_pfull);
      if (!(ok = mbar_wait_warp(bar_pvdone, j & 1, p.err, kErrWaitSoftmax, p.wait_ns))) break;
      tc_fence_after();
      const float f = beta * (1.0f / 127.0f);
      if (o_live && !o_scaled) to_vscale_units<HD>(tO + lane_base, sVSC);   // after approximate tiles
      if (o_live) fold_pv<HD, true>(ts, tO + lane_base, f);
      else fold_pv<HD, false>(ts, tO + lane_base, f);
      o_scaled = true;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_sfree);
      last_fold = true;
    }
    // epilogue: the last tile's P.V (unless these threads folded it), O / l -> bf16 ->
    // swizzled staging in region Q -> TMA store
    if (ok && j > 0 && !last_fold) ok = mbar_wait_warp(bar_pvdone, (j - 1) & 1, p.err, kErrWaitEpilogue, p.wait_ns);
    if (ok && j > 0) {
      tc_fence_after();
      const float inv = 1.f / l_sum;
      uint8_t* sO = sQ;
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + lane_base + c * 32, o);
        tmem_wait_ld();
        if (row < BLK) {
          const int box = (c * 32) / 64;
          const int col_byte0 = ((c * 32) % 64) * 2;
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            float sc[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) sc[t] = o_scaled ? inv * sVSC[c * 32 + v4 * 8 + t] : inv;
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o[v4 * 8 + 0]) * sc[0], __uint_as_float(o[v4 * 8 + 1]) * sc[1]);
            w.y = pack_bf16x2(__uint_as_float(o[v4 * 8 + 2]) * sc[2], __uint_as_float(o[v4 * 8 + 3]) * sc[3]);
            w.z = pack_bf16x2(__uint_as_float(o[v4 * 8 + 4]) * sc[4], __uint_as_float(o[v4 * 8 + 5]) * sc[5]);
            w.w = pack_bf16x2(__uint_as_float(o[v4 * 8 + 6]) * sc[6], __uint_as_float(o[v4 * 8 + 7]) * sc[7]);
            const int chunk = (col_byte0 >> 4) + v4;
            *reinterpret_cast<uint4*>(sO + box * (BLK * 128) + row * 128 + ((chunk ^ (row & 7)) << 4)) = w;
          }
        }
      }
      fence_proxy_async_smem();
    }
    named_bar_sync(1, 128);
    if (ok && j > 0 && p.perm) {
      store_rows_reordered<HD, BLK>(sQ, sTok, p, u, warp, 4, lane);
    } else if (ok && j > 0 && threadIdx.x == 0) {
      for (int i = 0; i < NBOX; ++i) tma_store_4d(&tm_o, sQ + i * (BLK * 128), i * 64, u.h, u.qb * BLK, u.b);
      bulk_commit_group();
      bulk_wait_group_read0();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// regions Q, K, V + key-scale ring + vscale + barriers + the output-token row (1 KB), plus
// 1 KB to align the tiles
static size_t fwd_int8_smem_bytes(int blk) { return (size_t)3 * 32768 + 4 * blk * 4 + 128 * 4 + 256 + 1024 + 1024; }

template <int HD, int BLK>
static cudaError_t launch_t(const FwdMaps& m, const FwdParams& p, cudaStream_t st) {
  auto kern = sol_fwd_int8_kernel<HD, BLK>;
  // the register split (40 + 216) adds up to the launch total only at 128 registers a
  // thread: with fewer, the softmax warpgroup's increase could never be granted
  static int launch_regs = 0;
  if (launch_regs == 0) {
    cudaFuncAttributes fa{};
    cudaError_t ea = cudaFuncGetAttributes(&fa, kern);
    if (ea != cudaSuccess) return ea;
    launch_regs = fa.numRegs;
  }
  if (launch_regs != 128) return cudaErrorInvalidConfiguration;
  const size_t smem = fwd_int8_smem_bytes(BLK);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const unsigned grid = (unsigned)((int64_t)p.B * p.H * p.N);
  return launch_pdl(kern, dim3(grid), dim3(256), smem, st, m.q, m.kc, m.vc, m.o, m.qi, m.ki, m.vi, m.v, p);
}

cudaError_t launch_fwd_int8(int hd, int blk, const FwdMaps& m, const FwdParams& p, cudaStream_t st) {
  if (hd == 128 && blk == 128) return launch_t<128, 128>(m, p, st);
  if (hd == 128 && blk == 64) return launch_t<128, 64>(m, p, st);
  if (hd == 64 && blk == 128) return launch_t<64, 128>(m, p, st);
  return launch_t<64, 64>(m, p, st);
}

}  // namespace solb200
