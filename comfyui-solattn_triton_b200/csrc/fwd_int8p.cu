// Pipelined INT8 Sol-Attn block-sparse forward for head_dim 128 and 128-token blocks
// (the video shapes); other shapes use the serial kernel in fwd_int8.cu.
//
// Tile walk and arithmetic follow _forward_int8_ptr (_int8_fwd.py:190-372):
//   approximate tiles (128 pooled keys): bf16 q . kc^T (kind::f16, q and kc in shared
//     memory), bf16 P . vc accumulated into O by the tensor core; the row sum weighs
//     each pooled column by its block length (_int8_fwd.py:288-308).
//   exact tiles (one routed 128-token block): S = qi . ki^T (_int8_fwd.py:311-332) on
//     kind::f16 over the int8 codes held as bf16 (qib, kib, written by the preprocess):
//     every product (<= 127^2) and partial sum (< 2^21) is an integer that fp32 holds
//     exactly, so S arrives in TMEM as the exact integer dot in fp32;
//     scores = S * (qs * s2) * ks.
//     INT8 P.V (int8_pv, _int8_fwd.py:336-353): pe = 2^(s - blockmax), codes
//       pi = int8(pe*127 rounded) as the reference; the reference's O += (pi . vi) *
//       (beta / 127) * vscale[d] with beta = 2^(blockmax - m) is computed as
//       P' = bf16(pi * beta / 127) (in TMEM, over the bf16 P columns) times
//       vdq = bf16(vi * vscale) (the dequantised V, written by the preprocess), on
//       kind::f16 accumulated into O by the tensor core: the int8 codes are the
//       reference's, each operand carries one more bf16 rounding (2^-9 relative).
//     BF16 P.V: P = 2^(s - m) in bf16 in TMEM, P . V (bf16) accumulated into O.
//
// One CTA per unit, one CTA per SM (all 512 TMEM columns):
//   TMEM  [0,128) bf16 P (64 columns) | [128,256) O | [256,384) S slot 0 |
//         [384,512) S slot 1
//   smem  q bf16 32 KB | qi codes bf16 32 KB | K ring 2 x 32 KB | V ring 2 x 32 KB |
//         ks ring of 4 tiles, mask row, max / sum exchange
// Warps 0-7 softmax (warps w and w+4 share the rows of TMEM lanes 32(w%4).. and split
// each tile's 128 columns), warp 8 TMA producer, warp 9 TMEM allocator + MMA issuer.
// The issuer keeps the tensor core idle while the softmax loads a tile's scores (a TMEM
// load waits behind in-flight MMAs): per tile, the softmax loads S(j+1), then P.V(j)
// and Q.K^T(j+2) run while it works on tile j+1. Every wait is bounded; every softmax
// thread runs every tile and every named barrier, also after a failed wait (the work is
// skipped, the barriers are not).
#include "common.cuh"
#include "fwd_common.cuh"

namespace solb200 {

namespace {

constexpr int kMaskCapI8 = 1024;   // routing-mask words of one unit kept in shared memory

// Maximum of this thread's 64 values (fp32 bits in `r`); with MASKED, columns whose bit
// in `cm` (2 words) is clear are set to -inf first.
template <bool MASKED>
__device__ __forceinline__ float max64(uint32_t (&r)[64], const uint32_t (&cm)[2]) {
  if (MASKED) {
#pragma unroll
    for (int i = 0; i < 64; ++i)
      if (!((cm[i >> 5] >> (i & 31)) & 1u)) r[i] = __float_as_uint(-INFINITY);
  }
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < 64; i += 8) {
    m4[(i >> 3) & 3] = max3(m4[(i >> 3) & 3],
                            max3(__uint_as_float(r[i]), __uint_as_float(r[i + 1]), __uint_as_float(r[i + 2])),
                            max3(__uint_as_float(r[i + 3]), __uint_as_float(r[i + 4]),
                                 max3(__uint_as_float(r[i + 5]), __uint_as_float(r[i + 6]),
                                      __uint_as_float(r[i + 7]))));
  }
  return max3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
}

// P = 2^(r * sc - m) as bf16 pairs in r[0..31] (pair k = columns 2k, 2k+1); returns the
// row sum of the 64 columns, weighing column `tail_col` by w_tail and every other by
// w_full when WEIGHTED.
template <bool WEIGHTED>
__device__ __forceinline__ float exp_bf16_64(uint32_t (&r)[64], float sc, float m, int tail_col, float w_tail,
                                             float w_full) {
  const float2 scv = make_float2(sc, sc), nmv = make_float2(-m, -m);
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  float tail_p = 0.f;
#pragma unroll
  for (int i = 0; i < 64; i += 2) {
    const float2 x = fma2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), scv, nmv);
    const float2 pp = make_float2(fast_exp2(x.x), fast_exp2(x.y));
    acc[(i >> 1) & 3] = add2(acc[(i >> 1) & 3], pp);
    if (WEIGHTED) tail_p += (i == tail_col ? pp.x : 0.f) + (i + 1 == tail_col ? pp.y : 0.f);
    r[i >> 1] = pack_bf16x2(pp.x, pp.y);
  }
  const float2 a = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
  float sum = a.x + a.y;
  if (WEIGHTED) sum = sum * w_full + tail_p * (w_tail - w_full);
  return sum;
}

// Exact tile with int8 P.V semantics: pe = 2^(r * sc - bm) in [0, 1] for the 64 columns
// (r: scores before the per-row factor sc; bm: the tile's row max in log2 units); the
// int8 code of pe (_int8_fwd.py:350: min(pe*127 + 0.5, 127) truncated) is the low part
// of RN(pe*127 + 2^23) = 2^23 + pe*127 rounded to the nearest integer (the reference's
// rounding except at exact ties, half-even here; the clamp never binds as pe <= 1);
// P' = code * pscale (= beta / 127) as bf16 pairs in r[0..31]; returns the sum of pe.
// Packed f32x2 arithmetic throughout.
__device__ __forceinline__ float exp_int8p_bf16_64(uint32_t (&r)[64], float sc, float bm, float pscale) {
  float2 acc = make_float2(0.f, 0.f);
  const float2 scv = make_float2(sc, sc), nbm = make_float2(-bm, -bm);
  const float2 k127 = make_float2(127.f, 127.f), mg = make_float2(8388608.f, 8388608.f);
  // (c - 2^23) * ps as one FMA: c * ps - 2^23 * ps, the product by 2^23 exact
  const float2 ps = make_float2(pscale, pscale), nps = make_float2(-8388608.f * pscale, -8388608.f * pscale);
#pragma unroll
  for (int i = 0; i < 64; i += 2) {
    const float2 x = fma2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), scv, nbm);
    const float2 pe = make_float2(fast_exp2(x.x), fast_exp2(x.y));
    acc = add2(acc, pe);
    const float2 v = fma2(fma2(pe, k127, mg), ps, nps);   // code * beta / 127
    r[i >> 1] = pack_bf16x2(v.x, v.y);
  }
  return acc.x + acc.y;
}

}  // namespace

__global__ void __launch_bounds__(320, 1)
sol_fwd_int8p_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kc,
                     const __grid_constant__ CUtensorMap tm_vc, const __grid_constant__ CUtensorMap tm_o,
                     const __grid_constant__ CUtensorMap tm_qi, const __grid_constant__ CUtensorMap tm_ki,
                     const __grid_constant__ CUtensorMap tm_vi, const __grid_constant__ CUtensorMap tm_v,
                     const FwdParams p) {
  pdl_begin();
  constexpr int HD = 128, BLK = 128;
  constexpr uint32_t BOX = 128 * 128;           // 128 rows x 128 bytes
  constexpr uint32_t TILE = 2 * BOX;            // 128 rows x 128 bf16
  constexpr int KST = 2, VST = 2;
  constexpr uint32_t IDESC_QK_BF16 = make_idesc(kFmtF32, kFmtBF16, kFmtBF16, 0, 0, 128, 128);
  constexpr uint32_t IDESC_PV_BF16 = make_idesc(kFmtF32, kFmtBF16, kFmtBF16, 0, 1, 128, HD);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                    // bf16 q (approximate tiles); later the O staging
  uint8_t* sQI = sQ + TILE;              // qi codes as bf16, 128 rows x 128 columns
  uint8_t* sK = sQI + TILE;              // KST stages: kc or the ki codes (bf16, 32 KB)
  uint8_t* sV = sK + KST * TILE;         // VST stages: vc, v or vdq (bf16)
  float* sKS = reinterpret_cast<float*>(sV + VST * TILE);   // [4][128] key scales, by tile j % 4
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKS + 4 * 128);
  uint64_t* bar_q = bars + 0;            // q, qi staged
  uint64_t* bar_kfull = bars + 1;        // [KST]
  uint64_t* bar_kfree = bars + 3;        // [KST] Q.K^T of the stage's tile complete
  uint64_t* bar_vfull = bars + 5;        // [VST]
  uint64_t* bar_vfree = bars + 7;        // [VST] P.V of the stage's tile complete
  uint64_t* bar_sfree = bars + 9;        // [2] scores of a slot loaded by the softmax (256)
  uint64_t* bar_pfull = bars + 11;       // P written (256)
  uint64_t* bar_drain = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  uint32_t* sMask = reinterpret_cast<uint32_t*>(bars + 16);    // kMaskCapI8 words
  float* sMax = reinterpret_cast<float*>(sMask + kMaskCapI8);   // [2 tiles][2 halves][128 rows]
  float* sSum = sMax + 512;                                      // [2 halves][128 rows]
  int* sBad = reinterpret_cast<int*>(sSum + 256);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  UnitInfo u = decode_unit(p, blockIdx.x);
  const int bh = u.b * p.H + u.h;
  const int tp = p.N * BLK;
  const bool pv8 = p.int8_pv != 0;
  if (p.nw <= kMaskCapI8)
    for (int i = threadIdx.x; i < p.nw; i += blockDim.x) sMask[i] = __ldg(u.row + i);

  if (threadIdx.x == 0) {
    *sBad = 0;
    mbar_init(bar_q, 1);
    for (int i = 0; i < KST; ++i) {
      mbar_init(bar_kfull + i, 1);
      mbar_init(bar_kfree + i, 1);
    }
    for (int i = 0; i < VST; ++i) {
      mbar_init(bar_vfull + i, 1);
      mbar_init(bar_vfree + i, 1);
    }
    for (int i = 0; i < 2; ++i) mbar_init(bar_sfree + i, 256);
    mbar_init(bar_pfull, 256);
    mbar_init(bar_drain, 1);
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (p.nw <= kMaskCapI8) u.row = sMask;
  const uint32_t tmem = *tmem_slot;
  const uint32_t tA = tmem, tO = tmem + 128, tS = tmem + 256;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    // q, qi; K0 K1, V0 V1; then per tile j: K(j+2) once Q.K^T(j) is done with
    // its stage (its key scales go to ring slot (j+2) % 4, which the softmax finished
    // with at tile j-2), V(j+2) once P.V(j) is done.
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_kc);
      tma_prefetch_desc(&tm_vc);
      tma_prefetch_desc(&tm_qi);
      tma_prefetch_desc(&tm_ki);
      tma_prefetch_desc(pv8 ? &tm_vi : &tm_v);
      mbar_arrive_expect_tx(bar_q, 2 * TILE);
      for (int i = 0; i < 2; ++i) {
        tma_load_4d(sQ + i * BOX, &tm_q, bar_q, i * 64, u.h, u.qb * BLK, u.b);
        tma_load_4d(sQI + i * BOX, &tm_qi, bar_q, i * 64, u.h, u.qb * BLK, u.b);
      }
      auto load_k = [&](int stage, int kind, int idx, int jt) {
        uint64_t* bar = bar_kfull + stage;
        uint8_t* dst = sK + stage * TILE;
        if (kind == kTileApprox) {
          mbar_arrive_expect_tx(bar, TILE);
          for (int i = 0; i < 2; ++i) tma_load_4d(dst + i * BOX, &tm_kc, bar, i * 64, u.h, idx * 128, u.b);
        } else {
          mbar_arrive_expect_tx(bar, TILE + BLK * 4);
          for (int i = 0; i < 2; ++i) tma_load_4d(dst + i * BOX, &tm_ki, bar, i * 64, u.h, idx * BLK, u.b);
          bulk_load(sKS + (jt & 3) * 128, p.ks + (int64_t)bh * tp + (int64_t)idx * BLK, BLK * 4, bar);
        }
      };
      auto load_v = [&](int stage, int kind, int idx) {
        uint64_t* bar = bar_vfull + stage;
        uint8_t* dst = sV + stage * TILE;
        if (kind == kTileApprox) {
          mbar_arrive_expect_tx(bar, TILE);
          for (int i = 0; i < 2; ++i) tma_load_4d(dst + i * BOX, &tm_vc, bar, i * 64, u.h, idx * 128, u.b);
        } else {
          // exact tile: the bf16 dequantised V (int8_pv; tm_vi maps it) or V
          const CUtensorMap* tmv = pv8 ? &tm_vi : &tm_v;
          mbar_arrive_expect_tx(bar, TILE);
          for (int i = 0; i < 2; ++i) tma_load_4d(dst + i * BOX, tmv, bar, i * 64, u.h, idx * BLK, u.b);
        }
      };
      TileIter itk(p, u), itv(p, u);
      int kind, idx, nk = 0, nv = 0;
      bool ok = true;
      while (nk < KST && itk.next(kind, idx)) load_k(nk % KST, kind, idx, nk), ++nk;
      while (nv < VST && itv.next(kind, idx)) load_v(nv % VST, kind, idx), ++nv;
      for (int j = 0; ok; ++j) {
        bool more = false;
        if (itk.next(kind, idx)) {
          more = true;
          if (!(ok = mbar_wait(bar_kfree + j % KST, (j / KST) & 1, p.err, kErrWaitLoad))) break;
          load_k(nk % KST, kind, idx, nk);
          ++nk;
        }
        if (itv.next(kind, idx)) {
          more = true;
          if (!(ok = mbar_wait(bar_vfree + j % VST, (j / VST) & 1, p.err, kErrWaitLoad))) break;
          load_v(nv % VST, kind, idx);
          ++nv;
        }
        if (!more) break;
      }
      if (!ok) {
        // exit path: the newest copy of every stage must land before shared memory goes away
        mbar_wait(bar_q, 0, p.err, kErrWaitDrain);
        for (int i = nk - 1; i >= 0 && i >= nk - KST; --i)
          mbar_wait(bar_kfull + i % KST, (i / KST) & 1, p.err, kErrWaitDrain);
        for (int i = nv - 1; i >= 0 && i >= nv - VST; --i)
          mbar_wait(bar_vfull + i % VST, (i / VST) & 1, p.err, kErrWaitDrain);
      }
    }
  } else if (warp == 9) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      // descriptors of the tile bases; a stage / K-step adds its byte offset >> 4 to
      // the start-address field (shared addresses stay below 2^18: nothing carries)
      const uint64_t qd = make_sw128_desc(smem_u32(sQ), 16, 1024);
      const uint64_t qid = make_sw128_desc(smem_u32(sQI), 16, 1024);   // qi codes, bf16
      const uint64_t kd0 = make_sw128_desc(smem_u32(sK), 16, 1024);
      const uint64_t vd0 = make_sw128_desc(smem_u32(sV), BOX, 1024);   // bf16 V, MN-major
      auto issue_qk = [&](int j, int kind) {
        const int st = j % KST;
        const uint32_t d = tS + (j & 1) * 128;
        const uint64_t kd = kd0 + (uint64_t)(st * (TILE >> 4));
        // approximate: bf16 q . kc; exact: the qi codes . the ki codes (both bf16)
        const uint64_t ad = kind == kTileApprox ? qd : qid;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = ((k >> 2) * BOX + (k & 3) * 32) >> 4;
          mma_bf16_ss(d, ad + (uint64_t)off, kd + (uint64_t)off, IDESC_QK_BF16, k > 0);
        }
        tc_commit(bar_kfree + st);
      };
      bool ok = mbar_wait(bar_q, 0, p.err, kErrWaitMma);
      tc_fence_after();
      TileIter itq(p, u), itp(p, u);
      int kind, idx, jq = 0;
      while (ok && jq < 2 && itq.next(kind, idx)) {
        if (!(ok = mbar_wait(bar_kfull + jq % KST, (jq / KST) & 1, p.err, kErrWaitMma))) break;
        tc_fence_after();
        issue_qk(jq++, kind);
      }
      for (int j = 0; ok && itp.next(kind, idx); ++j) {
        // P.V(j) once P(j) is written and the softmax holds the scores of tile j+1,
        // then Q.K^T(j+2) into the slot the softmax released at tile j
        if (!(ok = mbar_wait(bar_pfull, j & 1, p.err, kErrWaitMma))) break;
        int qkind, qidx;
        const bool more = itq.next(qkind, qidx);   // tile j+2
        TileIter peek = itp;
        int k1, i1;
        if (peek.next(k1, i1) &&
            !(ok = mbar_wait(bar_sfree + ((j + 1) & 1), ((j + 1) >> 1) & 1, p.err, kErrWaitMma)))
          break;
        if (!(ok = mbar_wait(bar_vfull + j % VST, (j / VST) & 1, p.err, kErrWaitMma))) break;
        tc_fence_after();
        const uint32_t vo = (j % VST) * (TILE >> 4);
        {
          const uint32_t acc0 = j > 0 ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16_ts(tO, tA + kk * 8, vd0 + (uint64_t)(vo + kk * (2048 >> 4)), IDESC_PV_BF16,
                        kk > 0 ? 1u : acc0);
        }
        tc_commit(bar_vfree + j % VST);
        if (more) {
          if (!(ok = mbar_wait(bar_sfree + (j & 1), (j >> 1) & 1, p.err, kErrWaitMma))) break;
          if (!(ok = mbar_wait(bar_kfull + (j + 2) % KST, ((j + 2) / KST) & 1, p.err, kErrWaitMma))) break;
          tc_fence_after();
          issue_qk(j + 2, qkind);
        }
      }
      // every MMA this thread issued has completed once bar_drain fires
      tc_commit(bar_drain);
      mbar_wait(bar_drain, 0, p.err, kErrWaitDrain);
    }
  } else {
    // -------------------------------- softmax and epilogue (rows x column halves)
    const int row = threadIdx.x & 127;                 // TMEM lane / query row
    const int h = threadIdx.x >> 7;                    // column half of tiles and of O
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int qrow = u.qb * BLK + row;
    const float qs_log2 = (qrow < p.T ? __ldg(p.qs + (int64_t)bh * tp + qrow) : 0.f) * p.s2;
    bool ok = mbar_wait_warp(bar_q, 0, p.err, kErrWaitSoftmax);
    float m_ref = -INFINITY, l_sum = 0.f;
    bool o_live = false;      // O holds a contribution
    int j = 0, kind, idx;
    TileIter it(p, u);
    for (; it.next(kind, idx); ++j) {
      const bool exact = kind == kTileExact;
      uint32_t r[64];
      if (ok) ok = mbar_wait_warp(bar_kfree + j % KST, (j / KST) & 1, p.err, kErrWaitSoftmax);
      if (ok) {
        tc_fence_after();
        tmem_ld32(tS + (j & 1) * 128 + lane_base + h * 64, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32(tS + (j & 1) * 128 + lane_base + h * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_wait_ld();
      }
      tc_fence_before();
      mbar_arrive(bar_sfree + (j & 1));
      if (ok && exact) {
        // exact integer scores (fp32) * ks (_int8_fwd.py:329-330); the per-row factor qs * s2 (positive)
        // is applied to the row max and inside the exponent
        const float4* ks4 = reinterpret_cast<const float4*>(sKS + (j & 3) * 128 + h * 64);
#pragma unroll
        for (int i = 0; i < 64; i += 4) {
          const float4 k4 = ks4[i >> 2];
          const float2 s01 = mul2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])),
                                  make_float2(k4.x, k4.y));
          const float2 s23 = mul2(make_float2(__uint_as_float(r[i + 2]), __uint_as_float(r[i + 3])),
                                  make_float2(k4.z, k4.w));
          r[i] = __float_as_uint(s01.x);
          r[i + 1] = __float_as_uint(s01.y);
          r[i + 2] = __float_as_uint(s23.x);
          r[i + 3] = __float_as_uint(s23.y);
        }
      }
      // P.V(j-1) complete: the P / P.V columns and the int8 P buffer are free again
      bool pv_prev = j == 0;
      auto wait_pv = [&]() {
        if (ok && !pv_prev) {
          ok = mbar_wait_warp(bar_vfree + (j - 1) % VST, ((j - 1) / VST) & 1, p.err, kErrWaitSoftmax);
          tc_fence_after();
          pv_prev = true;
        }
      };
      uint32_t colmask[4];
      int tail_col = -1;
      bool masked = true;
      if (!exact) {
        it.approx_bits(idx, colmask);
        tail_col = (p.N - 1 >= idx * 128 && p.N - 1 < idx * 128 + 128) ? p.N - 1 - idx * 128 - h * 64 : -1;
        if (tail_col >= 64) tail_col = -1;
      } else {
        token_bits<128>(p.T - idx * BLK, colmask);
        masked = idx * BLK + BLK > p.T;
      }
      const uint32_t cm[2] = {h ? colmask[2] : colmask[0], h ? colmask[3] : colmask[1]};
      const float sc = exact ? qs_log2 : p.s2;   // scores -> log2 units (both positive)
      float pm = -INFINITY;
      if (ok) pm = (masked ? max64<true>(r, cm) : max64<false>(r, cm)) * sc;
      float* xm = sMax + (j & 1) * 256;
      xm[h * 128 + row] = pm;
      named_bar_sync(1, 256);
      const float mx = fmaxf(pm, xm[(1 - h) * 128 + row]);   // the tile's row max
      const float m_new = fmaxf(m_ref, mx);
      float alpha = 1.f;
      bool need = false;
      if (m_ref == -INFINITY) {
        m_ref = m_new;
      } else if (m_new > m_ref + 8.f) {
        alpha = fast_exp2(m_ref - m_new);
        m_ref = m_new;
        need = true;
      }
      // P in TMEM as bf16, P.V accumulated into O by the tensor core; O is rescaled first
      // when a row's reference max moved (warp-uniform, after P.V(j-1) is complete)
      if (__any_sync(0xffffffffu, need) && o_live) {
        wait_pv();
        if (ok) rescale_rows<64>(tO + lane_base + h * 64, alpha);
      }
      float psum = 0.f;
      if (exact && pv8) {
        // int8 P relative to the tile's max, scaled by beta / 127 (see exp_int8p_bf16_64)
        const float bm = mx;
        const float beta = mx == -INFINITY ? 0.f : fast_exp2(bm - m_ref);
        if (ok) psum = exp_int8p_bf16_64(r, sc, bm == -INFINITY ? 0.f : bm, beta * (1.0f / 127.0f));
        l_sum = l_sum * alpha + beta * psum;
      } else {
        const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
        if (ok)
          psum = exact ? exp_bf16_64<false>(r, sc, m_use, -1, 0.f, 1.f)
                       : exp_bf16_64<true>(r, sc, m_use, tail_col, (float)(p.T - (p.N - 1) * BLK), (float)BLK);
        l_sum = l_sum * alpha + psum;
      }
      wait_pv();                       // P columns free
      if (ok) {
        tmem_st32(tA + lane_base + h * 32, *reinterpret_cast<const uint32_t(*)[32]>(&r[0]));
        tmem_wait_st();
      }
      o_live = true;
      tc_fence_before();
      mbar_arrive(bar_pfull);
    }
    // epilogue: the last P.V, l = both halves' sums, O / l -> bf16 -> swizzled staging
    // (the q buffer) -> TMA store when every softmax thread succeeded
    if (j > 0 && ok) {
      ok = mbar_wait_warp(bar_vfree + (j - 1) % VST, ((j - 1) / VST) & 1, p.err, kErrWaitEpilogue);
      tc_fence_after();
    }
    sSum[h * 128 + row] = l_sum;
    if (!ok) *sBad = 1;
    named_bar_sync(1, 256);
    const float inv = 1.f / (sSum[row] + sSum[128 + row]);
    ok = ok && *sBad == 0;
    if (ok && j > 0) {
      uint8_t* sO = sQ;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t r[32];
        tmem_ld32(tO + lane_base + h * 64 + c * 32, r);
        tmem_wait_ld();
        const int chunk0 = c * 4;   // 64 bf16 of O half h = box h, chunks 0..7
#pragma unroll
        for (int v4 = 0; v4 < 4; ++v4) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(r[v4 * 8 + 0]) * inv, __uint_as_float(r[v4 * 8 + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(r[v4 * 8 + 2]) * inv, __uint_as_float(r[v4 * 8 + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(r[v4 * 8 + 4]) * inv, __uint_as_float(r[v4 * 8 + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(r[v4 * 8 + 6]) * inv, __uint_as_float(r[v4 * 8 + 7]) * inv);
          const int chunk = chunk0 + v4;
          *reinterpret_cast<uint4*>(sO + h * BOX + row * 128 + ((chunk ^ (row & 7)) << 4)) = w;
        }
      }
      fence_proxy_async_smem();
    }
    if (!ok) *sBad = 1;
    named_bar_sync(1, 256);
    if (threadIdx.x == 0 && j > 0 && *sBad == 0) {
      for (int i = 0; i < 2; ++i) tma_store_4d(&tm_o, sQ + i * BOX, i * 64, u.h, u.qb * BLK, u.b);
      bulk_commit_group();
      bulk_wait_group_read0();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// q 32 KB + qi codes 32 KB + K ring 64 KB + V ring 64 KB + key scales + barriers + mask
// row + exchange, plus 1 KB to align the tiles to 1024 bytes
size_t fwd_int8p_smem_bytes() {
  return (size_t)(2 * 32768 + 2 * 32768 + 2 * 32768) + 4 * 128 * 4 + 128 + 4 * kMaskCapI8 +
         4 * (512 + 256) + 16 + 1024;
}

cudaError_t launch_fwd_int8p(const FwdMaps& m, const FwdParams& p, cudaStream_t st) {
  const size_t smem = fwd_int8p_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(sol_fwd_int8p_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const unsigned grid = (unsigned)((int64_t)p.B * p.H * p.N);
  return launch_pdl(sol_fwd_int8p_kernel, dim3(grid), dim3(320), smem, st, m.q, m.kc, m.vc, m.o, m.qi,
                    m.ki, m.vi, m.v, p);
}

}  // namespace solb200
