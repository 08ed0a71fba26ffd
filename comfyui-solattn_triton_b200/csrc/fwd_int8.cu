// INT8 Sol-Attn block-sparse forward on sm_100a tensor cores.
//
// Same unit / tile walk as the BF16 kernel (fwd_bf16.cu). Approximate tiles are
// identical (bf16 q against the centred pooled keys, bf16 P * vc into the fp32
// accumulator). Exact tiles follow _forward_int8_ptr (_int8_fwd.py:311-365):
//   S = qi . ki^T on tcgen05 kind::i8 (int32 in TMEM); scores = S * (qs * s2) * ks.
//   INT8 P*V (int8_pv = 1): pe = 2^(s - rowmax_tile) in [0, 1], pi = int8(min(pe*127
//     + 0.5, 127)) written to shared memory; PV = pi . vi on kind::i8 into TMEM (over
//     the consumed scores); the softmax warps then fold it into the fp32 accumulator
//     as O = O * alpha + PV * (beta / 127) * vscale[d], beta = 2^(rowmax_tile - m).
//   BF16 P*V (int8_pv = 0): P = 2^(s - m) in bf16 in TMEM, P * V (bf16) accumulated by
//     the tensor core, as the BF16 kernel.
//
// Shared memory (HD = 128): sQ 32 KB bf16 q | sK 32 KB: kc chunk, or ki tile + (int8
// P or qi) | sV 32 KB: vc chunk, or vi tile + qi, or the bf16 V tile | small: ks tile,
// vscale. TMEM: 128 score columns + HD accumulator columns, two CTAs per SM.
#include "common.cuh"
#include "fwd_common.cuh"

namespace solb200 {

// Descriptor of a K-major / MN-major operand whose rows are `rb` bytes (64 or 128).
__device__ __forceinline__ uint64_t make_desc_rows(uint32_t addr, int rb, uint32_t lbo, uint32_t sbo_rows8) {
  uint64_t d = make_sw128_desc(addr, lbo, sbo_rows8);
  if (rb == 64) d = (d & ~((uint64_t)7 << 61)) | ((uint64_t)4 << 61);   // 64-byte swizzle
  return d;
}

// byte offset of 16-byte chunk `c` of row `r` in a swizzled tile with `rb`-byte rows
__device__ __forceinline__ uint32_t swz_off(int r, int c, int rb) {
  return rb == 128 ? (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)) : (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

template <int HD, int BLK>
__global__ void __launch_bounds__(192, 2)
sol_fwd_int8_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kc,
                    const __grid_constant__ CUtensorMap tm_vc, const __grid_constant__ CUtensorMap tm_o,
                    const __grid_constant__ CUtensorMap tm_qi, const __grid_constant__ CUtensorMap tm_ki,
                    const __grid_constant__ CUtensorMap tm_vi, const __grid_constant__ CUtensorMap tm_v,
                    const FwdParams p) {
  pdl_begin();
  constexpr int NBOX = HD / 64;
  constexpr uint32_t BOX = 128 * 128;
  constexpr int RB = HD;                    // bytes per int8 q/k/v row
  constexpr int PB = BLK;                   // bytes per int8 P row
  constexpr uint32_t IDESC_QK_APPROX = make_idesc(kFmtF32, kFmtBF16, kFmtBF16, 0, 0, 128, 128);
  constexpr uint32_t IDESC_PV_BF16 = make_idesc(kFmtF32, kFmtBF16, kFmtBF16, 0, 1, 128, HD);
  constexpr uint32_t IDESC_QK_I8 = make_idesc(kFmtS32, kFmtS8, kFmtS8, 0, 0, 128, BLK);
  constexpr uint32_t IDESC_PV_I8 = make_idesc(kFmtS32, kFmtS8, kFmtS8, 0, 1, 128, HD);
  constexpr uint32_t REGION = 2 * BOX;        // 32 KB per operand region for any head_dim
  constexpr uint32_t HALF = REGION / 2;       // upper half of a region

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + REGION;
  uint8_t* sV = sK + REGION;
  float* sKS2 = reinterpret_cast<float*>(sV + REGION);      // 2 x BLK floats (by tile parity)
  float* sVSC = sKS2 + 256;                                  // HD floats
  uint64_t* bars = reinterpret_cast<uint64_t*>(sVSC + 128);
  uint64_t* bar_q = bars + 0;
  uint64_t* bar_kfull = bars + 1;
  uint64_t* bar_vfull = bars + 2;
  uint64_t* bar_sfull = bars + 3;
  uint64_t* bar_pfull = bars + 4;
  uint64_t* bar_pvdone = bars + 5;
  uint64_t* bar_sfree = bars + 6;
  uint64_t* bar_qi = bars + 7;
  uint64_t* bar_drain = bars + 8;
  uint64_t* bar_s8free = bars + 9;   // score columns released after an int8 P*V fold
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  const bool pv8 = p.int8_pv != 0;
  // int8 operand homes (see the header comment)
  uint8_t* sQI = pv8 ? sV + HALF : sK + HALF;
  uint8_t* sP = sK + HALF;   // int8 P (pv8 only)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const UnitInfo u = decode_unit(p, blockIdx.x);
  const int bh = u.b * p.H + u.h;
  const int tp = p.N * BLK;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    mbar_init(bar_kfull, 1);
    mbar_init(bar_vfull, 1);
    mbar_init(bar_sfull, 1);
    mbar_init(bar_pfull, 128);
    mbar_init(bar_pvdone, 1);
    mbar_init(bar_sfree, 1);
    mbar_init(bar_qi, 1);
    mbar_init(bar_drain, 1);
    mbar_init(bar_s8free, 128);
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

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_kc);
      tma_prefetch_desc(&tm_vc);
      tma_prefetch_desc(&tm_ki);
      mbar_arrive_expect_tx(bar_q, NBOX * BOX + (pv8 ? HD * 4 : 0));
      for (int i = 0; i < NBOX; ++i) tma_load_4d(sQ + i * BOX, &tm_q, bar_q, i * 64, u.h, u.qb * BLK, u.b);
      if (pv8) bulk_load(sVSC, p.vscale + (int64_t)bh * HD, HD * 4, bar_q);
      TileIter it(p, u);
      int t = 0, kind, idx;
      bool ok = true, qi_loaded = false;
      while (it.next(kind, idx)) {
        if (kind == kTileExact && !qi_loaded) {
          // the int8 query tile's home is free once the last approximate P*V is done
          if (t > 0 && !(ok = mbar_wait(bar_pvdone, (t - 1) & 1, p.err, kErrWaitLoad))) break;
          mbar_arrive_expect_tx(bar_qi, 128 * RB);
          tma_load_4d(sQI, &tm_qi, bar_qi, 0, u.h, u.qb * BLK, u.b);
          qi_loaded = true;
        }
        if (t > 0 && !(ok = mbar_wait(bar_sfull, (t - 1) & 1, p.err, kErrWaitLoad))) break;
        if (kind == kTileApprox) {
          mbar_arrive_expect_tx(bar_kfull, NBOX * BOX);
          for (int i = 0; i < NBOX; ++i) tma_load_4d(sK + i * BOX, &tm_kc, bar_kfull, i * 64, u.h, idx * 128, u.b);
        } else {
          // the K scales are double-buffered by tile parity: the softmax warps may still
          // be reading the previous tile's scales
          mbar_arrive_expect_tx(bar_kfull, BLK * RB + BLK * 4);
          tma_load_4d(sK, &tm_ki, bar_kfull, 0, u.h, idx * BLK, u.b);
          bulk_load(sKS2 + (t & 1) * 128, p.ks + (int64_t)bh * tp + (int64_t)idx * BLK, BLK * 4, bar_kfull);
        }
        if (t > 0 && !(ok = mbar_wait(bar_pvdone, (t - 1) & 1, p.err, kErrWaitLoad))) {
          ++t;
          break;
        }
        if (kind == kTileApprox) {
          mbar_arrive_expect_tx(bar_vfull, NBOX * BOX);
          for (int i = 0; i < NBOX; ++i) tma_load_4d(sV + i * BOX, &tm_vc, bar_vfull, i * 64, u.h, idx * 128, u.b);
        } else if (pv8) {
          mbar_arrive_expect_tx(bar_vfull, BLK * RB);
          tma_load_4d(sV, &tm_vi, bar_vfull, 0, u.h, idx * BLK, u.b);
        } else {
          mbar_arrive_expect_tx(bar_vfull, NBOX * BLK * 128);
          for (int i = 0; i < NBOX; ++i) tma_load_4d(sV + i * BOX, &tm_v, bar_vfull, i * 64, u.h, idx * BLK, u.b);
        }
        ++t;
      }
      if (!ok && t > 0) {
        mbar_wait(bar_kfull, (t - 1) & 1, p.err, kErrWaitDrain);
        mbar_wait(bar_vfull, (t - 1) & 1, nullptr, 0);
      }
    }
  } else if (warp == 5) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      const uint32_t qi_base = smem_u32(sQI), p_base = smem_u32(sP);
      (void)NBOX;
      bool ok = mbar_wait(bar_q, 0, p.err, kErrWaitMma);
      bool qi_ready = false;
      TileIter it(p, u);
      int t = 0, kind, idx;
      // the score columns of tile t-1 are released on bar_sfree (tensor-core P*V, n_mma
      // such tiles so far) or on bar_s8free (int8 P*V folded by the softmax warps, n_fold)
      int n_mma = 0, n_fold = 0, prev_fold = -1;
      while (ok && it.next(kind, idx)) {
        if (kind == kTileExact && !qi_ready) {
          if (!(ok = mbar_wait(bar_qi, 0, p.err, kErrWaitMma))) break;
          qi_ready = true;
        }
        if (!(ok = mbar_wait(bar_kfull, t & 1, p.err, kErrWaitMma))) break;
        if (prev_fold == 1 && !(ok = mbar_wait(bar_s8free, (n_fold - 1) & 1, p.err, kErrWaitMma))) break;
        if (prev_fold == 0 && !(ok = mbar_wait(bar_sfree, (n_mma - 1) & 1, p.err, kErrWaitMma))) break;
        tc_fence_after();
        if (kind == kTileApprox) {
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint32_t off = (k >> 2) * BOX + (k & 3) * 32;
            mma_bf16_ss(tS, make_sw128_desc(q_base + off, 16, 1024), make_sw128_desc(k_base + off, 16, 1024),
                        IDESC_QK_APPROX, k > 0);
          }
        } else {
#pragma unroll
          for (int k = 0; k < RB / 32; ++k) {
            mma_i8_ss(tS, make_desc_rows(qi_base + k * 32, RB, 16, 8 * RB),
                      make_desc_rows(k_base + k * 32, RB, 16, 8 * RB), IDESC_QK_I8, k > 0);
          }
        }
        tc_commit(bar_sfull);
        if (!(ok = mbar_wait(bar_pfull, t & 1, p.err, kErrWaitMma))) break;
        if (!(ok = mbar_wait(bar_vfull, t & 1, p.err, kErrWaitMma))) break;
        tc_fence_after();
        if (kind == kTileExact && pv8) {
          // PV (int32) into the score columns; the softmax warps fold it into O and
          // then release the score columns (bar_sfree)
#pragma unroll
          for (int kk = 0; kk < BLK / 32; ++kk) {
            mma_i8_ss(tS, make_desc_rows(p_base + kk * 32, PB, 16, 8 * PB),
                      make_desc_rows(v_base + kk * 32 * RB, RB, 0, 8 * RB), IDESC_PV_I8, kk > 0);
          }
          tc_commit(bar_pvdone);
          ++n_fold;
          prev_fold = 1;
        } else {
          const int keys = kind == kTileApprox ? 128 : BLK;
          for (int kk = 0; kk < keys / 16; ++kk) {
            mma_bf16_ts(tO, tS + kk * 8, make_sw128_desc(v_base + kk * 2048, BOX, 1024), IDESC_PV_BF16,
                        (t > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(bar_pvdone);
          tc_commit(bar_sfree);
          ++n_mma;
          prev_fold = 0;
        }
        ++t;
      }
      tc_commit(bar_drain);
      mbar_wait(bar_drain, 0, p.err, kErrWaitDrain);
    }
  } else {
    // ------------------------------------------------- softmax + epilogue (rows)
    const int row = threadIdx.x;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const int qrow = u.qb * BLK + row;
    const float qs_log2 = (qrow < p.T ? __ldg(p.qs + (int64_t)bh * tp + qrow) : 0.f) * p.s2;
    float m_ref = -INFINITY, l_sum = 0.f;
    bool o_live = false;   // has anything been accumulated into tO yet
    TileIter it(p, u);
    int t = 0, kind, idx;
    bool ok = mbar_wait_warp(bar_q, 0, p.err, kErrWaitSoftmax);   // vscale is staged with q
    int last_kind = kTileApprox;
    while (ok && it.next(kind, idx)) {
      last_kind = kind;
      if (!(ok = mbar_wait_warp(bar_sfull, t & 1, p.err, kErrWaitSoftmax))) break;
      tc_fence_after();
      const float* sKS = sKS2 + (t & 1) * 128;
      if (kind == kTileApprox || !pv8) {
        // ------------- scores -> bf16 P in TMEM (approximate, or exact with bf16 P*V)
        uint32_t colmask[4];
        float w_tail = 0.f, w_full = 1.f;
        int tail_col = -1;
        const bool approx = kind == kTileApprox;
        if (approx) {
          it.approx_bits(idx, colmask);
          if (p.N - 1 >= idx * 128 && p.N - 1 < idx * 128 + 128) {
            tail_col = p.N - 1 - idx * 128;
            w_tail = (float)(p.T - (p.N - 1) * BLK);
          }
          w_full = (float)BLK;
        } else {
          token_bits<BLK>(p.T - idx * BLK, colmask);
        }
        const int nchunks = (approx ? 128 : BLK) / 32;
        float mx = -INFINITY;
        for (int c = 0; c < nchunks; ++c) {
          uint32_t r[32];
          tmem_ld32(tS + lane_base + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if ((colmask[c] >> i) & 1u) {
              const float s = approx ? __uint_as_float(r[i]) * p.s2
                                     : (float)(int)r[i] * (qs_log2 * sKS[c * 32 + i]);
              mx = fmaxf(mx, s);
            }
          }
        }
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
        if (__any_sync(0xffffffffu, need) && o_live) {
          l_sum *= alpha;
          rescale_rows<HD>(tO + lane_base, alpha);
        }
        const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
        float lsum = 0.f;
        for (int c = 0; c < nchunks; ++c) {
          uint32_t r[32];
          tmem_ld32(tS + lane_base + c * 32, r);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float pr[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int col = c * 32 + i + e;
              const bool v = (colmask[c] >> (i + e)) & 1u;
              const float s = approx ? __uint_as_float(r[i + e]) * p.s2
                                     : (float)(int)r[i + e] * (qs_log2 * sKS[col]);
              pr[e] = v ? fast_exp2(s - m_use) : 0.f;
              lsum += pr[e] * (col == tail_col ? w_tail : w_full);
            }
            pk[i >> 1] = pack_bf16x2(pr[0], pr[1]);
          }
          tmem_st16(tS + lane_base + c * 16, pk);
        }
        l_sum += lsum;
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_pfull);
        o_live = true;
      } else {
        // ------------------------------- exact tile with int8 P*V (_int8_fwd.py:342-353)
        uint32_t colmask[4];
        token_bits<BLK>(p.T - idx * BLK, colmask);
        float bm = -INFINITY;
        for (int c = 0; c < BLK / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tS + lane_base + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if ((colmask[c] >> i) & 1u) bm = fmaxf(bm, (float)(int)r[i] * (qs_log2 * sKS[c * 32 + i]));
        }
        float alpha = 1.f;
        if (m_ref == -INFINITY) {
          m_ref = bm;
        } else if (bm > m_ref + 8.f) {
          alpha = fast_exp2(m_ref - bm);
          m_ref = bm;
        }
        const float beta = fast_exp2(bm - m_ref);
        float psum = 0.f;
        for (int c = 0; c < BLK / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tS + lane_base + c * 32, r);
          tmem_wait_ld();
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            uint32_t word = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const bool v = (colmask[c] >> (i + e)) & 1u;
              const float s = (float)(int)r[i + e] * (qs_log2 * sKS[c * 32 + i + e]);
              const float pe = v ? fast_exp2(s - bm) : 0.f;
              psum += pe;
              const int pi = __float2int_rz(fminf(__fadd_rn(__fmul_rn(pe, 127.f), 0.5f), 127.f));
              word |= (uint32_t)(pi & 0xff) << (8 * e);
            }
            w[i >> 2] = word;
          }
          // 32 int8 = two 16-byte chunks of this row's P
          uint8_t* prow = sP;
          *reinterpret_cast<uint4*>(prow + swz_off(row, c * 2, PB)) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(prow + swz_off(row, c * 2 + 1, PB)) = make_uint4(w[4], w[5], w[6], w[7]);
        }
        l_sum = l_sum * alpha + beta * psum;
        fence_proxy_async_smem();   // P (generic stores) -> tensor core (async proxy)
        tc_fence_before();
        mbar_arrive(bar_pfull);
        // fold PV into the fp32 accumulator once the int8 MMA is done
        if (!(ok = mbar_wait_warp(bar_pvdone, t & 1, p.err, kErrWaitSoftmax))) break;
        tc_fence_after();
        const float f = beta * (1.0f / 127.0f);
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t pv[32], o[32];
          tmem_ld32(tS + lane_base + c * 32, pv);
          if (o_live) tmem_ld32(tO + lane_base + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float add = (float)(int)pv[i] * (f * sVSC[c * 32 + i]);
            o[i] = __float_as_uint(o_live ? fmaf(__uint_as_float(o[i]), alpha, add) : add);
          }
          tmem_st32(tO + lane_base + c * 32, o);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_s8free);
        o_live = true;
      }
      ++t;
    }
    // epilogue
    // an int8-P*V exact tile was folded into O by these threads themselves; any other
    // last tile was accumulated by the tensor core: wait for it
    const bool last_by_mma = !(pv8 && last_kind == kTileExact);
    if (ok && t > 0 && last_by_mma) ok = mbar_wait_warp(bar_pvdone, (t - 1) & 1, p.err, kErrWaitEpilogue);
    if (ok && t > 0) {
      tc_fence_after();
      const float inv = 1.f / l_sum;
      uint8_t* sO = sQ;
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tO + lane_base + c * 32, r);
        tmem_wait_ld();
        if (row < BLK) {
          const int box = (c * 32) / 64;
          const int col_byte0 = ((c * 32) % 64) * 2;
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(r[v4 * 8 + 0]) * inv, __uint_as_float(r[v4 * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(r[v4 * 8 + 2]) * inv, __uint_as_float(r[v4 * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(r[v4 * 8 + 4]) * inv, __uint_as_float(r[v4 * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(r[v4 * 8 + 6]) * inv, __uint_as_float(r[v4 * 8 + 7]) * inv);
            const int chunk = (col_byte0 >> 4) + v4;
            *reinterpret_cast<uint4*>(sO + box * (BLK * 128) + row * 128 + ((chunk ^ (row & 7)) << 4)) = w;
          }
        }
      }
      fence_proxy_async_smem();
    }
    named_bar_sync(1, 128);
    if (ok && t > 0 && threadIdx.x == 0) {
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

size_t fwd_int8_smem_bytes(int) { return (size_t)3 * 32768 + 1024 + 1024 + 512 + 256; }

template <int HD, int BLK>
static cudaError_t launch_t(const FwdMaps& m, const FwdParams& p, cudaStream_t st) {
  auto kern = sol_fwd_int8_kernel<HD, BLK>;
  size_t smem = fwd_int8_smem_bytes(HD);
  if (smem < 100 * 1024) smem = 100 * 1024;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const unsigned grid = (unsigned)((int64_t)p.B * p.H * p.N);
  return launch_pdl(kern, dim3(grid), dim3(192), smem, st, m.q, m.kc, m.vc, m.o, m.qi, m.ki, m.vi, m.v, p);
}

cudaError_t launch_fwd_int8(int hd, int blk, const FwdMaps& m, const FwdParams& p, cudaStream_t st) {
  // head_dim 128 with 128-token blocks (the video shapes) runs the pipelined kernel
  if (hd == 128 && blk == 128) return launch_fwd_int8p(m, p, st);
  if (hd == 128 && blk == 64) return launch_t<128, 64>(m, p, st);
  if (hd == 64 && blk == 128) return launch_t<64, 128>(m, p, st);
  return launch_t<64, 64>(m, p, st);
}

}  // namespace solb200
