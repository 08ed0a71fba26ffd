// BF16 Sol-Attn block-sparse forward on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA per (batch, head, query block). The query tile is always 128 rows (the
// tcgen05 M); with 64-token blocks the upper 64 rows are the next block's queries
// and are computed but never stored. The CTA walks its keys in 64-row halves
// (HalfIter):
//   1. approximate halves: 64 pooled keys kc / pooled values vc holding at least one
//      non-routed block of this query block. Scores are q . kc_j * s2; columns of
//      routed or invalid blocks are masked; the row sum weighs column j by the block
//      length (a pooled block stands for len_j tokens of mean key kc_j and summed
//      value vc_j), as _tri_fwd.py:288-308.
//   2. exact halves of every routed block in ascending order: q . k^T * s2 with
//      tokens >= T masked (_tri_fwd.py:310-340).
// The online softmax keeps a per-row reference max that is raised only when a half
// exceeds it by more than 2^8; P is stored as bf16 in TMEM over the consumed scores
// and fed to the P*V MMA as the A operand.
//
// Pipeline: two slots (s & 1) for K, V, scores/P. The MMA issuer runs
//   QK(0) QK(1) | PV(0) QK(2) | PV(1) QK(3) | ...
// so the scores of half s+1 are ready while the softmax warps work on half s.
// Warp roles (192 threads): warps 0-3 softmax + epilogue (thread = row = TMEM lane),
// warp 4 TMA producer, warp 5 TMEM allocator + MMA issuer. 96 KB of shared memory and
// 256 TMEM columns per CTA: two CTAs share an SM.
#include "common.cuh"
#include "fwd_common.cuh"

namespace solb200 {

// BIAS: 0, or the mask kind (kBias*) of a masked dense instantiation (a mask added to the
// exact scores, see add_bias_row).
template <int HD, int BLK, int BIAS>
__global__ void __launch_bounds__(192, 2)
sol_fwd_bf16_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_kc,
                    const __grid_constant__ CUtensorMap tm_vc, const __grid_constant__ CUtensorMap tm_o,
                    const FwdParams p, const BiasParams bp) {
  pdl_begin();
  static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
  static_assert(BLK == 64 || BLK == 128, "block 64 or 128");
  constexpr int NBOX = HD / 64;                 // 64-column (128-byte) boxes per row
  constexpr uint32_t QBOX = 128 * 128;          // a 128-row box
  constexpr uint32_t HBOX = 64 * 128;           // a 64-row box
  constexpr uint32_t SLOT = NBOX * HBOX;        // one K (or V) half: 64 rows x HD
  constexpr uint32_t IDESC_QK = make_idesc(kFmtF32, kFmtBF16, kFmtBF16, 0, 0, 128, 64);
  constexpr uint32_t IDESC_PV = make_idesc(kFmtF32, kFmtBF16, kFmtBF16, 0, 1, 128, HD);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                    // NBOX x 16 KB
  uint8_t* sK = sQ + NBOX * QBOX;        // 2 slots x NBOX x 8 KB
  uint8_t* sV = sK + 2 * SLOT;           // 2 slots x NBOX x 8 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * SLOT);
  uint64_t* bar_q = bars + 0;
  uint64_t* bar_kfull = bars + 1;        // [2]
  uint64_t* bar_vfull = bars + 3;        // [2]
  uint64_t* bar_sfull = bars + 5;        // [2]
  uint64_t* bar_pfull = bars + 7;        // [2]
  uint64_t* bar_pvdone = bars + 9;       // [2]
  uint64_t* bar_drain = bars + 11;
  uint64_t* bar_never = bars + 12;       // completed by nothing (the stall_unit test hook)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  int64_t* sTok = reinterpret_cast<int64_t*>(bars + 32);   // [128] output tokens (reordered calls)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const UnitInfo u = decode_unit(p, blockIdx.x);

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_kfull + i, 1);
      mbar_init(bar_vfull + i, 1);
      mbar_init(bar_sfull + i, 1);
      mbar_init(bar_pfull + i, 128);
      mbar_init(bar_pvdone + i, 1);
    }
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
  const uint32_t tS = tmem;          // scores: slot 0 columns [0, 64), slot 1 [64, 128)
  const uint32_t tO = tmem + 128;    // output accumulator (HD columns)

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    // Loads are issued in the order the MMA issuer consumes them:
    //   K0 K1 | V0 K2 | V1 K3 | ...  K(s+2) waits for QK(s), V(s) for PV(s-2).
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_kc);
      tma_prefetch_desc(&tm_vc);
      mbar_arrive_expect_tx(bar_q, NBOX * QBOX);
      for (int i = 0; i < NBOX; ++i) tma_load_4d(sQ + i * QBOX, &tm_q, bar_q, i * 64, u.h, u.qb * BLK, u.b);
      auto load_half = [&](int s, int kind, int row0, bool is_v) {
        const int slot = s & 1;
        uint64_t* bar = (is_v ? bar_vfull : bar_kfull) + slot;
        uint8_t* dst = (is_v ? sV : sK) + slot * SLOT;
        const CUtensorMap* map = kind == kTileApprox ? (is_v ? &tm_vc : &tm_kc) : (is_v ? &tm_v : &tm_k);
        mbar_arrive_expect_tx(bar, SLOT);
        for (int i = 0; i < NBOX; ++i) tma_load_4d(dst + i * HBOX, map, bar, i * 64, u.h, row0, u.b);
      };
      HalfIter<BLK> itk(p, u), itv(p, u);
      int sk = 0, kind, row0;
      bool ok = true;
      int last_k = -1, last_v = -1;
      while (sk < 2 && itk.next(kind, row0)) {
        load_half(sk, kind, row0, false);
        last_k = sk++;
      }
      for (int s = 0; itv.next(kind, row0); ++s) {
        if (s >= 2 && !(ok = mbar_wait(bar_pvdone + (s & 1), ((s - 2) >> 1) & 1, p.err, kErrWaitLoad, p.wait_ns))) break;
        load_half(s, kind, row0, true);
        last_v = s;
        int kk, kr;
        if (itk.next(kk, kr)) {
          if (!(ok = mbar_wait(bar_sfull + (s & 1), (s >> 1) & 1, p.err, kErrWaitLoad, p.wait_ns))) break;
          load_half(s + 2, kk, kr, false);
          last_k = s + 2;
        }
      }
      if (!ok) {
        // exit path: let every issued copy land before the CTA's shared memory goes away
        if (last_k >= 0) mbar_wait(bar_kfull + (last_k & 1), (last_k >> 1) & 1, p.err, kErrWaitDrain);
        if (last_k >= 1) mbar_wait(bar_kfull + ((last_k - 1) & 1), ((last_k - 1) >> 1) & 1, nullptr, 0);
        if (last_v >= 0) mbar_wait(bar_vfull + (last_v & 1), (last_v >> 1) & 1, nullptr, 0);
        if (last_v >= 1) mbar_wait(bar_vfull + ((last_v - 1) & 1), ((last_v - 1) >> 1) & 1, nullptr, 0);
      }
    }
  } else if (warp == 5) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      auto issue_qk = [&](int s) {
        const int slot = s & 1;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t qo = (k >> 2) * QBOX + (k & 3) * 32;
          const uint32_t ko = slot * SLOT + (k >> 2) * HBOX + (k & 3) * 32;
          mma_bf16_ss(tS + slot * 64, make_sw128_desc(q_base + qo, 16, 1024),
                      make_sw128_desc(k_base + ko, 16, 1024), IDESC_QK, k > 0);
        }
        tc_commit(bar_sfull + slot);
      };
      bool ok = mbar_wait(bar_q, 0, p.err, kErrWaitMma, p.wait_ns);
      if (ok && u.unit == p.stall_unit) ok = mbar_wait(bar_never, 0, p.err, kErrWaitMma, p.wait_ns);
      HalfIter<BLK> itq(p, u), itp(p, u);
      int kind, row0, sq = 0;
      while (ok && sq < 2 && itq.next(kind, row0)) {
        if (!(ok = mbar_wait(bar_kfull + (sq & 1), (sq >> 1) & 1, p.err, kErrWaitMma, p.wait_ns))) break;
        tc_fence_after();
        issue_qk(sq++);
      }
      for (int s = 0; ok && itp.next(kind, row0); ++s) {
        const int slot = s & 1;
        const uint32_t par = (s >> 1) & 1;
        if (!(ok = mbar_wait(bar_pfull + slot, par, p.err, kErrWaitMma, p.wait_ns))) break;
        if (!(ok = mbar_wait(bar_vfull + slot, par, p.err, kErrWaitMma, p.wait_ns))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_bf16_ts(tO, tS + slot * 64 + kk * 8,
                      make_sw128_desc(v_base + slot * SLOT + kk * 2048, HBOX, 1024), IDESC_PV,
                      (s > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(bar_pvdone + slot);
        if (itq.next(kind, row0)) {
          // QK(s+2) overwrites slot s's P: let PV(s) finish reading it first
          if (!(ok = mbar_wait(bar_pvdone + slot, par, p.err, kErrWaitMma, p.wait_ns))) break;
          if (!(ok = mbar_wait(bar_kfull + slot, ((s + 2) >> 1) & 1, p.err, kErrWaitMma, p.wait_ns))) break;
          tc_fence_after();
          issue_qk(s + 2);
        }
      }
      // every MMA this thread issued has completed once bar_drain fires
      tc_commit(bar_drain);
      mbar_wait(bar_drain, 0, p.err, kErrWaitDrain);
    }
  } else {
    // ------------------------------------------------- softmax + epilogue (rows)
    const int row = threadIdx.x;                       // 0..127 = TMEM lane
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    if (p.perm) prefetch_row_token<BLK>(p, u, row, sTok);
    int64_t bias_off = -1;   // masked dense calls: this row's mask offset (row < BLK and q < T)
    if constexpr (BIAS) {
      const int64_t qtok = (int64_t)u.qb * BLK + row;
      if (row < BLK && qtok < p.T) bias_off = u.b * bp.bias_s[0] + u.h * bp.bias_s[1] + qtok * bp.bias_s[2];
    }
    float m_ref = -INFINITY, l_sum = 0.f;
    HalfIter<BLK> it(p, u);
    int s = 0, kind, row0;
    auto bias = [&](uint32_t (&ra)[32], uint32_t (&rb)[32]) {
      add_bias_row<BIAS == 0 ? kBiasF32 : BIAS>(p, bp, bias_off, row0, ra, rb);
    };
    bool ok = true;
    for (; it.next(kind, row0); ++s) {
      const int slot = s & 1;
      if (!(ok = mbar_wait_warp(bar_sfull + slot, (s >> 1) & 1, p.err, kErrWaitSoftmax, p.wait_ns))) break;
      tc_fence_after();
      const uint32_t ts = tS + lane_base + slot * 64;
      // before rescaling O, every P*V issued so far must be complete
      auto drain = [&]() {
        ok = mbar_wait_warp(bar_pvdone + ((s - 1) & 1), ((s - 1) >> 1) & 1, p.err, kErrWaitSoftmax, p.wait_ns);
        tc_fence_after();
      };
      uint32_t colmask[2];
      if (kind == kTileApprox) {
        it.approx_bits64(row0, colmask);
        const int tail_col = (p.N - 1 >= row0 && p.N - 1 < row0 + 64) ? p.N - 1 - row0 : -1;
        softmax_half<true, true, HD>(ts, tO + lane_base, colmask, p.s2, m_ref, l_sum, s > 0, tail_col,
                                     (float)(p.T - (p.N - 1) * BLK), (float)BLK, drain);
      } else if (row0 + 64 > p.Tk) {
        colmask[0] = low_bits(p.Tk - row0);
        colmask[1] = low_bits(p.Tk - row0 - 32);
        if constexpr (BIAS)
          softmax_half_pre<true, false, HD>(ts, tO + lane_base, colmask, p.s2, m_ref, l_sum, s > 0, -1, 0.f, 1.f,
                                            drain, bias);
        else
          softmax_half<true, false, HD>(ts, tO + lane_base, colmask, p.s2, m_ref, l_sum, s > 0, -1, 0.f, 1.f,
                                        drain);
      } else {
        if constexpr (BIAS)
          softmax_half_pre<false, false, HD>(ts, tO + lane_base, colmask, p.s2, m_ref, l_sum, s > 0, -1, 0.f,
                                             1.f, drain, bias);
        else
          softmax_half<false, false, HD>(ts, tO + lane_base, colmask, p.s2, m_ref, l_sum, s > 0, -1, 0.f, 1.f,
                                         drain);
      }
      if (!ok) break;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_pfull + slot);
    }
    // epilogue: O / l -> bf16 -> swizzled staging (the free Q buffer) -> TMA store
    if (ok && s > 0 && (ok = mbar_wait_warp(bar_pvdone + ((s - 1) & 1), ((s - 1) >> 1) & 1, p.err,
                                            kErrWaitEpilogue, p.wait_ns))) {
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
    if (ok && s > 0 && p.perm) {
      store_rows_reordered<HD, BLK>(sQ, sTok, p, u, warp, 4, lane);
    } else if (ok && s > 0 && threadIdx.x == 0) {
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

// q + K and V slots, barriers (256 B) and the output-token row (1 KB), plus 1 KB to align
size_t fwd_bf16_smem_bytes(int hd) { return (size_t)(hd / 64) * (128 * 128 + 4 * 64 * 128) + 1024 + 256 + 1024; }

template <int HD, int BLK, int BIAS = 0>
static cudaError_t launch_t(const FwdMaps& m, const FwdParams& p, cudaStream_t st, const BiasParams& bp = {}) {
  auto kern = sol_fwd_bf16_kernel<HD, BLK, BIAS>;
  // at least ~100 KB so that at most two CTAs (512 TMEM columns) share an SM
  size_t smem = fwd_bf16_smem_bytes(HD);
  if (smem < 100 * 1024) smem = 100 * 1024;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const unsigned grid = (unsigned)((int64_t)p.B * p.H * p.N);
  return launch_pdl(kern, dim3(grid), dim3(192), smem, st, m.q, m.k, m.v, m.kc, m.vc, m.o, p, bp);
}

cudaError_t launch_fwd_bf16(int hd, int blk, const FwdMaps& m, const FwdParams& p, cudaStream_t st) {
  if (hd == 128 && blk == 128) return launch_t<128, 128>(m, p, st);
  if (hd == 128 && blk == 64) return launch_t<128, 64>(m, p, st);
  if (hd == 64 && blk == 128) return launch_t<64, 128>(m, p, st);
  return launch_t<64, 64>(m, p, st);
}

// Masked dense calls: 128-token query tiles, every key block exact (p.mask null).
cudaError_t launch_fwd_bf16_masked(int hd, const FwdMaps& m, const FwdParams& p, const BiasParams& bp,
                                   cudaStream_t st) {
  if (p.mask || !bp.bias) return cudaErrorInvalidValue;
  switch (bp.bias_kind) {
    case kBiasBool:
      return hd == 128 ? launch_t<128, 128, kBiasBool>(m, p, st, bp) : launch_t<64, 128, kBiasBool>(m, p, st, bp);
    case kBiasF32:
      return hd == 128 ? launch_t<128, 128, kBiasF32>(m, p, st, bp) : launch_t<64, 128, kBiasF32>(m, p, st, bp);
    case kBiasBF16:
      return hd == 128 ? launch_t<128, 128, kBiasBF16>(m, p, st, bp) : launch_t<64, 128, kBiasBF16>(m, p, st, bp);
    case kBiasF16:
      return hd == 128 ? launch_t<128, 128, kBiasF16>(m, p, st, bp) : launch_t<64, 128, kBiasF16>(m, p, st, bp);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace solb200
