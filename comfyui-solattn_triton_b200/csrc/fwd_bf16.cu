// BF16 Sol-Attn block-sparse forward on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA per (batch, head, query block). The query tile is always 128 rows (the
// tcgen05 M); with 64-token blocks the upper 64 rows are the next block's queries
// and are computed but never stored. The CTA walks a list of "tiles":
//   1. approximate tiles: 128-row chunks of the pooled keys kc / pooled values vc
//      that contain at least one non-routed block of this query block. Scores are
//      q . kc_j * s2; columns of routed or invalid blocks are masked; the row sum
//      weighs column j by the block length (the pooled block stands for len_j
//      tokens of mean key kc_j and summed value vc_j), as _tri_fwd.py:288-308.
//   2. exact tiles: every routed block in ascending order, full q . k^T * s2 with
//      tokens >= T masked (_tri_fwd.py:310-340).
// The online softmax keeps a per-row reference max that is raised only when a tile
// exceeds it by more than 2^8 (the output rescale in TMEM is then warp-uniform);
// P is stored as bf16 in TMEM over the consumed scores and fed to the P*V MMA as
// the A operand.
//
// Warp roles (192 threads): warps 0-3 softmax + epilogue (thread = row = TMEM lane),
// warp 4 TMA producer, warp 5 TMEM allocator + MMA issuer. Each CTA uses 96 KB of
// shared memory and 256 TMEM columns, so two CTAs share an SM and their softmax and
// MMA phases interleave.
#include "common.cuh"
#include "fwd_common.cuh"

namespace solb200 {

template <int HD, int BLK>
__global__ void __launch_bounds__(192, 2)
sol_fwd_bf16_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_kc,
                    const __grid_constant__ CUtensorMap tm_vc, const __grid_constant__ CUtensorMap tm_o,
                    const FwdParams p) {
  static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
  static_assert(BLK == 64 || BLK == 128, "block 64 or 128");
  constexpr int NBOX = HD / 64;                 // 64-column (128-byte) boxes per row
  constexpr uint32_t BOX = 128 * 128;           // bytes per 128-row box region
  constexpr uint32_t IDESC_QK_APPROX = make_idesc(kFmtF32, kFmtBF16, kFmtBF16, 0, 0, 128, 128);
  constexpr uint32_t IDESC_QK_EXACT = make_idesc(kFmtF32, kFmtBF16, kFmtBF16, 0, 0, 128, BLK);
  constexpr uint32_t IDESC_PV = make_idesc(kFmtF32, kFmtBF16, kFmtBF16, 0, 1, 128, HD);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + NBOX * BOX;
  uint8_t* sV = sK + NBOX * BOX;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + NBOX * BOX);
  uint64_t* bar_q = bars + 0;
  uint64_t* bar_kfull = bars + 1;
  uint64_t* bar_vfull = bars + 2;
  uint64_t* bar_sfull = bars + 3;
  uint64_t* bar_pfull = bars + 4;
  uint64_t* bar_pvdone = bars + 5;
  uint64_t* bar_drain = bars + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const UnitInfo u = decode_unit(p, blockIdx.x);

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    mbar_init(bar_kfull, 1);
    mbar_init(bar_vfull, 1);
    mbar_init(bar_sfull, 1);
    mbar_init(bar_pfull, 128);
    mbar_init(bar_pvdone, 1);
    mbar_init(bar_drain, 1);
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
  const uint32_t tS = tmem;          // scores (128 columns); P aliases the first columns
  const uint32_t tO = tmem + 128;    // output accumulator (HD columns)

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_kc);
      tma_prefetch_desc(&tm_vc);
      mbar_arrive_expect_tx(bar_q, NBOX * BOX);
      for (int i = 0; i < NBOX; ++i) tma_load_4d(sQ + i * BOX, &tm_q, bar_q, i * 64, u.h, u.qb * BLK, u.b);
      TileIter it(p, u);
      int t = 0, kind, idx;
      bool ok = true;
      while (it.next(kind, idx)) {
        if (t > 0 && !(ok = mbar_wait(bar_sfull, (t - 1) & 1, p.err, kErrWaitLoad))) break;
        const uint32_t rows = kind == kTileApprox ? 128 : BLK;
        mbar_arrive_expect_tx(bar_kfull, NBOX * rows * 128);
        for (int i = 0; i < NBOX; ++i) {
          if (kind == kTileApprox) tma_load_4d(sK + i * BOX, &tm_kc, bar_kfull, i * 64, u.h, idx * 128, u.b);
          else tma_load_4d(sK + i * BOX, &tm_k, bar_kfull, i * 64, u.h, idx * BLK, u.b);
        }
        if (t > 0 && !(ok = mbar_wait(bar_pvdone, (t - 1) & 1, p.err, kErrWaitLoad))) {
          ++t;   // the K load above is in flight: drain it below
          break;
        }
        mbar_arrive_expect_tx(bar_vfull, NBOX * rows * 128);
        for (int i = 0; i < NBOX; ++i) {
          if (kind == kTileApprox) tma_load_4d(sV + i * BOX, &tm_vc, bar_vfull, i * 64, u.h, idx * 128, u.b);
          else tma_load_4d(sV + i * BOX, &tm_v, bar_vfull, i * 64, u.h, idx * BLK, u.b);
        }
        ++t;
      }
      if (!ok && t > 0) {
        // exit path: let every issued copy land before the CTA's shared memory goes away
        mbar_wait(bar_kfull, (t - 1) & 1, p.err, kErrWaitDrain);
        mbar_wait(bar_vfull, (t - 1) & 1, nullptr, 0);
      }
    }
  } else if (warp == 5) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      bool ok = mbar_wait(bar_q, 0, p.err, kErrWaitMma);
      TileIter it(p, u);
      int t = 0, kind, idx;
      while (ok && it.next(kind, idx)) {
        if (!(ok = mbar_wait(bar_kfull, t & 1, p.err, kErrWaitMma))) break;
        if (t > 0 && !(ok = mbar_wait(bar_pvdone, (t - 1) & 1, p.err, kErrWaitMma))) break;
        tc_fence_after();
        const uint32_t idesc_qk = kind == kTileApprox ? IDESC_QK_APPROX : IDESC_QK_EXACT;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * BOX + (k & 3) * 32;
          mma_bf16_ss(tS, make_sw128_desc(q_base + off, 16, 1024), make_sw128_desc(k_base + off, 16, 1024),
                      idesc_qk, k > 0);
        }
        tc_commit(bar_sfull);
        if (!(ok = mbar_wait(bar_pfull, t & 1, p.err, kErrWaitMma))) break;
        if (!(ok = mbar_wait(bar_vfull, t & 1, p.err, kErrWaitMma))) break;
        tc_fence_after();
        const int keys = kind == kTileApprox ? 128 : BLK;
        for (int kk = 0; kk < keys / 16; ++kk) {
          mma_bf16_ts(tO, tS + kk * 8, make_sw128_desc(v_base + kk * 2048, BOX, 1024), IDESC_PV,
                      (t > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(bar_pvdone);
        ++t;
      }
      // every MMA this thread issued has completed once bar_drain fires
      tc_commit(bar_drain);
      mbar_wait(bar_drain, 0, p.err, kErrWaitDrain);
    }
  } else {
    // ------------------------------------------------- softmax + epilogue (rows)
    const int row = threadIdx.x;                       // 0..127 = TMEM lane
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    float m_ref = -INFINITY, l_sum = 0.f;
    TileIter it(p, u);
    int t = 0, kind, idx;
    bool ok = true;
    while (it.next(kind, idx)) {
      if (!(ok = mbar_wait_warp(bar_sfull, t & 1, p.err, kErrWaitSoftmax))) break;
      tc_fence_after();
      uint32_t colmask[4];
      if (kind == kTileApprox) {
        // column of the last (ragged) block, weighed by its true length
        it.approx_bits(idx, colmask);
        const int tail_col = (p.N - 1 >= idx * 128 && p.N - 1 < idx * 128 + 128) ? p.N - 1 - idx * 128 : -1;
        softmax_tile<128, true, true, HD>(tS + lane_base, tO + lane_base, colmask, p.s2, m_ref, l_sum, t > 0,
                                          tail_col, (float)(p.T - (p.N - 1) * BLK), (float)BLK);
      } else if ((idx + 1) * BLK > p.T) {
        token_bits<BLK>(p.T - idx * BLK, colmask);
        softmax_tile<BLK, true, false, HD>(tS + lane_base, tO + lane_base, colmask, p.s2, m_ref, l_sum, t > 0,
                                           -1, 0.f, 1.f);
      } else {
        softmax_tile<BLK, false, false, HD>(tS + lane_base, tO + lane_base, colmask, p.s2, m_ref, l_sum,
                                            t > 0, -1, 0.f, 1.f);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_pfull);
      ++t;
    }
    // epilogue: O / l -> bf16 -> swizzled staging (the free Q buffer) -> TMA store
    if (ok && t > 0 && (ok = mbar_wait_warp(bar_pvdone, (t - 1) & 1, p.err, kErrWaitEpilogue))) {
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

size_t fwd_bf16_smem_bytes(int hd) { return (size_t)3 * (hd / 64) * 128 * 128 + 1024 + 128; }

template <int HD, int BLK>
static cudaError_t launch_t(const FwdMaps& m, const FwdParams& p, cudaStream_t st) {
  auto kern = sol_fwd_bf16_kernel<HD, BLK>;
  // at least ~100 KB so that at most two CTAs (512 TMEM columns) share an SM
  size_t smem = fwd_bf16_smem_bytes(HD);
  if (smem < 100 * 1024) smem = 100 * 1024;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const unsigned grid = (unsigned)((int64_t)p.B * p.H * p.N);
  kern<<<grid, 192, smem, st>>>(m.q, m.k, m.v, m.kc, m.vc, m.o, p);
  return cudaGetLastError();
}

cudaError_t launch_fwd_bf16(int hd, int blk, const FwdMaps& m, const FwdParams& p, cudaStream_t st) {
  if (hd == 128 && blk == 128) return launch_t<128, 128>(m, p, st);
  if (hd == 128 && blk == 64) return launch_t<128, 64>(m, p, st);
  if (hd == 64 && blk == 128) return launch_t<64, 128>(m, p, st);
  return launch_t<64, 64>(m, p, st);
}

}  // namespace solb200
