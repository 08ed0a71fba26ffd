// Pieces shared by the BF16 and INT8 block-sparse forward kernels.
#pragma once

#include "common.cuh"

namespace solb200 {

struct FwdParams {
  const uint32_t* mask;   // [B, H, N, nw] exact-block bits (routing output)
  int* err;               // device error word
  int B, T, H, N, nw;
  float s2;               // softmax scale * log2(e)
  // INT8 path only
  const float* qs;        // [B, H, T] per-token Q scales
  const float* ks;        // [B, H, T] per-token K scales
  const float* vscale;    // [B, H, D] per-channel V scales (int8 P*V)
  int int8_pv;
};

struct FwdMaps {
  CUtensorMap q, k, v, kc, vc, o;      // bf16 operands and output
  CUtensorMap qi, ki, vi;              // int8 operands (INT8 path)
};

struct UnitInfo {
  int b, h, qb;
  const uint32_t* row;   // this unit's nw mask words
};

// Units are numbered head-major, (b*H + h)*N + qb, so CTAs that run together share
// a head's K/V in L2.
__device__ __forceinline__ UnitInfo decode_unit(const FwdParams& p, int unit) {
  UnitInfo u;
  u.qb = unit % p.N;
  const int bh = unit / p.N;
  u.b = bh / p.H;
  u.h = bh % p.H;
  u.row = p.mask + ((int64_t)bh * p.N + u.qb) * p.nw;
  return u;
}

enum { kTileApprox = 0, kTileExact = 1 };

__device__ __forceinline__ uint32_t low_bits(int n) {
  return n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : ((1u << n) - 1u));
}

// The tile sequence of one unit, identical for every warp role: first each
// 128-block chunk of the pooled keys that holds at least one approximate (valid,
// non-routed) block, then every routed block in ascending order.
struct TileIter {
  const uint32_t* row;
  int nw, N, nchunks;
  int phase, c, w;
  uint32_t bits;

  __device__ TileIter(const FwdParams& p, const UnitInfo& u)
      : row(u.row), nw(p.nw), N(p.N), nchunks((p.N + 127) / 128), phase(0), c(0), w(-1), bits(0) {}

  // Approximate-column bits of pooled chunk `chunk` (128 columns = 4 words).
  __device__ __forceinline__ void approx_bits(int chunk, uint32_t (&out)[4]) const {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int wi = chunk * 4 + i;
      out[i] = wi < nw ? (~__ldg(row + wi)) & low_bits(N - wi * 32) : 0u;
    }
  }

  __device__ __forceinline__ bool next(int& kind, int& idx) {
    while (phase == 0) {
      if (c >= nchunks) {
        phase = 1;
        break;
      }
      uint32_t b4[4];
      approx_bits(c, b4);
      const int cc = c++;
      if (b4[0] | b4[1] | b4[2] | b4[3]) {
        kind = kTileApprox;
        idx = cc;
        return true;
      }
    }
    while (true) {
      if (bits) {
        const int bit = __ffs(bits) - 1;
        bits &= bits - 1;
        kind = kTileExact;
        idx = w * 32 + bit;
        return true;
      }
      if (++w >= nw) return false;
      bits = __ldg(row + w);
    }
  }
};

// Bits of the key columns of an exact tile that hold real tokens (valid = T - kv0).
template <int BLK>
__device__ __forceinline__ void token_bits(int valid, uint32_t (&out)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) out[i] = i < BLK / 32 ? low_bits(valid - 32 * i) : 0u;
}

// 2^x on the special-function unit (ex2.approx; 2^-inf = 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Multiply this warp's 32 TMEM lanes of an HD-column fp32 accumulator by a per-row
// factor (every thread passes its own row's factor).
template <int HD>
__device__ __forceinline__ void rescale_rows(uint32_t taddr, float f) {
#pragma unroll 1
  for (int c = 0; c < HD / 32; ++c) {
    uint32_t r[32];
    tmem_ld32(taddr + c * 32, r);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
    tmem_st32(taddr + c * 32, r);
  }
}

cudaError_t launch_fwd_bf16(int hd, int blk, const FwdMaps& m, const FwdParams& p, cudaStream_t st);
cudaError_t launch_fwd_int8(int hd, int blk, const FwdMaps& m, const FwdParams& p, cudaStream_t st);
size_t fwd_bf16_smem_bytes(int hd);

}  // namespace solb200
