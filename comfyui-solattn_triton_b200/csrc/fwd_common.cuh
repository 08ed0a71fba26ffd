// Pieces shared by the BF16 and INT8 block-sparse forward kernels.
#pragma once

#include <cuda_fp16.h>
#include "common.cuh"

namespace solb200 {

struct FwdParams {
  const uint32_t* mask;   // [B, H, N, nw] exact-block bits (routing output); null: dense
                          // attention (every key block exact, no approximate tiles)
  const int* order;       // [B*H*N] unit of each CTA (the schedule), or null: CTA i = unit i
  int* err;               // device error word
  int B, T, H, N, nw;     // T, N: query tokens and query blocks (units per head)
  int Tk, Nk;             // key tokens and key blocks (T and N except for dense cross-attention)
  float s2;               // softmax scale * log2(e)
  // INT8 path only
  const float* qs;        // [B, H, T] per-token Q scales
  const float* ks;        // [B, H, T] per-token K scales
  const float* vscale;    // [B, H, D] per-channel V scales (int8 P*V)
  int int8_pv;
  // bounded waits: limit of the pipeline's waits (the exit-path drains keep the default);
  // test hook: the CTA running unit `stall_unit` (-1: none) makes its MMA issuer wait on
  // a barrier that nothing completes, so that its pipeline waits run out
  uint64_t wait_ns;
  int stall_unit;
  // reordered calls: row i of the attention sequence is output token perm[i]; the
  // epilogue writes each row to out[b, perm[i], h, :] (dense BTHD) instead of the tile store
  const int64_t* perm;
  __nv_bfloat16* out;
};

// Masked dense calls (BF16 kernel, its bias instantiation only): an attention mask read as
// bias[b * bias_s[0] + h * bias_s[1] + q * bias_s[2] + k * bias_s[3]] (element strides, 0
// broadcasts) of kind kBias*: a bool false masks the key, a float value is added to the
// scaled score. bias_mul = 1 / scale, since the kernel adds the mask to the unscaled q . k.
// A kernel parameter of its own: growing FwdParams changes the other kernels' registers.
struct BiasParams {
  const void* bias;
  int bias_kind;
  float bias_mul;
  int64_t bias_s[4];
};

enum { kBiasNone = 0, kBiasBool = 1, kBiasF32 = 2, kBiasBF16 = 3, kBiasF16 = 4 };

struct FwdMaps {
  CUtensorMap q, k, v, kc, vc, o;      // bf16 operands and output
  CUtensorMap qi, ki, vi;              // int8 operands (INT8 path)
};

struct UnitInfo {
  int unit, b, h, qb;
  const uint32_t* row;   // this unit's nw mask words: global memory or a shared-memory
                         // copy, so they are read with generic (not ld.global.nc) loads
};

// Units are numbered head-major, (b*H + h)*N + qb. CTA i runs unit order[i]: the
// schedule keeps heads in order, so CTAs that run together share a head's K/V in L2,
// and within a head runs the query blocks with the most exact blocks first, so the
// grid's last wave is made of its shortest units.
__device__ __forceinline__ UnitInfo decode_unit(const FwdParams& p, int cta) {
  const int unit = p.order ? __ldg(p.order + cta) : cta;
  UnitInfo u;
  u.unit = unit;
  u.qb = unit % p.N;
  const int bh = unit / p.N;
  u.b = bh / p.H;
  u.h = bh % p.H;
  u.row = p.mask ? p.mask + ((int64_t)bh * p.N + u.qb) * p.nw : nullptr;
  return u;
}

enum { kTileApprox = 0, kTileExact = 1 };

// Reordered calls: the output token of this thread's tile row (row = query row of the
// unit), prefetched at the start of the unit into sTok[row] so that the epilogue's stores
// do not wait on it: perm[qb*BLK + row], or -1 for rows past T (not stored) and for an index
// outside [0, T) (recorded in the error word, not stored).
template <int BLK>
__device__ __forceinline__ void prefetch_row_token(const FwdParams& p, const UnitInfo& u, int row, int64_t* sTok) {
  if (row >= BLK) return;
  const int64_t pos = (int64_t)u.qb * BLK + row;
  int64_t tok = -1;
  if (pos < p.T) {
    tok = __ldg(p.perm + pos);
    if (tok < 0 || tok >= p.T) {
      atomicOr(p.err, kErrBadIndex);
      tok = -1;
    }
  }
  sTok[row] = tok;
}

// Epilogue of a reordered call: the unit's output tile, staged bf16 in shared memory as
// HD/64 boxes of BLK rows x 128 bytes (128-byte swizzle, box i at sO + i * BLK * 128), is
// written row by row to out[b, sTok[r], h, :] (the tokens prefetched by prefetch_row_token);
// warp w of the `nwarps` epilogue warps stores rows w, w + nwarps, ..., one coalesced row
// (HD * 2 bytes over the 32 lanes) per store; rows with token -1 are skipped.
template <int HD, int BLK>
__device__ __forceinline__ void store_rows_reordered(const uint8_t* sO, const int64_t* sTok, const FwdParams& p,
                                                     const UnitInfo& u, int warp, int nwarps, int lane) {
  constexpr int LB = HD * 2 / 32;                 // bytes per lane: 8 (HD 128) or 4 (HD 64)
  const int byte0 = lane * LB;                     // byte of the output row this lane stores
  const int box = byte0 >> 7, cb = byte0 & 127;    // 64-column box, byte inside its 128-byte row
  for (int r = warp; r < BLK; r += nwarps) {
    const int64_t tok = sTok[r];
    if (tok < 0) continue;
    const uint8_t* src = sO + box * (BLK * 128) + r * 128 + ((((cb >> 4) ^ (r & 7)) << 4) | (cb & 15));
    uint8_t* dst = reinterpret_cast<uint8_t*>(p.out + (((int64_t)u.b * p.T + tok) * p.H + u.h) * HD) + byte0;
    if (LB == 8) *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(src);
    else *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(src);
  }
}

__device__ __forceinline__ uint32_t low_bits(int n) {
  return n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : ((1u << n) - 1u));
}

// The tile sequence of one unit, identical for every warp role: first each
// 128-block chunk of the pooled keys that holds at least one approximate (valid,
// non-routed) block, then every routed block in ascending order.
struct TileIter {
  const uint32_t* row;    // null: dense (every one of the Nk key blocks is exact)
  int nw, N, nchunks;
  int phase, c, w;
  uint32_t bits;

  __device__ TileIter(const FwdParams& p, const UnitInfo& u)
      : row(u.row), nw(u.row ? p.nw : (p.Nk + 31) / 32), N(u.row ? p.N : p.Nk), nchunks((p.N + 127) / 128),
        phase(u.row ? 0 : 1), c(0), w(-1), bits(0) {}

  // Approximate-column bits of pooled chunk `chunk` (128 columns = 4 words).
  __device__ __forceinline__ void approx_bits(int chunk, uint32_t (&out)[4]) const {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int wi = chunk * 4 + i;
      out[i] = wi < nw ? (~row[wi]) & low_bits(N - wi * 32) : 0u;
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
      bits = row ? row[w] : low_bits(N - w * 32);
    }
  }
};

// The same walk in 64-row halves, the unit of the forward pipeline: each approximate
// chunk contributes the halves (64 pooled rows) that hold approximate columns, each
// routed block contributes its 64-token halves that hold at least one real token.
// row0 is the first pooled row (approximate) or token (exact) of the half.
template <int BLK>
struct HalfIter {
  TileIter tiles;
  int T;
  int pend0, pend1;   // the current tile's halves (scalars: no local-memory array)
  int npend, ipend, pkind;

  __device__ HalfIter(const FwdParams& p, const UnitInfo& u)
      : tiles(p, u), T(p.Tk), pend0(0), pend1(0), npend(0), ipend(0), pkind(0) {}

  __device__ __forceinline__ bool next(int& kind, int& row0) {
    while (ipend >= npend) {
      int k, idx;
      if (!tiles.next(k, idx)) return false;
      ipend = 0;
      pkind = k;
      if (k == kTileApprox) {
        uint32_t b[4];
        tiles.approx_bits(idx, b);
        const bool lo = (b[0] | b[1]) != 0, hi = (b[2] | b[3]) != 0;
        pend0 = lo ? idx * 128 : idx * 128 + 64;
        pend1 = idx * 128 + 64;
        npend = (lo ? 1 : 0) + (hi ? 1 : 0);
      } else {
        pend0 = idx * BLK;
        pend1 = idx * BLK + 64;
        npend = (BLK == 128 && idx * BLK + 64 < T) ? 2 : 1;
      }
    }
    kind = pkind;
    row0 = ipend == 0 ? pend0 : pend1;
    ++ipend;
    return true;
  }

  // approximate-column bits of the 64 pooled rows starting at row0 (a multiple of 64)
  __device__ __forceinline__ void approx_bits64(int row0, uint32_t (&out)[2]) const {
    uint32_t b[4];
    tiles.approx_bits(row0 >> 7, b);
    out[0] = (row0 & 64) ? b[2] : b[0];
    out[1] = (row0 & 64) ? b[3] : b[1];
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

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
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

// One tile of the online softmax for this thread's row (= TMEM lane), NCOLS score
// columns in TMEM at `t_s` (fp32). MASKED: columns whose bit in `colmask` is clear
// are excluded. WEIGHTED: the row sum weighs every column by `w_full`, except column
// `tail_col` by `w_tail` (pooled blocks stand for their token count).
// Updates the reference max m_ref (raised only when the tile exceeds it by more than
// 2^8; then this warp's accumulator rows in TMEM at `t_o` are rescaled when o_live)
// and the row sum l_sum, and writes bf16 P over the first NCOLS/2 score columns.
template <int NCOLS, bool MASKED, bool WEIGHTED, int HD>
__device__ __forceinline__ void softmax_tile(uint32_t t_s, uint32_t t_o, const uint32_t (&colmask)[4],
                                             float s2, float& m_ref, float& l_sum, bool o_live,
                                             int tail_col, float w_tail, float w_full) {
  uint32_t r[NCOLS];
#pragma unroll
  for (int c = 0; c < NCOLS / 32; ++c) tmem_ld32(t_s + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
  tmem_wait_ld();
  if (MASKED) {
#pragma unroll
    for (int i = 0; i < NCOLS; ++i)
      if (!((colmask[i >> 5] >> (i & 31)) & 1u)) r[i] = __float_as_uint(-INFINITY);
  }
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < NCOLS; i += 8) {
    m4[(i >> 3) & 3] = max3(m4[(i >> 3) & 3], max3(__uint_as_float(r[i]), __uint_as_float(r[i + 1]),
                                                   __uint_as_float(r[i + 2])),
                            max3(__uint_as_float(r[i + 3]), __uint_as_float(r[i + 4]),
                                 fmaxf(__uint_as_float(r[i + 5]),
                                       fmaxf(__uint_as_float(r[i + 6]), __uint_as_float(r[i + 7])))));
  }
  const float mx = max3(m4[0], m4[1], fmaxf(m4[2], m4[3])) * s2;
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
    rescale_rows<HD>(t_o, alpha);
  }
  const float neg_m = m_ref == -INFINITY ? 0.f : -m_ref;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float tail_p = 0.f;
#pragma unroll
  for (int i = 0; i < NCOLS; i += 2) {
    const float p0 = fast_exp2(fmaf(__uint_as_float(r[i]), s2, neg_m));
    const float p1 = fast_exp2(fmaf(__uint_as_float(r[i + 1]), s2, neg_m));
    acc[(i >> 1) & 3] += p0 + p1;
    if (WEIGHTED) tail_p += (i == tail_col ? p0 : 0.f) + (i + 1 == tail_col ? p1 : 0.f);
    r[i >> 1] = pack_bf16x2(p0, p1);   // P overwrites already-consumed registers
  }
  float s = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  if (WEIGHTED) s = s * w_full + tail_p * (w_tail - w_full);
  l_sum += s;
#pragma unroll
  for (int c = 0; c < NCOLS / 32; ++c)
    tmem_st16(t_s + c * 16, *reinterpret_cast<const uint32_t(*)[16]>(&r[c * 16]));
}

// One 64-column half of the online softmax for this thread's row. Same contract as
// softmax_tile, plus `before_rescale`, called (warp-uniformly) before the accumulator
// rows are rescaled so the caller can wait for in-flight P*V products first.
// `pre(ra, rb)` sees the half's raw scores (fp32 bits, columns 0-31 and 32-63) before
// the column mask and the row max; softmax_half passes none.
template <bool MASKED, bool WEIGHTED, int HD, typename Hook, typename Pre>
__device__ __forceinline__ void softmax_half_pre(uint32_t t_s, uint32_t t_o, const uint32_t (&colmask)[2],
                                                 float s2, float& m_ref, float& l_sum, bool o_live, int tail_col,
                                                 float w_tail, float w_full, Hook&& before_rescale, Pre&& pre) {
  uint32_t ra[32], rb[32];
  tmem_ld32(t_s, ra);
  tmem_ld32(t_s + 32, rb);
  tmem_wait_ld();
  pre(ra, rb);
  if (MASKED) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (!((colmask[0] >> i) & 1u)) ra[i] = __float_as_uint(-INFINITY);
      if (!((colmask[1] >> i) & 1u)) rb[i] = __float_as_uint(-INFINITY);
    }
  }
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    m4[(i >> 2) & 3] = max3(m4[(i >> 2) & 3],
                            max3(__uint_as_float(ra[i]), __uint_as_float(ra[i + 1]), __uint_as_float(ra[i + 2])),
                            max3(__uint_as_float(ra[i + 3]), __uint_as_float(rb[i]),
                                 max3(__uint_as_float(rb[i + 1]), __uint_as_float(rb[i + 2]),
                                      __uint_as_float(rb[i + 3]))));
  }
  const float mx = max3(m4[0], m4[1], fmaxf(m4[2], m4[3])) * s2;
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
    before_rescale();
    l_sum *= alpha;
    rescale_rows<HD>(t_o, alpha);
  }
  const float neg_m = m_ref == -INFINITY ? 0.f : -m_ref;
  const float2 s2v = make_float2(s2, s2), nmv = make_float2(neg_m, neg_m);
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  float tail_p = 0.f;
  uint32_t pa[16], pb[16];
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const float2 xa = fma2(make_float2(__uint_as_float(ra[i]), __uint_as_float(ra[i + 1])), s2v, nmv);
    const float2 xb = fma2(make_float2(__uint_as_float(rb[i]), __uint_as_float(rb[i + 1])), s2v, nmv);
    const float2 pa2 = make_float2(fast_exp2(xa.x), fast_exp2(xa.y));
    const float2 pb2 = make_float2(fast_exp2(xb.x), fast_exp2(xb.y));
    acc[(i >> 1) & 1] = add2(acc[(i >> 1) & 1], pa2);
    acc[2 + ((i >> 1) & 1)] = add2(acc[2 + ((i >> 1) & 1)], pb2);
    if (WEIGHTED) {
      tail_p += (i == tail_col ? pa2.x : 0.f) + (i + 1 == tail_col ? pa2.y : 0.f);
      tail_p += (i + 32 == tail_col ? pb2.x : 0.f) + (i + 33 == tail_col ? pb2.y : 0.f);
    }
    pa[i >> 1] = pack_bf16x2(pa2.x, pa2.y);
    pb[i >> 1] = pack_bf16x2(pb2.x, pb2.y);
  }
  const float2 a01 = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
  float s = a01.x + a01.y;
  if (WEIGHTED) s = s * w_full + tail_p * (w_tail - w_full);
  l_sum += s;
  tmem_st16(t_s, pa);
  tmem_st16(t_s + 16, pb);
}

template <bool MASKED, bool WEIGHTED, int HD, typename Hook>
__device__ __forceinline__ void softmax_half(uint32_t t_s, uint32_t t_o, const uint32_t (&colmask)[2], float s2,
                                             float& m_ref, float& l_sum, bool o_live, int tail_col,
                                             float w_tail, float w_full, Hook&& before_rescale) {
  softmax_half_pre<MASKED, WEIGHTED, HD>(t_s, t_o, colmask, s2, m_ref, l_sum, o_live, tail_col, w_tail, w_full,
                                         before_rescale, [](uint32_t (&)[32], uint32_t (&)[32]) {});
}

// Masked dense calls: adds this thread's mask row over keys k0 .. k0+63 to the raw scores
// (a bool false, or a -inf value, makes the score -inf; keys >= Tk are left alone, the
// column mask drops them). `row_off` is the element offset of mask[b, h, q, 0], or -1 for
// a row past Tq (nothing is read).
template <int KIND>
__device__ __forceinline__ float bias_value(const void* base, int64_t off) {
  if (KIND == kBiasBool) return __ldg(static_cast<const uint8_t*>(base) + off) ? 0.f : -INFINITY;
  if (KIND == kBiasF32) return __ldg(static_cast<const float*>(base) + off);
  if (KIND == kBiasBF16) return __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(base) + off));
  return __half2float(__ldg(static_cast<const __half*>(base) + off));
}

// element j of a 16-byte vector of mask elements, as the value added to a score
template <int KIND>
__device__ __forceinline__ float bias_lane(const uint4& w, int j) {
  constexpr int ES = KIND == kBiasBool ? 1 : (KIND == kBiasF32 ? 4 : 2);
  const int wi = (j * ES) >> 2;
  const uint32_t word = wi == 0 ? w.x : (wi == 1 ? w.y : (wi == 2 ? w.z : w.w));
  if (KIND == kBiasBool) return ((word >> ((j & 3) * 8)) & 0xffu) ? 0.f : -INFINITY;
  if (KIND == kBiasF32) return __uint_as_float(word);
  const uint16_t h = (uint16_t)(word >> ((j & 1) * 16));
  if (KIND == kBiasBF16) return __uint_as_float((uint32_t)h << 16);
  return __half2float(__ushort_as_half(h));
}

template <int KIND>
__device__ __forceinline__ void add_bias_value(uint32_t& r, float b, float mul) {
  r = __float_as_uint(b == -INFINITY ? -INFINITY : fmaf(b, mul, __uint_as_float(r)));
}

template <int KIND>
__device__ __forceinline__ void add_bias_row(const FwdParams& p, const BiasParams& bp, int64_t row_off, int k0,
                                             uint32_t (&ra)[32], uint32_t (&rb)[32]) {
  if (row_off < 0) return;
  constexpr int ES = KIND == kBiasBool ? 1 : (KIND == kBiasF32 ? 4 : 2);   // bytes per element
  constexpr int EPV = 16 / ES;                                              // elements per 16 bytes
  const int n = min(64, p.Tk - k0);
  const int64_t sk = bp.bias_s[3];
  const uint8_t* base = static_cast<const uint8_t*>(bp.bias) + (row_off + (int64_t)k0 * sk) * ES;
  if (n == 64 && sk == 1 && (reinterpret_cast<uintptr_t>(base) & 15u) == 0) {
    // a contiguous, 16-byte-aligned row of 64 elements: 64 * ES / 16 vector loads
#pragma unroll
    for (int v = 0; v < 64 / EPV; ++v) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(base) + v);
#pragma unroll
      for (int j = 0; j < EPV; ++j) {
        const int c = v * EPV + j;
        add_bias_value<KIND>(c < 32 ? ra[c & 31] : rb[c & 31], bias_lane<KIND>(w, j), bp.bias_mul);
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 64; ++j) {
    if (j < n)
      add_bias_value<KIND>(j < 32 ? ra[j & 31] : rb[j & 31], bias_value<KIND>(base, (int64_t)j * sk),
                           bp.bias_mul);
  }
}

cudaError_t launch_fwd_bf16(int hd, int blk, const FwdMaps& m, const FwdParams& p, cudaStream_t st);
cudaError_t launch_fwd_bf16_masked(int hd, const FwdMaps& m, const FwdParams& p, const BiasParams& bp,
                                   cudaStream_t st);
cudaError_t launch_fwd_int8(int hd, int blk, const FwdMaps& m, const FwdParams& p, cudaStream_t st);
size_t fwd_bf16_smem_bytes(int hd);

}  // namespace solb200
