// Bandwidth-bound stages of the Sol-Attn path (sm_100a):
//   pool_kernel      one pass over Q, K, V: kc (block mean of K), vc (block sum of V),
//                    q-block centroids, optional per-block |V| max
//   moments_kernel   per (b, h): kc mean/variance (INT8: k_mean, kc centred in place,
//                    V scales)
//   route_kernel     per-q-block routing threshold, exact-block bitmask [B,H,N,NW],
//                    counts, optional index lists
//   quant_qkv_kernel per-token int8 of Q and of K - k_mean, per-channel int8 of V
//   morton kernels   Z-order ranks (no sort) and a row gather for the reorder
//
// Reductions that the reference performs in a defined order are done here in the
// same order (documented at each kernel) so that pooled keys, thresholds and int8
// values agree bit for bit with the reference.
#include "prep.cuh"

namespace solb200 {

// ---------------------------------------------------------------------- pool


__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&x)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8_bf16(const float (&x)[8]) {
  uint4 u;
  u.x = pack_bf16x2(x[0], x[1]);
  u.y = pack_bf16x2(x[2], x[3]);
  u.z = pack_bf16x2(x[4], x[5]);
  u.w = pack_bf16x2(x[6], x[7]);
  return u;
}

// RN(x / s) for s > 0 from y = RN(1/s) (__frcp_rn, computed once per scale) without a
// division per element, by Markstein's theorem (Markstein 1990; Muller et al.,
// Handbook of Floating-Point Arithmetic, section on FMA-based division): if y is within
// half an ulp of 1/s, q within one ulp of x/s and r = x - s*q exact (an FMA), then
// RN(q + r*y) = RN(x/s). q0 = RN(x*y) can be 1.5 ulp off, so one correction first
// brings it within half an ulp (plus a rounding of its remainder), then the second
// is the theorem's step. Exact while the remainders are normal numbers, which holds
// for every quotient the int8 codes depend on (|x/s| >= 2^-2 with s >= 1e-8); tiny
// quotients may differ in the last place and still round to the code 0.
__device__ __forceinline__ float quotient_rn(float x, float s, float y) {
  const float q0 = __fmul_rn(x, y);
  const float q1 = __fmaf_rn(__fmaf_rn(-s, q0, x), y, q0);
  return __fmaf_rn(__fmaf_rn(-s, q1, x), y, q1);
}

// eight int8 codes (low bytes of c[0..7]) packed into two words, c[0] lowest
__device__ __forceinline__ uint2 pack_codes(const uint32_t (&c)[8]) {
  uint32_t a, b, lo, hi;
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(a) : "r"(c[0]), "r"(c[1]));
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(b) : "r"(c[2]), "r"(c[3]));
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(lo) : "r"(a), "r"(b));
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(a) : "r"(c[4]), "r"(c[5]));
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(b) : "r"(c[6]), "r"(c[7]));
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(hi) : "r"(a), "r"(b));
  return make_uint2(lo, hi);
}

// One thread owns 8 consecutive channels (16 bytes) of one head and one of the three
// tensors (role 0: Q -> centroid; role 1: K -> kc; role 2:
// V -> vc and |V| max), so a call with few heads still has three threads per channel
// group in flight. Rows are accumulated in token order (row 0 first) in fp32, the
// order of the reference's block sums; the loads of ROWS rows are issued before any of
// them is added, so a thread keeps ROWS x 16 bytes in flight.
// Grid: (3*ceil(H*D/8 / NT), Npad, B), role = blockIdx.x % 3 so that the three roles
// interleave in launch order; NT = 32 or 64 threads (launch_pool_t). The INT8 codes of
// Q are formed by quant_qkv_kernel, with those of K and V.
template <int HD, bool VAMAX>
__global__ void __launch_bounds__(64) pool_kernel(PoolParams p) {
  pdl_begin();
  constexpr int LANES_PER_HEAD = HD / 8;
  constexpr int ROWS = 16;
  const int g = (blockIdx.x / 3) * blockDim.x + threadIdx.x;
  const int n = blockIdx.y, role = blockIdx.x % 3, b = blockIdx.z;
  const bool active = g < p.H * LANES_PER_HEAD;
  const int h = g / LANES_PER_HEAD;
  const int d0 = (g % LANES_PER_HEAD) * 8;
  const int64_t out_off = (((int64_t)b * p.npad + n) * p.H + h) * HD + d0;
  if (n >= p.N) {   // zero padding rows of kc / vc
    if (active && role > 0)
      *reinterpret_cast<uint4*>((role == 1 ? p.kc : p.vc) + out_off) = make_uint4(0, 0, 0, 0);
    return;
  }
  const int r0 = n * p.blk;
  const int r1 = min(p.T, r0 + p.blk);
  // reordered calls: the block's tokens, read once per CTA (checked) so that the row loads
  // below do not wait behind an index load each
  __shared__ int64_t s_tok[128];
  if (p.perm) {
    for (int i = threadIdx.x; i < r1 - r0; i += blockDim.x) s_tok[i] = order_row(p.perm, r0 + i, p.T, p.err);
    __syncthreads();
  }
  const __nv_bfloat16* src;
  int64_t st;
  __nv_bfloat16* copy;   // the reordered dense copy of this role's tensor, or null
  if (role == 0) {
    src = p.q + (int64_t)b * p.sq_b + (int64_t)h * p.sq_h + d0;
    st = p.sq_t;
    copy = p.qcopy;
  } else if (role == 1) {
    src = p.k + (int64_t)b * p.sk_b + (int64_t)h * p.sk_h + d0;
    st = p.sk_t;
    copy = p.kcopy;
  } else {
    src = p.v + (int64_t)b * p.sv_b + (int64_t)h * p.sv_h + d0;
    st = p.sv_t;
    copy = p.vcopy;
  }
  float sum[8], vmax[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sum[i] = vmax[i] = 0.f;
  for (int rb = r0; rb < r1; rb += ROWS) {
    uint4 u[ROWS];
#pragma unroll
    for (int j = 0; j < ROWS; ++j)
      u[j] = (active && rb + j < r1)
                 ? __ldg(reinterpret_cast<const uint4*>(src + (p.perm ? s_tok[rb + j - r0] : (int64_t)(rb + j)) * st))
                 : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < ROWS; ++j) {
      const int r = rb + j;
      if (r >= r1) break;   // uniform over the CTA
      if (copy && active)
        *reinterpret_cast<uint4*>(copy + (((int64_t)b * p.T + r) * p.H + h) * HD + d0) = u[j];
      float x[8];
      {
        const __nv_bfloat162* hx = reinterpret_cast<const __nv_bfloat162*>(&u[j]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(hx[i]);
          x[2 * i] = f.x;
          x[2 * i + 1] = f.y;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) sum[i] = __fadd_rn(sum[i], x[i]);
      if (VAMAX && role == 2) {
#pragma unroll
        for (int i = 0; i < 8; ++i) vmax[i] = fmaxf(vmax[i], fabsf(x[i]));
      }
    }
  }
  if (!active) return;
  const float len = (float)(r1 - r0);
  const int64_t c_off = (((int64_t)b * p.N + n) * p.H + h) * HD + d0;
  if (role == 0) {
    float4* cp = reinterpret_cast<float4*>(p.centroid + c_off);
    cp[0] = make_float4(__fdiv_rn(sum[0], len), __fdiv_rn(sum[1], len),
                        __fdiv_rn(sum[2], len), __fdiv_rn(sum[3], len));
    cp[1] = make_float4(__fdiv_rn(sum[4], len), __fdiv_rn(sum[5], len),
                        __fdiv_rn(sum[6], len), __fdiv_rn(sum[7], len));
  } else if (role == 1) {
    float kcv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) kcv[i] = __fdiv_rn(bf16_round(sum[i]), len);   // bf16 block sum, then / len
    *reinterpret_cast<uint4*>(p.kc + out_off) = pack8_bf16(kcv);
  } else {
    *reinterpret_cast<uint4*>(p.vc + out_off) = pack8_bf16(sum);
    if (VAMAX) {
      float4* ap = reinterpret_cast<float4*>(p.vamax + c_off);
      ap[0] = make_float4(vmax[0], vmax[1], vmax[2], vmax[3]);
      ap[1] = make_float4(vmax[4], vmax[5], vmax[6], vmax[7]);
    }
  }
}

// ------------------------------------------------------------------- moments

// Sum of `count` values x(i) in the order of ATen's CPU cascade sum for a strided
// (outer) reduction: rows are added in order into level 0; every 2^lp rows level 0
// is folded into level 1, every 2^(2 lp) rows level 1 into level 2, and so on;
// finally the levels are added from 0 up. lp = max(4, ceil(log2(count)) / 4).
// This is the order torch.mean uses for the reference's kc moments, so the result
// matches it bit for bit.
template <typename F>
__device__ float cascade_sum(int count, F x) {
  int lp = 0;
  while ((1 << lp) < count) ++lp;
  lp = max(4, lp / 4);
  const int step = 1 << lp;
  const int mask = step - 1;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int i = 0;
  while (i + step <= count) {
    for (int j = 0; j < step; ++j, ++i) acc[0] = __fadd_rn(acc[0], x(i));
    for (int j = 1; j < 4; ++j) {
      acc[j] = __fadd_rn(acc[j], acc[j - 1]);
      acc[j - 1] = 0.f;
      if ((i & (mask << (j * lp))) != 0) break;
    }
  }
  for (; i < count; ++i) acc[0] = __fadd_rn(acc[0], x(i));
  for (int j = 1; j < 4; ++j) acc[0] = __fadd_rn(acc[0], acc[j]);
  return acc[0];
}

// numpy's float32 sum of n (a multiple of 8, <= 128) values: eight interleaved
// partial sums combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)).
template <int N, typename F>
__device__ __forceinline__ float pairwise_sum(F x) {
  static_assert(N % 8 == 0 && N <= 128, "pairwise_sum: n must be a multiple of 8, <= 128");
  float r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) r[j] = x(j);
#pragma unroll
  for (int i = 8; i < N; i += 8)
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(r[j], x(i + j));
  return __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                   __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
}


// ATen's cascade sum (above) of `count` values in parallel, bit for bit: level 0 always
// restarts from zero, so each chunk of 2^lp values can be summed by its own thread in
// order; one thread per channel then replays the level folds over the chunk sums and
// adds the tail. x(n, d) gives value n of channel d; the result for channel d is
// written to out[d]. Called by all NT threads of the CTA.
template <int HD, int NT, typename F>
__device__ void cascade_sum_par(int count, F x, float* s_chunk /* [64][HD] */, float* out) {
  int lp = 0;
  while ((1 << lp) < count) ++lp;
  lp = max(4, lp / 4);
  const int step = 1 << lp;            // <= 64 for count < 2^24
  const int mask = step - 1;
  const int full = count / step;       // chunks taken by the cascade's main loop
  const int d = threadIdx.x;           // the folding thread of channel d (d < HD)
  float acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
  for (int g0 = 0; g0 < full; g0 += step) {
    const int gn = min(step, full - g0);   // chunks in this group
    for (int it = threadIdx.x; it < gn * HD; it += NT) {
      const int c = it / HD, dd = it % HD;
      const int n0 = (g0 + c) * step;
      float a = 0.f;
      for (int j = 0; j < step; ++j) a = __fadd_rn(a, x(n0 + j, dd));
      s_chunk[c * HD + dd] = a;
    }
    __syncthreads();
    if (d < HD) {
      for (int c = 0; c < gn; ++c) {
        const int i = (g0 + c + 1) * step;   // values consumed after this chunk
        acc1 = __fadd_rn(acc1, s_chunk[c * HD + d]);
        if ((i & (mask << lp)) != 0) continue;
        acc2 = __fadd_rn(acc2, acc1);
        acc1 = 0.f;
        if ((i & (mask << (2 * lp))) != 0) continue;
        acc3 = __fadd_rn(acc3, acc2);
        acc2 = 0.f;
      }
    }
    __syncthreads();
  }
  if (d < HD) {
    float tail = 0.f;
    for (int n = full * step; n < count; ++n) tail = __fadd_rn(tail, x(n, d));
    out[d] = __fadd_rn(__fadd_rn(__fadd_rn(tail, acc1), acc2), acc3);
  }
  __syncthreads();
}

// One CTA per (b, h, 16-channel slab), 256 threads. The slab's kc values (N x 16 bf16)
// are staged in shared memory once and both cascade passes read them there (STAGED;
// slabs too large for shared memory read them from global memory).
// BF16 mode (_preprocess.py:240-243): kcm = mean_n kc, kcv = mean_n (kc-kcm)^2.
// INT8 mode (_fused_prep.py:77-81; _fused_quant.py:103): k_mean = mean_n kc,
//   kc <- bf16(kc - k_mean), kcv = mean_n kc^2, vscale = max(amax/127, 1e-8).
// The per-q-block thresholds that use these moments are computed by route_kernel.
constexpr int kMomentsCh = 16;
constexpr int kMomentsThreads = 256;

template <int HD, bool INT8, bool STAGED>
__global__ void __launch_bounds__(kMomentsThreads) moments_kernel(MomentsParams p) {
  pdl_begin();
  constexpr int NT = kMomentsThreads, CH = kMomentsCh;
  extern __shared__ __align__(16) __nv_bfloat16 s_x[];   // [N][CH] when STAGED
  __shared__ float s_chunk[64 * CH];
  __shared__ float s_mean[CH], s_var[CH];
  const int bh = blockIdx.x, c0 = blockIdx.y * CH;
  const int b = bh / p.H, h = bh % p.H;
  const int64_t row = (int64_t)p.H * HD;
  __nv_bfloat16* kc0 = p.kc + ((int64_t)b * p.npad) * row + (int64_t)h * HD + c0;
  if (STAGED) {
    for (int i = threadIdx.x; i < p.N * (CH / 8); i += NT) {
      const int n = i / (CH / 8), part = i % (CH / 8);
      *reinterpret_cast<uint4*>(s_x + n * CH + part * 8) =
          __ldg(reinterpret_cast<const uint4*>(kc0 + (int64_t)n * row + part * 8));
    }
    __syncthreads();
  }
  auto kc_at = [&](int n, int d) {
    return __bfloat162float(STAGED ? s_x[n * CH + d] : kc0[(int64_t)n * row + d]);
  };
  cascade_sum_par<CH, NT>(p.N, kc_at, s_chunk, s_mean);
  if (threadIdx.x < CH) s_mean[threadIdx.x] = __fdiv_rn(s_mean[threadIdx.x], (float)p.N);
  __syncthreads();
  if (INT8) {
    for (int i = threadIdx.x; i < p.N * CH; i += NT) {
      const int n = i / CH, d = i % CH;
      const __nv_bfloat16 cb = __float2bfloat16_rn(__fsub_rn(kc_at(n, d), s_mean[d]));
      kc0[(int64_t)n * row + d] = cb;
      if (STAGED) s_x[n * CH + d] = cb;
    }
    __syncthreads();
    cascade_sum_par<CH, NT>(p.N, [&](int n, int d) {
      const float x = kc_at(n, d);
      return __fmul_rn(x, x);
    }, s_chunk, s_var);
    if (p.vamax) {
      // |V| max over the blocks: order-free, partial maxima over row strips
      float* s_max = s_chunk;
      constexpr int STRIPS = NT / CH;
      const int d = threadIdx.x % CH, strip = threadIdx.x / CH;
      const float* vam = p.vamax + ((int64_t)b * p.N) * row + (int64_t)h * HD + c0 + d;
      float amax = 0.f;
#pragma unroll 4
      for (int n = strip; n < p.N; n += STRIPS) amax = fmaxf(amax, __ldg(vam + (int64_t)n * row));
      s_max[strip * CH + d] = amax;
      __syncthreads();
      if (threadIdx.x < CH) {
        float m = 0.f;
        for (int k = 0; k < STRIPS; ++k) m = fmaxf(m, s_max[k * CH + threadIdx.x]);
        p.vscale[(int64_t)bh * HD + c0 + threadIdx.x] = fmaxf(__fdiv_rn(m, 127.f), 1e-8f);
      }
    }
  } else {
    cascade_sum_par<CH, NT>(p.N, [&](int n, int d) {
      const float x = __fsub_rn(kc_at(n, d), s_mean[d]);
      return __fmul_rn(x, x);
    }, s_chunk, s_var);
  }
  if (threadIdx.x < CH) {
    p.kmean[(int64_t)bh * HD + c0 + threadIdx.x] = s_mean[threadIdx.x];
    p.kvar[(int64_t)bh * HD + c0 + threadIdx.x] = __fdiv_rn(s_var[threadIdx.x], (float)p.N);
  }
}

// --------------------------------------------------------------------- route


// Block j is exact for q-block n when (c_n . kc_j) * s2 > thr_n (the block-mean
// score of _tri_fwd.py:279-286, with the row mean taken before the dot), or
// |n - j| <= 1, or j is a sink KV block; a q-block inside the sink query range
// attends every valid block exactly.
//
// A CTA scores QB = 8 q-blocks against every key block of one (b, h). The key rows are
// staged in shared memory a chunk of 8 words (256 rows) at a time with coalesced 16-byte
// cp.async copies (the first chunk's are issued before anything else), rows padded to
// kRowStride bytes so that lane l reading row l is free of bank conflicts. Warp w scores
// word w of the chunk: lane l holds key row 32w + l in registers and scores it against
// the 8 centroids (broadcast from shared memory) with packed f32x2 FMAs. Each score is
// four interleaved partial sums over the channels d = 0, 1, 2, 3 (mod 4), in channel
// order, added as (a0 + a1) + (a2 + a3). Grid: (ceil(N/8), B*H); 256 threads.
//
// The threshold of each q-block is computed here from its centroid:
//   BF16 (_preprocess.py:149-164): thr = (c.kcm)*s2 + tau*sqrt(max((c^2.kcv)*s2^2, 0) + 1e-6)
//   INT8 (_fused_prep.py:50-59):   thr = tau*sqrt((c^2.kcv)*s2^2 + 1e-6)
// with the D-sums in numpy's 8-way pairwise order: lane j of each 8-lane group runs
// partial sum j, and three xor shuffles combine them as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)).
constexpr int kRouteQB = 8;
constexpr int kRouteChunkWords = 8;   // one word per warp per chunk

template <int HD>
constexpr int route_row_stride() { return HD * 2 + 16; }

template <int HD>
constexpr size_t route_smem_bytes() { return (size_t)kRouteChunkWords * 32 * route_row_stride<HD>(); }

__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr), "l"(gmem) : "memory");
}

template <int HD>
__global__ void __launch_bounds__(256) route_kernel(RouteParams p) {
  pdl_begin();
  constexpr int QB = kRouteQB;
  constexpr int KCH = HD / 8;                       // 16-byte chunks of a kc row
  constexpr int RS = route_row_stride<HD>();        // staged row stride, bytes
  extern __shared__ __align__(16) uint8_t s_rows[];  // [256][RS]
  __shared__ __align__(16) float s_c[QB][HD];
  __shared__ float s_km[HD], s_kv[HD];
  __shared__ float s_thr[QB];
  __shared__ uint32_t s_words[QB][64];
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nbase = blockIdx.x * QB;
  const int64_t krow = (int64_t)p.H * HD;
  const __nv_bfloat16* kc0 = p.kc + (int64_t)b * p.npad * krow + (int64_t)h * HD;
  const uint32_t rows_addr = smem_u32(s_rows);
  // rows j < 32 * nw <= npad lie inside the zero-padded kc buffer
  auto stage = [&](int w0, int cw) {
    for (int i = threadIdx.x; i < cw * 32 * KCH; i += 256) {
      const int r = i / KCH, c = i % KCH;
      cp_async16(rows_addr + r * RS + c * 16, kc0 + (int64_t)(w0 * 32 + r) * krow + c * 8);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  stage(0, min(kRouteChunkWords, p.nw));
  for (int i = threadIdx.x; i < QB * HD; i += 256) {
    const int w = i / HD, d = i % HD, nn = nbase + w;
    s_c[w][d] = nn < p.N ? p.centroid[(((int64_t)b * p.N + nn) * p.H + h) * HD + d] : 0.f;
  }
  for (int d = threadIdx.x; d < HD; d += 256) {
    s_km[d] = p.kmean[(int64_t)bh * HD + d];
    s_kv[d] = p.kvar[(int64_t)bh * HD + d];
  }
  __syncthreads();
  {
    const int n = nbase + warp;
    const int j8 = lane & 7;
    float rv = 0.f, rm = 0.f;
#pragma unroll
    for (int i = 0; i < HD; i += 8) {
      const float ci = s_c[warp][i + j8];
      const float tv = __fmul_rn(__fmul_rn(ci, ci), s_kv[i + j8]);
      rv = i == 0 ? tv : __fadd_rn(rv, tv);
      if (!p.int8) {
        const float tm = __fmul_rn(ci, s_km[i + j8]);
        rm = i == 0 ? tm : __fadd_rn(rm, tm);
      }
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) {
      rv = __fadd_rn(rv, __shfl_xor_sync(0xffffffffu, rv, off));
      rm = __fadd_rn(rm, __shfl_xor_sync(0xffffffffu, rm, off));
    }
    const float v = __fmul_rn(rv, __fmul_rn(p.s2, p.s2));
    float t;
    if (p.int8) {
      t = __fmul_rn(p.tau, __fsqrt_rn(__fadd_rn(v, 1.0e-6f)));
    } else {
      t = __fadd_rn(__fmul_rn(rm, p.s2),
                    __fmul_rn(p.tau, __fsqrt_rn(__fadd_rn(fmaxf(v, 0.f), 1.0e-6f))));
    }
    if (lane == 0) {
      s_thr[warp] = t;
      if (n < p.N) p.thr[((int64_t)b * p.N + n) * p.H + h] = t;
    }
  }
  float thr[QB];
  const float4* c4 = reinterpret_cast<const float4*>(&s_c[0][0]);
  for (int w0 = 0; w0 < p.nw; w0 += kRouteChunkWords) {
    const int cw = min(kRouteChunkWords, p.nw - w0);
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();   // the chunk (and, the first time, the thresholds) is visible
    if (w0 == 0) {
#pragma unroll
      for (int q = 0; q < QB; ++q) thr[q] = s_thr[q];
    }
    if (warp < cw) {
      const int jw = w0 + warp;
      const int j = jw * 32 + lane;
      const bool valid = j < p.N;
      const uint4* kr = reinterpret_cast<const uint4*>(s_rows + (warp * 32 + lane) * RS);
      float2 acc[QB][2];
#pragma unroll
      for (int q = 0; q < QB; ++q) acc[q][0] = acc[q][1] = make_float2(0.f, 0.f);
#pragma unroll
      for (int t = 0; t < KCH; ++t) {
        // channels 8t .. 8t+7 of row j as (k0,k1) (k2,k3) (k4,k5) (k6,k7)
        const uint4 kv4 = kr[t];
        const float2 k01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kv4.x));
        const float2 k23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kv4.y));
        const float2 k45 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kv4.z));
        const float2 k67 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kv4.w));
#pragma unroll
        for (int q = 0; q < QB; ++q) {
          const float4 ca = c4[q * (HD / 4) + 2 * t], cb = c4[q * (HD / 4) + 2 * t + 1];
          acc[q][0] = __ffma2_rn(make_float2(ca.x, ca.y), k01, acc[q][0]);
          acc[q][1] = __ffma2_rn(make_float2(ca.z, ca.w), k23, acc[q][1]);
          acc[q][0] = __ffma2_rn(make_float2(cb.x, cb.y), k45, acc[q][0]);
          acc[q][1] = __ffma2_rn(make_float2(cb.z, cb.w), k67, acc[q][1]);
        }
      }
      uint32_t mine = 0;
#pragma unroll
      for (int q = 0; q < QB; ++q) {
        const int n = nbase + q;
        const float score = __fmul_rn(__fadd_rn(__fadd_rn(acc[q][0].x, acc[q][0].y),
                                                __fadd_rn(acc[q][1].x, acc[q][1].y)), p.s2);
        bool exact = (score > thr[q]) || (abs(n - j) <= 1) || (j >= p.sink_kv0 && j < p.sink_kv1);
        if (n >= p.sink_q0 && n < p.sink_q1) exact = true;
        const uint32_t word = __ballot_sync(0xffffffffu, exact && valid);
        if (lane == q) mine = word;
        if (p.stat && valid && n < p.N) p.stat[(((int64_t)b * p.H + h) * p.N + n) * p.N + j] = score;
      }
      if (lane < QB && nbase + lane < p.N) {
        p.mask[(((int64_t)b * p.H + h) * p.N + nbase + lane) * p.nw + jw] = mine;
        if (jw < 64) s_words[lane][jw] = mine;
      }
    }
    if (w0 + kRouteChunkWords < p.nw) {
      __syncthreads();   // every warp is done with this chunk
      stage(w0 + kRouteChunkWords, min(kRouteChunkWords, p.nw - w0 - kRouteChunkWords));
    }
  }
  __syncthreads();   // every word of the CTA's q-blocks is in s_words / mask
  const int n = nbase + warp;   // warps 0 .. QB-1 finish one q-block each
  if (warp >= QB || n >= p.N) return;
  const int64_t urow = ((int64_t)b * p.H + h) * p.N + n;
  auto word_at = [&](int w) { return w < 64 ? s_words[warp][w] : p.mask[urow * p.nw + w]; };
  int total = 0;
  for (int w = lane; w < p.nw; w += 32) total += __popc(word_at(w));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) total += __shfl_xor_sync(0xffffffffu, total, off);
  if (lane == 0) p.count[urow] = total;
  if (p.lists) {
    int* out = p.lists + urow * p.N;
    int base = 0;
    for (int w0 = 0; w0 < p.nw; w0 += 32) {
      const int w = w0 + lane;
      uint32_t bits = w < p.nw ? word_at(w) : 0u;
      const int c = __popc(bits);
      int incl = c;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      int pos = base + incl - c;
      while (bits) {
        const int bit = __ffs(bits) - 1;
        bits &= bits - 1;
        out[pos++] = w * 32 + bit;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    for (int i = total + lane; i < p.N; i += 32) out[i] = -1;
  }
}

// ------------------------------------------------------------- quant Q, K, V

// Q: per-(token, head) symmetric int8 (_fused_prep.py:36-44); K: per-(token, head) int8 of
//    K - k_mean (_fused_quant.py:8-42); both s = max|x| / 127, floor 1e-8, round half away
//    from zero of x / s (the clamp to +-127 never acts, see code_pair).
// V: per-channel int8 with the (b, h, d) scale (_fused_quant.py:61-88).
// One thread per 16 channels of a (head, token); a head's lanes share a warp. The
// quotients are formed two lanes at a time (f32x2), with the same IEEE operations as
// quotient_rn.
constexpr int kQuantStages = 4;

// quotient_rn of two values at once
__device__ __forceinline__ float2 quotient_rn2(float2 x, float2 s, float2 y) {
  const float2 ns = make_float2(-s.x, -s.y);
  const float2 q0 = mul2(x, y);
  const float2 q1 = fma2(fma2(ns, q0, x), y, q0);
  return fma2(fma2(ns, q1, x), y, q1);
}

// The int8 codes of two quotients, round half away from zero: trunc(RN(q + copysign(0.5,
// q))), the arithmetic of the reference's conversion (x / s, then + or - 0.5, then a
// truncating cast), as two's-complement words (the code in the low byte). Valid for
// |q| <= 127.5, where clamping to +-127 (the reference's, before or after rounding) changes
// nothing: the quantisers divide by s >= max|x| / 127 (rounded), so |q| <= 127 (1 + 2^-23).
__device__ __forceinline__ void code_pair(float2 q, uint32_t& c0, uint32_t& c1) {
  const float2 v = add2(q, make_float2(copysignf(0.5f, q.x), copysignf(0.5f, q.y)));
  c0 = (uint32_t)__float2int_rz(v.x);
  c1 = (uint32_t)__float2int_rz(v.y);
}

// int8 codes round half away from zero of x / den (|x| <= 127 den, see code_pair);
// rcp = RN(1 / den)
__device__ __forceinline__ uint2 quant8(const float (&x)[8], const float (&den)[8], const float (&rcp)[8]) {
  uint32_t c[8];
#pragma unroll
  for (int i = 0; i < 8; i += 2)
    code_pair(quotient_rn2(make_float2(x[i], x[i + 1]), make_float2(den[i], den[i + 1]),
                             make_float2(rcp[i], rcp[i + 1])),
                c[i], c[i + 1]);
  return pack_codes(c);
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&x)[8]) {
  const __nv_bfloat162* hx = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(hx[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// Per-(token, head) codes of this lane's 16 values: the head's max |x| over its LPH lanes,
// s = max(RN(max / 127), 1e-8) (returned), codes of x / s.
template <int LPH>
__device__ __forceinline__ uint4 token_codes(const float (&x)[16], float& s_out) {
  float amax = 0.f;
#pragma unroll
  for (int c = 0; c < 16; ++c) amax = fmaxf(amax, fabsf(x[c]));
#pragma unroll
  for (int off = 1; off < LPH; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  // RN(amax / 127) by quotient_rn with RN(1 / 127): exact for every amax that is not
  // subnormal, and a subnormal amax gives s < 1e-8, replaced by the floor below
  const float s = quotient_rn(amax, 127.f, 0.007874015718698502f);
  const float s_safe = s > 1e-8f ? s : 1e-8f;
  const float y = __frcp_rn(s_safe);
  float den[8], rcp[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    den[c] = s_safe;
    rcp[c] = y;
  }
  s_out = s_safe;
  const float(&lo)[8] = *reinterpret_cast<const float(*)[8]>(&x[0]);
  const float(&hi)[8] = *reinterpret_cast<const float(*)[8]>(&x[8]);
  const uint2 a = quant8(lo, den, rcp), b = quant8(hi, den, rcp);
  return make_uint4(a.x, a.y, b.x, b.y);
}

// 16-byte cp.async that reads `src_bytes` (16 or 0: zero fill) from gmem
__device__ __forceinline__ void cp_async16_zfill(uint32_t smem_addr, const void* gmem, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr), "l"(gmem), "r"(src_bytes)
               : "memory");
}

// Grid layout of quant_qkv_kernel: a stripe of CTAs covers whole tokens (lcm(per_grp, 256)
// threads, per_grp = H * HD / 16 lanes per token), so a thread keeps one (head, 16-channel)
// lane for all the tokens it visits, stepping by the grid's stripes.
static inline int64_t quant_stripe_threads(int64_t per_grp) {
  int64_t a = per_grp, b = 256;
  while (b) {
    const int64_t t = a % b;
    a = b;
    b = t;
  }
  return per_grp / a * 256;   // lcm(per_grp, 256)
}

// (batch, token) of a row index bg = b * T + t, advanced by a fixed step without a division
struct RowCursor {
  int64_t b, t;
  __device__ void advance(int64_t step, int64_t T) {
    t += step;
    while (t >= T) {
      t -= T;
      ++b;
    }
  }
};

// Persistent form: one thread per 16 channels of a (head, token); each thread walks its
// tokens with kQuantStages tokens of Q / K / V rows in flight (cp.async into its own
// shared-memory slots; no thread reads another's), and quantises one token while the next
// ones load.
template <int HD>
__global__ void __launch_bounds__(256, 2) quant_qkv_kernel(QuantParams p, int stripe_ctas) {
  pdl_begin();
  constexpr int LPH = HD / 16, NS = kQuantStages, SLOTS = 6;   // Q, K, V x two 16-byte halves
  extern __shared__ __align__(16) uint4 qbuf[];                // [NS][SLOTS][256]
  const int64_t per_grp = (int64_t)p.H * LPH;
  const int64_t total = (int64_t)p.B * p.T;
  const int64_t stripe_rows = (int64_t)stripe_ctas * 256 / per_grp;
  const int64_t lin = (int64_t)(blockIdx.x % stripe_ctas) * 256 + threadIdx.x;
  const int hl = (int)(lin % per_grp);
  const int h = hl / LPH, d0 = (hl % LPH) * 16;
  const int64_t row0 = (int64_t)(blockIdx.x / stripe_ctas) * stripe_rows;   // the CTA's first row
  const int64_t step = (int64_t)(gridDim.x / stripe_ctas) * stripe_rows;
  const int64_t first = row0 + lin / per_grp;
  const bool with_q = p.qi != nullptr, with_v = p.vi != nullptr;
  const uint32_t base = smem_u32(qbuf) + threadIdx.x * 16;
  const __nv_bfloat16* qh = p.q + (int64_t)h * p.sq_h + d0;
  const __nv_bfloat16* kh = p.k + (int64_t)h * p.sk_h + d0;
  const __nv_bfloat16* vh = p.v + (int64_t)h * p.sv_h + d0;
  // rows visited: first + k * step for k < nk (nk uniform over the CTA, so every lane of a
  // head takes part in every shuffle; rows past the end load zeros and store nothing)
  const int64_t nk = row0 < total ? (total - row0 + step - 1) / step : 0;
  RowCursor in{first / p.T, first % p.T}, out = in;
  auto issue = [&](int64_t k) {
    const uint32_t sb = base + (uint32_t)((k % NS) * SLOTS * 256 * 16);
    const bool ok = in.b < p.B;
    const int64_t b = ok ? in.b : 0;
    const int64_t src_t = ok ? order_row(p.perm, in.t, p.T, p.err) : 0;   // token of row t
    const __nv_bfloat16* q = qh + b * p.sq_b + src_t * p.sq_t;
    const __nv_bfloat16* k_ = kh + b * p.sk_b + src_t * p.sk_t;
    const __nv_bfloat16* v = vh + b * p.sv_b + src_t * p.sv_t;
    const uint32_t nq = ok && with_q ? 16u : 0u, nkb = ok ? 16u : 0u, nv = ok && with_v ? 16u : 0u;
    cp_async16_zfill(sb + 0 * 256 * 16, q, nq);
    cp_async16_zfill(sb + 1 * 256 * 16, q + 8, nq);
    cp_async16_zfill(sb + 2 * 256 * 16, k_, nkb);
    cp_async16_zfill(sb + 3 * 256 * 16, k_ + 8, nkb);
    cp_async16_zfill(sb + 4 * 256 * 16, v, nv);
    cp_async16_zfill(sb + 5 * 256 * 16, v + 8, nv);
    in.advance(step, p.T);
  };
#pragma unroll
  for (int s = 0; s < NS - 1; ++s) {
    if (s < nk) issue(s);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  int64_t cur_b = -1;
  float m[16], sc[16], sc_rcp[16];
  for (int64_t k = 0; k < nk; ++k) {
    if (k + NS - 1 < nk) issue(k + NS - 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group %0;" ::"n"(NS - 1) : "memory");
    const bool ok = out.b < p.B;
    const int64_t b = ok ? out.b : 0, t = out.t;
    out.advance(step, p.T);
    if (b != cur_b) {   // per-(b, h) constants of this lane
      cur_b = b;
      const float4* mp = reinterpret_cast<const float4*>(p.kmean + (b * p.H + h) * HD + d0);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 mj = __ldg(mp + j);
        m[4 * j] = mj.x; m[4 * j + 1] = mj.y; m[4 * j + 2] = mj.z; m[4 * j + 3] = mj.w;
      }
      if (with_v) {
        const float4* sp = reinterpret_cast<const float4*>(p.vscale + (b * p.H + h) * HD + d0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 sj = __ldg(sp + j);
          sc[4 * j] = sj.x; sc[4 * j + 1] = sj.y; sc[4 * j + 2] = sj.z; sc[4 * j + 3] = sj.w;
        }
      }
#pragma unroll
      for (int c = 0; c < 16; ++c) sc_rcp[c] = with_v ? __frcp_rn(sc[c]) : 0.f;
    }
    const uint4* sl = qbuf + (k % NS) * SLOTS * 256 + threadIdx.x;
    const int64_t o = ((b * p.T + t) * p.H + h) * HD + d0;
    const int64_t so = (b * p.H + h) * p.tp + t;
    float x[16];
    if (with_q) {
      float s;
      unpack8(sl[0], *reinterpret_cast<float(*)[8]>(&x[0]));
      unpack8(sl[256], *reinterpret_cast<float(*)[8]>(&x[8]));
      const uint4 cq = token_codes<LPH>(x, s);
      if (ok) {
        *reinterpret_cast<uint4*>(p.qi + o) = cq;
        if (d0 == 0) p.qs[so] = s;
      }
    }
    {
      float s;
      unpack8(sl[2 * 256], *reinterpret_cast<float(*)[8]>(&x[0]));
      unpack8(sl[3 * 256], *reinterpret_cast<float(*)[8]>(&x[8]));
#pragma unroll
      for (int c = 0; c < 16; ++c) x[c] = __fsub_rn(x[c], m[c]);
      const uint4 ck = token_codes<LPH>(x, s);
      if (ok) {
        *reinterpret_cast<uint4*>(p.ki + o) = ck;
        if (d0 == 0) p.ks[so] = s;
      }
    }
    if (with_v) {
      unpack8(sl[4 * 256], *reinterpret_cast<float(*)[8]>(&x[0]));
      unpack8(sl[5 * 256], *reinterpret_cast<float(*)[8]>(&x[8]));
      const uint2 a = quant8(*reinterpret_cast<const float(*)[8]>(&x[0]), *reinterpret_cast<const float(*)[8]>(&sc[0]),
                             *reinterpret_cast<const float(*)[8]>(&sc_rcp[0]));
      const uint2 c2 = quant8(*reinterpret_cast<const float(*)[8]>(&x[8]), *reinterpret_cast<const float(*)[8]>(&sc[8]),
                              *reinterpret_cast<const float(*)[8]>(&sc_rcp[8]));
      if (ok) *reinterpret_cast<uint4*>(p.vi + o) = make_uint4(a.x, a.y, c2.x, c2.y);
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Self-test of the quantisers' arithmetic against CUDA's IEEE division and conversion on
// caller-given (x, s) pairs, two at a time as in quant8: counts the pairs whose quotient
// (quotient_rn2) differs in value from __fdiv_rn(x, s) (bad[0]) and whose int8 code
// (code_pair of the quotient clamped to +-127, which equals the reference's clamp after
// rounding for any quotient) differs (bad[1]).
__global__ void __launch_bounds__(256) quotient_selftest_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ s, int64_t n,
                                                                unsigned long long* bad) {
  pdl_begin();
  unsigned long long nq = 0, nc = 0;
  const int64_t pairs = (n + 1) / 2;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < pairs; i += (int64_t)gridDim.x * 256) {
    const int64_t i0 = 2 * i, i1 = 2 * i + 1 < n ? 2 * i + 1 : 2 * i;
    const float2 xi = make_float2(x[i0], x[i1]), si = make_float2(s[i0], s[i1]);
    const float2 got = quotient_rn2(xi, si, make_float2(__frcp_rn(si.x), __frcp_rn(si.y)));
    uint32_t c[2];
    code_pair(make_float2(fminf(fmaxf(got.x, -127.f), 127.f), fminf(fmaxf(got.y, -127.f), 127.f)), c[0], c[1]);
    const float g2[2] = {got.x, got.y}, x2[2] = {xi.x, xi.y}, s2[2] = {si.x, si.y};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      if (e == 1 && i1 == i0) break;
      const float want = __fdiv_rn(x2[e], s2[e]);
      if (!(g2[e] == want)) ++nq;
      const float wc = fminf(fmaxf(want, -256.f), 256.f);
      const int want_code = max(-127, min(127, wc >= 0.f ? __float2int_rz(__fadd_rn(wc, 0.5f))
                                                         : __float2int_rz(__fsub_rn(wc, 0.5f))));
      if ((int)(int8_t)(c[e] & 0xffu) != want_code) ++nc;
    }
  }
  if (nq) atomicAdd(bad, nq);
  if (nc) atomicAdd(bad + 1, nc);
}

void launch_quotient_selftest(const float* x, const float* s, int64_t n, unsigned long long* bad,
                              cudaStream_t st) {
  int64_t blocks = (n + 255) / 256;
  blocks = blocks < 1 ? 1 : (blocks > 4096 ? 4096 : blocks);
  launch_pdl(quotient_selftest_kernel, dim3((unsigned)blocks), dim3(256), 0, st, x, s, n, bad);
}

// -------------------------------------------------------------------- Morton

// Rank of token (z, y, x) among all tokens of the box grid ordered by their Morton
// code, computed digit by digit instead of by sorting: for every set bit of the
// code, count the grid points that agree with it above that bit and have a 0 there.
// Axis a in {0: x (width), 1: y (height), 2: z (frames)} holds code bits 3l + a.
// naxes = 3 for the "3d" curve; 2 for the within-frame part of "2d_frame".
__device__ __forceinline__ int64_t clamp_count(int64_t dim, int64_t base, int64_t span) {
  const int64_t c = dim - base;
  return c <= 0 ? 0 : (c < span ? c : span);
}

__device__ int64_t morton_rank(const int64_t (&c)[3], const int64_t (&dim)[3], int naxes,
                               int levels) {
  int64_t rank = 0;
  for (int l = levels - 1; l >= 0; --l) {
    for (int a = naxes - 1; a >= 0; --a) {
      if (((c[a] >> l) & 1) == 0) continue;
      int64_t term = 1;
      for (int e = 0; e < naxes && term; ++e) {
        int64_t cnt;
        if (e == a) {
          cnt = clamp_count(dim[e], (c[e] >> (l + 1)) << (l + 1), (int64_t)1 << l);
        } else if (e < a) {
          cnt = clamp_count(dim[e], (c[e] >> (l + 1)) << (l + 1), (int64_t)1 << (l + 1));
        } else {
          cnt = clamp_count(dim[e], (c[e] >> l) << l, (int64_t)1 << l);
        }
        term *= cnt;
      }
      rank += term;
    }
  }
  return rank;
}

// perm[pos] = token, inverse[token] = pos, with pos = (rank + roll) mod T; roll is the
// block-alignment rotation of _morton_h3.py:42-61 (0 for the plain permutation).
__global__ void morton_kernel(int64_t frames, int64_t height, int64_t width, int curve,
                              int64_t roll, int64_t* perm, int64_t* inverse) {
  pdl_begin();
  const int64_t T = frames * height * width;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T) return;
  const int64_t area = height * width;
  const int64_t z = i / area, rem = i - z * area, y = rem / width, x = rem - y * width;
  int64_t rank;
  if (curve == 1) {   // "2d_frame": frame index most significant, Z-order inside a frame
    const int64_t c[3] = {x, y, 0};
    const int64_t dim[3] = {width, height, 1};
    int levels = 1;
    while (levels < 21 && ((int64_t)1 << levels) < (width > height ? width : height)) ++levels;
    rank = z * area + morton_rank(c, dim, 2, levels);
  } else {
    const int64_t c[3] = {x, y, z};
    const int64_t dim[3] = {width, height, frames};
    int64_t mx = width > height ? width : height;
    mx = mx > frames ? mx : frames;
    int levels = 1;
    while (levels < 21 && ((int64_t)1 << levels) < mx) ++levels;
    rank = morton_rank(c, dim, 3, levels);
  }
  int64_t pos = (rank + roll) % T;
  if (pos < 0) pos += T;
  perm[pos] = i;
  inverse[i] = pos;
}

// dst[b, i, :] = src[b, index[i], :] for up to 4 tensors of identical geometry; one
// warp per destination row, 16-byte vectors (row_bytes % 16 == 0).

__global__ void __launch_bounds__(256) gather_rows_kernel(GatherParams p) {
  pdl_begin();
  const int64_t warp_id = ((int64_t)blockIdx.x * 256 + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= p.batch * p.rows) return;
  const int64_t b = warp_id / p.rows, i = warp_id - b * p.rows;
  const int64_t srow = __ldg(p.index + i);
  const int64_t nvec = p.row_bytes >> 4;
  for (int t = 0; t < p.ntensors; ++t) {
    const uint4* s = reinterpret_cast<const uint4*>(p.src[t] + b * p.src_stride_b +
                                                    srow * p.src_stride_row);
    uint4* d = reinterpret_cast<uint4*>(p.dst[t] + b * p.dst_stride_b + i * p.dst_stride_row);
    for (int64_t c = lane; c < nvec; c += 32) d[c] = __ldg(s + c);
  }
}

// ------------------------------------------------------------- host launches

template <int HD>
static void launch_pool_t(const PoolParams& p, bool vamax, cudaStream_t st) {
  // 64-thread CTAs when the channel groups fill them, else 32 (fewer idle lanes at small H)
  const int lanes = p.H * (HD / 8);
  const int nt = lanes % 64 == 0 ? 64 : 32;
  dim3 grid(3 * ((lanes + nt - 1) / nt), p.npad, p.B);
  if (vamax) launch_pdl(pool_kernel<HD, true>, grid, dim3(nt), 0, st, p);
  else launch_pdl(pool_kernel<HD, false>, grid, dim3(nt), 0, st, p);
}

void launch_pool(const PoolParams& p, int hd, bool vamax, cudaStream_t st) {
  if (hd == 128) launch_pool_t<128>(p, vamax, st);
  else launch_pool_t<64>(p, vamax, st);
}

template <int HD, bool INT8>
static void launch_moments_t(const MomentsParams& p, cudaStream_t st) {
  constexpr int kMaxStaged = 200 * 1024;
  const size_t staged = (size_t)p.N * kMomentsCh * sizeof(__nv_bfloat16);
  const dim3 grid(p.B * p.H, HD / kMomentsCh);
  if (staged <= kMaxStaged) {
    if (staged > 48 * 1024)   // opt-in on the current device (the attribute is per device)
      cudaFuncSetAttribute(moments_kernel<HD, INT8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kMaxStaged);
    launch_pdl(moments_kernel<HD, INT8, true>, grid, dim3(kMomentsThreads), staged, st, p);
  } else {
    launch_pdl(moments_kernel<HD, INT8, false>, grid, dim3(kMomentsThreads), 0, st, p);
  }
}

void launch_moments(const MomentsParams& p, int hd, bool int8, cudaStream_t st) {
  if (hd == 128) {
    if (int8) launch_moments_t<128, true>(p, st);
    else launch_moments_t<128, false>(p, st);
  } else {
    if (int8) launch_moments_t<64, true>(p, st);
    else launch_moments_t<64, false>(p, st);
  }
}

// ------------------------------------------------------------------- schedule

// One CTA per (b, h): counting sort of the head's query blocks by exact-block count,
// descending (counts above 1023 share the top bin). The order inside a bin does not
// matter: every unit's output is independent of when it runs.
__global__ void __launch_bounds__(256) order_kernel(const int* __restrict__ count, int* __restrict__ order,
                                                    int n) {
  pdl_begin();
  constexpr int kBins = 1024;
  __shared__ int hist[kBins];
  __shared__ int warp_tot[8];
  const int bh = blockIdx.x;
  const int* c = count + (int64_t)bh * n;
  int* o = order + (int64_t)bh * n;
  for (int i = threadIdx.x; i < kBins; i += 256) hist[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += 256) atomicAdd(&hist[kBins - 1 - min(c[i], kBins - 1)], 1);
  __syncthreads();
  // exclusive prefix sum of the bins (bin 0 = largest count): 4 bins per thread
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int v[4], s = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[k] = hist[threadIdx.x * 4 + k];
    s += v[k];
  }
  int incl = s;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int base = 0;
  for (int w = 0; w < warp; ++w) base += warp_tot[w];
  int run = base + incl - s;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    hist[threadIdx.x * 4 + k] = run;
    run += v[k];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += 256) {
    const int pos = atomicAdd(&hist[kBins - 1 - min(c[i], kBins - 1)], 1);
    o[pos] = bh * n + i;
  }
}

void launch_order(const int* count, int* order, int bh_count, int n, cudaStream_t st) {
  launch_pdl(order_kernel, dim3(bh_count), dim3(256), 0, st, count, order, n);
}

template <int HD>
static void launch_route_t(const RouteParams& p, cudaStream_t st) {
  constexpr size_t smem = route_smem_bytes<HD>();
  if (smem > 48 * 1024)   // opt-in on the current device (the attribute is per device)
    cudaFuncSetAttribute(route_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const dim3 grid((p.N + kRouteQB - 1) / kRouteQB, p.B * p.H);
  launch_pdl(route_kernel<HD>, grid, dim3(256), smem, st, p);
}

void launch_route(const RouteParams& p, int hd, cudaStream_t st) {
  if (hd == 128) launch_route_t<128>(p, st);
  else launch_route_t<64>(p, st);
}

void launch_quant_qkv(const QuantParams& p, int hd, cudaStream_t st) {
  static int sms = 0;   // SM count of the device (same on every GPU of a node)
  if (sms == 0) {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    sms = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : 148;
  }
  const int64_t per_grp = (int64_t)p.H * (hd / 16);
  const int64_t stripe_threads = quant_stripe_threads(per_grp);
  const int stripe_ctas = (int)(stripe_threads / 256);
  const int64_t total = (int64_t)p.B * p.T, stripe_rows = stripe_threads / per_grp;
  int64_t stripes = std::max<int64_t>(1, (2 * (int64_t)sms) / stripe_ctas);   // two CTAs per SM
  stripes = std::min<int64_t>(stripes, (total + stripe_rows - 1) / stripe_rows);
  const dim3 grid((unsigned)(stripes * stripe_ctas));
  const size_t smem = (size_t)kQuantStages * 6 * 256 * 16;
  if (hd == 128) {
    cudaFuncSetAttribute(quant_qkv_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(quant_qkv_kernel<128>, grid, dim3(256), smem, st, p, stripe_ctas);
  } else {
    cudaFuncSetAttribute(quant_qkv_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(quant_qkv_kernel<64>, grid, dim3(256), smem, st, p, stripe_ctas);
  }
}

void launch_morton(int64_t frames, int64_t height, int64_t width, int curve, int64_t roll,
                   int64_t* perm, int64_t* inverse, cudaStream_t st) {
  const int64_t T = frames * height * width;
  launch_pdl(morton_kernel, dim3((unsigned)((T + 255) / 256)), dim3(256), 0, st, frames, height, width, curve,
             roll, perm, inverse);
}

void launch_gather(const GatherParams& p, cudaStream_t st) {
  const int64_t warps = p.batch * p.rows;
  launch_pdl(gather_rows_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, st, p);
}

}  // namespace solb200
