// Bandwidth-bound stages of the Sol-Attn path (sm_100a):
//   pool_kernel      one pass over Q, K, V: kc (block mean of K), vc (block sum of V),
//                    q-block centroids, optional per-block |V| max and per-token Q int8
//   moments_kernel   per (b, h): kc mean/variance (INT8: k_mean, kc centred in place,
//                    V scales) and the per-q-block routing threshold
//   route_kernel     exact-block bitmask [B,H,N,NW], counts, optional index lists
//   quant_kv_kernel  per-token int8 of K - k_mean, per-channel int8 of V
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

// round half away from zero of an already clamped value, as trunc(x +- 0.5)
__device__ __forceinline__ int round_half_away(float x) {
  return x >= 0.f ? __float2int_rz(__fadd_rn(x, 0.5f)) : __float2int_rz(__fsub_rn(x, 0.5f));
}

// One thread owns 8 consecutive channels (16 bytes) of one head and one of the three
// tensors (role 0: Q -> centroid and, for INT8, qi / qs; role 1: K -> kc; role 2:
// V -> vc and |V| max), so a call with few heads still has three threads per channel
// group in flight. Rows are accumulated in token order (row 0 first) in fp32, the
// order of the reference's block sums. Grid: (ceil(H*D/8 / 64), Npad, 3*B); 64 threads.
template <int HD, bool VAMAX, bool QQUANT>
__global__ void __launch_bounds__(64) pool_kernel(PoolParams p) {
  constexpr int LANES_PER_HEAD = HD / 8;
  const int g = blockIdx.x * 64 + threadIdx.x;
  const int n = blockIdx.y, b = blockIdx.z / 3, role = blockIdx.z % 3;
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
  const __nv_bfloat16* src;
  int64_t st;
  if (role == 0) {
    src = p.q + (int64_t)b * p.sq_b + (int64_t)h * p.sq_h + d0;
    st = p.sq_t;
  } else if (role == 1) {
    src = p.k + (int64_t)b * p.sk_b + (int64_t)h * p.sk_h + d0;
    st = p.sk_t;
  } else {
    src = p.v + (int64_t)b * p.sv_b + (int64_t)h * p.sv_h + d0;
    st = p.sv_t;
  }
  float sum[8], vmax[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sum[i] = vmax[i] = 0.f;
#pragma unroll 8
  for (int r = r0; r < r1; ++r) {
    float x[8];
    if (active) {
      load8(src + (int64_t)r * st, x);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) sum[i] = __fadd_rn(sum[i], x[i]);
    if (VAMAX && role == 2) {
#pragma unroll
      for (int i = 0; i < 8; ++i) vmax[i] = fmaxf(vmax[i], fabsf(x[i]));
    }
    if (QQUANT && role == 0) {
      // per-token symmetric int8 of Q (_fused_prep.py:36-44): s = max|x| / 127,
      // floor at 1e-8, clamp(x / s, +-127), round half away from zero.
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(x[i]));
#pragma unroll
      for (int off = 1; off < LANES_PER_HEAD; off <<= 1)
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      const float s = __fdiv_rn(amax, 127.f);
      const float s_safe = s > 1e-8f ? s : 1e-8f;
      if (active) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float xv = fminf(fmaxf(__fdiv_rn(x[i], s_safe), -127.f), 127.f);
          const uint32_t byte = (uint32_t)(round_half_away(xv) & 0xff);
          if (i < 4) lo |= byte << (8 * i); else hi |= byte << (8 * (i - 4));
        }
        const int64_t qo = (((int64_t)b * p.T + r) * p.H + h) * HD + d0;
        *reinterpret_cast<uint2*>(p.qi + qo) = make_uint2(lo, hi);
        if (d0 == 0) p.qs[((int64_t)b * p.H + h) * p.tp + r] = s_safe;
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

// One CTA per (b, h), 512 threads.
// BF16 mode (_preprocess.py:240-243, 149-164): kcm = mean_n kc, kcv = mean_n (kc-kcm)^2,
//   thr = (c.kcm)*s2 + tau*sqrt(max((c^2.kcv)*s2^2, 0) + 1e-6).
// INT8 mode (_fused_prep.py:77-81, 50-59; _fused_quant.py:103): k_mean = mean_n kc,
//   kc <- bf16(kc - k_mean), kcv = mean_n kc^2, vscale = max(amax/127, 1e-8),
//   thr = tau*sqrt((c^2.kcv)*s2^2 + 1e-6).
// The D-sums of the threshold follow numpy's 8-way pairwise order: lane j of an 8-lane
// group runs partial sum j, and three xor shuffles combine them as
// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)).
template <int HD, bool INT8>
__global__ void __launch_bounds__(512) moments_kernel(MomentsParams p) {
  constexpr int NT = 512;
  __shared__ float s_chunk[64 * HD];
  __shared__ float s_mean[HD], s_var[HD];
  const int bh = blockIdx.x;
  const int b = bh / p.H, h = bh % p.H;
  const int64_t row = (int64_t)p.H * HD;
  __nv_bfloat16* kc0 = p.kc + ((int64_t)b * p.npad) * row + (int64_t)h * HD;
  auto kc_at = [&](int n, int d) { return __bfloat162float(kc0[(int64_t)n * row + d]); };
  const float inv_n = (float)p.N;
  cascade_sum_par<HD, NT>(p.N, kc_at, s_chunk, s_mean);
  if (threadIdx.x < HD) s_mean[threadIdx.x] = __fdiv_rn(s_mean[threadIdx.x], inv_n);
  __syncthreads();
  if (INT8) {
    for (int it = threadIdx.x; it < p.N * HD; it += NT) {
      const int n = it / HD, d = it % HD;
      kc0[(int64_t)n * row + d] = __float2bfloat16_rn(__fsub_rn(kc_at(n, d), s_mean[d]));
    }
    __syncthreads();
    cascade_sum_par<HD, NT>(p.N, [&](int n, int d) {
      const float x = kc_at(n, d);
      return __fmul_rn(x, x);
    }, s_chunk, s_var);
    if (p.vamax) {
      // |V| max over the blocks: order-free, partial maxima over row strips
      float* s_max = s_chunk;
      constexpr int STRIPS = NT / HD;
      const int d = threadIdx.x % HD, strip = threadIdx.x / HD;
      const float* vam = p.vamax + ((int64_t)b * p.N) * row + (int64_t)h * HD + d;
      float amax = 0.f;
      for (int n = strip; n < p.N; n += STRIPS) amax = fmaxf(amax, vam[(int64_t)n * row]);
      s_max[strip * HD + d] = amax;
      __syncthreads();
      if (threadIdx.x < HD) {
        float m = 0.f;
        for (int k = 0; k < STRIPS; ++k) m = fmaxf(m, s_max[k * HD + threadIdx.x]);
        p.vscale[(int64_t)bh * HD + threadIdx.x] = fmaxf(__fdiv_rn(m, 127.f), 1e-8f);
      }
    }
  } else {
    cascade_sum_par<HD, NT>(p.N, [&](int n, int d) {
      const float x = __fsub_rn(kc_at(n, d), s_mean[d]);
      return __fmul_rn(x, x);
    }, s_chunk, s_var);
  }
  if (threadIdx.x < HD) {
    s_var[threadIdx.x] = __fdiv_rn(s_var[threadIdx.x], inv_n);
    p.kmean[(int64_t)bh * HD + threadIdx.x] = s_mean[threadIdx.x];
    p.kvar[(int64_t)bh * HD + threadIdx.x] = s_var[threadIdx.x];
  }
  __syncthreads();
  // thresholds: 8 lanes per query block, 4 blocks per warp, 64 per pass of the CTA
  const float s2sq = __fmul_rn(p.s2, p.s2);
  const int lane = threadIdx.x & 31, j = lane & 7;
  for (int n0 = 0; n0 < p.N; n0 += NT / 8) {
    const int n = n0 + (threadIdx.x >> 3);
    const bool ok = n < p.N;
    const float* c = p.centroid + (((int64_t)b * p.N + (ok ? n : 0)) * p.H + h) * HD;
    float rv = 0.f, rm = 0.f;
#pragma unroll
    for (int i = 0; i < HD; i += 8) {
      const float ci = c[i + j];
      const float tv = __fmul_rn(__fmul_rn(ci, ci), s_var[i + j]);
      rv = i == 0 ? tv : __fadd_rn(rv, tv);
      if (!INT8) {
        const float tm = __fmul_rn(ci, s_mean[i + j]);
        rm = i == 0 ? tm : __fadd_rn(rm, tm);
      }
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) {
      rv = __fadd_rn(rv, __shfl_xor_sync(0xffffffffu, rv, off));
      if (!INT8) rm = __fadd_rn(rm, __shfl_xor_sync(0xffffffffu, rm, off));
    }
    if (ok && j == 0) {
      const float v = __fmul_rn(rv, s2sq);
      float t;
      if (INT8) {
        t = __fmul_rn(p.tau, __fsqrt_rn(__fadd_rn(v, 1.0e-6f)));
      } else {
        const float m = __fmul_rn(rm, p.s2);
        t = __fadd_rn(m, __fmul_rn(p.tau, __fsqrt_rn(__fadd_rn(fmaxf(v, 0.f), 1.0e-6f))));
      }
      p.thr[((int64_t)b * p.N + n) * p.H + h] = t;
    }
  }
}

// --------------------------------------------------------------------- route


// Block j is exact for q-block n when (c_n . kc_j) * s2 > thr_n (the block-mean
// score of _tri_fwd.py:279-286, with the row mean taken before the dot), or
// |n - j| <= 1, or j is a sink KV block; a q-block inside the sink query range
// attends every valid block exactly. One warp per q-block, lane = block within a
// 32-block word. Grid: (ceil(N/8), B*H); 256 threads.
template <int HD>
__global__ void __launch_bounds__(256) route_kernel(RouteParams p) {
  constexpr int KPAD = HD + 2;   // bf16 row stride: consecutive rows shift one bank
  __shared__ float s_c[8][HD];
  __shared__ __align__(16) __nv_bfloat16 s_kc[32][KPAD];
  __shared__ uint32_t s_words[8][64];
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp;
  const bool row_ok = n < p.N;
  for (int i = threadIdx.x; i < 8 * HD; i += 256) {
    const int w = i / HD, d = i % HD, nn = blockIdx.x * 8 + w;
    s_c[w][d] = nn < p.N ? p.centroid[(((int64_t)b * p.N + nn) * p.H + h) * HD + d] : 0.f;
  }
  const float thr = row_ok ? p.thr[((int64_t)b * p.N + n) * p.H + h] : 0.f;
  const bool q_sink = n >= p.sink_q0 && n < p.sink_q1;
  int total = 0;
  for (int jw = 0; jw < p.nw; ++jw) {
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * (HD / 8); i += 256) {
      const int r = i / (HD / 8), c8 = (i % (HD / 8)) * 8;
      const int j = jw * 32 + r;
      uint4 u = make_uint4(0, 0, 0, 0);
      if (j < p.N)
        u = __ldg(reinterpret_cast<const uint4*>(
            p.kc + (((int64_t)b * p.npad + j) * p.H + h) * HD + c8));
      uint32_t* dst = reinterpret_cast<uint32_t*>(&s_kc[r][c8]);
      dst[0] = u.x; dst[1] = u.y; dst[2] = u.z; dst[3] = u.w;
    }
    __syncthreads();
    const int j = jw * 32 + lane;
    float acc = 0.f;
    const __nv_bfloat162* kr = reinterpret_cast<const __nv_bfloat162*>(&s_kc[lane][0]);
#pragma unroll 16
    for (int d2 = 0; d2 < HD / 2; ++d2) {
      const float2 kv = __bfloat1622float2(kr[d2]);
      acc = fmaf(s_c[warp][2 * d2], kv.x, acc);
      acc = fmaf(s_c[warp][2 * d2 + 1], kv.y, acc);
    }
    const float score = __fmul_rn(acc, p.s2);
    const bool valid = j < p.N;
    bool exact = (score > thr) || (abs(n - j) <= 1) || (j >= p.sink_kv0 && j < p.sink_kv1);
    if (q_sink) exact = true;
    exact = exact && valid;
    const uint32_t word = __ballot_sync(0xffffffffu, exact);
    if (row_ok) {
      if (lane == 0) {
        p.mask[(((int64_t)b * p.H + h) * p.N + n) * p.nw + jw] = word;
        if (jw < 64) s_words[warp][jw] = word;
      }
      if (p.stat && valid) p.stat[(((int64_t)b * p.H + h) * p.N + n) * p.N + j] = score;
      total += __popc(word);
    }
  }
  if (!row_ok) return;
  const int64_t urow = ((int64_t)b * p.H + h) * p.N + n;
  if (lane == 0) p.count[urow] = total;
  if (p.lists) {
    __syncwarp();
    int* out = p.lists + urow * p.N;
    int base = 0;
    for (int w0 = 0; w0 < p.nw; w0 += 32) {
      const int w = w0 + lane;
      uint32_t bits = 0;
      if (w < p.nw) bits = w < 64 ? s_words[warp][w] : p.mask[urow * p.nw + w];
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

// ---------------------------------------------------------------- quant K, V


// K: per-(token, head) int8 of K - k_mean (_fused_quant.py:8-42): s = max|x|/127,
//    floor 1e-8, round half away from zero of x/s, clamp +-127.
// V: per-channel int8 with the (b, h, d) scale (_fused_quant.py:61-88).
// One thread per 8 channels of a (token, head); a head's lanes share a warp.
template <int HD>
__global__ void __launch_bounds__(256) quant_kv_kernel(QuantParams p) {
  constexpr int LPH = HD / 8;
  const int64_t gid = (int64_t)blockIdx.x * 256 + threadIdx.x;
  const int64_t per_tok = (int64_t)p.H * LPH;
  const int64_t total = (int64_t)p.B * p.T * per_tok;
  const bool active = gid < total;
  const int64_t g = active ? gid : 0;
  const int b = (int)(g / ((int64_t)p.T * per_tok));
  const int64_t rem = g - (int64_t)b * p.T * per_tok;
  const int t = (int)(rem / per_tok);
  const int hl = (int)(rem % per_tok);
  const int h = hl / LPH, d0 = (hl % LPH) * 8;
  float xk[8];
  load8(p.k + (int64_t)b * p.sk_b + (int64_t)t * p.sk_t + (int64_t)h * p.sk_h + d0, xk);
  const float* m = p.kmean + ((int64_t)b * p.H + h) * HD + d0;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    xk[i] = __fsub_rn(xk[i], m[i]);
    amax = fmaxf(amax, fabsf(xk[i]));
  }
#pragma unroll
  for (int off = 1; off < LPH; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float s = __fdiv_rn(amax, 127.f);
  const float s_safe = s > 1e-8f ? s : 1e-8f;
  const int64_t o = (((int64_t)b * p.T + t) * p.H + h) * HD + d0;
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int qv = max(-127, min(127, round_half_away(__fdiv_rn(xk[i], s_safe))));
    const uint32_t byte = (uint32_t)(qv & 0xff);
    if (i < 4) lo |= byte << (8 * i); else hi |= byte << (8 * (i - 4));
  }
  if (!active) return;
  *reinterpret_cast<uint2*>(p.ki + o) = make_uint2(lo, hi);
  if (d0 == 0) p.ks[((int64_t)b * p.H + h) * p.tp + t] = s_safe;
  if (p.vi) {
    float xv[8];
    load8(p.v + (int64_t)b * p.sv_b + (int64_t)t * p.sv_t + (int64_t)h * p.sv_h + d0, xv);
    const float* sc = p.vscale + ((int64_t)b * p.H + h) * HD + d0;
    lo = hi = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int qv = max(-127, min(127, round_half_away(__fdiv_rn(xv[i], sc[i]))));
      const uint32_t byte = (uint32_t)(qv & 0xff);
      if (i < 4) lo |= byte << (8 * i); else hi |= byte << (8 * (i - 4));
    }
    *reinterpret_cast<uint2*>(p.vi + o) = make_uint2(lo, hi);
  }
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
static void launch_pool_t(const PoolParams& p, bool vamax, bool qquant, cudaStream_t st) {
  dim3 grid((p.H * (HD / 8) + 63) / 64, p.npad, 3 * p.B);
  if (vamax && qquant) pool_kernel<HD, true, true><<<grid, 64, 0, st>>>(p);
  else if (vamax) pool_kernel<HD, true, false><<<grid, 64, 0, st>>>(p);
  else if (qquant) pool_kernel<HD, false, true><<<grid, 64, 0, st>>>(p);
  else pool_kernel<HD, false, false><<<grid, 64, 0, st>>>(p);
}

void launch_pool(const PoolParams& p, int hd, bool vamax, bool qquant, cudaStream_t st) {
  if (hd == 128) launch_pool_t<128>(p, vamax, qquant, st);
  else launch_pool_t<64>(p, vamax, qquant, st);
}

void launch_moments(const MomentsParams& p, int hd, bool int8, cudaStream_t st) {
  const int grid = p.B * p.H;
  if (hd == 128) {
    if (int8) moments_kernel<128, true><<<grid, 512, 0, st>>>(p);
    else moments_kernel<128, false><<<grid, 512, 0, st>>>(p);
  } else {
    if (int8) moments_kernel<64, true><<<grid, 512, 0, st>>>(p);
    else moments_kernel<64, false><<<grid, 512, 0, st>>>(p);
  }
}

// ------------------------------------------------------------------- schedule

// One CTA per (b, h): counting sort of the head's query blocks by exact-block count,
// descending (counts above 1023 share the top bin). The order inside a bin does not
// matter: every unit's output is independent of when it runs.
__global__ void __launch_bounds__(256) order_kernel(const int* __restrict__ count, int* __restrict__ order,
                                                    int n) {
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
  order_kernel<<<bh_count, 256, 0, st>>>(count, order, n);
}

void launch_route(const RouteParams& p, int hd, cudaStream_t st) {
  dim3 grid((p.N + 7) / 8, p.B * p.H);
  if (hd == 128) route_kernel<128><<<grid, 256, 0, st>>>(p);
  else route_kernel<64><<<grid, 256, 0, st>>>(p);
}

void launch_quant_kv(const QuantParams& p, int hd, cudaStream_t st) {
  const int64_t total = (int64_t)p.B * p.T * p.H * (hd / 8);
  const int64_t grid = (total + 255) / 256;
  if (hd == 128) quant_kv_kernel<128><<<(unsigned)grid, 256, 0, st>>>(p);
  else quant_kv_kernel<64><<<(unsigned)grid, 256, 0, st>>>(p);
}

void launch_morton(int64_t frames, int64_t height, int64_t width, int curve, int64_t roll,
                   int64_t* perm, int64_t* inverse, cudaStream_t st) {
  const int64_t T = frames * height * width;
  morton_kernel<<<(unsigned)((T + 255) / 256), 256, 0, st>>>(frames, height, width, curve, roll,
                                                             perm, inverse);
}

void launch_gather(const GatherParams& p, cudaStream_t st) {
  const int64_t warps = p.batch * p.rows;
  gather_rows_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(p);
}

}  // namespace solb200
