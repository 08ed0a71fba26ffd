// Parameter blocks and host launchers of the preprocessing kernels (prep.cu).
#pragma once

#include "common.cuh"

namespace solb200 {

struct PoolParams {
  const __nv_bfloat16* q; const __nv_bfloat16* k; const __nv_bfloat16* v;
  int64_t sq_b, sq_t, sq_h, sk_b, sk_t, sk_h, sv_b, sv_t, sv_h;   // element strides
  __nv_bfloat16* kc; __nv_bfloat16* vc;      // [B, Npad, H, D]
  float* centroid;                            // [B, N, H, D]
  float* vamax;                               // [B, N, H, D] or null
  // token order (reordered calls): row r of every tensor is input token perm[r]; the
  // rows are also written, in that order, to the dense copies that are non-null
  const int64_t* perm;                        // [T] or null
  __nv_bfloat16* qcopy; __nv_bfloat16* kcopy; __nv_bfloat16* vcopy;   // [B, T, H, D] or null
  int* err;                                   // device error word (perm index out of range)
  int B, T, H, N, npad, blk;
};

struct MomentsParams {
  __nv_bfloat16* kc;          // [B, Npad, H, D]; centred in place in INT8 mode
  const float* vamax;         // [B, N, H, D] (INT8 mode)
  float* kmean;               // [B, H, D]
  float* kvar;                // [B, H, D]
  float* vscale;              // [B, H, D] (INT8 mode)
  int B, H, N, npad;
};

struct RouteParams {
  const __nv_bfloat16* kc;   // [B, Npad, H, D]
  const float* centroid;     // [B, N, H, D]
  const float* kmean;        // [B, H, D] kc mean (BF16 mode; unused in INT8 mode)
  const float* kvar;         // [B, H, D] kc variance (INT8: mean of centred kc^2)
  float* thr;                // [B, N, H] written: the routing threshold of each q-block
  uint32_t* mask;            // [B, H, N, NW]
  int* count;                // [B, H, N]
  int* lists;                // [B, H, N, N] or null
  float* stat;               // [B, H, N, N] or null: (c . kc_j) * s2
  int B, H, N, npad, nw;
  float s2, tau;
  int int8;                  // threshold formula of the INT8 path
  int sink_kv0, sink_kv1, sink_q0, sink_q1;
};

struct QuantParams {
  const __nv_bfloat16* q; const __nv_bfloat16* k; const __nv_bfloat16* v;
  int64_t sq_b, sq_t, sq_h, sk_b, sk_t, sk_h, sv_b, sv_t, sv_h;
  const float* kmean;    // [B, H, D]
  const float* vscale;   // [B, H, D] or null
  int8_t* qi; float* qs; // [B, T, H, D], [B, H, tp]
  int8_t* ki; float* ks; // [B, T, H, D], [B, H, tp]
  int8_t* vi;            // [B, T, H, D] or null
  const int64_t* perm;   // [T] token order (reordered calls) or null
  int* err;              // device error word (perm index out of range)
  int B, T, H, tp;       // tp = N * blk (row stride of ks)
};

struct GatherParams {
  const char* src[4];
  char* dst[4];
  int ntensors;
  int64_t src_stride_b, src_stride_row, dst_stride_b, dst_stride_row;   // bytes
  const int64_t* index;
  int64_t batch, rows, row_bytes;
};

void launch_pool(const PoolParams& p, int hd, bool vamax, cudaStream_t st);
void launch_moments(const MomentsParams& p, int hd, bool int8, cudaStream_t st);
void launch_route(const RouteParams& p, int hd, cudaStream_t st);
// order[bh*N ..] = the units of head bh, its query blocks by descending count
void launch_order(const int* count, int* order, int bh_count, int n, cudaStream_t st);
void launch_quant_qkv(const QuantParams& p, int hd, cudaStream_t st);
void launch_morton(int64_t frames, int64_t height, int64_t width, int curve, int64_t roll,
                   int64_t* perm, int64_t* inverse, cudaStream_t st);
void launch_gather(const GatherParams& p, cudaStream_t st);
// bad[0] += quotients differing from __fdiv_rn, bad[1] += int8 codes differing
void launch_quotient_selftest(const float* x, const float* s, int64_t n, unsigned long long* bad,
                              cudaStream_t st);

}  // namespace solb200
