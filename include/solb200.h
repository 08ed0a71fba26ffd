/*
 * solb200: B200-native (sm_100a) Sol-Attn block-sparse attention, C ABI.
 *
 * Plain pointers, sizes and a CUDA stream; no framework types. Every entry point
 * returns an int status (SOLB200_OK = 0) and never allocates device memory: the
 * caller passes a workspace of solb200_workspace_bytes() bytes. All launches go on
 * the given stream, asynchronously; nothing synchronises except
 * solb200_read_device_error(). The text of the last failure on the calling thread
 * is available from solb200_last_error().
 *
 * Tensors are BTHD: [batch, tokens, heads, head_dim] with head_dim contiguous and
 * element strides {batch, token, head} given by the caller (strides must be
 * multiples of 8 elements and pointers 16-byte aligned). Outputs are dense BTHD.
 *
 * Reference interfaces these entry points replace (kijai/ComfyUI-SolAttn_triton):
 *   solb200_sol_attn_bf16   sol_attn          _tri_fwd.py:354-434 (with prepare,
 *                                             _preprocess.py:268-280)
 *   solb200_sol_attn_int8   sol_attn_int8     _int8_fwd.py:379-458 (with
 *                                             fused_preprocess, _fused_prep.py:62-98,
 *                                             quantize_bthd / quantize_v_per_channel,
 *                                             _fused_quant.py:45-58, 91-113)
 *   solb200_morton_perm     morton_perm       _morton.py:35-73 and the block-aligned
 *                                             roll of _perm_for, _morton_h3.py:42-61
 *   solb200_gather_rows     x.index_select(1, perm) of the Morton hooks,
 *                                             _morton.py:128,148, _morton_h3.py:192-217
 *   solb200_sol_attn_reordered  the Morton hooks' gathers (_morton.py:115-148,
 *                                             _morton_h3.py:161-218) fused around one call
 */
#ifndef SOLB200_H
#define SOLB200_H

#include <stdint.h>

#if defined(_WIN32)
#define SOLB200_API __declspec(dllexport)
#else
#define SOLB200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum solb200_status {
  SOLB200_OK = 0,
  SOLB200_ERR_INVALID = 1,    /* unsupported shape, dtype, block or argument */
  SOLB200_ERR_ALIGNMENT = 2,  /* pointer or stride not 16-byte aligned */
  SOLB200_ERR_WORKSPACE = 3,  /* workspace missing or too small */
  SOLB200_ERR_CUDA = 4,       /* a CUDA runtime / driver call failed */
  SOLB200_ERR_DEVICE = 5,     /* current device is not sm_100 */
  SOLB200_ERR_TIMEOUT = 6     /* a device-side bounded wait gave up (see below) */
};

/* Stage selection for the attention entry points. */
enum solb200_stages {
  SOLB200_STAGES_ALL = 0,     /* preprocess, route, forward */
  SOLB200_STAGES_PREPARE = 1, /* preprocess and route only (no output written) */
  SOLB200_STAGES_FORWARD = 2, /* forward only, over a workspace that an earlier ALL or PREPARE
                                 call with the same inputs and geometry filled (profiling) */
  /* PREPARE in parts, for per-stage timing: run in this order on one workspace, they leave
     it as one PREPARE call does (profiling) */
  SOLB200_STAGES_POOL = 3,    /* K / V / Q pooling and the kc moments (INT8: k_mean, centred kc,
                                 V scales) */
  SOLB200_STAGES_QUANT = 4,   /* INT8 only: the Q / K / V codes and scales, after POOL */
  SOLB200_STAGES_ROUTE = 5    /* routing (thresholds, mask, counts) and the forward's schedule,
                                 after POOL */
};

/* Workspace intermediates whose byte offsets solb200_workspace_offset() reports. */
enum solb200_buffer {
  SOLB200_BUF_ERROR = 0,      /* int32 device error word */
  SOLB200_BUF_KC = 1,         /* bf16 [B, Npad, H, D] pooled keys (INT8: centred) */
  SOLB200_BUF_VC = 2,         /* bf16 [B, Npad, H, D] pooled values (block sums) */
  SOLB200_BUF_CENTROID = 3,   /* fp32 [B, N, H, D] query-block means */
  SOLB200_BUF_KMEAN = 4,      /* fp32 [B, H, D] kc mean (INT8: k_mean) */
  SOLB200_BUF_KVAR = 5,       /* fp32 [B, H, D] kc variance */
  SOLB200_BUF_THR = 6,        /* fp32 [B, N, H] routing thresholds */
  SOLB200_BUF_MASK = 7,       /* uint32 [B, H, N, ceil(N/32)] exact-block bits */
  SOLB200_BUF_COUNT = 8,      /* int32 [B, H, N] exact blocks per query block */
  SOLB200_BUF_VAMAX = 9,      /* fp32 [B, N, H, D] per-block |V| max (INT8) */
  SOLB200_BUF_VSCALE = 10,    /* fp32 [B, H, D] V scales (INT8) */
  SOLB200_BUF_QI = 11,        /* int8 [B, T, H, D] (INT8) */
  SOLB200_BUF_QS = 12,        /* fp32 [B, H, N*block] (INT8; entries >= T unused) */
  SOLB200_BUF_KI = 13,        /* int8 [B, T, H, D] (INT8) */
  SOLB200_BUF_KS = 14,        /* fp32 [B, H, N*block] (INT8; entries >= T unused) */
  SOLB200_BUF_VI = 15,        /* int8 [B, T, H, D] (INT8) */
  SOLB200_BUF_ORDER = 16      /* int32 [B*H*N] the forward's schedule: unit ids (b*H + h)*N + n,
                                 head by head, each head's query blocks by descending
                                 exact-block count (the cheapest units run last) */
};

/* Thread-local text of the last failure (empty string if none). */
SOLB200_API const char* solb200_last_error(void);

/* ABI version of this library (bumped on any signature change). */
SOLB200_API int32_t solb200_abi_version(void);

/* Bytes of workspace for one call with this geometry. block: 64 or 128; head_dim:
 * 64 or 128; int8: 0 for the BF16 path, 1 for the INT8 path. */
SOLB200_API int32_t solb200_workspace_bytes(int64_t batch, int64_t tokens, int64_t heads, int64_t head_dim,
                                int32_t block, int32_t int8, int64_t* bytes);

/* Byte offset of an intermediate (enum solb200_buffer) inside that workspace. */
SOLB200_API int32_t solb200_workspace_offset(int64_t batch, int64_t tokens, int64_t heads, int64_t head_dim,
                                 int32_t block, int32_t int8, int32_t which, int64_t* offset);

/* BF16 Sol-Attn. q/k/v: bf16 BTHD with strides {batch, token, head} (elements);
 * out: dense bf16 [B, T, H, D]. scale: softmax scale (pass head_dim^-0.5 for the
 * reference default). tau: routing threshold multiplier. sink_kv / sink_q:
 * half-open block ranges [2] (pass {0, 0} for none). lists (nullable): int32
 * [B, H, N, N] receives each query block's exact KV blocks in ascending order,
 * padded with -1. route_stat (nullable): fp32 [B, H, N, N] routing scores. */
SOLB200_API int32_t solb200_sol_attn_bf16(const void* q, const int64_t* q_strides, const void* k,
                              const int64_t* k_strides, const void* v, const int64_t* v_strides,
                              void* out, int64_t batch, int64_t tokens, int64_t heads,
                              int64_t head_dim, int32_t block, float scale, float tau,
                              const int64_t* sink_kv, const int64_t* sink_q, int32_t stages,
                              void* workspace, int64_t workspace_bytes, int32_t* lists,
                              float* route_stat, void* stream);

/* INT8 Sol-Attn (per-token int8 Q and K with K smoothed by the pooled-key mean; with
 * int8_pv, per-channel int8 V and per-row int8 P). Same arguments as the BF16 entry
 * point plus int8_pv (1 = INT8 P*V, 0 = BF16 P*V). */
SOLB200_API int32_t solb200_sol_attn_int8(const void* q, const int64_t* q_strides, const void* k,
                              const int64_t* k_strides, const void* v, const int64_t* v_strides,
                              void* out, int64_t batch, int64_t tokens, int64_t heads,
                              int64_t head_dim, int32_t block, float scale, float tau,
                              const int64_t* sink_kv, const int64_t* sink_q, int32_t int8_pv,
                              int32_t stages, void* workspace, int64_t workspace_bytes,
                              int32_t* lists, float* route_stat, void* stream);

/* Bytes of workspace for solb200_sol_attn_reordered with this geometry: the workspace of
 * solb200_workspace_bytes (same offsets) plus dense copies of q / k / v in the call's token
 * order for the tensors the forward reads by tiles (q; k for BF16; v for BF16 or without
 * int8 P*V). */
SOLB200_API int32_t solb200_workspace_bytes_reordered(int64_t batch, int64_t tokens, int64_t heads,
                                                      int64_t head_dim, int32_t block, int32_t int8,
                                                      int32_t int8_pv, int64_t* bytes);

/* Sol-Attn with the tokens taken in the order `order` (int64 device array of `tokens`
 * entries, a permutation of [0, tokens); position i of the attention sequence is input
 * token order[i]) and the output written back in input order: the same result, bit for bit,
 * as gathering q/k/v by order, calling solb200_sol_attn_bf16 (int8 = 0) or
 * solb200_sol_attn_int8 (int8 = 1, int8_pv as there) and gathering the output by the
 * inverse order. That is the Morton reordering of the reference's model hooks
 * (_morton.py:115-148, _morton_h3.py:161-218: x.index_select(1, perm) before the blocks,
 * index_select(1, inverse) after) applied around one call, without the gather passes: the
 * pooling pass reads q/k/v rows through `order` (writing the copies the forward's tile
 * loads need) and the forward writes each output row to its input position. An index
 * outside [0, tokens) is recorded in the device error word (solb200_read_device_error then
 * returns SOLB200_ERR_INVALID) and never dereferenced; repeated indices are the caller's
 * error. Workspace: solb200_workspace_bytes_reordered. */
SOLB200_API int32_t solb200_sol_attn_reordered(const void* q, const int64_t* q_strides, const void* k,
                                               const int64_t* k_strides, const void* v,
                                               const int64_t* v_strides, void* out, int64_t batch,
                                               int64_t tokens, int64_t heads, int64_t head_dim,
                                               int32_t block, float scale, float tau,
                                               const int64_t* sink_kv, const int64_t* sink_q,
                                               const int64_t* order, int32_t int8, int32_t int8_pv,
                                               void* workspace, int64_t workspace_bytes, void* stream);

/* Dense BF16 attention on the same tensor cores, for the calls the Sol-Attn path does not
 * take (the reference hands them back to the host's attention, __init__.py:170-189,
 * 271-279): softmax(q k^T * scale) v with every key block computed exactly, no routing.
 * q: [batch, q_tokens, heads, head_dim], k/v: [batch, kv_tokens, heads, head_dim] (cross-
 * attention when the lengths differ), bf16 with strides as above; head_dim 64 or 128; out:
 * dense bf16 [batch, q_tokens, heads, head_dim]. workspace: >= 256 bytes (the device error
 * word). No counterpart in the reference (it runs no kernel of its own for these calls). */
SOLB200_API int32_t solb200_attn_dense(const void* q, const int64_t* q_strides, const void* k,
                                       const int64_t* k_strides, const void* v, const int64_t* v_strides,
                                       void* out, int64_t batch, int64_t q_tokens, int64_t kv_tokens,
                                       int64_t heads, int64_t head_dim, float scale, void* workspace,
                                       int64_t workspace_bytes, void* stream);

/* Element types of the mask of solb200_attn_dense_masked. */
enum {
  SOLB200_MASK_BOOL = 1,  /* one byte per element: nonzero attends, zero masks the key */
  SOLB200_MASK_F32 = 2,   /* float added to the scaled score (-inf masks the key) */
  SOLB200_MASK_BF16 = 3,
  SOLB200_MASK_F16 = 4
};

/* solb200_attn_dense with an attention mask, as the host's scaled_dot_product_attention
 * applies one: out = softmax(q k^T * scale + M) v. A bool mask puts -inf where it is false;
 * a float mask is added. The mask element for (batch b, head h, query token i, key token j)
 * is mask[b * s[0] + h * s[1] + i * s[2] + j * s[3]], s = mask_strides in elements. A stride
 * of 0 broadcasts that dimension, so [1, 1, 1, kv_tokens] key-padding masks and
 * [q_tokens, kv_tokens] masks are passed without a copy. The caller guarantees that every
 * such element lies inside the mask's allocation. A query row whose keys are all masked comes
 * out NaN (0 / 0). The override routes masked calls here; the reference declines every
 * masked call to the host's attention (__init__.py:170-189). */
SOLB200_API int32_t solb200_attn_dense_masked(const void* q, const int64_t* q_strides, const void* k,
                                              const int64_t* k_strides, const void* v, const int64_t* v_strides,
                                              const void* mask, int32_t mask_kind, const int64_t* mask_strides,
                                              void* out, int64_t batch, int64_t q_tokens, int64_t kv_tokens,
                                              int64_t heads, int64_t head_dim, float scale, void* workspace,
                                              int64_t workspace_bytes, void* stream);

/* BF16 Sol-Attn that allocates nothing, for hosts that cannot hand this library device
 * memory at call time (an application that plans all device allocations up front and
 * forbids allocating later, a plugin whose host owns the allocator, or a caller that
 * cannot afford cudaMalloc's implicit synchronisation in the attention path).
 * No counterpart in the reference. Same arguments and result as
 * solb200_sol_attn_bf16 without stages, workspace, lists and route_stat: the scratch
 * is a fixed 16 MiB __device__ array inside this library (held on every GPU that loads
 * the library, until exit). The 40-head, 32760-token, head_dim-128 call needs 10.9 MB
 * at 128-token blocks and fits; at 64-token blocks it needs 22.5 MB and, like any call
 * whose solb200_workspace_bytes exceeds 16 MiB, returns SOLB200_ERR_WORKSPACE. The first call
 * on a device (and the first after the device's context is recreated) looks up the
 * array's address on that device; make it before any stream capture. All calls on a device
 * share the array: calls that overlap on the GPU race and must be serialised by the caller.
 * A bounded-wait timeout inside the call leaves the output unwritten and is recorded in the
 * array's device error word, which the next call clears: read it after each call with
 * solb200_noalloc_read_device_error. */
SOLB200_API int32_t solb200_sol_attn_bf16_noalloc(const void* q, const int64_t* q_strides, const void* k,
                                                  const int64_t* k_strides, const void* v,
                                                  const int64_t* v_strides, void* out, int64_t batch,
                                                  int64_t tokens, int64_t heads, int64_t head_dim,
                                                  int32_t block, float scale, float tau,
                                                  const int64_t* sink_kv, const int64_t* sink_q,
                                                  void* stream);

/* Synchronise `stream`, read the workspace's device error word into *code and clear
 * it. Returns SOLB200_ERR_TIMEOUT when a kernel recorded a bounded-wait timeout. */
SOLB200_API int32_t solb200_read_device_error(void* workspace, int32_t* code, void* stream);

/* Test hook for the device-side bounded waits (no counterpart in the reference). For
 * attention calls made later from the calling thread: the forward kernel's pipeline waits
 * give up after wait_ns nanoseconds (<= 0: the default, 2 s; the exit-path drains of copies
 * and MMAs already issued always keep the default), and the CTA that runs unit stall_unit
 * ((b * heads + h) * N + query block; -1 = none) waits on a barrier that nothing completes,
 * so that its waits run out: that unit's output is not written, the kernel still returns,
 * and solb200_read_device_error reports SOLB200_ERR_TIMEOUT. Call (0, -1) to restore. */
SOLB200_API int32_t solb200_debug_set_wait(int64_t wait_ns, int32_t stall_unit);

/* solb200_read_device_error for the allocation-free entry point: synchronise `stream`,
 * read the device error word of the current device's static scratch into *code and clear
 * it (SOLB200_ERR_TIMEOUT when the last solb200_sol_attn_bf16_noalloc call on this device
 * recorded a bounded-wait timeout). Allocates nothing. No counterpart in the reference. */
SOLB200_API int32_t solb200_noalloc_read_device_error(int32_t* code, void* stream);

/* Morton (Z-order) permutation of a (frames, height, width) token grid in row-major
 * order: perm[i] = token at position i, inverse[token] = position. curve: 0 = "3d",
 * 1 = "2d_frame". roll: rotation of the permutation (the H3 block alignment uses
 * (-span_start) mod block); 0 for the plain permutation. perm/inverse: int64 device
 * arrays of frames*height*width entries. */
SOLB200_API int32_t solb200_morton_perm(int64_t frames, int64_t height, int64_t width, int32_t curve,
                            int64_t roll, int64_t* perm, int64_t* inverse, void* stream);

/* Copy heads [h0, h0+hc) of a bf16 BTHD tensor between a host array [B, T, H, D]
 * (head_dim contiguous, dense) and a dense device array [B, T, hc, D], as one strided
 * 2-D copy on `stream`: to_device = 1 copies host -> device, 0 device -> host. With a
 * page-locked host array the copy is asynchronous and overlaps kernels and copies in the
 * other direction. No counterpart in the reference (it is handed device tensors); it
 * lets a caller holding q/k/v in host memory stream them through the GPU head chunk by
 * head chunk (solb200.sol_attn_host). */
SOLB200_API int32_t solb200_copy_heads(void* device, void* host, int64_t batch, int64_t tokens, int64_t heads,
                                       int64_t head_dim, int64_t h0, int64_t hc, int32_t to_device,
                                       void* stream);

/* dst[b, i, :] = src[b, index[i], :] for up to 4 tensors that share one geometry:
 * rows of row_bytes (a multiple of 16) with byte strides {batch, row}. */
SOLB200_API int32_t solb200_gather_rows(const void* const* src, void* const* dst, int32_t ntensors,
                            const int64_t* index, int64_t batch, int64_t rows, int64_t row_bytes,
                            int64_t src_stride_b, int64_t src_stride_row, int64_t dst_stride_b,
                            int64_t dst_stride_row, void* stream);

/* Self-test of the arithmetic of the int8 quantisers (no counterpart in the
 * reference): for n pairs (x[i], s[i]) of device float arrays (s > 0), adds to the
 * device counters bad[0] the pairs whose division-free quotient differs from the
 * IEEE quotient x/s, and to bad[1] those whose int8 code clamp(round half away from
 * zero of x/s, +-127) differs. The caller zeroes bad (2 x uint64) first. */
SOLB200_API int32_t solb200_selftest_quotient(const float* x, const float* s, int64_t n, uint64_t* bad,
                                              void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SOLB200_H */
