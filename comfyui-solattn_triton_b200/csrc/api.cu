// Host side of the C ABI (include/solb200.h): argument checks, the workspace plan,
// TMA tensor maps and the launch sequence of each entry point. Nothing here
// allocates device memory or synchronises, except solb200_read_device_error.
#include <mutex>
#include <string>

#include <nvtx3/nvToolsExt.h>

#include "fwd_common.cuh"
#include "internal.h"
#include "prep.cuh"
#include "solb200.h"

using namespace solb200;

namespace {

// Host-side NVTX range: a named interval on the launching thread under which profilers
// group the kernels launched inside it (a few ns when no profiler is attached).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

thread_local std::string g_last_error;

// Test hook (solb200_debug_set_wait): the forward kernels' pipeline wait limit and the
// unit whose CTA stalls on purpose, for calls made from this thread.
struct DebugWait {
  uint64_t wait_ns = SOLB200_WAIT_NS;
  int32_t stall_unit = -1;
};
thread_local DebugWait g_debug_wait;

int32_t fail(int32_t code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int32_t cuda_fail(cudaError_t e, const char* what) {
  // clear the runtime's last-error slot (a launch error stays there otherwise and the
  // next call's launch check would report it again); faults of the context stay sticky
  (void)cudaGetLastError();
  return fail(SOLB200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// ----------------------------------------------------------------- geometry

struct Plan {
  int64_t B, T, H, D;
  int blk, N, npad, nw;
  bool int8;
  int64_t off[20];
  int64_t total;
  // reordered calls: dense copies of q / k / v in the call's token order (offsets, -1 if
  // the path does not read that tensor by tiles), after every other buffer
  int64_t off_copy[3];
};

int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

int32_t make_plan(int64_t B, int64_t T, int64_t H, int64_t D, int32_t blk, int32_t int8, Plan& p) {
  if (B < 1 || T < 1 || H < 1) return fail(SOLB200_ERR_INVALID, "batch, tokens and heads must be >= 1");
  if (D != 64 && D != 128) return fail(SOLB200_ERR_INVALID, "head_dim must be 64 or 128");
  if (blk != 64 && blk != 128) return fail(SOLB200_ERR_INVALID, "block must be 64 or 128");
  if (T > (int64_t)1 << 30) return fail(SOLB200_ERR_INVALID, "tokens must be < 2^30");
  p.B = B; p.T = T; p.H = H; p.D = D; p.blk = blk; p.int8 = int8 != 0;
  p.N = (int)((T + blk - 1) / blk);
  p.npad = (p.N + 63) / 64 * 64;   // zero-padded to whole 64-block groups, as the reference
  p.nw = (p.N + 31) / 32;
  if (B * H * p.N >= ((int64_t)1 << 31)) return fail(SOLB200_ERR_INVALID, "too many query blocks");
  int64_t cur = 0;
  auto take = [&](int64_t bytes) {
    const int64_t o = cur;
    cur = align_up(cur + bytes, 256);
    return o;
  };
  for (auto& o : p.off) o = -1;
  p.off[SOLB200_BUF_ERROR] = take(256);
  p.off[SOLB200_BUF_KC] = take(B * p.npad * H * D * 2);
  p.off[SOLB200_BUF_VC] = take(B * p.npad * H * D * 2);
  p.off[SOLB200_BUF_CENTROID] = take(B * p.N * H * D * 4);
  p.off[SOLB200_BUF_KMEAN] = take(B * H * D * 4);
  p.off[SOLB200_BUF_KVAR] = take(B * H * D * 4);
  p.off[SOLB200_BUF_THR] = take(B * p.N * H * 4);
  p.off[SOLB200_BUF_MASK] = take(B * H * p.N * p.nw * 4);
  p.off[SOLB200_BUF_COUNT] = take(B * H * p.N * 4);
  if (p.int8) {
    p.off[SOLB200_BUF_VAMAX] = take(B * p.N * H * D * 4);
    p.off[SOLB200_BUF_VSCALE] = take(B * H * D * 4);
    p.off[SOLB200_BUF_QI] = take(B * T * H * D);
    p.off[SOLB200_BUF_QS] = take(B * H * (int64_t)p.N * blk * 4);
    p.off[SOLB200_BUF_KI] = take(B * T * H * D);
    p.off[SOLB200_BUF_KS] = take(B * H * (int64_t)p.N * blk * 4);
    p.off[SOLB200_BUF_VI] = take(B * T * H * D);
  }
  p.off[SOLB200_BUF_ORDER] = take(B * H * p.N * 4);
  p.total = cur;
  p.off_copy[0] = p.off_copy[1] = p.off_copy[2] = -1;
  return SOLB200_OK;
}

// The plan of a reordered call: the forward reads q (both paths), k (BF16) and v (BF16, or
// INT8 without int8 P.V) by TMA tiles, so those are copied in the call's token order.
int32_t make_plan_reordered(int64_t B, int64_t T, int64_t H, int64_t D, int32_t blk, int32_t int8, int32_t int8_pv,
                            Plan& p) {
  const int32_t rc = make_plan(B, T, H, D, blk, int8, p);
  if (rc) return rc;
  const bool need[3] = {true, !p.int8, !p.int8 || !int8_pv};
  for (int i = 0; i < 3; ++i) {
    if (!need[i]) continue;
    p.off_copy[i] = p.total;
    p.total = align_up(p.total + B * T * H * D * 2, 256);
  }
  return SOLB200_OK;
}

template <typename T>
T* at(void* ws, const Plan& p, int which) {
  return reinterpret_cast<T*>(static_cast<char*>(ws) + p.off[which]);
}

int32_t check_device() {
  int dev = 0, major = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  if (major != 10) return fail(SOLB200_ERR_DEVICE, "solb200 kernels are built for sm_100a (B200) only");
  return SOLB200_OK;
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

int32_t check_tensor(const char* name, const void* ptr, const int64_t* s, int64_t B) {
  if (!ptr || !s) return fail(SOLB200_ERR_INVALID, std::string(name) + ": null pointer");
  if (!aligned16(ptr)) return fail(SOLB200_ERR_ALIGNMENT, std::string(name) + ": base not 16-byte aligned");
  for (int i = 0; i < 3; ++i) {
    if (i == 0 && B == 1) continue;
    if (s[i] <= 0 || s[i] % 8 != 0)
      return fail(SOLB200_ERR_ALIGNMENT,
                  std::string(name) + ": batch/token/head strides must be positive multiples of 8 elements");
  }
  return SOLB200_OK;
}

// -------------------------------------------------------------- tensor maps

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 4-D map over a BTHD-like tensor: dims {D, H, rows, B}, byte strides {head, row, batch},
// box {64 bf16 (or 128 int8) = 128 bytes, 1, box_rows, 1}, 128-byte swizzle, OOB = zeros.
int32_t make_map(CUtensorMap* m, const void* ptr, bool int8, int64_t D, int64_t H, int64_t rows, int64_t B,
                 int64_t s_h, int64_t s_row, int64_t s_b, int box_rows, const char* name) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SOLB200_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int64_t esz = int8 ? 1 : 2;
  if (B == 1) s_b = rows * s_row;   // unused; any aligned value
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)rows, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(s_h * esz), (cuuint64_t)(s_row * esz), (cuuint64_t)(s_b * esz)};
  // 128-byte rows (64 bf16 or 128 int8) use the 128-byte swizzle; int8 rows of a
  // 64-wide head are 64 bytes and use the 64-byte swizzle.
  const cuuint32_t inner = int8 ? (cuuint32_t)(D < 128 ? D : 128) : 64;
  const CUtensorMapSwizzle swz = inner * esz == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  cuuint32_t box[4] = {inner, 1, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, int8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(SOLB200_ERR_CUDA, std::string("cuTensorMapEncodeTiled failed for ") + name +
                                      " (code " + std::to_string((int)r) + ")");
  return SOLB200_OK;
}

// --------------------------------------------------------------- pipeline

struct Call {
  const void *q, *k, *v;
  const int64_t *sq, *sk, *sv;
  void* out;
  float scale, tau;
  int64_t sink_kv[2], sink_q[2];
  int32_t stages;
  bool int8, int8_pv;
  void* ws;
  int64_t ws_bytes;
  int32_t* lists;
  float* stat;
  const int64_t* perm;   // token order of a reordered call, or null
  cudaStream_t st;
};

int32_t run(const Plan& P, const Call& c) {
  int32_t rc = check_device();
  if (rc) return rc;
  if ((rc = check_tensor("q", c.q, c.sq, P.B))) return rc;
  if ((rc = check_tensor("k", c.k, c.sk, P.B))) return rc;
  if ((rc = check_tensor("v", c.v, c.sv, P.B))) return rc;
  if (c.stages < SOLB200_STAGES_ALL || c.stages > SOLB200_STAGES_ROUTE)
    return fail(SOLB200_ERR_INVALID, "unknown stages value");
  const bool whole_prep = c.stages == SOLB200_STAGES_ALL || c.stages == SOLB200_STAGES_PREPARE;
  const bool do_pool = whole_prep || c.stages == SOLB200_STAGES_POOL;
  const bool do_quant = whole_prep || c.stages == SOLB200_STAGES_QUANT;
  const bool do_route = whole_prep || c.stages == SOLB200_STAGES_ROUTE;
  const bool do_fwd = c.stages == SOLB200_STAGES_ALL || c.stages == SOLB200_STAGES_FORWARD;
  if (do_fwd && (!c.out || !aligned16(c.out)))
    return fail(SOLB200_ERR_ALIGNMENT, "out: null or not 16-byte aligned");
  if (!c.ws || c.ws_bytes < P.total)
    return fail(SOLB200_ERR_WORKSPACE, "workspace is " + std::to_string(c.ws_bytes) + " bytes, needs " +
                                           std::to_string(P.total));
  if (!aligned16(c.ws)) return fail(SOLB200_ERR_ALIGNMENT, "workspace not 16-byte aligned");
  if (!(c.scale > 0.f)) return fail(SOLB200_ERR_INVALID, "scale must be > 0");
  const int hd = (int)P.D;
  const float s2 = c.scale * 1.4426950408889634f;
  int* err = at<int>(c.ws, P, SOLB200_BUF_ERROR);
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), c.st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(error word)");

  PoolParams pp{};
  pp.q = static_cast<const __nv_bfloat16*>(c.q);
  pp.k = static_cast<const __nv_bfloat16*>(c.k);
  pp.v = static_cast<const __nv_bfloat16*>(c.v);
  pp.sq_b = c.sq[0]; pp.sq_t = c.sq[1]; pp.sq_h = c.sq[2];
  pp.sk_b = c.sk[0]; pp.sk_t = c.sk[1]; pp.sk_h = c.sk[2];
  pp.sv_b = c.sv[0]; pp.sv_t = c.sv[1]; pp.sv_h = c.sv[2];
  pp.kc = at<__nv_bfloat16>(c.ws, P, SOLB200_BUF_KC);
  pp.vc = at<__nv_bfloat16>(c.ws, P, SOLB200_BUF_VC);
  pp.centroid = at<float>(c.ws, P, SOLB200_BUF_CENTROID);
  pp.vamax = (c.int8 && c.int8_pv) ? at<float>(c.ws, P, SOLB200_BUF_VAMAX) : nullptr;
  int8_t* const qi_buf = c.int8 ? at<int8_t>(c.ws, P, SOLB200_BUF_QI) : nullptr;
  float* const qs_buf = c.int8 ? at<float>(c.ws, P, SOLB200_BUF_QS) : nullptr;
  pp.perm = c.perm;
  pp.err = err;
  __nv_bfloat16* copies[3] = {nullptr, nullptr, nullptr};
  for (int i = 0; i < 3; ++i)
    if (c.perm && P.off_copy[i] >= 0)
      copies[i] = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(c.ws) + P.off_copy[i]);
  pp.qcopy = copies[0]; pp.kcopy = copies[1]; pp.vcopy = copies[2];
  pp.B = (int)P.B; pp.T = (int)P.T; pp.H = (int)P.H; pp.N = P.N; pp.npad = P.npad; pp.blk = P.blk;
  if (do_pool) {
    NvtxRange r("solb200.pool");
    launch_pool(pp, hd, pp.vamax != nullptr, c.st);
  }

  MomentsParams mp{};
  mp.kc = pp.kc;
  mp.vamax = pp.vamax;
  mp.kmean = at<float>(c.ws, P, SOLB200_BUF_KMEAN);
  mp.kvar = at<float>(c.ws, P, SOLB200_BUF_KVAR);
  mp.vscale = c.int8 ? at<float>(c.ws, P, SOLB200_BUF_VSCALE) : nullptr;
  mp.B = (int)P.B; mp.H = (int)P.H; mp.N = P.N; mp.npad = P.npad;
  if (do_pool) {
    NvtxRange r("solb200.moments");
    launch_moments(mp, hd, c.int8, c.st);
  }

  if (c.int8 && do_quant) {
    NvtxRange r("solb200.quant");
    QuantParams qp{};
    qp.q = pp.q; qp.k = pp.k; qp.v = pp.v;
    qp.sq_b = pp.sq_b; qp.sq_t = pp.sq_t; qp.sq_h = pp.sq_h;
    qp.sk_b = pp.sk_b; qp.sk_t = pp.sk_t; qp.sk_h = pp.sk_h;
    qp.sv_b = pp.sv_b; qp.sv_t = pp.sv_t; qp.sv_h = pp.sv_h;
    qp.kmean = mp.kmean;
    qp.vscale = c.int8_pv ? mp.vscale : nullptr;
    qp.qi = qi_buf;
    qp.qs = qs_buf;
    qp.ki = at<int8_t>(c.ws, P, SOLB200_BUF_KI);
    qp.ks = at<float>(c.ws, P, SOLB200_BUF_KS);
    qp.vi = c.int8_pv ? at<int8_t>(c.ws, P, SOLB200_BUF_VI) : nullptr;
    qp.B = (int)P.B; qp.T = (int)P.T; qp.H = (int)P.H; qp.tp = P.N * P.blk;
    qp.perm = c.perm;
    qp.err = err;
    launch_quant_qkv(qp, hd, c.st);
  }

  RouteParams rp{};
  rp.kc = pp.kc;
  rp.centroid = pp.centroid;
  rp.kmean = mp.kmean;
  rp.kvar = mp.kvar;
  rp.thr = at<float>(c.ws, P, SOLB200_BUF_THR);
  rp.mask = at<uint32_t>(c.ws, P, SOLB200_BUF_MASK);
  rp.count = at<int>(c.ws, P, SOLB200_BUF_COUNT);
  rp.lists = c.lists;
  rp.stat = c.stat;
  rp.B = (int)P.B; rp.H = (int)P.H; rp.N = P.N; rp.npad = P.npad; rp.nw = P.nw;
  rp.s2 = s2; rp.tau = c.tau; rp.int8 = c.int8 ? 1 : 0;
  const int64_t lim = (int64_t)1 << 30;
  auto clampi = [&](int64_t x) { return (int)(x < -lim ? -lim : (x > lim ? lim : x)); };
  rp.sink_kv0 = clampi(c.sink_kv[0]); rp.sink_kv1 = clampi(c.sink_kv[1]);
  rp.sink_q0 = clampi(c.sink_q[0]); rp.sink_q1 = clampi(c.sink_q[1]);
  if (do_route) {
    NvtxRange r("solb200.route");
    launch_route(rp, hd, c.st);
    launch_order(rp.count, at<int>(c.ws, P, SOLB200_BUF_ORDER), (int)(P.B * P.H), P.N, c.st);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "preprocess launch");
  if (!do_fwd) return SOLB200_OK;

  FwdParams fp{};
  fp.mask = rp.mask;
  fp.order = at<int>(c.ws, P, SOLB200_BUF_ORDER);
  fp.err = err;
  fp.B = (int)P.B; fp.T = (int)P.T; fp.H = (int)P.H; fp.N = P.N; fp.nw = P.nw;
  fp.Tk = (int)P.T; fp.Nk = P.N;
  fp.s2 = s2;
  fp.wait_ns = g_debug_wait.wait_ns;
  fp.stall_unit = g_debug_wait.stall_unit;
  fp.perm = c.perm;
  fp.out = static_cast<__nv_bfloat16*>(c.out);
  FwdMaps m;
  const int64_t npad = P.npad;
  // reordered calls read the dense copies in the call's token order
  const int64_t TD = P.H * P.D;
  const int64_t dense_s[3] = {TD * P.T, TD, P.D};
  const void* qsrc = copies[0] ? copies[0] : c.q;
  const void* ksrc = copies[1] ? copies[1] : c.k;
  const void* vsrc = copies[2] ? copies[2] : c.v;
  const int64_t* sqm = copies[0] ? dense_s : c.sq;
  const int64_t* skm = copies[1] ? dense_s : c.sk;
  const int64_t* svm = copies[2] ? dense_s : c.sv;
  if ((rc = make_map(&m.q, qsrc, false, P.D, P.H, P.T, P.B, sqm[2], sqm[1], sqm[0], 128, "q"))) return rc;
  // the BF16 kernel streams 64-row halves; the INT8 kernel 128-row pooled chunks
  const int pooled_rows = c.int8 ? 128 : 64;
  const int kv_rows = c.int8 ? P.blk : 64;
  if ((rc = make_map(&m.kc, pp.kc, false, P.D, P.H, npad, P.B, P.D, P.H * P.D, npad * P.H * P.D, pooled_rows,
                     "kc")))
    return rc;
  if ((rc = make_map(&m.vc, pp.vc, false, P.D, P.H, npad, P.B, P.D, P.H * P.D, npad * P.H * P.D, pooled_rows,
                     "vc")))
    return rc;
  if ((rc = make_map(&m.o, c.out, false, P.D, P.H, P.T, P.B, P.D, P.H * P.D, P.T * P.H * P.D, P.blk, "out")))
    return rc;
  if (!c.int8) {
    if ((rc = make_map(&m.k, ksrc, false, P.D, P.H, P.T, P.B, skm[2], skm[1], skm[0], kv_rows, "k"))) return rc;
    if ((rc = make_map(&m.v, vsrc, false, P.D, P.H, P.T, P.B, svm[2], svm[1], svm[0], kv_rows, "v"))) return rc;
    NvtxRange r("solb200.forward");
    e = launch_fwd_bf16(hd, P.blk, m, fp, c.st);
    if (e != cudaSuccess) return cuda_fail(e, "bf16 forward launch");
    return SOLB200_OK;
  }
  // int8 operands: qi (128-row query tiles), ki and vi (one routed block per tile)
  if ((rc = make_map(&m.qi, qi_buf, true, P.D, P.H, P.T, P.B, P.D, TD, P.T * TD, 128, "qi"))) return rc;
  if ((rc = make_map(&m.ki, at<int8_t>(c.ws, P, SOLB200_BUF_KI), true, P.D, P.H, P.T, P.B, P.D, TD, P.T * TD,
                     P.blk, "ki")))
    return rc;
  if (c.int8_pv) {
    if ((rc = make_map(&m.vi, at<int8_t>(c.ws, P, SOLB200_BUF_VI), true, P.D, P.H, P.T, P.B, P.D, TD,
                       P.T * TD, P.blk, "vi")))
      return rc;
  } else {
    if ((rc = make_map(&m.v, vsrc, false, P.D, P.H, P.T, P.B, svm[2], svm[1], svm[0], kv_rows, "v"))) return rc;
  }
  fp.qs = qs_buf;
  fp.ks = at<float>(c.ws, P, SOLB200_BUF_KS);
  fp.vscale = mp.vscale;
  fp.int8_pv = c.int8_pv ? 1 : 0;
  {
    NvtxRange r("solb200.forward_int8");
    e = launch_fwd_int8(hd, P.blk, m, fp, c.st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "int8 forward launch");
  return SOLB200_OK;
}

}  // namespace

extern "C" {

const char* solb200_last_error(void) { return g_last_error.c_str(); }

int32_t solb200_abi_version(void) { return 2; }

int32_t solb200_workspace_bytes(int64_t batch, int64_t tokens, int64_t heads, int64_t head_dim, int32_t block,
                                int32_t int8, int64_t* bytes) {
  Plan p;
  const int32_t rc = make_plan(batch, tokens, heads, head_dim, block, int8, p);
  if (rc) return rc;
  if (!bytes) return fail(SOLB200_ERR_INVALID, "bytes: null pointer");
  *bytes = p.total;
  return SOLB200_OK;
}

int32_t solb200_workspace_offset(int64_t batch, int64_t tokens, int64_t heads, int64_t head_dim, int32_t block,
                                 int32_t int8, int32_t which, int64_t* offset) {
  Plan p;
  const int32_t rc = make_plan(batch, tokens, heads, head_dim, block, int8, p);
  if (rc) return rc;
  if (which < 0 || which > SOLB200_BUF_ORDER || p.off[which] < 0)
    return fail(SOLB200_ERR_INVALID, "buffer not part of this workspace");
  if (!offset) return fail(SOLB200_ERR_INVALID, "offset: null pointer");
  *offset = p.off[which];
  return SOLB200_OK;
}

static int32_t attn_entry(const void* q, const int64_t* sq, const void* k, const int64_t* sk, const void* v,
                          const int64_t* sv, void* out, int64_t B, int64_t T, int64_t H, int64_t D, int32_t blk,
                          float scale, float tau, const int64_t* sink_kv, const int64_t* sink_q, bool int8,
                          bool int8_pv, int32_t stages, void* ws, int64_t ws_bytes, int32_t* lists, float* stat,
                          void* stream, const int64_t* perm = nullptr) {
  Plan P;
  int32_t rc = perm ? make_plan_reordered(B, T, H, D, blk, int8 ? 1 : 0, int8_pv ? 1 : 0, P)
                    : make_plan(B, T, H, D, blk, int8 ? 1 : 0, P);
  if (rc) return rc;
  Call c{};
  c.q = q; c.k = k; c.v = v; c.sq = sq; c.sk = sk; c.sv = sv; c.out = out;
  c.scale = scale; c.tau = tau;
  c.sink_kv[0] = sink_kv ? sink_kv[0] : 0; c.sink_kv[1] = sink_kv ? sink_kv[1] : 0;
  c.sink_q[0] = sink_q ? sink_q[0] : 0; c.sink_q[1] = sink_q ? sink_q[1] : 0;
  c.stages = stages; c.int8 = int8; c.int8_pv = int8_pv;
  c.ws = ws; c.ws_bytes = ws_bytes; c.lists = lists; c.stat = stat; c.perm = perm;
  c.st = static_cast<cudaStream_t>(stream);
  return run(P, c);
}

int32_t solb200_sol_attn_bf16(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                              const void* v, const int64_t* v_strides, void* out, int64_t batch, int64_t tokens,
                              int64_t heads, int64_t head_dim, int32_t block, float scale, float tau,
                              const int64_t* sink_kv, const int64_t* sink_q, int32_t stages, void* workspace,
                              int64_t workspace_bytes, int32_t* lists, float* route_stat, void* stream) {
  return attn_entry(q, q_strides, k, k_strides, v, v_strides, out, batch, tokens, heads, head_dim, block, scale,
                    tau, sink_kv, sink_q, false, false, stages, workspace, workspace_bytes, lists, route_stat,
                    stream);
}

int32_t solb200_sol_attn_int8(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                              const void* v, const int64_t* v_strides, void* out, int64_t batch, int64_t tokens,
                              int64_t heads, int64_t head_dim, int32_t block, float scale, float tau,
                              const int64_t* sink_kv, const int64_t* sink_q, int32_t int8_pv, int32_t stages,
                              void* workspace, int64_t workspace_bytes, int32_t* lists, float* route_stat,
                              void* stream) {
  return attn_entry(q, q_strides, k, k_strides, v, v_strides, out, batch, tokens, heads, head_dim, block, scale,
                    tau, sink_kv, sink_q, true, int8_pv != 0, stages, workspace, workspace_bytes, lists,
                    route_stat, stream);
}

int32_t solb200_workspace_bytes_reordered(int64_t batch, int64_t tokens, int64_t heads, int64_t head_dim,
                                          int32_t block, int32_t int8, int32_t int8_pv, int64_t* bytes) {
  Plan p;
  const int32_t rc = make_plan_reordered(batch, tokens, heads, head_dim, block, int8, int8_pv, p);
  if (rc) return rc;
  if (!bytes) return fail(SOLB200_ERR_INVALID, "bytes: null pointer");
  *bytes = p.total;
  return SOLB200_OK;
}

int32_t solb200_sol_attn_reordered(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                   const void* v, const int64_t* v_strides, void* out, int64_t batch, int64_t tokens,
                                   int64_t heads, int64_t head_dim, int32_t block, float scale, float tau,
                                   const int64_t* sink_kv, const int64_t* sink_q, const int64_t* order, int32_t int8,
                                   int32_t int8_pv, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!order) return fail(SOLB200_ERR_INVALID, "order: null pointer");
  if (reinterpret_cast<uintptr_t>(order) & 7u) return fail(SOLB200_ERR_ALIGNMENT, "order: not 8-byte aligned");
  return attn_entry(q, q_strides, k, k_strides, v, v_strides, out, batch, tokens, heads, head_dim, block, scale,
                    tau, sink_kv, sink_q, int8 != 0, int8_pv != 0, SOLB200_STAGES_ALL, workspace,
                    workspace_bytes, nullptr, nullptr, stream, order);
}

// Dense attention on the BF16 kernel (every key block exact); `bp` adds a mask (null: none).
static int32_t attn_dense_impl(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                               const void* v, const int64_t* v_strides, void* out, int64_t batch,
                               int64_t q_tokens, int64_t kv_tokens, int64_t heads, int64_t head_dim, float scale,
                               void* workspace, int64_t workspace_bytes, void* stream, const BiasParams* bp) {
  int32_t rc = check_device();
  if (rc) return rc;
  if (batch < 1 || q_tokens < 1 || kv_tokens < 1 || heads < 1)
    return fail(SOLB200_ERR_INVALID, "batch, tokens and heads must be >= 1");
  if (head_dim != 64 && head_dim != 128) return fail(SOLB200_ERR_INVALID, "head_dim must be 64 or 128");
  if (q_tokens > ((int64_t)1 << 30) || kv_tokens > ((int64_t)1 << 30))
    return fail(SOLB200_ERR_INVALID, "tokens must be < 2^30");
  constexpr int BLK = 128;
  const int64_t nq = (q_tokens + BLK - 1) / BLK, nk = (kv_tokens + BLK - 1) / BLK;
  if (batch * heads * nq >= ((int64_t)1 << 31)) return fail(SOLB200_ERR_INVALID, "too many query blocks");
  if ((rc = check_tensor("q", q, q_strides, batch))) return rc;
  if ((rc = check_tensor("k", k, k_strides, batch))) return rc;
  if ((rc = check_tensor("v", v, v_strides, batch))) return rc;
  if (!out || !aligned16(out)) return fail(SOLB200_ERR_ALIGNMENT, "out: null or not 16-byte aligned");
  if (!workspace || workspace_bytes < 256)
    return fail(SOLB200_ERR_WORKSPACE, "the dense call needs a workspace of at least 256 bytes");
  if (!aligned16(workspace)) return fail(SOLB200_ERR_ALIGNMENT, "workspace not 16-byte aligned");
  if (!(scale > 0.f)) return fail(SOLB200_ERR_INVALID, "scale must be > 0");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* err = static_cast<int*>(workspace);
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(error word)");
  FwdParams fp{};
  fp.mask = nullptr;   // dense: every key block exact
  fp.order = nullptr;
  fp.err = err;
  fp.B = (int)batch; fp.T = (int)q_tokens; fp.H = (int)heads; fp.N = (int)nq; fp.nw = (int)((nk + 31) / 32);
  fp.Tk = (int)kv_tokens; fp.Nk = (int)nk;
  fp.s2 = scale * 1.4426950408889634f;
  fp.wait_ns = g_debug_wait.wait_ns;
  fp.stall_unit = g_debug_wait.stall_unit;
  fp.perm = nullptr;
  fp.out = static_cast<__nv_bfloat16*>(out);
  FwdMaps m;
  const int64_t D = head_dim, H = heads;
  if ((rc = make_map(&m.q, q, false, D, H, q_tokens, batch, q_strides[2], q_strides[1], q_strides[0], 128, "q")))
    return rc;
  if ((rc = make_map(&m.k, k, false, D, H, kv_tokens, batch, k_strides[2], k_strides[1], k_strides[0], 64, "k")))
    return rc;
  if ((rc = make_map(&m.v, v, false, D, H, kv_tokens, batch, v_strides[2], v_strides[1], v_strides[0], 64, "v")))
    return rc;
  if ((rc = make_map(&m.o, out, false, D, H, q_tokens, batch, D, H * D, q_tokens * H * D, BLK, "out"))) return rc;
  m.kc = m.k;   // no pooled keys / values in a dense call: valid maps that are never loaded
  m.vc = m.v;
  {
    NvtxRange r(bp ? "solb200.dense_masked" : "solb200.dense");
    e = bp ? launch_fwd_bf16_masked((int)head_dim, m, fp, *bp, st) : launch_fwd_bf16((int)head_dim, BLK, m, fp, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "dense forward launch");
  return SOLB200_OK;
}

int32_t solb200_attn_dense(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                           const void* v, const int64_t* v_strides, void* out, int64_t batch, int64_t q_tokens,
                           int64_t kv_tokens, int64_t heads, int64_t head_dim, float scale, void* workspace,
                           int64_t workspace_bytes, void* stream) {
  return attn_dense_impl(q, q_strides, k, k_strides, v, v_strides, out, batch, q_tokens, kv_tokens, heads,
                         head_dim, scale, workspace, workspace_bytes, stream, nullptr);
}

int32_t solb200_attn_dense_masked(const void* q, const int64_t* q_strides, const void* k,
                                  const int64_t* k_strides, const void* v, const int64_t* v_strides,
                                  const void* mask, int32_t mask_kind, const int64_t* mask_strides, void* out,
                                  int64_t batch, int64_t q_tokens, int64_t kv_tokens, int64_t heads,
                                  int64_t head_dim, float scale, void* workspace, int64_t workspace_bytes,
                                  void* stream) {
  if (!mask || !mask_strides) return fail(SOLB200_ERR_INVALID, "mask: null pointer or strides");
  size_t esize = 0;
  switch (mask_kind) {
    case SOLB200_MASK_BOOL: esize = 1; break;
    case SOLB200_MASK_F32: esize = 4; break;
    case SOLB200_MASK_BF16:
    case SOLB200_MASK_F16: esize = 2; break;
    default: return fail(SOLB200_ERR_INVALID, "mask_kind must be SOLB200_MASK_BOOL, _F32, _BF16 or _F16");
  }
  if (reinterpret_cast<uintptr_t>(mask) % esize)
    return fail(SOLB200_ERR_ALIGNMENT, "mask: not aligned to its element size");
  BiasParams bp{};
  bp.bias = mask;
  bp.bias_kind = mask_kind;
  bp.bias_mul = scale > 0.f ? 1.f / scale : 0.f;
  for (int i = 0; i < 4; ++i) {
    if (mask_strides[i] < 0 || mask_strides[i] > ((int64_t)1 << 40))
      return fail(SOLB200_ERR_INVALID, "mask strides must be in [0, 2^40] elements (0 broadcasts)");
    bp.bias_s[i] = mask_strides[i];
  }
  return attn_dense_impl(q, q_strides, k, k_strides, v, v_strides, out, batch, q_tokens, kv_tokens, heads,
                         head_dim, scale, workspace, workspace_bytes, stream, &bp);
}

int32_t solb200_debug_set_wait(int64_t wait_ns, int32_t stall_unit) {
  if (stall_unit < -1) return fail(SOLB200_ERR_INVALID, "stall_unit must be -1 (none) or a unit id");
  g_debug_wait.wait_ns = wait_ns > 0 ? (uint64_t)wait_ns : SOLB200_WAIT_NS;
  g_debug_wait.stall_unit = stall_unit;
  return SOLB200_OK;
}

int32_t solb200_read_device_error(void* workspace, int32_t* code, void* stream) {
  if (!workspace || !code) return fail(SOLB200_ERR_INVALID, "null workspace or code pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  e = cudaMemsetAsync(workspace, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the device error word");
  *code = host;
  if (host & kErrBadIndex)
    return fail(SOLB200_ERR_INVALID, "the token order holds an index outside [0, tokens) (device error bits " +
                                         std::to_string(host) + ")");
  if (host != 0)
    return fail(SOLB200_ERR_TIMEOUT, "a kernel gave up on a bounded wait (device error bits " +
                                         std::to_string(host) + ")");
  return SOLB200_OK;
}

int32_t solb200_morton_perm(int64_t frames, int64_t height, int64_t width, int32_t curve, int64_t roll,
                            int64_t* perm, int64_t* inverse, void* stream) {
  int32_t rc = check_device();
  if (rc) return rc;
  if (frames < 1 || height < 1 || width < 1) return fail(SOLB200_ERR_INVALID, "grid dims must be >= 1");
  if (curve != 0 && curve != 1) return fail(SOLB200_ERR_INVALID, "curve must be 0 (3d) or 1 (2d_frame)");
  const int64_t lim = curve == 0 ? ((int64_t)1 << 21) : ((int64_t)1 << 14);
  if (width >= lim || height >= lim || (curve == 0 && frames >= lim))
    return fail(SOLB200_ERR_INVALID, "grid dims exceed the Morton code's bit budget");
  if (frames * height * width >= ((int64_t)1 << 40)) return fail(SOLB200_ERR_INVALID, "grid too large");
  if (!perm || !inverse) return fail(SOLB200_ERR_INVALID, "perm/inverse: null pointer");
  launch_morton(frames, height, width, curve, roll, perm, inverse, static_cast<cudaStream_t>(stream));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SOLB200_OK : cuda_fail(e, "morton launch");
}

int32_t solb200_gather_rows(const void* const* src, void* const* dst, int32_t ntensors, const int64_t* index,
                            int64_t batch, int64_t rows, int64_t row_bytes, int64_t src_stride_b,
                            int64_t src_stride_row, int64_t dst_stride_b, int64_t dst_stride_row, void* stream) {
  int32_t rc = check_device();
  if (rc) return rc;
  if (ntensors < 1 || ntensors > 4) return fail(SOLB200_ERR_INVALID, "ntensors must be 1..4");
  if (!src || !dst || !index) return fail(SOLB200_ERR_INVALID, "null pointer");
  if (batch < 1 || rows < 1 || row_bytes < 16 || row_bytes % 16)
    return fail(SOLB200_ERR_INVALID, "row_bytes must be a positive multiple of 16");
  if (src_stride_row % 16 || dst_stride_row % 16 || (batch > 1 && (src_stride_b % 16 || dst_stride_b % 16)))
    return fail(SOLB200_ERR_ALIGNMENT, "strides must be multiples of 16 bytes");
  GatherParams gp{};
  for (int i = 0; i < ntensors; ++i) {
    if (!src[i] || !dst[i] || !aligned16(src[i]) || !aligned16(dst[i]))
      return fail(SOLB200_ERR_ALIGNMENT, "tensor pointers must be non-null and 16-byte aligned");
    gp.src[i] = static_cast<const char*>(src[i]);
    gp.dst[i] = static_cast<char*>(dst[i]);
  }
  gp.ntensors = ntensors;
  gp.src_stride_b = src_stride_b; gp.src_stride_row = src_stride_row;
  gp.dst_stride_b = dst_stride_b; gp.dst_stride_row = dst_stride_row;
  gp.index = index; gp.batch = batch; gp.rows = rows; gp.row_bytes = row_bytes;
  launch_gather(gp, static_cast<cudaStream_t>(stream));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SOLB200_OK : cuda_fail(e, "gather launch");
}

int32_t solb200_selftest_quotient(const float* x, const float* s, int64_t n, uint64_t* bad, void* stream) {
  int32_t rc = check_device();
  if (rc) return rc;
  if (!x || !s || !bad || n < 0) return fail(SOLB200_ERR_INVALID, "null pointer or negative count");
  if (n == 0) return SOLB200_OK;
  launch_quotient_selftest(x, s, n, reinterpret_cast<unsigned long long*>(bad), static_cast<cudaStream_t>(stream));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SOLB200_OK : cuda_fail(e, "selftest launch");
}

int32_t solb200_copy_heads(void* device, void* host, int64_t batch, int64_t tokens, int64_t heads,
                           int64_t head_dim, int64_t h0, int64_t hc, int32_t to_device, void* stream) {
  if (!device || !host) return fail(SOLB200_ERR_INVALID, "null pointer");
  if (batch < 1 || tokens < 1 || heads < 1 || head_dim < 1 || hc < 1 || h0 < 0 || h0 + hc > heads)
    return fail(SOLB200_ERR_INVALID, "head range [h0, h0+hc) must lie in [0, heads)");
  const size_t esz = 2;   // bf16
  const size_t host_pitch = (size_t)heads * head_dim * esz, dev_pitch = (size_t)hc * head_dim * esz;
  const size_t width = dev_pitch, height = (size_t)batch * tokens;
  char* h = static_cast<char*>(host) + (size_t)h0 * head_dim * esz;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = to_device
      ? cudaMemcpy2DAsync(device, dev_pitch, h, host_pitch, width, height, cudaMemcpyHostToDevice, st)
      : cudaMemcpy2DAsync(h, host_pitch, device, dev_pitch, width, height, cudaMemcpyDeviceToHost, st);
  return e == cudaSuccess ? SOLB200_OK : cuda_fail(e, "cudaMemcpy2DAsync (head chunk)");
}

}  // extern "C"

namespace solb200 {

int32_t set_last_error(int32_t code, const std::string& msg) { return fail(code, msg); }

int32_t set_cuda_error(cudaError_t e, const char* what) { return cuda_fail(e, what); }

int32_t plan_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t D, int32_t block, int32_t int8,
                             int64_t* bytes) {
  return solb200_workspace_bytes(B, T, H, D, block, int8, bytes);
}

int32_t run_attention(const void* q, const int64_t* sq, const void* k, const int64_t* sk, const void* v,
                      const int64_t* sv, void* out, int64_t B, int64_t T, int64_t H, int64_t D, int32_t blk,
                      float scale, float tau, const int64_t* sink_kv, const int64_t* sink_q, bool int8,
                      bool int8_pv, int32_t stages, void* ws, int64_t ws_bytes, int32_t* lists, float* stat,
                      void* stream) {
  return attn_entry(q, sq, k, sk, v, sv, out, B, T, H, D, blk, scale, tau, sink_kv, sink_q, int8, int8_pv,
                    stages, ws, ws_bytes, lists, stat, stream);
}

}  // namespace solb200
