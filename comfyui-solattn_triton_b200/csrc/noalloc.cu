// The allocation-free attention entry point (solb200_sol_attn_bf16_noalloc).
//
// Some hosts cannot give this library device memory at call time: an application
// that plans every device allocation up front and forbids allocating afterwards (a
// fixed-budget inference server, a plugin inside an engine that owns the allocator),
// or a caller that cannot afford cudaMalloc's implicit device-wide synchronisation in
// the attention path. For them this entry point runs the BF16 Sol-Attn call with its
// scratch (the workspace of solb200_sol_attn_bf16) in a file-scope __device__ array of
// fixed size, so the call itself allocates nothing: no cudaMalloc, no cudaFree, no
// allocating library routine. The caller still provides q, k, v and the output.
//
// The array's host-side name is only a stand-in; its device address is looked up with
// cudaGetSymbolAddress on the first call made with a device current, and cached for
// that device's CUDA context (a context created anew after a device reset reloads the
// module, so its address is looked up again). Every GPU that loads this library holds
// the array until the process exits. All calls on a device share it, so calls that
// overlap on the GPU (concurrent streams, or calls from several host threads) race on
// it: serialise them. The array's first 256 bytes hold the device error word of the
// last call (bounded-wait timeouts); solb200_noalloc_read_device_error reads and clears it.
#include <cuda.h>

#include <mutex>

#include "internal.h"
#include "solb200.h"

namespace {

constexpr int64_t kStaticScratchBytes = int64_t(16) << 20;   // 16 MiB
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
struct ScratchSlot {
  CUcontext ctx;   // the context the address belongs to
  void* address;
};
ScratchSlot g_scratch[kMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (this library does not link
// libcuda directly).
CUcontext current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  CUcontext ctx = nullptr;
  if (fn) fn(&ctx);
  return ctx;
}

// Device address of the static scratch on the current device (looked up once per
// device context).
int32_t static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return solb200::set_cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return solb200::set_last_error(SOLB200_ERR_INVALID, "device ordinal beyond the static scratch table");
  // Before any runtime call has used the device, its primary context may not exist yet
  // (ctx is null here); the symbol lookup creates it, and the context is read again after.
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  CUcontext ctx = current_context();
  ScratchSlot& slot = g_scratch[dev];
  if (slot.address == nullptr || ctx == nullptr || slot.ctx != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return solb200::set_cuda_error(e, "cudaGetSymbolAddress(static scratch)");
    slot.address = p;
    slot.ctx = current_context();
  }
  *out = slot.address;
  return SOLB200_OK;
}

}  // namespace

extern "C" int32_t solb200_sol_attn_bf16_noalloc(const void* q, const int64_t* q_strides, const void* k,
                                                 const int64_t* k_strides, const void* v,
                                                 const int64_t* v_strides, void* out, int64_t batch,
                                                 int64_t tokens, int64_t heads, int64_t head_dim,
                                                 int32_t block, float scale, float tau, const int64_t* sink_kv,
                                                 const int64_t* sink_q, void* stream) {
  int64_t need = 0;
  int32_t rc = solb200::plan_workspace_bytes(batch, tokens, heads, head_dim, block, 0, &need);
  if (rc) return rc;
  if (need > kStaticScratchBytes)
    return solb200::set_last_error(
        SOLB200_ERR_WORKSPACE,
        "this call needs " + std::to_string(need) + " bytes of scratch; the allocation-free entry point's "
        "static scratch holds " + std::to_string(kStaticScratchBytes) +
        " bytes (use solb200_sol_attn_bf16 with a caller workspace)");
  void* scratch = nullptr;
  if ((rc = static_scratch(&scratch))) return rc;
  // Nothing in the scratch needs clearing by this entry point: the pipeline zeroes the
  // error word on every call and every other buffer is fully rewritten before use.
  return solb200::run_attention(q, q_strides, k, k_strides, v, v_strides, out, batch, tokens, heads, head_dim,
                                block, scale, tau, sink_kv, sink_q, false, false, SOLB200_STAGES_ALL, scratch,
                                kStaticScratchBytes, nullptr, nullptr, stream);
}

extern "C" int32_t solb200_noalloc_read_device_error(int32_t* code, void* stream) {
  void* scratch = nullptr;
  const int32_t rc = static_scratch(&scratch);
  if (rc) return rc;
  // the error word sits at offset 0 of the scratch, as of a caller workspace
  return solb200_read_device_error(scratch, code, stream);
}
