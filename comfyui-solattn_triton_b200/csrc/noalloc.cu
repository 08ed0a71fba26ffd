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
// The array's host-side name is only a stand-in; its device address is looked up
// once per device with cudaGetSymbolAddress, on the first call made with that device
// current, and cached. Every GPU that loads this library holds the array until the
// process exits. All calls on a device share it, so calls that overlap on the GPU
// (concurrent streams, or calls from several host threads) race on it: serialise them.
#include <mutex>

#include "internal.h"
#include "solb200.h"

namespace {

constexpr int64_t kStaticScratchBytes = int64_t(16) << 20;   // 16 MiB
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of the static scratch on the current device (looked up once).
int32_t static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return solb200::set_cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return solb200::set_last_error(SOLB200_ERR_INVALID, "device ordinal beyond the static scratch table");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return solb200::set_cuda_error(e, "cudaGetSymbolAddress(static scratch)");
    g_scratch_address[dev] = p;
  }
  *out = g_scratch_address[dev];
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
