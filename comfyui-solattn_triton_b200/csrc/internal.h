// Internal (not exported) hooks of api.cu for the library's other entry-point files.
#pragma once

#include <stdint.h>

#include <string>

#include <cuda_runtime.h>

namespace solb200 {

// Record the calling thread's last-error text and return `code`.
int32_t set_last_error(int32_t code, const std::string& msg);
int32_t set_cuda_error(cudaError_t e, const char* what);

// Workspace bytes of one attention call with this geometry (solb200_workspace_bytes).
int32_t plan_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t D, int32_t block, int32_t int8,
                             int64_t* bytes);

// The attention pipeline of solb200_sol_attn_bf16 / _int8 on a given workspace.
int32_t run_attention(const void* q, const int64_t* sq, const void* k, const int64_t* sk, const void* v,
                      const int64_t* sv, void* out, int64_t B, int64_t T, int64_t H, int64_t D, int32_t blk,
                      float scale, float tau, const int64_t* sink_kv, const int64_t* sink_q, bool int8,
                      bool int8_pv, int32_t stages, void* ws, int64_t ws_bytes, int32_t* lists, float* stat,
                      void* stream);

}  // namespace solb200
