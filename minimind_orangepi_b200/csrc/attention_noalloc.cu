// Allocation-free variant of the fused decode-attention operator.
//
// mmc_op_attention needs a caller-provided workspace (split partials, arrival
// counters, an error word). Some callers cannot provide one: code that runs
// where cudaMalloc is forbidden or unsafe (a custom allocator's own hooks, a
// real-time loop with a no-allocation rule, or a plugin host that owns all
// device memory). For them this file keeps a fixed workspace in a file-scope
// __device__ array that every GPU loading the library holds until the process
// exits, and passes it to the same kernel.
//
// The array's address is looked up once per device and cached for the life of
// the process; it belongs to that device's primary context, so the entry point
// must not be used after cudaDeviceReset (or from a non-primary context).
// With lazy module loading (the CUDA 12 default) the first call on a device
// loads the module, which may allocate the array's backing memory: make one
// warm-up call, or run with CUDA_MODULE_LOADING=EAGER, before entering a
// region where allocation is forbidden.
#include "../../include/minimind_cuda.h"

#include <cuda_runtime.h>

#include <mutex>
#include <string>

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per GPU
static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};
}  // namespace

// Sets the thread-local text mmc_last_error() returns (defined in mmc_api.cu).
void mmc_set_last_error(const std::string& msg);

extern "C" int mmc_op_attention_noalloc(int32_t batch, int32_t nq, int32_t nkv, int32_t hd, int32_t layer,
                                        int32_t layers, const float* d_qkv, const float* d_q_norm,
                                        const float* d_k_norm, const float* d_rope_cos, const float* d_rope_sin,
                                        int32_t max_pos, float eps, void* d_kv_pool, const int32_t* d_block_table,
                                        int32_t max_pages, const int32_t* d_seq_pos, const int32_t* d_slots,
                                        int32_t max_ctx, float* d_out, void* stream) {
  size_t need = 0;
  int rc = mmc_op_attention_workspace_size(batch, nq, nkv, hd, max_ctx, &need);
  if (rc != MMC_OK) return rc;
  if (need > kNoAllocScratchBytes) {
    mmc_set_last_error("mmc_op_attention_noalloc: this batch/context needs " + std::to_string(need) +
                       " bytes of scratch, more than the fixed " + std::to_string(kNoAllocScratchBytes) +
                       " (use mmc_op_attention with a workspace)");
    return MMC_ERR_INVALID;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    mmc_set_last_error("mmc_op_attention_noalloc: no usable current device");
    return MMC_ERR_CUDA;
  }
  void* scratch = nullptr;
  {
    // First call on a device: look up the array's device address with that
    // device current. Host code must never use g_attn_scratch's own name as a
    // device pointer: on the host it is only a stand-in symbol.
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_ptr[dev] == nullptr) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
      if (e != cudaSuccess || p == nullptr) {
        mmc_set_last_error(std::string("mmc_op_attention_noalloc: cudaGetSymbolAddress failed: ") +
                           cudaGetErrorString(e));
        return MMC_ERR_CUDA;
      }
      g_scratch_ptr[dev] = p;
    }
    scratch = g_scratch_ptr[dev];
  }
  // mmc_op_attention zeroes the counters and error word of its workspace on
  // `stream` before the launch, so stale contents from an earlier call are
  // harmless. Calls that overlap on the GPU share this array and race.
  rc = mmc_op_attention(batch, nq, nkv, hd, layer, layers, d_qkv, d_q_norm, d_k_norm, d_rope_cos, d_rope_sin, max_pos,
                        eps, d_kv_pool, d_block_table, max_pages, d_seq_pos, d_slots, max_ctx, d_out, scratch,
                        kNoAllocScratchBytes, stream);
  if (rc != MMC_OK) return rc;
  // The caller cannot see the error word inside this library's array, so the
  // call waits for the kernel and reports a device-side error (a missing KV
  // page, a position past max_pos, a bounded wait that ran out) itself.
  return mmc_op_attention_status(scratch, stream);
}
