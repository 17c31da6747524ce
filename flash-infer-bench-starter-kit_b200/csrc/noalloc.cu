// Allocation-free variant of the layer call.
//
// Some callers cannot allocate GPU memory at the point where they call the
// layer: a custom memory manager that owns every device allocation of the
// process, a runtime that forbids cudaMalloc on its serving path (it would
// synchronise the device and stall other streams), or a plugin host that
// gives the plugin no allocator at all.  For them, moe_fp8_ds_run_noalloc
// runs the same six kernels as moe_fp8_ds_run, but on a workspace that lives
// in a file-scope __device__ array of this library instead of a buffer the
// caller passes.  That array (kNoAllocScratchBytes) is reserved on every GPU
// that loads the library and stays reserved until the process exits, and it
// limits the entry point to small decode batches (T <= 16 tokens).
#include <mutex>

#include "kernels.cuh"

namespace moe {
namespace {

constexpr uint64_t kNoAllocScratchBytes = 16ull << 20;   // 16 MiB per device
constexpr int kNoAllocMaxTokens = 16;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once
// per device; the array's host-side name is not a device address).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices)
    return MOE_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return MOE_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return MOE_OK;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_fp8_ds_run_noalloc(const moe_fp8_ds_args* args, void* stream) {
  if (!args) return MOE_ERR_INVALID_ARGUMENT;
  if (args->num_tokens > kNoAllocMaxTokens) return MOE_ERR_TOO_LARGE;
  if (args->num_tokens <= 0) return args->num_tokens == 0 ? MOE_OK : MOE_ERR_INVALID_ARGUMENT;
  uint64_t need = 0;
  int st = moe_fp8_ds_workspace_size(args->num_tokens, args->num_local_experts, &need);
  if (st != MOE_OK) return st;
  if (need > kNoAllocScratchBytes) return MOE_ERR_TOO_LARGE;
  void* ws = nullptr;
  st = scratch_address(&ws);
  if (st != MOE_OK) return st;
  // The error word must start at zero; the rest is rewritten by every call.
  if (cudaMemsetAsync(ws, 0, 16, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return MOE_ERR_CUDA;
  return run_layer_with_workspace(args, ws, kNoAllocScratchBytes, stream, false);
}
