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
struct ScratchSlot {
  void* ctx = nullptr;    // CUcontext the address below belongs to
  void* ptr = nullptr;    // device address of g_noalloc_scratch in that context
};
ScratchSlot g_noalloc_slot[kNoAllocMaxDevices];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn g_ctx_get_current = nullptr;

// Set-up, once per device and context: the device address of the scratch
// array on the current device (the array's host-side name is not a device
// address), and a zeroed error block.  A context re-created after
// cudaDeviceReset reloads this library's module, so the address is looked up
// again for the new context.
int scratch_address(cudaStream_t stream, void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices)
    return MOE_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_ctx_get_current) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return MOE_ERR_NO_DEVICE;
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  CUcontext ctx = nullptr;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) return MOE_ERR_NO_DEVICE;
  ScratchSlot& slot = g_noalloc_slot[dev];
  if (!ctx || slot.ctx != static_cast<void*>(ctx) || !slot.ptr) {
    void* p = nullptr;
    // Also makes the device's primary context current if none was.
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return MOE_ERR_CUDA;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || !ctx) return MOE_ERR_NO_DEVICE;
    if (cudaMemsetAsync(p, 0, 16, stream) != cudaSuccess) return MOE_ERR_CUDA;
    slot.ctx = ctx;
    slot.ptr = p;
  }
  *out = slot.ptr;
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* ws = nullptr;
  st = scratch_address(s, &ws);
  if (st != MOE_OK) return st;
  // Words 1..3 of the error block (grid-barrier state) must start at zero;
  // word 0, the device error code, stays set until it is read.
  if (cudaMemsetAsync(static_cast<int*>(ws) + 1, 0, 12, s) != cudaSuccess) return MOE_ERR_CUDA;
  return run_layer_with_workspace(args, ws, kNoAllocScratchBytes, stream, false);
}

extern "C" int moe_fp8_ds_noalloc_read_device_error(void* stream, int32_t* device_error) {
  if (!device_error) return MOE_ERR_INVALID_ARGUMENT;
  void* ws = nullptr;
  const int st = scratch_address(static_cast<cudaStream_t>(stream), &ws);
  if (st != MOE_OK) return st;
  return moe_fp8_ds_read_device_error(ws, stream, device_error);
}
