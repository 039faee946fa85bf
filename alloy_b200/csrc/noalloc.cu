// alloy_ssd_combined_noalloc: the fused prefill for callers that cannot
// allocate device memory.
//
// Some callers of this library are not allowed to call cudaMalloc: a serving
// process that hands all device memory to its own pool at start-up and forbids
// allocation afterwards, or a host runtime that reaches the library only
// through raw pointers owned by another framework's allocator (a Go or Java
// service calling in through FFI has no CUDA allocator of its own).  The
// tensor-core prefill needs scratch for the conv + SiLU of the B/C columns;
// this entry point takes it from one fixed array compiled into the library
// instead of asking the caller for a workspace.
//
// The array is a file-scope __device__ variable: every device context that
// loads the library holds kNoAllocScratchBytes of it until the process exits.
// Its name is only a host-side handle, so its device address is looked up
// with cudaGetSymbolAddress, with the call's device current, the first time a
// call runs in a context, and kept per device together with that context's
// unique id.  A context that is destroyed and created again (cudaDeviceReset)
// gets a new id and loads the module anew, possibly at another address, so
// the next call looks the address up again instead of using a stale one.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace alloy {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;   // 8 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct ScratchSlot {
  unsigned long long ctx_id;   // unique id of the context the address belongs to
  void* addr;
};
std::mutex g_scratch_mu;
ScratchSlot g_scratch[kMaxDevices] = {};

// The current context's unique id in *id (cuCtxGetCurrent + cuCtxGetId,
// through the runtime's driver entry points; the library links no driver
// stub), or 0 when this thread has no current context yet.
int current_context_id(unsigned long long* id) {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  if (get_current == nullptr || get_id == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return fail(ALLOY_ERR_CUDA, "ssd_combined_noalloc: cuCtxGetCurrent unavailable");
    get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return fail(ALLOY_ERR_CUDA, "ssd_combined_noalloc: cuCtxGetId unavailable");
    get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  }
  *id = 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS)
    return fail(ALLOY_ERR_CUDA, "ssd_combined_noalloc: cuCtxGetCurrent failed");
  if (ctx == nullptr) return ALLOY_OK;
  if (get_id(ctx, id) != CUDA_SUCCESS) return fail(ALLOY_ERR_CUDA, "ssd_combined_noalloc: cuCtxGetId failed");
  return ALLOY_OK;
}

int scratch_of_current_device(void** out) {
  int dev = 0;
  ALLOY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(ALLOY_ERR_DEVICE, "device index %d out of range", dev);
  unsigned long long ctx = 0;
  ALLOY_TRY(current_context_id(&ctx));
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& s = g_scratch[dev];
  if (ctx == 0 || s.addr == nullptr || s.ctx_id != ctx) {
    // set-up for this device's context: the lookup makes the device's primary
    // context current if nothing has yet, and may load the module into it
    void* p = nullptr;
    ALLOY_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    if (ctx == 0) ALLOY_TRY(current_context_id(&ctx));
    if (ctx == 0) return fail(ALLOY_ERR_CUDA, "ssd_combined_noalloc: no current CUDA context");
    s.addr = p;
    s.ctx_id = ctx;
  }
  *out = s.addr;
  return ALLOY_OK;
}

}  // namespace
}  // namespace alloy

using namespace alloy;

extern "C" int alloy_ssd_combined_noalloc(
    const alloy_tensor_t* xBC, const alloy_tensor_t* dt_raw, const alloy_tensor_t* conv_w,
    const alloy_tensor_t* conv_b, const alloy_tensor_t* dt_bias, const alloy_tensor_t* A_log,
    const alloy_tensor_t* D, const alloy_tensor_t* ssm_in, const alloy_tensor_t* conv_in,
    alloy_tensor_t* y, alloy_tensor_t* ssm_out, alloy_tensor_t* conv_out,
    const alloy_ssd_dims_t* dims, void* stream) {
  size_t need = 0;
  if (xBC != nullptr && xBC->ndim == 3 && dims != nullptr)
    need = ssd_combined_workspace(xBC->shape[0], xBC->shape[1], xBC->dtype, dims, false);
  if (need > kNoAllocScratchBytes) {
    last_error().clear();
    return fail(ALLOY_ERR_UNSUPPORTED,
                "ssd_combined_noalloc: this call needs %zu bytes of scratch but the fixed "
                "scratch holds %zu; use alloy_ssd_combined with a workspace",
                need, kNoAllocScratchBytes);
  }
  void* ws = nullptr;
  if (need > 0) {
    const int st = scratch_of_current_device(&ws);
    if (st != ALLOY_OK) return st;
  }
  // Every element of the scratch that the scan reads is written earlier in
  // the same call (by the B/C pre-pass, or by the state-only pass of a
  // segmented call), so nothing needs clearing between calls.
  return alloy_ssd_combined(xBC, dt_raw, conv_w, conv_b, dt_bias, A_log, D, ssm_in, conv_in, y,
                            ssm_out, conv_out, ws, need > 0 ? kNoAllocScratchBytes : 0, dims,
                            stream);
}
