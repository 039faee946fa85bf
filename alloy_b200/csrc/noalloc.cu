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
// Its name is only a host-side handle, so the device address is looked up
// here with cudaGetSymbolAddress, once per device, on the first call made with
// that device current (which may also load the library's device code).
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace alloy {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;   // 8 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {nullptr};

int scratch_of_current_device(void** out) {
  int dev = 0;
  ALLOY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(ALLOY_ERR_DEVICE, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    ALLOY_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
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
