// Shared helpers for liballoy_ssd: element conversion, host-side argument
// checking and the per-thread last-error message.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <atomic>
#include <string>

#include "alloy_ssd.h"

namespace alloy {

// ---------------------------------------------------------------------------
// last-error message (thread local, never shared between caller threads)
// ---------------------------------------------------------------------------
std::string& last_error();

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  last_error() = buf;
  return code;
}

inline int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ALLOY_OK;
  return fail(ALLOY_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define ALLOY_TRY(expr)                 \
  do {                                  \
    int _st = (expr);                   \
    if (_st != ALLOY_OK) return _st;    \
  } while (0)

#define ALLOY_CUDA(expr) ALLOY_TRY(::alloy::cuda_status((expr), #expr))

// kernels this library launched in this process (alloy_kernel_launch_count)
std::atomic<uint64_t>& launch_counter();

// Reports a failed launch (bad configuration, missing device code, ...) and
// counts the ones that went out.  Every kernel launch of the library is
// followed by this check.
inline int check_launch(const char* name) {
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(ALLOY_ERR_CUDA, "launch of %s failed: %s", name, cudaGetErrorString(e));
  }
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  return ALLOY_OK;
}

// ---------------------------------------------------------------------------
// host-side tensor checks
// ---------------------------------------------------------------------------
inline bool present(const alloy_tensor_t* t) { return t != nullptr && t->data != nullptr; }

inline const char* dtype_name(int d) {
  return d == ALLOY_F32 ? "f32" : d == ALLOY_BF16 ? "bf16" : "?";
}

inline int elem_size(int d) { return d == ALLOY_F32 ? 4 : d == ALLOY_BF16 ? 2 : 0; }

// Checks rank, shape (entries < 0 are free) and dtype (bitmask of 1<<dtype).
inline int check_tensor(const alloy_tensor_t* t, const char* name, int ndim,
                        const int64_t* shape, unsigned dtype_mask) {
  if (t == nullptr || t->data == nullptr)
    return fail(ALLOY_ERR_INVALID_ARG, "%s: null tensor", name);
  if (t->ndim != ndim)
    return fail(ALLOY_ERR_INVALID_ARG, "%s: expected %d dims, got %d", name, ndim, t->ndim);
  if (t->dtype < 0 || t->dtype > 1 || !((1u << t->dtype) & dtype_mask))
    return fail(ALLOY_ERR_INVALID_ARG, "%s: unsupported dtype %d", name, t->dtype);
  for (int i = 0; i < ndim; ++i) {
    if (t->shape[i] < 0)
      return fail(ALLOY_ERR_INVALID_ARG, "%s: negative extent in dim %d", name, i);
    if (shape && shape[i] >= 0 && t->shape[i] != shape[i])
      return fail(ALLOY_ERR_INVALID_ARG, "%s: dim %d is %lld, expected %lld", name, i,
                  (long long)t->shape[i], (long long)shape[i]);
  }
  return ALLOY_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr unsigned kF32 = 1u << ALLOY_F32;
constexpr unsigned kBF16 = 1u << ALLOY_BF16;
constexpr unsigned kAnyFloat = kF32 | kBF16;

// Per-device one-time flags (max dynamic shared memory opt-in and the like).
constexpr int kMaxDevices = 64;

int current_device_checked(int* dev);

// ---------------------------------------------------------------------------
// device-side element access
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Load an element of a runtime-typed tensor (dtype given by flag).
__device__ __forceinline__ float load_any(const void* p, int64_t i, int is_bf16) {
  return is_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i])
                 : static_cast<const float*>(p)[i];
}
__device__ __forceinline__ void store_any(void* p, int64_t i, int is_bf16, float v) {
  if (is_bf16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<float*>(p)[i] = v;
}

// softplus(x) = log(1 + exp(x)) computed stably as max(x,0) + log1p(exp(-|x|)).
__device__ __forceinline__ float softplus_f32(float x) {
  return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x)));
}

__device__ __forceinline__ float silu_f32(float x) { return x / (1.f + expf(-x)); }

}  // namespace alloy
