// Gated RMS norm of the mixer output (alloy/models/mamba_block.py:495-499):
//   g   = y * silu(gate)                     (Zamba2RMSNormGated order: gate first)
//   out = g * rsqrt(mean over the group of g^2 + eps) * weight
// with the group the whole row (nn.RMSNorm(d_inner), :137) or `group_size`
// channels of it.  Math in fp32, out written in the activation dtype.
//
// HBM-bound: per row it reads y and gate once and writes out once.  The vector
// kernel keeps a row's g in registers between the reduction and the scaling;
// the scalar kernel (unaligned rows, channel counts the vector kernel does not
// cover) reads y and gate twice.
#include "common.cuh"
#include "kernels.h"

namespace alloy {
namespace {

constexpr int kNormThreads = 256;

// silu(x) = x / (1 + e^-x) with the hardware exponential and reciprocal (a few
// ulp; the accurate library forms would make this memory-bound kernel issue-bound)
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.f + __expf(-x)); }
// bf16 outputs: silu(x) = h + h tanh(h) with h = x/2, one hardware tanh
// (relative error ~2^-11, below the 2^-9 rounding of the bf16 result)
__device__ __forceinline__ float silu_tanh(float x) {
  float t;
  const float h = 0.5f * x;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
}
template <typename T>
__device__ __forceinline__ float silu_for(float x) {
  if constexpr (sizeof(T) == 2) return silu_tanh(x);
  else return silu_fast(x);
}
constexpr int kMaxVecPerThread = 8;   // the vector kernel holds up to 8 x 16 bytes of g a thread

template <typename T>
struct Vec;
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int n = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ static void store(__nv_bfloat16* p, const float (&v)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <>
struct Vec<float> {
  static constexpr int n = 4;
  __device__ static void load(const float* p, float (&v)[4]) {
    const float4 u = *reinterpret_cast<const float4*>(p);
    v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
  }
  __device__ static void store(float* p, const float (&v)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};

struct NormArgs {
  const void* y; int64_t y_s;
  const void* gate; int64_t g_s;
  void* out; int64_t o_s;
  const float* w; int64_t w_s;   // null: gate only
  int w_vec;                     // w contiguous and 16-byte aligned
  int D, group;                  // channels per row, per norm group
  float eps;
};

// One CTA per row.  Thread i holds vectors i, i + 256, ... of the row; all its
// loads are issued before the first use.
template <typename T, int VPT>
__global__ void __launch_bounds__(kNormThreads) gated_rmsnorm_vec_kernel(NormArgs a) {
  constexpr int V = Vec<T>::n;
  extern __shared__ float sh[];   // [D / V] partial sums, then [D / group] scales
  const int64_t row = blockIdx.x;
  const T* y = static_cast<const T*>(a.y) + row * a.y_s;
  const T* gt = static_cast<const T*>(a.gate) + row * a.g_s;
  T* out = static_cast<T*>(a.out) + row * a.o_s;
  const int nvec = a.D / V;
  // every load of the thread first (all in flight at once), then the math
  uint4 ry[VPT], rg[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = threadIdx.x + j * kNormThreads;
    if (v < nvec) {
      ry[j] = __ldg(reinterpret_cast<const uint4*>(y + (int64_t)v * V));
      rg[j] = __ldg(reinterpret_cast<const uint4*>(gt + (int64_t)v * V));
    }
  }
  float g[VPT][V];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = threadIdx.x + j * kNormThreads;
    if (v < nvec) {
      float yv[V], gv[V];
      Vec<T>::load(reinterpret_cast<const T*>(&ry[j]), yv);
      Vec<T>::load(reinterpret_cast<const T*>(&rg[j]), gv);
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        g[j][i] = yv[i] * silu_for<T>(gv[i]);
        ss = fmaf(g[j][i], g[j][i], ss);
      }
      if (a.w) sh[v] = ss;
    }
  }
  float* scale = sh + nvec;
  if (a.w) {
    __syncthreads();
    // one warp per group: sum its vectors' partial sums
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gvec = a.group / V, ngroups = a.D / a.group;
    for (int grp = warp; grp < ngroups; grp += kNormThreads / 32) {
      float s = 0.f;
      for (int i = lane; i < gvec; i += 32) s += sh[grp * gvec + i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) scale[grp] = rsqrtf(s / (float)a.group + a.eps);
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = threadIdx.x + j * kNormThreads;
    if (v < nvec) {
      if (a.w) {
        const float r = scale[(v * V) / a.group];
        if (a.w_vec) {   // contiguous, 16-byte aligned weights
#pragma unroll
          for (int i = 0; i < V; i += 4) {
            const float4 w4 = __ldg(reinterpret_cast<const float4*>(a.w + v * V + i));
            g[j][i] *= r * w4.x; g[j][i + 1] *= r * w4.y; g[j][i + 2] *= r * w4.z; g[j][i + 3] *= r * w4.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < V; ++i) g[j][i] *= r * a.w[(int64_t)(v * V + i) * a.w_s];
        }
      }
      Vec<T>::store(out + (int64_t)v * V, g[j]);
    }
  }
}

// Any D and alignment: per-group sums of squares by shared-memory atomics,
// then a second read of y and gate for the output.
template <typename T>
__global__ void __launch_bounds__(kNormThreads) gated_rmsnorm_scalar_kernel(NormArgs a) {
  extern __shared__ float gs[];   // [D / group] sums, then scales
  const int64_t row = blockIdx.x;
  const T* y = static_cast<const T*>(a.y) + row * a.y_s;
  const T* gt = static_cast<const T*>(a.gate) + row * a.g_s;
  T* out = static_cast<T*>(a.out) + row * a.o_s;
  const int ngroups = a.D / a.group;
  auto gated = [&](int c) { return to_f32(y[c]) * silu_for<T>(to_f32(gt[c])); };
  if (a.w) {
    for (int i = threadIdx.x; i < ngroups; i += kNormThreads) gs[i] = 0.f;
    __syncthreads();
    for (int c = threadIdx.x; c < a.D; c += kNormThreads) {
      const float v = gated(c);
      atomicAdd(&gs[c / a.group], v * v);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < ngroups; i += kNormThreads) gs[i] = rsqrtf(gs[i] / (float)a.group + a.eps);
    __syncthreads();
  }
  for (int c = threadIdx.x; c < a.D; c += kNormThreads) {
    float v = gated(c);
    if (a.w) v *= gs[c / a.group] * a.w[(int64_t)c * a.w_s];
    out[c] = from_f32<T>(v);
  }
}

template <typename T>
int launch_norm(const NormArgs& a, int64_t rows, bool vec_ok, cudaStream_t s) {
  constexpr int V = Vec<T>::n;
  const int nvec = a.D / V;
  const int vpt = (nvec + kNormThreads - 1) / kNormThreads;
  if (vec_ok && vpt <= kMaxVecPerThread) {
    const size_t smem = (size_t)(nvec + a.D / a.group) * sizeof(float);
    if (smem > 48 * 1024) return fail(ALLOY_ERR_UNSUPPORTED, "gated_rmsnorm: %d channels too many", a.D);
#define ALLOY_NORM_VEC(VP)                                                                       \
    case VP:                                                                                     \
      gated_rmsnorm_vec_kernel<T, VP><<<(unsigned)rows, kNormThreads, smem, s>>>(a);             \
      break;
    switch (vpt) {
      ALLOY_NORM_VEC(1) ALLOY_NORM_VEC(2) ALLOY_NORM_VEC(3) ALLOY_NORM_VEC(4)
      ALLOY_NORM_VEC(5) ALLOY_NORM_VEC(6) ALLOY_NORM_VEC(7) ALLOY_NORM_VEC(8)
      default: break;
    }
#undef ALLOY_NORM_VEC
    return check_launch("gated_rmsnorm_vec_kernel");
  }
  const size_t smem = (size_t)(a.D / a.group) * sizeof(float);
  if (smem > 48 * 1024) return fail(ALLOY_ERR_UNSUPPORTED, "gated_rmsnorm: %d norm groups too many", a.D / a.group);
  gated_rmsnorm_scalar_kernel<T><<<(unsigned)rows, kNormThreads, smem, s>>>(a);
  return check_launch("gated_rmsnorm_scalar_kernel");
}

}  // namespace

int gated_rmsnorm(const alloy_tensor_t* y, const alloy_tensor_t* gate, const alloy_tensor_t* w,
                  alloy_tensor_t* out, float eps, int group, cudaStream_t s) {
  NormArgs a;
  a.y = y->data; a.y_s = y->stride[0];
  a.gate = gate->data; a.g_s = gate->stride[0];
  a.out = out->data; a.o_s = out->stride[0];
  a.w = w ? static_cast<const float*>(w->data) : nullptr;
  a.w_s = w ? w->stride[0] : 0;
  a.w_vec = a.w && a.w_s == 1 && (reinterpret_cast<uintptr_t>(a.w) & 15) == 0;
  a.D = (int)y->shape[1];
  a.group = group;
  a.eps = eps;
  const int64_t rows = y->shape[0];
  if (rows == 0 || a.D == 0) return ALLOY_OK;
  const int esz = elem_size(y->dtype), V = 16 / esz;
  auto aligned = [&](const void* p, int64_t row_stride) {
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && row_stride % V == 0;
  };
  const bool vec_ok = a.D % V == 0 && a.group % V == 0 && aligned(a.y, a.y_s) && aligned(a.gate, a.g_s) &&
                      aligned(a.out, a.o_s);
  if (y->dtype == ALLOY_BF16) return launch_norm<__nv_bfloat16>(a, rows, vec_ok, s);
  return launch_norm<float>(a, rows, vec_ok, s);
}

}  // namespace alloy
