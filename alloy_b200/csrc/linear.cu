// Projections of a decode step: y[b, o] = sum_i W[o, i] x[b, i] for up to 4
// tokens, the in_proj / out_proj of MambaBlock (alloy/models/
// mamba_block.py:438, :501) when a cached step runs one token per sequence.
// At that size the product is a weight-streaming GEMV: every weight is read
// once and used for at most 4 multiply-adds, so the kernel is built to keep
// HBM busy.  The token rows (bf16) sit in shared memory; each warp takes
// output rows in turn and its lanes stream the row's 16-byte chunks with
// non-allocating loads, 8 chunks a lane in flight, multiply them in packed
// f32x2 FMAs against the token chunks and reduce across the warp.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace alloy {
namespace {

using tc::f2_fma;
using tc::f2_from_bf2;
using tc::f2_unpack;

constexpr int kLinWarps = 8;
constexpr int kLinUnroll = 8;

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

template <int NB>
__global__ void __launch_bounds__(kLinWarps * 32)
decode_linear_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_sb, const __nv_bfloat16* __restrict__ w,
                     int64_t w_so, __nv_bfloat16* __restrict__ y, int64_t y_sb, int in, int out) {
  extern __shared__ uint4 xs[];   // [NB][in / 8]
  const int nchunk = in / 8;
  for (int i = threadIdx.x; i < NB * nchunk; i += blockDim.x) {
    const int b = i / nchunk, c = i % nchunk;
    xs[i] = reinterpret_cast<const uint4*>(x + (int64_t)b * x_sb)[c];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int o = blockIdx.x * kLinWarps + warp; o < out; o += gridDim.x * kLinWarps) {
    const uint4* wrow = reinterpret_cast<const uint4*>(w + (int64_t)o * w_so);
    uint64_t acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0;
    for (int c0 = lane; c0 < nchunk; c0 += 32 * kLinUnroll) {
      uint4 wv[kLinUnroll];
#pragma unroll
      for (int u = 0; u < kLinUnroll; ++u) {
        const int c = c0 + 32 * u;
        wv[u] = c < nchunk ? ld_stream(wrow + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kLinUnroll; ++u) {
        const int c = c0 + 32 * u;
        if (c >= nchunk) break;
        const uint32_t ww[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const uint4 xv = xs[b * nchunk + c];
          const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[b] = f2_fma(f2_from_bf2(ww[q]), f2_from_bf2(xx[q]), acc[b]);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float lo, hi;
      f2_unpack(acc[b], lo, hi);
      float s = lo + hi;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (lane == 0) y[(int64_t)b * y_sb + o] = __float2bfloat16_rn(s);
    }
  }
}

}  // namespace

int decode_linear(const alloy_tensor_t* x, const alloy_tensor_t* w, alloy_tensor_t* y, cudaStream_t s) {
  const int NB = (int)x->shape[0], in = (int)x->shape[1], out = (int)w->shape[0];
  if (NB == 0 || out == 0) return ALLOY_OK;
  const size_t smem = (size_t)NB * in * 2;
  // one output row a warp up to 8 CTAs an SM of a 148-SM part, then several
  const int blocks = std::max(1, std::min((out + kLinWarps - 1) / kLinWarps, 148 * 8));
  auto launch = [&](auto kernel) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kernel<<<blocks, kLinWarps * 32, smem, s>>>(
        static_cast<const __nv_bfloat16*>(x->data), x->stride[0], static_cast<const __nv_bfloat16*>(w->data),
        w->stride[0], static_cast<__nv_bfloat16*>(y->data), y->stride[0], in, out);
  };
  switch (NB) {
    case 1: launch(decode_linear_kernel<1>); break;
    case 2: launch(decode_linear_kernel<2>); break;
    case 3: launch(decode_linear_kernel<3>); break;
    default: launch(decode_linear_kernel<4>); break;
  }
  return check_launch("decode_linear_kernel");
}

}  // namespace alloy
