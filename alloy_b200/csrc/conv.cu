// Causal depthwise conv1d + SiLU (alloy/models/mamba_kernels.py:17-50,
// alloy/models/mamba_block.py:144-158 + :455).
//
// Tiled kernel: a CTA owns TT timesteps x (32 x 16-byte) channel vectors of
// one batch row.  It stages the TT + K - 1 input rows of its channel window
// in shared memory with 128-bit channel-contiguous loads (the K-1 row halo is
// shared by all outputs of the tile), then each thread produces 8 timesteps
// of one 16-byte channel vector with an fp32 sliding window.  HBM traffic is
// one read of the input and one write of the output; the halo re-read is
// (K-1)/TT of the input and hits L2.
#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace alloy {

namespace {

constexpr int kConvThreads = 256;
constexpr int kConvTT = 64;                     // timesteps per tile
constexpr int kConvRowsPerThread = kConvTT / (kConvThreads / 32);  // 8

template <typename T> struct Vec;
template <> struct Vec<float> { static constexpr int N = 4; };
template <> struct Vec<__nv_bfloat16> { static constexpr int N = 8; };

__device__ __forceinline__ uint4 ldg_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

template <typename T>
__device__ __forceinline__ void unpack(const uint4& u, float* f);
template <>
__device__ __forceinline__ void unpack<float>(const uint4& u, float* f) {
  f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
}
template <>
__device__ __forceinline__ void unpack<__nv_bfloat16>(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack(const float* f);
template <>
__device__ __forceinline__ uint4 pack<float>(const float* f) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}
template <>
__device__ __forceinline__ uint4 pack<__nv_bfloat16>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename T, int K, bool SILU>
__global__ void __launch_bounds__(kConvThreads)
conv1d_silu_tile_kernel(const T* __restrict__ xp, int64_t xp_sb, int64_t xp_st,
                        const void* __restrict__ w, int w_bf16, int64_t w_sc, int64_t w_sk,
                        const void* __restrict__ bias, int b_bf16, int64_t b_s,
                        T* __restrict__ out, int64_t o_sb, int64_t o_st, int L, int C) {
  constexpr int V = Vec<T>::N;
  constexpr int CW = 32 * V;
  __shared__ uint4 tile[(kConvTT + K - 1) * 32];

  const int b = blockIdx.z;
  const int t0 = blockIdx.y * kConvTT;
  const int c0 = blockIdx.x * CW;
  const int nt = min(kConvTT, L - t0);
  const int rows = nt + K - 1;
  const int nvec = min(CW, C - c0) / V;

  const T* src = xp + (int64_t)b * xp_sb + (int64_t)t0 * xp_st + c0;
  for (int i = threadIdx.x; i < rows * 32; i += kConvThreads) {
    const int r = i >> 5, v = i & 31;
    if (v < nvec) tile[i] = ldg_v4(src + (int64_t)r * xp_st + v * V);
  }
  __syncthreads();

  const int v = threadIdx.x & 31;
  const int r0 = (threadIdx.x >> 5) * kConvRowsPerThread;
  if (v >= nvec || r0 >= nt) return;

  const int c = c0 + v * V;
  float wr[V][K], br[V];
#pragma unroll
  for (int j = 0; j < V; ++j) {
#pragma unroll
    for (int k = 0; k < K; ++k) wr[j][k] = load_any(w, (int64_t)(c + j) * w_sc + k * w_sk, w_bf16);
    br[j] = bias ? load_any(bias, (int64_t)(c + j) * b_s, b_bf16) : 0.f;
  }

  float win[K][V];
#pragma unroll
  for (int k = 0; k < K - 1; ++k) unpack<T>(tile[(r0 + k) * 32 + v], win[k]);

  T* dst = out + (int64_t)b * o_sb + (int64_t)(t0 + r0) * o_st + c;
#pragma unroll
  for (int i = 0; i < kConvRowsPerThread; ++i) {
    if (r0 + i >= nt) break;
    unpack<T>(tile[(r0 + i + K - 1) * 32 + v], win[K - 1]);
    float o[V];
#pragma unroll
    for (int j = 0; j < V; ++j) {
      float acc = br[j];
#pragma unroll
      for (int k = 0; k < K; ++k) acc = fmaf(win[k][j], wr[j][k], acc);
      o[j] = SILU ? silu_f32(acc) : acc;
    }
    *reinterpret_cast<uint4*>(dst + (int64_t)i * o_st) = pack<T>(o);
#pragma unroll
    for (int k = 0; k < K - 1; ++k)
#pragma unroll
      for (int j = 0; j < V; ++j) win[k][j] = win[k + 1][j];
  }
}

// bf16 activations, K = 4 (the layer case): a CTA owns kBfTiles consecutive
// tiles of 64 output rows x 256 channels of one batch row.  The 67 input rows of
// a tile (the K-1-row halo shared by its outputs) arrive in shared memory by
// cp.async 16-byte copies into one of two buffers: the copies of tile i + 1 are
// in flight while tile i is computed, and two CTAs share an SM (at three a CTA
// the registers spill, which cost more than the third CTA gained).  Each thread
// convolves 8 channels over 8 rows in packed f32x2 FMAs with the taps and bias
// halved, which gives h = x / 2 and silu(x) = h + h tanh(h) from one hardware
// tanh (its error is below the bf16 rounding of the output).
constexpr int kBfRows = 64;                        // output rows per tile
constexpr int kBfTiles = 8;                        // tiles per CTA
constexpr int kBfCols = 256;                       // channels per CTA
constexpr int kBfBuf = (kBfRows + 3) * kBfCols * 2;
constexpr int kBfSmem = 2 * kBfBuf;

template <bool SILU>
__global__ void __launch_bounds__(256, 2)
conv1d_silu_bf16_kernel(const __nv_bfloat16* __restrict__ xp, int64_t xp_sb, int64_t xp_st,
                        const void* __restrict__ w, int w_bf16, int64_t w_sc, int64_t w_sk,
                        const void* __restrict__ bias, int b_bf16, int64_t b_s,
                        __nv_bfloat16* __restrict__ out, int64_t o_sb, int64_t o_st, int L, int C) {
  using namespace tc;
  extern __shared__ __align__(16) unsigned char tile_raw[];
  __shared__ float4 taps_s[kBfCols];
  __shared__ float bias_s[kBfCols];
  const uint32_t tiles = static_cast<uint32_t>(__cvta_generic_to_shared(tile_raw));
  const int b = blockIdx.z;
  const int c0 = blockIdx.y * kBfCols;
  const int Lp = L + 3;
  const int nvec = min(kBfCols, C - c0) / 8;        // 16-byte channel vectors of this CTA
  const int tile0 = blockIdx.x * kBfTiles;
  const int ntiles = min(kBfTiles, (L + kBfRows - 1) / kBfRows - tile0);
  const __nv_bfloat16* src = xp + (int64_t)b * xp_sb + c0;
  // input rows [t0, t0 + 67) x vectors [0, nvec) of tile i into buffer i & 1;
  // rows past the input are zero-filled (they only feed rows past L)
  auto load_tile = [&](int i) {
    const int t0 = (tile0 + i) * kBfRows;
    const uint32_t buf = tiles + (i & 1) * kBfBuf;
    for (int k = threadIdx.x; k < (kBfRows + 3) * 32; k += 256) {
      const int r = k >> 5, v = k & 31;
      const bool ok = v < nvec && t0 + r < Lp;
      const void* g = ok ? (const void*)(src + (int64_t)(t0 + r) * xp_st + v * 8) : (const void*)src;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(buf + k * 16), "l"(g), "r"(ok ? 16 : 0)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_tile(0);
  if (threadIdx.x < kBfCols) {
    const int ch = min(c0 + (int)threadIdx.x, C - 1);
    const float f = SILU ? 0.5f : 1.f;   // halved for the tanh form of silu
    taps_s[threadIdx.x] = make_float4(f * load_any(w, (int64_t)ch * w_sc, w_bf16),
                                      f * load_any(w, (int64_t)ch * w_sc + w_sk, w_bf16),
                                      f * load_any(w, (int64_t)ch * w_sc + 2 * w_sk, w_bf16),
                                      f * load_any(w, (int64_t)ch * w_sc + 3 * w_sk, w_bf16));
    bias_s[threadIdx.x] = bias ? f * load_any(bias, (int64_t)ch * b_s, b_bf16) : 0.f;
  }
  __syncthreads();
  const int cg = threadIdx.x & 31, strip = threadIdx.x >> 5;   // 8 channels x 8 rows
  uint64_t w2[4][4], b2[4];   // [tap][channel pair]
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int cc = min(cg, max(nvec - 1, 0)) * 8;
    const float4 ta = taps_s[cc + 2 * i], tb = taps_s[cc + 2 * i + 1];
    w2[0][i] = f2_pack(ta.x, tb.x);
    w2[1][i] = f2_pack(ta.y, tb.y);
    w2[2][i] = f2_pack(ta.z, tb.z);
    w2[3][i] = f2_pack(ta.w, tb.w);
    b2[i] = f2_pack(bias_s[cc + 2 * i], bias_s[cc + 2 * i + 1]);
  }
  const int r0 = strip * 8;
#pragma unroll 1
  for (int i = 0; i < ntiles; ++i) {
    // tile i + 1 in flight while tile i is computed (its buffer was last read
    // by tile i - 1, which every thread finished before the barrier below)
    if (i + 1 < ntiles) load_tile(i + 1);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();
    const int t0 = (tile0 + i) * kBfRows;
    if (cg < nvec) {
      const uint32_t col = tiles + (i & 1) * kBfBuf + cg * 16;
      uint64_t win[3][4];
#pragma unroll
      for (int r = 0; r < 3; ++r) {
        uint32_t u0, u1, u2, u3;
        asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(u0), "=r"(u1), "=r"(u2), "=r"(u3)
                     : "r"(col + (r0 + r) * 512));
        win[r][0] = f2_from_bf2(u0); win[r][1] = f2_from_bf2(u1);
        win[r][2] = f2_from_bf2(u2); win[r][3] = f2_from_bf2(u3);
      }
      __nv_bfloat16* dst = out + (int64_t)b * o_sb + (int64_t)(t0 + r0) * o_st + c0 + cg * 8;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        uint32_t u0, u1, u2, u3;
        asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(u0), "=r"(u1), "=r"(u2), "=r"(u3)
                     : "r"(col + (r0 + r + 3) * 512));
        const uint64_t x[4] = {f2_from_bf2(u0), f2_from_bf2(u1), f2_from_bf2(u2), f2_from_bf2(u3)};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint64_t acc = f2_fma(win[0][q], w2[0][q], b2[q]);
          acc = f2_fma(win[1][q], w2[1][q], acc);
          acc = f2_fma(win[2][q], w2[2][q], acc);
          acc = f2_fma(x[q], w2[3][q], acc);
          if (SILU) {
            float hl, hh;
            f2_unpack(acc, hl, hh);
            acc = f2_fma(acc, f2_pack(tanh_approx(hl), tanh_approx(hh)), acc);
          }
          o[q] = f2_to_bf2(acc);
          win[0][q] = win[1][q];
          win[1][q] = win[2][q];
          win[2][q] = x[q];
        }
        if (t0 + r0 + r < L)
          *reinterpret_cast<uint4*>(dst + (int64_t)r * o_st) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    __syncthreads();   // buffer i & 1 is free for tile i + 2
  }
}

// Any layout / alignment / K: one thread per output element.
__global__ void conv1d_silu_scalar_kernel(const void* __restrict__ xp, int x_bf16, int64_t xp_sb,
                                          int64_t xp_st, int64_t xp_sc,
                                          const void* __restrict__ w, int w_bf16, int64_t w_sc,
                                          int64_t w_sk, const void* __restrict__ bias, int b_bf16,
                                          int64_t b_s, void* __restrict__ out, int o_bf16,
                                          int64_t o_sb, int64_t o_st, int64_t o_sc, int B, int L,
                                          int C, int K, int silu) {
  const int64_t total = (int64_t)B * L * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const int t = (int)((i / C) % L);
    const int b = (int)(i / ((int64_t)C * L));
    float acc = bias ? load_any(bias, (int64_t)c * b_s, b_bf16) : 0.f;
    for (int k = 0; k < K; ++k)
      acc = fmaf(load_any(xp, b * xp_sb + (int64_t)(t + k) * xp_st + c * xp_sc, x_bf16),
                 load_any(w, (int64_t)c * w_sc + k * w_sk, w_bf16), acc);
    store_any(out, b * o_sb + (int64_t)t * o_st + c * o_sc, o_bf16, silu ? silu_f32(acc) : acc);
  }
}

template <typename T, bool SILU>
int launch_tile(const alloy_tensor_t* x, const alloy_tensor_t* w, const alloy_tensor_t* bias,
                alloy_tensor_t* out, int B, int L, int C, cudaStream_t s) {
  constexpr int V = Vec<T>::N;
  dim3 grid((C + 32 * V - 1) / (32 * V), (L + kConvTT - 1) / kConvTT, B);
  const void* bptr = present(bias) ? bias->data : nullptr;
  conv1d_silu_tile_kernel<T, 4, SILU><<<grid, kConvThreads, 0, s>>>(
      static_cast<const T*>(x->data), x->stride[0], x->stride[1], w->data,
      w->dtype == ALLOY_BF16, w->stride[0], w->stride[1], bptr,
      bptr ? bias->dtype == ALLOY_BF16 : 0, bptr ? bias->stride[0] : 0,
      static_cast<T*>(out->data), out->stride[0], out->stride[1], L, C);
  return check_launch("conv1d_silu_tile_kernel");
}

}  // namespace

int conv1d_silu(const alloy_tensor_t* x, const alloy_tensor_t* w, const alloy_tensor_t* bias,
                alloy_tensor_t* out, bool silu, cudaStream_t s) {
  const int B = (int)x->shape[0], Lp = (int)x->shape[1], C = (int)x->shape[2];
  const int K = (int)w->shape[1];
  const int L = Lp - K + 1;
  if (B == 0 || L == 0 || C == 0) return ALLOY_OK;
  const int es = elem_size(x->dtype);
  const int V = 16 / es;
  const bool vec_ok = K == 4 && x->stride[2] == 1 && out->stride[2] == 1 && C % V == 0 &&
                      aligned16(x->data) && aligned16(out->data) &&
                      (x->stride[0] * es) % 16 == 0 && (x->stride[1] * es) % 16 == 0 &&
                      (out->stride[0] * es) % 16 == 0 && (out->stride[1] * es) % 16 == 0;
  if (vec_ok && x->dtype == ALLOY_BF16) {
    dim3 grid(((L + kBfRows - 1) / kBfRows + kBfTiles - 1) / kBfTiles, (C + kBfCols - 1) / kBfCols, B);
    const void* bptr = present(bias) ? bias->data : nullptr;
    auto launch = [&](auto kernel) {
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBfSmem);
      kernel<<<grid, 256, kBfSmem, s>>>(
          static_cast<const __nv_bfloat16*>(x->data), x->stride[0], x->stride[1], w->data,
          w->dtype == ALLOY_BF16, w->stride[0], w->stride[1], bptr, bptr ? bias->dtype == ALLOY_BF16 : 0,
          bptr ? bias->stride[0] : 0, static_cast<__nv_bfloat16*>(out->data), out->stride[0],
          out->stride[1], L, C);
    };
    if (silu) launch(conv1d_silu_bf16_kernel<true>);
    else launch(conv1d_silu_bf16_kernel<false>);
    return check_launch("conv1d_silu_bf16_kernel");
  }
  if (vec_ok) {
    if (silu)
      return x->dtype == ALLOY_BF16 ? launch_tile<__nv_bfloat16, true>(x, w, bias, out, B, L, C, s)
                                    : launch_tile<float, true>(x, w, bias, out, B, L, C, s);
    return x->dtype == ALLOY_BF16 ? launch_tile<__nv_bfloat16, false>(x, w, bias, out, B, L, C, s)
                                  : launch_tile<float, false>(x, w, bias, out, B, L, C, s);
  }
  const int64_t total = (int64_t)B * L * C;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 32);
  const void* bptr = present(bias) ? bias->data : nullptr;
  conv1d_silu_scalar_kernel<<<blocks, 256, 0, s>>>(
      x->data, x->dtype == ALLOY_BF16, x->stride[0], x->stride[1], x->stride[2], w->data,
      w->dtype == ALLOY_BF16, w->stride[0], w->stride[1], bptr,
      bptr ? bias->dtype == ALLOY_BF16 : 0, bptr ? bias->stride[0] : 0, out->data,
      out->dtype == ALLOY_BF16, out->stride[0], out->stride[1], out->stride[2], B, L, C, K,
      silu ? 1 : 0);
  return check_launch("conv1d_silu_scalar_kernel");
}

}  // namespace alloy
