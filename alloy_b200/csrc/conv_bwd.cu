// Backward of the causal depthwise conv1d + SiLU: the VJP that alloy attaches
// to its Metal conv kernel (_metal_conv1d_silu_vjp, alloy/models/mamba_block.py:25-47).
//
//   pre[t]    = bias + sum_k x_padded[t+k] w_k               (t in [0, L))
//   g[t]      = dy[t] * sig (1 + pre (1 - sig)),  sig = sigmoid(pre)
//   dx[t']    = sum_k g[t'-k] w_k                             (t' in [0, L+K-1), g = 0 outside [0, L))
//   dw_k      = sum_{b,t} g[t] x_padded[t+k],   dbias = sum_{b,t} g[t]
//
// Kernel 1 (one pass over x_padded and dy, one write of dx): a warp owns 4
// channels per lane (128 consecutive channels, coalesced 8- or 16-byte row
// loads) and walks kRowsPerWarp rows of dx in time order.  It carries the
// last K-1 rows of x and of g in registers, so every row of x and dy is
// loaded once (plus a K-1 row halo at the start of the warp's rows, whose g
// is recomputed).  The rows arrive through a per-warp ring in shared memory
// filled with cp.async kRing - 1 rows ahead of their use: each lane copies
// and later reads only its own 4 channels, so the ring needs no barrier, and
// a warp keeps ~15 rows of x and dy in flight.  The warp also sums g x_{t+k} and g over its rows; the 8
// warps of a CTA (consecutive row ranges of the same channels) are summed in
// shared memory in a fixed order into one partial per CTA in the workspace.
// Kernel 2 sums the partials of every CTA of a channel in a fixed order, so
// dweight and dbias do not depend on scheduling.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace alloy {

namespace {

using tc::ex2_approx;
using tc::tanh_approx;
using tc::f2_fma;
using tc::f2_from_bf2;
using tc::f2_mul;
using tc::f2_pack;
using tc::f2_splat;
using tc::f2_to_bf2;
using tc::f2_unpack;

constexpr int kBwdWarps = 8;
constexpr int kBwdThreads = kBwdWarps * 32;
constexpr int kRowsPerWarp = 64;
constexpr int kRowsPerCta = kBwdWarps * kRowsPerWarp;
constexpr int kChanPerLane = 4;
constexpr int kChanPerCta = 32 * kChanPerLane;
// ring slots per warp: kRing - 1 rows in flight (bf16: 8 KB a warp; fp32: 16 KB)
template <typename T> struct Ring { static constexpr int N = 16; };
template <> struct Ring<float> { static constexpr int N = 16; };

// asynchronous global -> shared copy of n (8 or 16) bytes, zero-filled when
// `valid` is false (no global bytes are read then)
template <int NB>
__device__ __forceinline__ void cp_async(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(dst), "l"(src), "n"(NB),
               "r"(valid ? NB : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
template <typename T>
__device__ __forceinline__ void lds4(uint32_t addr, float (&f)[4]);
template <>
__device__ __forceinline__ void lds4<float>(uint32_t addr, float (&f)[4]) {
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(f[0]), "=f"(f[1]), "=f"(f[2]), "=f"(f[3])
               : "r"(addr) : "memory");
}

// 4 consecutive channels of one row: one 8-byte (bf16) or 16-byte (fp32) load
template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&f)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&f)[4]) {
  const float4 v = __ldg(reinterpret_cast<const float4*>(p));
  f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&f)[4]) {
  const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
  f[0] = __uint_as_float(v.x << 16); f[1] = __uint_as_float(v.x & 0xffff0000u);
  f[2] = __uint_as_float(v.y << 16); f[3] = __uint_as_float(v.y & 0xffff0000u);
}

// a lane's 4 channels of a ring slot as two f32 pairs
template <typename T>
__device__ __forceinline__ void lds_pairs(uint32_t addr, uint64_t (&p)[2]);
template <>
__device__ __forceinline__ void lds_pairs<float>(uint32_t addr, uint64_t (&p)[2]) {
  float f[4];
  lds4<float>(addr, f);
  p[0] = f2_pack(f[0], f[1]);
  p[1] = f2_pack(f[2], f[3]);
}
template <>
__device__ __forceinline__ void lds_pairs<__nv_bfloat16>(uint32_t addr, uint64_t (&p)[2]) {
  uint32_t a, b;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr) : "memory");
  p[0] = f2_from_bf2(a);
  p[1] = f2_from_bf2(b);
}
template <typename T>
__device__ __forceinline__ void store_pairs(T* p, const uint64_t (&o)[2]);
template <>
__device__ __forceinline__ void store_pairs<float>(float* p, const uint64_t (&o)[2]) {
  float f[4];
  f2_unpack(o[0], f[0], f[1]);
  f2_unpack(o[1], f[2], f[3]);
  *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
}
template <>
__device__ __forceinline__ void store_pairs<__nv_bfloat16>(__nv_bfloat16* p, const uint64_t (&o)[2]) {
  *reinterpret_cast<uint2*>(p) = make_uint2(f2_to_bf2(o[0]), f2_to_bf2(o[1]));
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

// sigmoid of an f32 pair.  fp32: 1 / (1 + 2^(-x log2 e)) from the hardware
// exponential and reciprocal (a few ulp; 0 once the power overflows).  bf16
// activations: 0.5 + 0.5 tanh(x / 2) from the hardware tanh (absolute error
// ~1e-4, below the bf16 rounding of the results it feeds).
template <typename T>
__device__ __forceinline__ uint64_t sigmoid2(uint64_t x) {
  const uint64_t one = f2_splat(1.f);
  float e0, e1;
  f2_unpack(f2_mul(x, f2_splat(-kLog2e)), e0, e1);
  float u0, u1;
  f2_unpack(f2_fma(f2_pack(ex2_approx(e0), ex2_approx(e1)), one, one), u0, u1);
  return f2_pack(rcp_approx(u0), rcp_approx(u1));
}
template <>
__device__ __forceinline__ uint64_t sigmoid2<__nv_bfloat16>(uint64_t x) {
  const uint64_t half = f2_splat(0.5f);
  float h0, h1;
  f2_unpack(f2_mul(x, half), h0, h1);
  return f2_fma(f2_pack(tanh_approx(h0), tanh_approx(h1)), half, half);
}

// sigmoid from the hardware exponential and reciprocal (relative error of a
// few ulp; 0 for x below about -87, where the exponential overflows)
__device__ __forceinline__ float sigmoid_f32(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// Vector path: channel stride 1, 4 | C, rows aligned for 4-channel loads.
template <typename T, int K>
__global__ void __launch_bounds__(kBwdThreads, K <= 5 ? 2 : 1)
conv1d_silu_bwd_kernel(const T* __restrict__ xp, int64_t x_sb, int64_t x_st,
                       const T* __restrict__ dy, int64_t dy_sb, int64_t dy_st,
                       T* __restrict__ dx, int64_t dx_sb, int64_t dx_st,
                       const void* __restrict__ w, int w_bf16, int64_t w_sc, int64_t w_sk,
                       const void* __restrict__ bias, int b_bf16, int64_t b_s,
                       float* __restrict__ partial, int L, int C) {
  constexpr int VB = 4 * sizeof(T);    // bytes of a lane's 4 channels
  constexpr int D = Ring<T>::N;
  __shared__ float red[kBwdWarps][K + 1][kChanPerCta];
  extern __shared__ __align__(16) unsigned char ring_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // slot s of this warp: x row at +0, dy row at +32 VB (lane-major inside)
  const uint32_t ring = static_cast<uint32_t>(__cvta_generic_to_shared(ring_raw)) +
                        warp * D * 64 * VB + lane * VB;
  const int b = blockIdx.z;
  const int c = blockIdx.x * kChanPerCta + lane * kChanPerLane;
  const int Lp = L + K - 1;
  const int r0 = blockIdx.y * kRowsPerCta + warp * kRowsPerWarp;
  const int r1 = min(r0 + kRowsPerWarp, Lp);
  const bool active = c < C;

  // channel pairs (j = 0: channels c, c+1; j = 1: c+2, c+3) in packed f32x2
  // registers: every product and sum below is one IEEE fp32 operation per
  // channel, two channels per instruction
  uint64_t dw[K][2], db[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    db[j] = 0;
#pragma unroll
    for (int k = 0; k < K; ++k) dw[k][j] = 0;
  }
  if (active && r0 < r1) {
    const uint64_t one = f2_splat(1.f), neg_log2e = f2_splat(-kLog2e);
    uint64_t wr[K][2], br[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int k = 0; k < K; ++k)
        wr[k][j] = f2_pack(load_any(w, (int64_t)(c + 2 * j) * w_sc + k * w_sk, w_bf16),
                           load_any(w, (int64_t)(c + 2 * j + 1) * w_sc + k * w_sk, w_bf16));
      br[j] = bias ? f2_pack(load_any(bias, (int64_t)(c + 2 * j) * b_s, b_bf16),
                             load_any(bias, (int64_t)(c + 2 * j + 1) * b_s, b_bf16))
                   : 0;
    }
    const T* xrow = xp + (int64_t)b * x_sb + c;
    const T* dyrow = dy + (int64_t)b * dy_sb + c;
    T* dxrow = dx + (int64_t)b * dx_sb + c;
    // xw[i] = x_padded[t + i] (i < K - 1), gw[i] = g[t - 1 - i], zero outside the rows
    uint64_t xw[K - 1 > 0 ? K - 1 : 1][2], gw[K - 1 > 0 ? K - 1 : 1][2];
    const int t_begin = r0 - (K - 1);
#pragma unroll
    for (int i = 0; i < K - 1; ++i) {
      const int tt = t_begin + i;
      gw[i][0] = gw[i][1] = 0;
      xw[i][0] = xw[i][1] = 0;
      if (tt >= 0 && tt < Lp) {
        float f[4];
        load4<T>(xrow + (int64_t)tt * x_st, f);
        xw[i][0] = f2_pack(f[0], f[1]);
        xw[i][1] = f2_pack(f[2], f[3]);
      }
    }
    // iteration i handles row t = t_begin + i: x row t + K - 1 and dy row t,
    // copied into slot i % D (zeros outside the rows)
    const int n_iter = r1 - t_begin;
    // issue() is called for iterations 0, 1, 2, ... in order: the source rows
    // advance by one stride per call
    int it = 0;
    const T* xs = xrow + (int64_t)(t_begin + K - 1) * x_st;
    const T* ds = dyrow + (int64_t)t_begin * dy_st;
    auto issue = [&]() {
      if (it < n_iter) {
        const int t = t_begin + it, tn = t + K - 1;
        const uint32_t slot = ring + (it % D) * 64 * VB;
        const bool xv = tn >= 0 && tn < Lp, dv = t >= 0 && t < L;
        cp_async<VB>(slot, xv ? (const void*)xs : (const void*)xrow, xv);
        cp_async<VB>(slot + 32 * VB, dv ? (const void*)ds : (const void*)dyrow, dv);
      }
      cp_async_commit();
      ++it;
      xs += x_st;
      ds += dy_st;
    };
#pragma unroll 1
    for (int i = 0; i < D - 1; ++i) issue();
    // rows in blocks of kU: one wait for the block's copies, the g of its rows
    // computed side by side (independent chains), then their dx in order
    constexpr int kU = 4;
    static_assert(D % kU == 0 && D > kU, "ring slots");
#pragma unroll 1
    for (int i0 = 0; i0 < n_iter; i0 += kU) {
      // groups i0 .. i0 + kU - 1 have landed: D - 1 + i0 committed, at most
      // D - 1 - kU of them pending
      cp_async_wait<D - 1 - kU>();
      uint64_t xn[kU][2], g[kU][2], dv[kU][2];
#pragma unroll
      for (int u = 0; u < kU; ++u) {   // every load of the block before any use
        const uint32_t slot = ring + ((i0 + u) % D) * 64 * VB;
        lds_pairs<T>(slot, xn[u]);
        lds_pairs<T>(slot + 32 * VB, dv[u]);
      }
      // g of the block's rows and their dweight / dbias terms; rows outside
      // [0, L) have g = 0, halo rows (before r0) only feed dx
      auto rows = [&](auto interior) {
        constexpr bool kIn = decltype(interior)::value;
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int t = t_begin + i0 + u;
          g[u][0] = g[u][1] = 0;
          if (kIn || (i0 + u < n_iter && t >= 0 && t < L)) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              // pre[t] = bias + sum_k x[t + k] w_k: the window of row t is
              // xw[u ..] (rows before this block) then xn[.. u] (this block)
              uint64_t pre = br[j];
#pragma unroll
              for (int k = 0; k < K; ++k) {
                const int m = u + k;   // x row t + k = window position m
                const uint64_t xv = m < K - 1 ? xw[m < K - 1 ? m : 0][j] : xn[m - (K - 1) < kU ? m - (K - 1) : 0][j];
                pre = f2_fma(xv, wr[k][j], pre);
              }
              const uint64_t sg = sigmoid2<T>(pre);
              // g = dy sig (1 + pre (1 - sig))
              const uint64_t oms = f2_fma(sg, f2_splat(-1.f), one);
              g[u][j] = f2_mul(dv[u][j], f2_mul(sg, f2_fma(pre, oms, one)));
              if (kIn || t >= r0) {
                db[j] = f2_fma(g[u][j], one, db[j]);
#pragma unroll
                for (int k = 0; k < K; ++k) {
                  const int m = u + k;
                  const uint64_t xv = m < K - 1 ? xw[m < K - 1 ? m : 0][j] : xn[m - (K - 1) < kU ? m - (K - 1) : 0][j];
                  dw[k][j] = f2_fma(g[u][j], xv, dw[k][j]);
                }
              }
            }
          }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          // dx[t] = sum_k g[t - k] w_k: g of this block, then gw (rows before it)
          const int t = t_begin + i0 + u;
          if (kIn || (i0 + u < n_iter && t >= r0)) {
            uint64_t o[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              uint64_t acc = f2_mul(g[u][j], wr[0][j]);
#pragma unroll
              for (int k = 1; k < K; ++k) {
                const int m = u - k;   // >= 0: this block's row; < 0: gw[-m - 1]
                const uint64_t gv = m >= 0 ? g[m >= 0 ? m : 0][j] : gw[(-m - 1) < K - 1 ? -m - 1 : 0][j];
                acc = f2_fma(gv, wr[k][j], acc);
              }
              o[j] = acc;
            }
            store_pairs<T>(dxrow + (int64_t)t * dx_st, o);
          }
        }
      };
      // interior blocks (the common case): every row in [max(r0, 0), min(r1, L))
      const int tb = t_begin + i0;
      if (tb >= r0 && tb >= 0 && tb + kU <= r1 && tb + kU <= L)
        rows(std::true_type{});
      else
        rows(std::false_type{});
      // windows for the next block: the last K - 1 rows of x / g seen so far
#pragma unroll
      for (int m = 0; m < K - 1; ++m) {
        // new xw[m] = x row (t_begin + i0 + kU) + m = old position m + kU
        const int q = m + kU;
#pragma unroll
        for (int j = 0; j < 2; ++j)
          xw[m][j] = q < K - 1 ? xw[q < K - 1 ? q : 0][j] : xn[q - (K - 1) < kU ? q - (K - 1) : 0][j];
      }
#pragma unroll
      for (int m = K - 2; m >= 0; --m) {
        // new gw[m] = g of row (t_begin + i0 + kU - 1) - m; descending m, so an
        // old gw[m - kU] is read before it is replaced
        const int q = kU - 1 - m;
#pragma unroll
        for (int j = 0; j < 2; ++j) gw[m][j] = q >= 0 ? g[q >= 0 ? q : 0][j] : gw[(-q - 1) < K - 1 ? -q - 1 : 0][j];
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) issue();   // rows i0 + D - 1 .. i0 + D + kU - 2
    }
    cp_async_wait<0>();
  }
  // the CTA's partial sums: warps in a fixed order
#pragma unroll
  for (int j = 0; j < 2; ++j) {
#pragma unroll
    for (int k = 0; k < K; ++k) f2_unpack(dw[k][j], red[warp][k][lane * 4 + 2 * j], red[warp][k][lane * 4 + 2 * j + 1]);
    f2_unpack(db[j], red[warp][K][lane * 4 + 2 * j], red[warp][K][lane * 4 + 2 * j + 1]);
  }
  __syncthreads();
  const int nslot = gridDim.y * gridDim.z;
  const int slot = blockIdx.z * gridDim.y + blockIdx.y;
  for (int i = threadIdx.x; i < (K + 1) * kChanPerCta; i += kBwdThreads) {
    const int k = i / kChanPerCta, cc = i % kChanPerCta;
    const int ch = blockIdx.x * kChanPerCta + cc;
    if (ch >= C) continue;
    float s = 0.f;
#pragma unroll
    for (int wq = 0; wq < kBwdWarps; ++wq) s += red[wq][k][cc];
    // partial[k][slot][c]: the reduction kernel reads consecutive channels
    partial[((int64_t)k * nslot + slot) * C + ch] = s;
  }
}

// Any strides, any C: one thread per (batch row, channel), walking all rows.
template <int K>
__global__ void conv1d_silu_bwd_scalar_kernel(const void* __restrict__ xp, int x_bf16, int64_t x_sb,
                                              int64_t x_st, int64_t x_sc, const void* __restrict__ dy,
                                              int64_t dy_sb, int64_t dy_st, int64_t dy_sc,
                                              void* __restrict__ dx, int64_t dx_sb, int64_t dx_st,
                                              int64_t dx_sc, const void* __restrict__ w, int w_bf16,
                                              int64_t w_sc, int64_t w_sk, const void* __restrict__ bias,
                                              int b_bf16, int64_t b_s, float* __restrict__ partial,
                                              int B, int L, int C) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * C) return;
  const int b = (int)(i / C), c = (int)(i % C);
  const int Lp = L + K - 1;
  float wr[K];
#pragma unroll
  for (int k = 0; k < K; ++k) wr[k] = load_any(w, (int64_t)c * w_sc + k * w_sk, w_bf16);
  const float br = bias ? load_any(bias, (int64_t)c * b_s, b_bf16) : 0.f;
  auto X = [&](int t) {
    return t >= 0 && t < Lp ? load_any(xp, b * x_sb + (int64_t)t * x_st + c * x_sc, x_bf16) : 0.f;
  };
  auto G = [&](int t) {
    if (t < 0 || t >= L) return 0.f;
    float pre = br;
    for (int k = 0; k < K; ++k) pre = fmaf(X(t + k), wr[k], pre);
    const float s = sigmoid_f32(pre);
    return load_any(dy, b * dy_sb + (int64_t)t * dy_st + c * dy_sc, x_bf16) * (s * fmaf(pre, 1.f - s, 1.f));
  };
  float dw[K], db = 0.f;
#pragma unroll
  for (int k = 0; k < K; ++k) dw[k] = 0.f;
  for (int t = 0; t < Lp; ++t) {
    float acc = 0.f;
    for (int k = 0; k < K; ++k) acc = k == 0 ? G(t) * wr[0] : fmaf(G(t - k), wr[k], acc);
    store_any(dx, b * dx_sb + (int64_t)t * dx_st + c * dx_sc, x_bf16, acc);
    if (t < L) {
      const float g = G(t);
      db += g;
      for (int k = 0; k < K; ++k) dw[k] = fmaf(g, X(t + k), dw[k]);
    }
  }
  for (int k = 0; k < K; ++k) partial[((int64_t)k * B + b) * C + c] = dw[k];
  partial[((int64_t)K * B + b) * C + c] = db;
}

// dweight[c, k] = sum over slots of partial[k][slot][c]; dbias from row K
__global__ void conv1d_silu_bwd_reduce_kernel(const float* __restrict__ partial, int nslot, int C, int K,
                                              void* __restrict__ dw, int dw_bf16, int64_t dw_sc,
                                              int64_t dw_sk, void* __restrict__ db, int db_bf16,
                                              int64_t db_s) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)(K + 1) * C) return;
  const int k = (int)(i / C), c = (int)(i % C);
  float s = 0.f;
  for (int p = 0; p < nslot; ++p) s += partial[((int64_t)k * nslot + p) * C + c];
  if (k < K) store_any(dw, (int64_t)c * dw_sc + (int64_t)k * dw_sk, dw_bf16, s);
  else if (db) store_any(db, (int64_t)c * db_s, db_bf16, s);
}

struct BwdPlan {
  bool vec;
  int nslot;
};

BwdPlan plan(const alloy_tensor_t* x, const alloy_tensor_t* dy, const alloy_tensor_t* dx, int B, int L,
             int C, int K) {
  const int es = elem_size(x->dtype);
  const int64_t al = 4 * es;   // bytes of one 4-channel load
  auto rows_ok = [&](const alloy_tensor_t* t) {
    return t->stride[2] == 1 && (reinterpret_cast<uintptr_t>(t->data) % al) == 0 &&
           (t->stride[0] * es) % al == 0 && (t->stride[1] * es) % al == 0;
  };
  BwdPlan p;
  p.vec = C % 4 == 0 && rows_ok(x) && rows_ok(dy) && rows_ok(dx);
  p.nslot = p.vec ? B * ((L + K - 1 + kRowsPerCta - 1) / kRowsPerCta) : B;
  return p;
}

template <typename T, int K>
void launch_vec(const alloy_tensor_t* x, const alloy_tensor_t* w, const alloy_tensor_t* bias,
                const alloy_tensor_t* dy, alloy_tensor_t* dx, float* partial, int B, int L, int C,
                cudaStream_t s) {
  const void* bptr = present(bias) ? bias->data : nullptr;
  dim3 grid((C + kChanPerCta - 1) / kChanPerCta, (L + K - 1 + kRowsPerCta - 1) / kRowsPerCta, B);
  const int ring_bytes = kBwdWarps * Ring<T>::N * 64 * 4 * (int)sizeof(T);
  cudaFuncSetAttribute(conv1d_silu_bwd_kernel<T, K>, cudaFuncAttributeMaxDynamicSharedMemorySize, ring_bytes);
  conv1d_silu_bwd_kernel<T, K><<<grid, kBwdThreads, ring_bytes, s>>>(
      static_cast<const T*>(x->data), x->stride[0], x->stride[1], static_cast<const T*>(dy->data),
      dy->stride[0], dy->stride[1], static_cast<T*>(dx->data), dx->stride[0], dx->stride[1], w->data,
      w->dtype == ALLOY_BF16, w->stride[0], w->stride[1], bptr, bptr ? bias->dtype == ALLOY_BF16 : 0,
      bptr ? bias->stride[0] : 0, partial, L, C);
}

template <int K>
void launch_scalar(const alloy_tensor_t* x, const alloy_tensor_t* w, const alloy_tensor_t* bias,
                   const alloy_tensor_t* dy, alloy_tensor_t* dx, float* partial, int B, int L, int C,
                   cudaStream_t s) {
  const void* bptr = present(bias) ? bias->data : nullptr;
  const int64_t n = (int64_t)B * C;
  conv1d_silu_bwd_scalar_kernel<K><<<(unsigned)((n + 127) / 128), 128, 0, s>>>(
      x->data, x->dtype == ALLOY_BF16, x->stride[0], x->stride[1], x->stride[2], dy->data, dy->stride[0],
      dy->stride[1], dy->stride[2], dx->data, dx->stride[0], dx->stride[1], dx->stride[2], w->data,
      w->dtype == ALLOY_BF16, w->stride[0], w->stride[1], bptr, bptr ? bias->dtype == ALLOY_BF16 : 0,
      bptr ? bias->stride[0] : 0, partial, B, L, C);
}

template <int K>
void launch_k(bool vec, bool bf16, const alloy_tensor_t* x, const alloy_tensor_t* w,
              const alloy_tensor_t* bias, const alloy_tensor_t* dy, alloy_tensor_t* dx, float* partial,
              int B, int L, int C, cudaStream_t s) {
  if (!vec) launch_scalar<K>(x, w, bias, dy, dx, partial, B, L, C, s);
  else if (bf16) launch_vec<__nv_bfloat16, K>(x, w, bias, dy, dx, partial, B, L, C, s);
  else launch_vec<float, K>(x, w, bias, dy, dx, partial, B, L, C, s);
}

}  // namespace

// sized for the vector path's partials (B per 512 rows of dx), which is at
// least the B partials of the strided path
size_t conv1d_silu_backward_workspace(int64_t B, int64_t Lp, int64_t C, int64_t K) {
  const int64_t slices = std::max<int64_t>(1, (Lp + kRowsPerCta - 1) / kRowsPerCta);
  return (size_t)((K + 1) * B * slices * C) * sizeof(float);
}

int conv1d_silu_backward(const alloy_tensor_t* x, const alloy_tensor_t* w, const alloy_tensor_t* bias,
                         const alloy_tensor_t* dy, alloy_tensor_t* dx, alloy_tensor_t* dw,
                         alloy_tensor_t* db, void* workspace, int B, int L, int C, int K,
                         cudaStream_t s) {
  const BwdPlan p = plan(x, dy, dx, B, L, C, K);
  float* partial = static_cast<float*>(workspace);
  const bool bf16 = x->dtype == ALLOY_BF16;
  const bool any_rows = B > 0 && C > 0 && L + K - 1 > 0;
  if (any_rows) {
    switch (K) {
      case 1: launch_k<1>(p.vec, bf16, x, w, bias, dy, dx, partial, B, L, C, s); break;
      case 2: launch_k<2>(p.vec, bf16, x, w, bias, dy, dx, partial, B, L, C, s); break;
      case 3: launch_k<3>(p.vec, bf16, x, w, bias, dy, dx, partial, B, L, C, s); break;
      case 4: launch_k<4>(p.vec, bf16, x, w, bias, dy, dx, partial, B, L, C, s); break;
      case 5: launch_k<5>(p.vec, bf16, x, w, bias, dy, dx, partial, B, L, C, s); break;
      case 6: launch_k<6>(p.vec, bf16, x, w, bias, dy, dx, partial, B, L, C, s); break;
      case 7: launch_k<7>(p.vec, bf16, x, w, bias, dy, dx, partial, B, L, C, s); break;
      default: launch_k<8>(p.vec, bf16, x, w, bias, dy, dx, partial, B, L, C, s); break;
    }
    ALLOY_TRY(check_launch("conv1d_silu_bwd_kernel"));
  }
  if (C > 0) {
    const int64_t n = (int64_t)(K + 1) * C;
    conv1d_silu_bwd_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        partial, any_rows ? p.nslot : 0, C, K, dw->data, dw->dtype == ALLOY_BF16, dw->stride[0],
        dw->stride[1], present(db) ? db->data : nullptr, present(db) && db->dtype == ALLOY_BF16,
        present(db) ? db->stride[0] : 0);
    ALLOY_TRY(check_launch("conv1d_silu_bwd_reduce_kernel"));
  }
  return ALLOY_OK;
}

}  // namespace alloy
