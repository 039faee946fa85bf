// One decode token through the conv cache and the SSM cache, in place
// (the L = 1 path of alloy/models/mamba_block.py:446-493 with
// _selective_scan_sequential :160-204).
//
// A CTA owns one (batch row, head group).  That makes it the only writer of
// every conv-cache channel it touches (the group's x channels and its B and C
// columns), so the roll can be done in place without races.  Phase 1 rolls
// the conv cache and produces the token's x, B, C (fp32, in shared memory);
// phase 2 streams the fp32 state of the group's heads once: 16-byte loads,
// s' = exp(A dt) s + dt x B^T, y = C s' + D x, 16-byte stores.  The state
// traffic (read + write of [heads, N, P] fp32) is the whole cost.
//
// When the batch is small (fewer (row, group) pairs than SMs) each group's
// heads are split over several CTAs so that the state streams from most of
// the SMs.  The B and C channels are then read by every slice of the group,
// so the slices leave them unrolled and a second small kernel rolls them.
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace alloy {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

// the state is read and written once per token: streaming (evict-first)
// cache policy for both, so it does not displace the rest of L2
__device__ __forceinline__ float4 ld_state(const float* p) {
  return __ldcs(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ void st_state(float* p, const float4& v) {
  __stcs(reinterpret_cast<float4*>(p), v);
}

// Phase 2 for the [.., P, N] layout (N contiguous): a row p is NV float4s,
// handled by NV lanes (NV a power of two <= 32); y[p] is a segmented
// shuffle reduction.  NV == 0 selects the generic loop (a warp per row).
template <int NV>
__device__ __forceinline__ void state_rows_pn(const DecodeArgs& a, float* st, const float* xs,
                                              const float* Bs, const float* Cs, float dA,
                                              float dt, float Dh, int P, int N, void* yrow,
                                              int64_t y_off) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int nwarps = kThreads / 32;
  if constexpr (NV > 0) {
    constexpr int RPW = 32 / NV;  // rows per warp per step
    const int sub = lane / NV, j = lane % NV;
    const float4 bv = reinterpret_cast<const float4*>(Bs)[j];
    const float4 cv = reinterpret_cast<const float4*>(Cs)[j];
    for (int p0 = warp * RPW * kUnroll; p0 < P; p0 += nwarps * RPW * kUnroll) {
      float4 s[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        s[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        const int p = p0 + u * RPW + sub;
        if (p < P) s[u] = ld_state(st + (int64_t)p * a.st_row + 4 * j);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int p = p0 + u * RPW + sub;
        const float xd = (p < P ? xs[p] : 0.f) * dt;
        float4 v = s[u];
        v.x = fmaf(dA, v.x, xd * bv.x);
        v.y = fmaf(dA, v.y, xd * bv.y);
        v.z = fmaf(dA, v.z, xd * bv.z);
        v.w = fmaf(dA, v.w, xd * bv.w);
        float part = v.x * cv.x + v.y * cv.y + v.z * cv.z + v.w * cv.w;
#pragma unroll
        for (int o = NV / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (p < P) {
          st_state(st + (int64_t)p * a.st_row + 4 * j, v);
          if (j == 0) store_any(yrow, y_off + p, a.y_bf16, fmaf(Dh, xs[p], part));
        }
      }
    }
  } else {
    for (int p = warp; p < P; p += nwarps) {
      const float xd = xs[p] * dt;
      float part = 0.f;
      for (int n = lane; n < N; n += 32) {
        float v = st[(int64_t)p * a.st_row + n];
        v = fmaf(dA, v, xd * Bs[n]);
        st[(int64_t)p * a.st_row + n] = v;
        part = fmaf(Cs[n], v, part);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (lane == 0) store_any(yrow, y_off + p, a.y_bf16, fmaf(Dh, xs[p], part));
    }
  }
}

// Phase 2 for the [.., N, P] layout (P contiguous): thread owns float4 column
// groups and accumulates y over its rows; row groups reduce through smem.
__device__ __forceinline__ void state_rows_np(const DecodeArgs& a, float* st, const float* xs,
                                              const float* Bs, const float* Cs, float dA,
                                              float dt, float Dh, int P, int N, void* yrow,
                                              int64_t y_off, float* red, bool vec) {
  const int tid = threadIdx.x;
  if (vec) {
    const int PV = P / 4;                 // float4 columns
    const int groups = kThreads / PV;     // row groups (PV divides 256)
    const int j = tid % PV, rg = tid / PV;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 xv = reinterpret_cast<const float4*>(xs)[j];
    for (int n0 = rg * kUnroll; n0 < N; n0 += groups * kUnroll) {
      float4 s[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        s[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        const int n = n0 + u;
        if (n < N) s[u] = ld_state(st + (int64_t)n * a.st_row + 4 * j);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int n = n0 + u;
        if (n < N) {
          const float bd = Bs[n] * dt, c = Cs[n];
          float4 v = s[u];
          v.x = fmaf(dA, v.x, bd * xv.x);
          v.y = fmaf(dA, v.y, bd * xv.y);
          v.z = fmaf(dA, v.z, bd * xv.z);
          v.w = fmaf(dA, v.w, bd * xv.w);
          st_state(st + (int64_t)n * a.st_row + 4 * j, v);
          acc.x = fmaf(c, v.x, acc.x);
          acc.y = fmaf(c, v.y, acc.y);
          acc.z = fmaf(c, v.z, acc.z);
          acc.w = fmaf(c, v.w, acc.w);
        }
      }
    }
    // red: [groups][P]
    reinterpret_cast<float4*>(red)[rg * PV + j] = acc;
    __syncthreads();
    for (int p = tid; p < P; p += kThreads) {
      float sum = 0.f;
      for (int r = 0; r < groups; ++r) sum += red[r * P + p];
      store_any(yrow, y_off + p, a.y_bf16, fmaf(Dh, xs[p], sum));
    }
    __syncthreads();
  } else {
    for (int p = tid; p < P; p += kThreads) {
      float sum = 0.f;
      const float xd = xs[p] * dt;
      for (int n = 0; n < N; ++n) {
        float v = st[(int64_t)n * a.st_row + p];
        v = fmaf(dA, v, xd * Bs[n]);
        st[(int64_t)n * a.st_row + p] = v;
        sum = fmaf(Cs[n], v, sum);
      }
      store_any(yrow, y_off + p, a.y_bf16, fmaf(Dh, xs[p], sum));
    }
  }
}

template <int NV>
__global__ void __launch_bounds__(kThreads) decode_step_kernel(const DecodeArgs a, int hsplit, int roll_bc) {
  const int b = blockIdx.y;
  const int hpg = a.H / a.G;
  const int g = a.head_begin / hpg + blockIdx.x / hsplit;
  const int gb = max(a.head_begin, g * hpg);
  const int ge = min(a.head_begin + a.head_count, (g + 1) * hpg);
  // this CTA's slice of the group's heads (the whole group when hsplit == 1)
  const int per = (ge - gb + hsplit - 1) / hsplit;
  const int hb = gb + (blockIdx.x % hsplit) * per;
  const int he = min(ge, hb + per);
  if (hb >= he) return;
  const int nh = he - hb;
  const int P = a.P, N = a.N, K = a.K;

  extern __shared__ __align__(16) float sm[];
  const int n4 = (N + 3) & ~3;
  float* red = sm;                 // [kThreads * 4] reduction scratch (NP layout)
  float* Bs = red + kThreads * 4;  // [N]
  float* Cs = Bs + n4;             // [N]
  float* xs = Cs + n4;             // [nh][P]

  // ---- phase 1: conv + SiLU for this CTA's channels ----------------------
  // The CTA rolls the conv cache of its own x channels.  The group's B and C
  // channels are shared by every slice of the group: with roll_bc == 0 they
  // are only read here and decode_bc_roll_kernel rolls them afterwards.
  const int nx = nh * P;
  const int nch = nx + 2 * N;
  for (int i = threadIdx.x; i < nch; i += kThreads) {
    const int c = i < nx ? hb * P + i
                         : (i < nx + N ? a.H * P + g * N + (i - nx)
                                       : a.H * P + a.G * N + g * N + (i - nx - N));
    float win[8];
    const int64_t cs_base = b * a.cs_sb + (int64_t)c * a.cs_sc;
    for (int k = 0; k < K - 1; ++k) win[k] = load_any(a.conv_state, cs_base + k * a.cs_sk, a.cs_bf16);
    win[K - 1] = load_any(a.xbc, b * a.x_sb + c, a.x_bf16);
    float acc = a.conv_b ? a.conv_b[c * a.cb_s] : 0.f;
    for (int k = 0; k < K; ++k) acc = fmaf(win[k], a.conv_w[c * a.cw_sc + k * a.cw_sk], acc);
    if (i < nx || roll_bc)
      for (int k = 0; k < K - 1; ++k) store_any(a.conv_state, cs_base + k * a.cs_sk, a.cs_bf16, win[k + 1]);
    const float v = silu_f32(acc);
    if (i < nx) xs[i] = v;
    else if (i < nx + N) Bs[i - nx] = v;
    else Cs[i - nx - N] = v;
  }
  __syncthreads();

  // ---- phase 2: stream each head's state once ----------------------------
  const bool np_vec = (P % 4 == 0) && (kThreads % (P / 4) == 0) && ((a.st_row & 3) == 0);
  for (int hl = 0; hl < nh; ++hl) {
    const int h = hb + hl;
    const float dt = softplus_f32(load_any(a.dt, b * a.dt_sb + h * a.dt_sh, a.dt_bf16) +
                                  a.dt_bias[h * a.dtb_s]);
    const float dA = expf(-expf(a.A_log[h * a.al_s]) * dt);
    const float Dh = a.Dp ? a.Dp[h * a.d_s] : 0.f;
    float* st = a.state + b * a.st_sb + h * a.st_sh;
    const int64_t y_off = b * a.y_sb + h * a.y_sh;
    if (a.state_pn)
      state_rows_pn<NV>(a, st, xs + hl * P, Bs, Cs, dA, dt, Dh, P, N, a.y, y_off);
    else
      state_rows_np(a, st, xs + hl * P, Bs, Cs, dA, dt, Dh, P, N, a.y, y_off, red, np_vec);
  }
}

// Conv-cache roll of the B and C channels of groups g0 .. g0 + ngroups - 1,
// after decode_step_kernel has read them (split-head launches): one thread
// per (batch row, channel).
__global__ void __launch_bounds__(kThreads) decode_bc_roll_kernel(const DecodeArgs a, int g0, int ngroups) {
  const int per_row = 2 * ngroups * a.N;
  const int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (i >= (int64_t)a.B * per_row) return;
  const int b = (int)(i / per_row), r = (int)(i % per_row);
  const int which = r / (ngroups * a.N), q = r % (ngroups * a.N);  // 0: B, 1: C
  const int c = a.H * a.P + which * a.G * a.N + g0 * a.N + q;
  const int64_t cs_base = b * a.cs_sb + (int64_t)c * a.cs_sc;
  for (int k = 0; k + 1 < a.K - 1; ++k)
    store_any(a.conv_state, cs_base + k * a.cs_sk, a.cs_bf16,
              load_any(a.conv_state, cs_base + (k + 1) * a.cs_sk, a.cs_bf16));
  if (a.K >= 2)
    store_any(a.conv_state, cs_base + (a.K - 2) * a.cs_sk, a.cs_bf16, load_any(a.xbc, b * a.x_sb + c, a.x_bf16));
}

}  // namespace

int ssd_decode_step(const DecodeArgs& a, cudaStream_t s) {
  if (a.B == 0 || a.head_count == 0) return ALLOY_OK;
  const int hpg = a.H / a.G;
  const int g0 = a.head_begin / hpg, g1 = (a.head_begin + a.head_count - 1) / hpg;
  const int ngroups = g1 - g0 + 1;
  const int max_heads = std::min(hpg, a.head_count);
  // Few (batch row, group) pairs leave most SMs idle: split each group's heads
  // over several CTAs, aiming at two CTAs an SM of a 148-SM part.
  const int64_t pairs = (int64_t)ngroups * a.B;
  // vectorised PN rows need 16-byte aligned rows of N floats
  const bool pn_vec = a.state_pn && (a.N % 4 == 0) && (a.st_row % 4 == 0) &&
                      ((reinterpret_cast<uintptr_t>(a.state) & 15) == 0) &&
                      (a.st_sb % 4 == 0) && (a.st_sh % 4 == 0);
  const int nv = pn_vec ? a.N / 4 : 0;
  auto smem_for = [&](int hs) {
    const int slice_heads = (max_heads + hs - 1) / hs;
    return sizeof(float) * ((size_t)slice_heads * a.P + 2 * ((a.N + 3) & ~3) + kThreads * 4);
  };
  auto kernel_of = [&](int v) -> void (*)(const DecodeArgs, int, int) {
    switch (v) {
      case 4: return decode_step_kernel<4>;
      case 8: return decode_step_kernel<8>;
      case 16: return decode_step_kernel<16>;
      case 32: return decode_step_kernel<32>;
      default: return decode_step_kernel<0>;
    }
  };
  int hsplit = 1;
  if (pairs < 148) {
    hsplit = (int)std::min<int64_t>(max_heads, (296 + pairs - 1) / pairs);
    const int per = (max_heads + hsplit - 1) / hsplit;
    hsplit = (max_heads + per - 1) / per;
  } else if (max_heads >= 2) {
    // Many pairs: one CTA a pair can leave the last wave mostly empty (the
    // Nemotron shape at batch 256: 2,048 CTAs at 4 an SM on 148 SMs are 3.46
    // waves).  Split the heads in two when that packs the waves better.
    const int sms = sm_count_of_current_device();
    auto waste = [&](int hs) {   // idle fraction of the last wave
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel_of(nv), kThreads, smem_for(hs)) !=
              cudaSuccess || per_sm <= 0 || sms <= 0)
        return 0.0;
      const double waves = (double)(pairs * hs) / ((double)sms * per_sm);
      return (std::ceil(waves) - waves) / std::ceil(waves);
    };
    if (waste(2) + 0.02 < waste(1)) hsplit = 2;
  }
  const size_t smem = smem_for(hsplit);
  if (smem > 200 * 1024)
    return fail(ALLOY_ERR_UNSUPPORTED, "decode: heads per group * head_dim too large");
  dim3 grid(ngroups * hsplit, a.B);
  const int roll_bc = hsplit == 1;
#define ALLOY_DEC(NVV)                                                                       \
  do {                                                                                       \
    ALLOY_CUDA(cudaFuncSetAttribute(decode_step_kernel<NVV>,                                 \
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    decode_step_kernel<NVV><<<grid, kThreads, smem, s>>>(a, hsplit, roll_bc);                \
  } while (0)
  switch (nv) {
    case 4: ALLOY_DEC(4); break;
    case 8: ALLOY_DEC(8); break;
    case 16: ALLOY_DEC(16); break;
    case 32: ALLOY_DEC(32); break;
    default: ALLOY_DEC(0); break;
  }
#undef ALLOY_DEC
  int rc = check_launch("decode_step_kernel");
  if (rc != ALLOY_OK || roll_bc) return rc;
  const int64_t n = (int64_t)a.B * 2 * ngroups * a.N;
  decode_bc_roll_kernel<<<(unsigned)((n + kThreads - 1) / kThreads), kThreads, 0, s>>>(a, g0, ngroups);
  return check_launch("decode_bc_roll_kernel");
}

}  // namespace alloy
