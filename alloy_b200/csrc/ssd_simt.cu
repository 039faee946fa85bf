// fp32 CUDA-core chunked SSD scan (the exact-precision path).
//
// Used for fp32 inputs (where a bf16 tensor-core path cannot meet an fp32
// tolerance) and for pre-discretised inputs (alloy_selective_scan).  One CTA
// owns one (batch, head) and walks its chunks in order, keeping the fp32
// state [N, P] in shared memory.  Per chunk of QS steps (the SSD dual form of
// alloy/models/mamba_block.py:206-285; the result does not depend on QS):
//   cum[t]  = sum_{u<=t} log a_u                       (inclusive, this chunk)
//   W[t,s]  = exp(cum[t]-cum[s]) * <C_t, B_s>, s <= t   (decay-masked scores)
//   y[t,:]  = sum_s W[t,s] x_s + exp(cum[t]) C_t h + D x_t
//   h       = exp(cum[Q-1]) h + sum_s exp(cum[Q-1]-cum[s]) B_s x_s^T
// In mode 0 the chunk's x, B and C are produced in place from the raw xBC
// rows by the causal conv + SiLU (mamba_block.py:446-455) and dt, log a by
// the discretisation (:471-486).
#include "common.cuh"
#include "kernels.h"

namespace alloy {
namespace {

constexpr int QS = 32;        // chunk length (one warp lane per step)
constexpr int kThreads = 256;

__device__ __forceinline__ float raw_xbc(const SsdArgs& a, int b, int t, int c) {
  // x_padded[b, t + K - 1, c] of mamba_block.py:446-452
  if (t >= 0) return load_any(a.xBC, b * a.xbc_sb + (int64_t)t * a.xbc_st + c, a.xbc_bf16);
  if (a.conv_in == nullptr) return 0.f;
  return load_any(a.conv_in, b * a.ci_sb + (int64_t)(a.K - 1 + t) * a.ci_sk + c * a.ci_sc,
                  a.ci_bf16);
}

__global__ void __launch_bounds__(kThreads) ssd_simt_kernel(const SsdArgs a) {
  const int b = blockIdx.y;
  const int h = a.head_begin + blockIdx.x;
  const int P = a.P, N = a.N, H = a.H, L = a.L;
  const int tid = threadIdx.x;

  extern __shared__ float sm[];
  float* hs = sm;               // [N][P] state
  float* xs = hs + N * P;       // [QS][P] dt-scaled x
  float* xu = xs + QS * P;      // [QS][P] unscaled x (D skip)
  float* Bs = xu + QS * P;      // [N][QS] (transposed: conflict-free score loop)
  float* Cs = Bs + N * QS;      // [QS][N]
  float* W = Cs + QS * N;       // [QS][QS]
  float* cum = W + QS * QS;     // [QS]
  float* av = cum + QS;         // [QS] log a, later the chunk-end decay per step
  float* dtv = av + QS;         // [QS]

  for (int i = tid; i < N * P; i += kThreads) {
    const int n = i / P, p = i % P;
    hs[i] = a.ssm_in ? a.ssm_in[b * a.si_sb + h * a.si_sh + n * a.si_sn + p * a.si_sp] : 0.f;
  }

  float A = 0.f, dtb = 0.f, Dh = 0.f;
  int g;
  if (a.mode == 0) {
    A = -expf(a.A_log[h * a.al_s]);
    dtb = a.dt_bias[h * a.dtb_s];
    Dh = a.Dp ? a.Dp[h * a.d_s] : 0.f;
    g = h / (H / a.G);
  } else {
    g = h / (H / a.Gbc);
  }
  const int xoff = h * P;                 // channel offsets inside xBC
  const int boff = H * P + g * N;
  const int coff = H * P + a.G * N + g * N;

  for (int t0 = 0; t0 < L; t0 += QS) {
    const int qn = min(QS, L - t0);
    __syncthreads();  // previous chunk fully consumed
    // ---- load / produce the chunk ----------------------------------------
    if (a.mode == 0) {
      for (int i = tid; i < QS; i += kThreads) {
        float dt = 0.f;
        if (i < qn) {
          const float raw = load_any(a.dt_raw, b * a.dt_sb + (int64_t)(t0 + i) * a.dt_st +
                                                   h * a.dt_sh, a.dt_bf16);
          dt = softplus_f32(raw + dtb);
        }
        dtv[i] = dt;
        av[i] = A * dt;
      }
      const int W3 = P + 2 * N;
      for (int i = tid; i < QS * W3; i += kThreads) {
        const int r = i / W3, j = i % W3;
        const int c = j < P ? xoff + j : (j < P + N ? boff + (j - P) : coff + (j - P - N));
        float v = 0.f;
        if (r < qn) {
          const int t = t0 + r;
          float acc = a.conv_b ? a.conv_b[c * a.cb_s] : 0.f;
          for (int k = 0; k < a.K; ++k)
            acc = fmaf(raw_xbc(a, b, t - (a.K - 1) + k, c), a.conv_w[c * a.cw_sc + k * a.cw_sk],
                       acc);
          v = silu_f32(acc);
        }
        if (j < P) xu[r * P + j] = v;
        else if (j < P + N) Bs[(j - P) * QS + r] = v;
        else Cs[r * N + (j - P - N)] = v;
      }
      __syncthreads();
      for (int i = tid; i < QS * P; i += kThreads) xs[i] = xu[i] * dtv[i / P];
    } else {
      for (int i = tid; i < QS; i += kThreads) {
        float la = 0.f;
        if (i < qn) {
          const int64_t t = t0 + i;
          if (a.log_a) la = a.log_a[b * a.la_sb + t * a.la_st + h * a.la_sh];
          else la = logf(fmaxf(load_any(a.A_disc, b * a.ad_sb + t * a.ad_st + h * a.ad_sh,
                                        a.ad_bf16), 1e-10f));
        }
        av[i] = la;
      }
      for (int i = tid; i < QS * P; i += kThreads) {
        const int r = i / P, p = i % P;
        xs[i] = r < qn ? load_any(a.x, b * a.x_sb + (int64_t)(t0 + r) * a.x_st + h * a.x_sh + p,
                                  a.x_bf16) : 0.f;
      }
      for (int i = tid; i < QS * N; i += kThreads) {
        const int r = i / N, n = i % N;
        float bv = 0.f, cv = 0.f;
        if (r < qn) {
          const int64_t t = t0 + r;
          bv = load_any(a.Bm, b * a.bm_sb + t * a.bm_st + g * a.bm_sg + n * a.bm_sn, a.bm_bf16);
          cv = load_any(a.Cm, b * a.cm_sb + t * a.cm_st + g * a.cm_sg + n * a.cm_sn, a.cm_bf16);
        }
        Bs[n * QS + r] = bv;
        Cs[r * N + n] = cv;
      }
    }
    __syncthreads();
    // ---- inclusive cumsum of log a over the chunk (one warp) --------------
    if (tid < 32) {
      float v = av[tid];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (tid >= o) v += u;
      }
      cum[tid] = v;
    }
    __syncthreads();
    const float cl = cum[qn - 1];
    // ---- decay-masked scores W and chunk-end decay per step ---------------
    if ((N & 3) == 0) {
      // 4 consecutive sources s of one step t a thread: per n one broadcast C
      // and one float4 of B (stored [n][s]) feed 4 FMAs
      for (int i = tid; i < QS * QS / 4; i += kThreads) {
        const int t = i / (QS / 4), s4 = (i % (QS / 4)) * 4;
        float dot[4] = {0.f, 0.f, 0.f, 0.f};
        if (s4 <= t) {
          for (int n = 0; n < N; ++n) {
            const float cv = Cs[t * N + n];
            const float4 bv = *reinterpret_cast<const float4*>(Bs + n * QS + s4);
            dot[0] = fmaf(cv, bv.x, dot[0]);
            dot[1] = fmaf(cv, bv.y, dot[1]);
            dot[2] = fmaf(cv, bv.z, dot[2]);
            dot[3] = fmaf(cv, bv.w, dot[3]);
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int s2 = s4 + j;
          W[t * QS + s2] = s2 <= t ? dot[j] * expf(cum[t] - cum[s2]) : 0.f;
        }
      }
    } else
    for (int i = tid; i < QS * QS; i += kThreads) {
      const int t = i / QS, s = i % QS;
      float v = 0.f;
      if (s <= t) {
        float dot = 0.f;
        for (int n = 0; n < N; ++n) dot = fmaf(Cs[t * N + n], Bs[n * QS + s], dot);
        v = dot * expf(cum[t] - cum[s]);
      }
      W[i] = v;
    }
    __syncthreads();
    if (tid < QS) av[tid] = tid < qn ? expf(cl - cum[tid]) : 0.f;
    // ---- outputs -----------------------------------------------------------
    if ((P & 3) == 0 && (N & 3) == 0) {
      // register tiles of 4 steps x 2 columns: per reduction index one float2
      // of x (or h) and 4 broadcast scalars of W (or C) feed 8 FMAs
      const int ntile = (QS / 4) * (P / 2);
      for (int tile = tid; tile < ntile; tile += kThreads) {
        const int pp = (tile % (P / 2)) * 2, t0r = (tile / (P / 2)) * 4;
        if (t0r >= qn) continue;
        float intra[4][2], inter[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) intra[i][0] = intra[i][1] = inter[i][0] = inter[i][1] = 0.f;
        const int smax = min(t0r + 4, qn);
        for (int s2 = 0; s2 < smax; ++s2) {   // W is zero above the diagonal
          const float2 xv = *reinterpret_cast<const float2*>(xs + s2 * P + pp);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float wv = W[(t0r + i) * QS + s2];
            intra[i][0] = fmaf(wv, xv.x, intra[i][0]);
            intra[i][1] = fmaf(wv, xv.y, intra[i][1]);
          }
        }
        for (int n = 0; n < N; ++n) {
          const float2 hv = *reinterpret_cast<const float2*>(hs + n * P + pp);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float cv = Cs[(t0r + i) * N + n];
            inter[i][0] = fmaf(cv, hv.x, inter[i][0]);
            inter[i][1] = fmaf(cv, hv.y, inter[i][1]);
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int t = t0r + i;
          if (t >= qn) break;
          const float e = expf(cum[t]);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            float yv = fmaf(e, inter[i][j], intra[i][j]);
            if (a.mode == 0) yv = fmaf(Dh, xu[t * P + pp + j], yv);
            store_any(a.y, b * a.y_sb + (int64_t)(t0 + t) * a.y_st + h * a.y_sh + (pp + j) * a.y_sp,
                      a.y_bf16, yv);
          }
        }
      }
    } else
    for (int i = tid; i < qn * P; i += kThreads) {
      const int t = i / P, p = i % P;
      float intra = 0.f;
      for (int s = 0; s <= t; ++s) intra = fmaf(W[t * QS + s], xs[s * P + p], intra);
      float inter = 0.f;
      for (int n = 0; n < N; ++n) inter = fmaf(Cs[t * N + n], hs[n * P + p], inter);
      float yv = fmaf(expf(cum[t]), inter, intra);
      if (a.mode == 0) yv = fmaf(Dh, xu[t * P + p], yv);
      store_any(a.y, b * a.y_sb + (int64_t)(t0 + t) * a.y_st + h * a.y_sh + p * a.y_sp,
                a.y_bf16, yv);
    }
    __syncthreads();
    // ---- state update --------------------------------------------------------
    const float dl = expf(cl);
    if ((P & 3) == 0 && (N & 3) == 0) {
      // B_s decayed to the chunk end, transposed to [s][n] in the C buffer (read
      // by the outputs above, complete at the barrier), then register tiles of
      // 4 n x 4 p: per step one float4 of it and one of x feed 16 FMAs
      float* Bv = Cs;
      for (int i = tid; i < QS * N; i += kThreads) {
        const int s2 = i / N, n = i % N;
        Bv[i] = Bs[n * QS + s2] * av[s2];
      }
      __syncthreads();
      const int ntile = (N / 4) * (P / 4);
      for (int tile = tid; tile < ntile; tile += kThreads) {
        const int p4 = (tile % (P / 4)) * 4, n4 = (tile / (P / 4)) * 4;
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
        for (int s2 = 0; s2 < qn; ++s2) {
          const float4 bv = *reinterpret_cast<const float4*>(Bv + s2 * N + n4);
          const float4 xv = *reinterpret_cast<const float4*>(xs + s2 * P + p4);
          const float bb[4] = {bv.x, bv.y, bv.z, bv.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(bb[i], xx[j], acc[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float4* hrow = reinterpret_cast<float4*>(hs + (n4 + i) * P + p4);
          const float4 ho = *hrow;
          *hrow = make_float4(fmaf(dl, ho.x, acc[i][0]), fmaf(dl, ho.y, acc[i][1]),
                              fmaf(dl, ho.z, acc[i][2]), fmaf(dl, ho.w, acc[i][3]));
        }
      }
    } else
    for (int i = tid; i < N * P; i += kThreads) {
      const int n = i / P, p = i % P;
      float acc = 0.f;
      for (int s = 0; s < qn; ++s) acc = fmaf(Bs[n * QS + s] * av[s], xs[s * P + p], acc);
      hs[i] = fmaf(dl, hs[i], acc);
    }
  }
  __syncthreads();
  if (a.ssm_out) {
    for (int i = tid; i < N * P; i += kThreads) {
      const int n = i / P, p = i % P;
      a.ssm_out[b * a.so_sb + h * a.so_sh + n * a.so_sn + p * a.so_sp] = hs[i];
    }
  }
}

template <typename T>
__global__ void conv_state_update_kernel(const T* __restrict__ xbc, int64_t x_sb, int64_t x_st,
                                         const T* conv_in, int64_t ci_sb, int64_t ci_sk,
                                         int64_t ci_sc, T* conv_out, int64_t co_sb,
                                         int64_t co_sk, int64_t co_sc, int B, int L, int K,
                                         int c0, int n0, int c1, int n1, int c2, int n2) {
  const int nch = n0 + n1 + n2;
  const int64_t total = (int64_t)B * nch;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / nch);
    int j = (int)(i % nch);
    const int c = j < n0 ? c0 + j : (j < n0 + n1 ? c1 + (j - n0) : c2 + (j - n0 - n1));
    T v[8];
    for (int k = 0; k < K - 1; ++k) {
      const int t = L - (K - 1) + k;  // raw time index of x_padded row L + k
      if (t >= 0) v[k] = xbc[b * x_sb + (int64_t)t * x_st + c];
      else if (conv_in) v[k] = conv_in[b * ci_sb + (int64_t)(K - 1 + t) * ci_sk + c * ci_sc];
      else v[k] = from_f32<T>(0.f);
    }
    for (int k = 0; k < K - 1; ++k) conv_out[b * co_sb + (int64_t)k * co_sk + c * co_sc] = v[k];
  }
}

}  // namespace

size_t ssd_simt_smem_bytes(int P, int N) {
  return sizeof(float) * ((size_t)N * P + 2 * QS * P + 2 * (size_t)QS * N + QS * QS + 3 * QS);
}

int ssd_simt(const SsdArgs& a, cudaStream_t s) {
  const size_t smem = ssd_simt_smem_bytes(a.P, a.N);
  if (smem > 227 * 1024)
    return fail(ALLOY_ERR_UNSUPPORTED, "ssd: head_dim*d_state too large for the fp32 path");
  if (a.B == 0 || a.head_count == 0) return ALLOY_OK;
  ALLOY_CUDA(cudaFuncSetAttribute(ssd_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
  dim3 grid(a.head_count, a.B);
  ssd_simt_kernel<<<grid, kThreads, smem, s>>>(a);
  return check_launch("ssd_simt_kernel");
}

int conv_state_update(const alloy_tensor_t* xBC, const alloy_tensor_t* conv_in,
                      alloy_tensor_t* conv_out, int H, int P, int N, int G, int K,
                      int head_begin, int head_count, cudaStream_t s) {
  const int B = (int)xBC->shape[0], L = (int)xBC->shape[1];
  if (B == 0 || head_count == 0 || K < 2) return ALLOY_OK;
  const int hpg = H / G;
  const int g0 = head_begin / hpg, g1 = (head_begin + head_count - 1) / hpg;
  const int c0 = head_begin * P, n0 = head_count * P;
  const int c1 = H * P + g0 * N, n1 = (g1 - g0 + 1) * N;
  const int c2 = H * P + G * N + g0 * N, n2 = n1;
  const int64_t total = (int64_t)B * (n0 + n1 + n2);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  const bool ci = present(conv_in);
#define ALLOY_CSU(T)                                                                          \
  conv_state_update_kernel<T><<<blocks, 256, 0, s>>>(                                         \
      static_cast<const T*>(xBC->data), xBC->stride[0], xBC->stride[1],                       \
      ci ? static_cast<const T*>(conv_in->data) : nullptr, ci ? conv_in->stride[0] : 0,       \
      ci ? conv_in->stride[1] : 0, ci ? conv_in->stride[2] : 0,                               \
      static_cast<T*>(conv_out->data), conv_out->stride[0], conv_out->stride[1],              \
      conv_out->stride[2], B, L, K, c0, n0, c1, n1, c2, n2)
  if (xBC->dtype == ALLOY_BF16) ALLOY_CSU(__nv_bfloat16);
  else ALLOY_CSU(float);
#undef ALLOY_CSU
  return check_launch("conv_state_update_kernel");
}

}  // namespace alloy
