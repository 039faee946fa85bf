// Tensor-core (tcgen05) chunked scan on pre-discretised bf16 inputs: the
// scan of MambaBlock._selective_scan / _scan_chunk (alloy/models/
// mamba_block.py:206-366) when x (dt-scaled), B and C arrive as separate bf16
// tensors, as in the split mode and in the gradient scans of training.
//
//   h_t = exp(la_t) h_{t-1} + B_t x_t^T,   y_t = C_t h_t        (h: [N, P] fp32)
//
// One CTA per (batch row, head) walks chunks of Q = 128 steps in order with
// the fp32 state resident in tensor memory.  Per chunk (t, s < Q):
//   cum[t]   = sum_{u<=t} la_u                               (score warps)
//   CB       = C B^T                                         (tcgen05 -> TMEM)
//   S[t,s]   = CB[t,s] exp(cum[t] - cum[s]) for s <= t, else 0  (bf16 pairs, in place over CB)
//   C~[t,:]  = exp(cum[t]) C[t,:]                            (bf16 pairs, next to S)
//   H        = bf16(state); state *= exp(cum[Q-1])           (state warps)
//   X'[s,:]  = exp(cum[Q-1] - cum[s]) x[s,:]                 (state warps)
//   Y        = [S | C~] [x ; H]                              (tcgen05, A from TMEM)
//   state   += B^T X'                                        (tcgen05)
// so y needs no separate inter-chunk product or epilogue combination.  The
// decays must satisfy la <= 0 (A_disc <= 1), as A = -exp(A_log) gives, which
// keeps every exponential above at or below 1.
//
// Operand tiles in shared memory use the 128-byte swizzle: x, B and C as
// [64-column blocks][128 steps][64] bf16 (double-buffered, filled by cp.async
// from any strides, negative time strides included), X' like x, H as
// [64-column blocks of p][N rows][64].  For N = 64 the B tile carries a zero
// second block, so the state MMA runs at M = 128 with the state's rows
// 64..127 identically zero.
//
// Warp roles (17 warps): 0-3 cumulative decay, scores and C~ (row t = lane
// quadrant); 4-7 state copy/decay (row n) and X' (row s); 8-11 output rows;
// 12-15 loads; 16 TMEM allocation and MMA issue.  Every mbarrier wait is
// bounded: on timeout the CTA records an error word, drains its copies and
// MMAs, frees its tensor memory and exits.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace alloy {

// error word written by a CTA whose bounded wait ran out (0 = none):
// [0] = 1 + site id, [1] = blockIdx.x, [2] = blockIdx.y
__device__ unsigned int g_scan_tc_error[3];

namespace {

using namespace tc;

constexpr int Q = 128;
constexpr int kWarps = 17;
constexpr int kThreads = kWarps * 32;
constexpr int kMmaWarp = 16;
constexpr long long kWaitCycles = 4000000000LL;   // ~2 s at 1.9 GHz
constexpr float kLog2e = 1.4426950408889634f;

enum {
  B_FULL0 = 0, B_FULL1,      // loads -> all: x, B, C, la of a buffer (4 loader warps)
  B_EMPTY0, B_EMPTY1,        // MMA -> loads: buffer read by every MMA
  B_CB_FULL,                 // MMA -> score warps
  B_CUM0, B_CUM1,            // score warps -> state warps: cum of a buffer (4)
  B_S_READY,                 // score warps -> MMA: S and C~ in TMEM (4)
  B_ST_READY,                // state warps -> MMA: H, X' written, state decayed (4)
  B_Y_FULL0, B_Y_FULL1,      // MMA -> output warps (per TMEM buffer)
  B_Y_EMPTY0, B_Y_EMPTY1,    // output warps -> MMA (4)
  B_ST_DONE,                 // MMA -> state warps: state update complete
  B_PWG,                     // score warps: warp totals of the decay scan (4)
  B_DRAIN,
  NBAR
};

template <int PP, int NN>
struct Layout {
  static constexpr uint32_t kX = PP * 256;           // x tile of one buffer
  static constexpr uint32_t kB = 32768;              // B tile (two 64-column blocks)
  static constexpr uint32_t kC = NN * 256;
  static constexpr uint32_t kBuf = kX + kB + kC;
  static constexpr uint32_t OFF_BUF = 0;             // 2 buffers [x | B | C]
  static constexpr uint32_t OFF_XP = 2 * kBuf;       // X' [PP/64][128][64]
  static constexpr uint32_t OFF_H = OFF_XP + kX;     // H [PP/64][NN][64]
  static constexpr uint32_t OFF_LA = OFF_H + PP * NN * 2;   // [2][128] f32
  static constexpr uint32_t OFF_CUM = OFF_LA + 1024;        // [2][128] f32
  static constexpr uint32_t OFF_WSUM = OFF_CUM + 1024;      // [2][4] f32
  static constexpr uint32_t OFF_BAR = OFF_WSUM + 64;
  static constexpr uint32_t OFF_TMEMPTR = OFF_BAR + NBAR * 8;
  static constexpr uint32_t OFF_ABORT = OFF_TMEMPTR + 8;
  static constexpr uint32_t kSmem = OFF_ABORT + 16 + 1024;  // + alignment slack
  // tensor memory columns
  static constexpr uint32_t T_CB = 0;                // CB, then S (cols 0-63) and C~ (64-)
  static constexpr uint32_t T_Y = 128;               // 2 x PP: output accumulators
  static constexpr uint32_t T_ST = 128 + 2 * PP;     // PP: state rows n
  static_assert(T_ST + PP <= 512, "tensor memory");
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ void signal_abort(volatile int* abort_flag, int site) {
  *abort_flag = 1;
  if (atomicCAS(&g_scan_tc_error[0], 0u, 1u + site) == 0u) {
    g_scan_tc_error[1] = blockIdx.x;
    g_scan_tc_error[2] = blockIdx.y;
  }
}

// single-thread wait (MMA issuer)
__device__ __forceinline__ bool wait1(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site) {
  const long long t0 = clock64();
  for (uint32_t it = 0; it < (1u << 30); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) break;
  }
  signal_abort(abort_flag, site);
  return false;
}

// warp-uniform wait: every lane polls (bounded by the clock and the CTA's
// abort flag), one vote makes the outcome the same on all lanes
__device__ __forceinline__ bool waitw(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site) {
  const long long t0 = clock64();
  bool ok;
  while (!(ok = mbar_try_wait(bar, parity) != 0)) {
    if (*abort_flag || clock64() - t0 > kWaitCycles) break;
  }
  ok = __all_sync(0xffffffffu, ok);
  if (!ok && (threadIdx.x & 31) == 0 && !*abort_flag) signal_abort(abort_flag, site);
  __syncwarp();
  return ok;
}

// byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a 128-byte-swizzled block
__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src))
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// copies the rows [c*Q, c*Q + Q) of one [L, cols] bf16 operand (row stride
// `st` elements, 64-column blocks of a swizzled tile); rows past L are zeroed
template <int COLS>
__device__ __forceinline__ void load_rows(uint32_t tile, const __nv_bfloat16* src, int64_t st, int row0, int L,
                                          int i) {
  constexpr int CPR = COLS / 8;   // 16-byte chunks a row
#pragma unroll 4
  for (int k = i; k < Q * CPR; k += 128) {
    const int r = k / CPR, j = k % CPR;
    const uint32_t dst = tile + (j >> 3) * 16384 + sw_off(r, j & 7);
    if (row0 + r < L)
      cp_async16(dst, src + (int64_t)(row0 + r) * st + 8 * j);
    else
      st_shared_v4(dst, make_uint4(0u, 0u, 0u, 0u));
  }
}

template <int PP, int NN>
__global__ void __launch_bounds__(kThreads, 1) scan_tc_kernel(const SsdArgs a, int y_vec) {
  using Lo = Layout<PP, NN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);
  float* la_s = reinterpret_cast<float*>(smem + Lo::OFF_LA);
  float* cum_s = reinterpret_cast<float*>(smem + Lo::OFF_CUM);
  float* wsum = reinterpret_cast<float*>(smem + Lo::OFF_WSUM);
  volatile uint32_t* tmem_ptr = reinterpret_cast<volatile uint32_t*>(smem + Lo::OFF_TMEMPTR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Lo::OFF_ABORT);
  auto bar = [&](int i) { return base + Lo::OFF_BAR + 8u * i; };
  auto xt = [&](int buf) { return base + Lo::OFF_BUF + buf * Lo::kBuf; };
  auto bt = [&](int buf) { return xt(buf) + Lo::kX; };
  auto ct = [&](int buf) { return bt(buf) + Lo::kB; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, b = blockIdx.y;
  const int L = a.L;
  const int nk = (L + Q - 1) / Q;
  const int g = h / (a.H / a.Gbc);

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    // FULL0/1 EMPTY0/1 CB_FULL CUM0/1 S_READY ST_READY Y_FULL0/1 Y_EMPTY0/1 ST_DONE PWG DRAIN
    const int counts[NBAR] = {4, 4, 1, 1, 1, 4, 4, 4, 4, 1, 1, 4, 4, 1, 4, 1};
    for (int i = 0; i < NBAR; ++i) mbar_init(bar(i), counts[i]);
    mbar_fence_init();
  }
  if (NN == 64) {
    // the zero second block of both B tiles (never written by the loads)
    for (int i = threadIdx.x; i < 2 * 1024; i += kThreads) {
      const int buf = i >> 10;
      st_shared_v4(bt(buf) + 16384 + (i & 1023) * 16, make_uint4(0u, 0u, 0u, 0u));
    }
    fence_async_smem();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(base + Lo::OFF_TMEMPTR, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_ptr;
  const int q = warp & 3;                       // TMEM lane quadrant
  const int r = q * 32 + lane;                  // row of this thread (t, s or n)
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);

  if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t ID_CB = idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t ID_Y = idesc_bf16(128, PP, 0, 1);
      constexpr uint32_t ID_ST = idesc_bf16(128, PP, 1, 1);
      for (int c = 0; c < nk; ++c) {
        const int buf = c & 1, yb = c & 1;
        if (!wait1(bar(B_FULL0 + buf), (c >> 1) & 1, abort_flag, 1)) break;
        // CB overwrites the S / C~ columns that Y(c-1) read
        if (c > 0 && !wait1(bar(B_Y_FULL0 + (yb ^ 1)), ((c - 1) >> 1) & 1, abort_flag, 2)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < NN / 16; ++k)
          umma_bf16(tmem + Lo::T_CB, sw128_desc(ct(buf) + (k >> 2) * 16384 + 32 * (k & 3), 16, 1024),
                    sw128_desc(bt(buf) + (k >> 2) * 16384 + 32 * (k & 3), 16, 1024), ID_CB, k != 0);
        umma_commit(bar(B_CB_FULL));
        if (!wait1(bar(B_S_READY), c & 1, abort_flag, 3)) break;
        if (!wait1(bar(B_ST_READY), c & 1, abort_flag, 4)) break;
        if (c >= 2 && !wait1(bar(B_Y_EMPTY0 + yb), ((c >> 1) - 1) & 1, abort_flag, 5)) break;
        tc_fence_after();
        // Y = S x + C~ H
        const uint32_t ty = tmem + Lo::T_Y + yb * PP;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_bf16_ta(ty, tmem + Lo::T_CB + 8 * k, sw128_desc(xt(buf) + 2048 * k, 16384, 1024), ID_Y, k != 0);
#pragma unroll
        for (int k = 0; k < NN / 16; ++k)
          umma_bf16_ta(ty, tmem + Lo::T_CB + 64 + 8 * k,
                       sw128_desc(base + Lo::OFF_H + 2048 * k, NN * 128, 1024), ID_Y, 1);
        umma_commit(bar(B_Y_FULL0 + yb));
        // state[n, p] += sum_s B[s, n] X'[s, p]
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_bf16(tmem + Lo::T_ST, sw128_desc(bt(buf) + 2048 * k, 16384, 1024),
                    sw128_desc(base + Lo::OFF_XP + 2048 * k, 16384, 1024), ID_ST, 1);
        umma_commit(bar(B_ST_DONE));
        umma_commit(bar(B_EMPTY0 + buf));
      }
      // wait (bounded) for every MMA this thread issued
      umma_commit(bar(B_DRAIN));
      const long long t0 = clock64();
      while (!mbar_try_wait(bar(B_DRAIN), 0) && clock64() - t0 < kWaitCycles) {
      }
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------------ loads
    const int i = threadIdx.x - 384;
    const int xh = a.x_hpg > 1 ? h / a.x_hpg : h;
    const __nv_bfloat16* xs = static_cast<const __nv_bfloat16*>(a.x) + (int64_t)b * a.x_sb + (int64_t)xh * a.x_sh;
    const __nv_bfloat16* bs = static_cast<const __nv_bfloat16*>(a.Bm) + (int64_t)b * a.bm_sb + (int64_t)g * a.bm_sg;
    const __nv_bfloat16* cs = static_cast<const __nv_bfloat16*>(a.Cm) + (int64_t)b * a.cm_sb + (int64_t)g * a.cm_sg;
    for (int c = 0; c < nk; ++c) {
      const int buf = c & 1;
      if (c >= 2 && !waitw(bar(B_EMPTY0 + buf), ((c >> 1) - 1) & 1, abort_flag, 10)) break;
      const int row0 = c * Q;
      load_rows<PP>(xt(buf), xs, a.x_st, row0, L, i);
      load_rows<NN>(bt(buf), bs, a.bm_st, row0, L, i);
      load_rows<NN>(ct(buf), cs, a.cm_st, row0, L, i);
      {
        const int t = row0 + i;
        float la = 0.f;
        if (t < L) {
          if (a.log_a)
            la = a.log_a[(int64_t)b * a.la_sb + (int64_t)t * a.la_st + (int64_t)h * a.la_sh];
          else
            la = logf(fmaxf(load_any(a.A_disc, (int64_t)b * a.ad_sb + (int64_t)t * a.ad_st + (int64_t)h * a.ad_sh,
                                     a.ad_bf16), 1e-10f));
        }
        la_s[buf * 128 + i] = la;
      }
      cp_async_wait_all();
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_FULL0 + buf));
    }
    cp_async_wait_all();
  } else if (warp < 4) {
    // ------------------------------------------------------------------ scores
    const int t = r;
    for (int c = 0; c < nk; ++c) {
      const int buf = c & 1;
      if (!waitw(bar(B_FULL0 + buf), (c >> 1) & 1, abort_flag, 20)) break;
      // cum[t] = inclusive sum of la over the chunk
      float v = la_s[buf * 128 + t];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      // warp totals: wsum[buf] for chunk c+2 is written only after every warp
      // passed the PWG wait of chunk c+1, which follows its reads for chunk c
      if (lane == 31) wsum[buf * 4 + q] = v;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PWG));
      if (!waitw(bar(B_PWG), c & 1, abort_flag, 21)) break;
      float pre = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) pre += k < q ? wsum[buf * 4 + k] : 0.f;
      const float cum_t = v + pre;
      cum_s[buf * 128 + t] = cum_t;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_CUM0 + buf));
      if (!waitw(bar(B_CUM0 + buf), (c >> 1) & 1, abort_flag, 22)) break;
      if (!waitw(bar(B_CB_FULL), c & 1, abort_flag, 23)) break;
      tc_fence_after();
      // S: K-step k (sources 16k .. 16k+15) as bf16 pairs in columns [8k, 8k+8)
      const float* cm = cum_s + buf * 128;
      const float ct2 = cum_t * kLog2e;
      auto score = [&](int k, const uint32_t (&rv)[16]) {
        uint32_t o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int s = 16 * k + 2 * e;
          const float f0 = s <= t ? __uint_as_float(rv[2 * e]) * ex2_approx(fmaf(-cm[s], kLog2e, ct2)) : 0.f;
          const float f1 = s + 1 <= t ? __uint_as_float(rv[2 * e + 1]) * ex2_approx(fmaf(-cm[s + 1], kLog2e, ct2)) : 0.f;
          o[e] = pack_bf16x2(f0, f1);
        }
        tmem_st8(lane_base + Lo::T_CB + 8 * k, o);
      };
      const int kmax = 2 * q + 1;   // pieces at or left of this warp's diagonal block
      uint32_t ra[16], rb[16];
      tmem_ld16(lane_base + Lo::T_CB, ra);
#pragma unroll 1
      for (int k = 0; k <= kmax; k += 2) {
        tmem_ld_wait_regs(ra);
        tmem_ld16(lane_base + Lo::T_CB + 16 * (k + 1), rb);
        score(k, ra);
        tmem_ld_wait_regs(rb);
        if (k + 2 <= kmax) tmem_ld16(lane_base + Lo::T_CB + 16 * (k + 2), ra);
        score(k + 1, rb);
      }
      {
        uint32_t z[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) z[e] = 0u;
#pragma unroll 1
        for (int k = kmax + 1; k < 8; ++k) tmem_st8(lane_base + Lo::T_CB + 8 * k, z);
      }
      // C~ = exp(cum[t]) C[t, :]: K-step k of the C~ H product in columns [64 + 8k, 64 + 8k + 8)
      {
        const float e = ex2_approx(ct2);
        const uint32_t crow = ct(buf);
#pragma unroll 1
        for (int k = 0; k < NN / 16; ++k) {
          uint32_t o[8];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int j = 2 * k + hh;   // 16-byte chunk of the row
            const uint4 w = ld_shared_v4(crow + (j >> 3) * 16384 + sw_off(t, j & 7));
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int m = 0; m < 4; ++m) o[4 * hh + m] = pack_bf16x2(e * bf16_lo(ww[m]), e * bf16_hi(ww[m]));
          }
          tmem_st8(lane_base + Lo::T_CB + 64 + 8 * k, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_S_READY));
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------------ state and X'
    const bool has_row = r < NN;   // warp-uniform
    // initial state (rows n >= NN stay zero)
#pragma unroll 1
    for (int p0 = 0; p0 < PP; p0 += 16) {
      uint32_t v[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        float f = 0.f;
        if (has_row && a.ssm_in)
          f = a.ssm_in[(int64_t)b * a.si_sb + (int64_t)h * a.si_sh + (int64_t)r * a.si_sn + (int64_t)(p0 + k) * a.si_sp];
        v[k] = __float_as_uint(f);
      }
      tmem_st16(lane_base + Lo::T_ST + p0, v);
    }
    tmem_st_wait();
    for (int c = 0; c < nk; ++c) {
      const int buf = c & 1;
      if (!waitw(bar(B_FULL0 + buf), (c >> 1) & 1, abort_flag, 30)) break;
      if (!waitw(bar(B_CUM0 + buf), (c >> 1) & 1, abort_flag, 31)) break;
      // the previous state update (and Y(c-1), issued before it) has completed
      if (c > 0 && !waitw(bar(B_ST_DONE), (c - 1) & 1, abort_flag, 32)) break;
      tc_fence_after();
      const float* cm = cum_s + buf * 128;
      const float last = cm[127];
      if (has_row) {
        const float e = ex2_approx(last * kLog2e);
        const uint32_t hrow = base + Lo::OFF_H;
#pragma unroll 1
        for (int p0 = 0; p0 < PP; p0 += 16) {
          uint32_t v[16];
          tmem_ld16(lane_base + Lo::T_ST + p0, v);
          tmem_ld_wait();
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int j = p0 / 8 + hh;   // 16-byte chunk of the state row (8 p)
            st_shared_v4(hrow + (j >> 3) * (NN * 128) + sw_off(r, j & 7),
                         make_uint4(pack_bf16x2(__uint_as_float(v[8 * hh + 0]), __uint_as_float(v[8 * hh + 1])),
                                    pack_bf16x2(__uint_as_float(v[8 * hh + 2]), __uint_as_float(v[8 * hh + 3])),
                                    pack_bf16x2(__uint_as_float(v[8 * hh + 4]), __uint_as_float(v[8 * hh + 5])),
                                    pack_bf16x2(__uint_as_float(v[8 * hh + 6]), __uint_as_float(v[8 * hh + 7]))));
          }
#pragma unroll
          for (int k = 0; k < 16; ++k) v[k] = __float_as_uint(e * __uint_as_float(v[k]));
          tmem_st16(lane_base + Lo::T_ST + p0, v);
        }
      }
      {
        // X'[s, :] = exp(cum[Q-1] - cum[s]) x[s, :]
        const float w = ex2_approx((last - cm[r]) * kLog2e);
        const uint32_t src = xt(buf), dst = base + Lo::OFF_XP;
#pragma unroll
        for (int j = 0; j < PP / 8; ++j) {
          const uint32_t off = (j >> 3) * 16384 + sw_off(r, j & 7);
          const uint4 u = ld_shared_v4(src + off);
          st_shared_v4(dst + off, make_uint4(pack_bf16x2(w * bf16_lo(u.x), w * bf16_hi(u.x)),
                                             pack_bf16x2(w * bf16_lo(u.y), w * bf16_hi(u.y)),
                                             pack_bf16x2(w * bf16_lo(u.z), w * bf16_hi(u.z)),
                                             pack_bf16x2(w * bf16_lo(u.w), w * bf16_hi(u.w))));
        }
      }
      fence_async_smem();
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_ST_READY));
    }
    // the final state
    if (!*abort_flag && a.ssm_out && nk > 0 && waitw(bar(B_ST_DONE), (nk - 1) & 1, abort_flag, 33)) {
      tc_fence_after();
      if (has_row) {
#pragma unroll 1
        for (int p0 = 0; p0 < PP; p0 += 16) {
          uint32_t v[16];
          tmem_ld16(lane_base + Lo::T_ST + p0, v);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 16; ++k)
            a.ssm_out[(int64_t)b * a.so_sb + (int64_t)h * a.so_sh + (int64_t)r * a.so_sn + (int64_t)(p0 + k) * a.so_sp] =
                __uint_as_float(v[k]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ output rows
    // y (optional) and the row dot products with z (optional)
    const int zh = a.z_hpg > 1 ? h / a.z_hpg : h;
    for (int c = 0; c < nk; ++c) {
      const int yb = c & 1;
      if (!waitw(bar(B_Y_FULL0 + yb), (c >> 1) & 1, abort_flag, 40)) break;
      tc_fence_after();
      const int t = c * Q + r;
      const int64_t yoff = (int64_t)b * a.y_sb + (int64_t)t * a.y_st + (int64_t)h * a.y_sh;
      const int64_t zoff = (int64_t)b * a.z_sb + (int64_t)t * a.z_st + (int64_t)zh * a.z_sh;
      float dot = 0.f;
#pragma unroll 1
      for (int p0 = 0; p0 < PP; p0 += 16) {
        uint32_t v[16];
        tmem_ld16(lane_base + Lo::T_Y + yb * PP + p0, v);
        tmem_ld_wait();
        if (t < L) {
          if (a.dot) {
            // z rows: 16-byte aligned with unit column stride (checked on the host)
            if (a.z_bf16) {
              const uint4* zp = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.z) + zoff + p0);
#pragma unroll
              for (int m = 0; m < 2; ++m) {
                const uint4 zz = __ldg(zp + m);
                const uint32_t zw[4] = {zz.x, zz.y, zz.z, zz.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  dot = fmaf(__uint_as_float(v[8 * m + 2 * e]), bf16_lo(zw[e]), dot);
                  dot = fmaf(__uint_as_float(v[8 * m + 2 * e + 1]), bf16_hi(zw[e]), dot);
                }
              }
            } else {
              const float4* zp = reinterpret_cast<const float4*>(static_cast<const float*>(a.z) + zoff + p0);
#pragma unroll
              for (int m = 0; m < 4; ++m) {
                const float4 zz = __ldg(zp + m);
                dot = fmaf(__uint_as_float(v[4 * m]), zz.x, dot);
                dot = fmaf(__uint_as_float(v[4 * m + 1]), zz.y, dot);
                dot = fmaf(__uint_as_float(v[4 * m + 2]), zz.z, dot);
                dot = fmaf(__uint_as_float(v[4 * m + 3]), zz.w, dot);
              }
            }
          }
          if (!a.y) {
          } else if (y_vec) {
            if (a.y_bf16) {
              uint4* d = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.y) + yoff + p0);
#pragma unroll
              for (int m = 0; m < 2; ++m)
                d[m] = make_uint4(pack_bf16x2(__uint_as_float(v[8 * m + 0]), __uint_as_float(v[8 * m + 1])),
                                  pack_bf16x2(__uint_as_float(v[8 * m + 2]), __uint_as_float(v[8 * m + 3])),
                                  pack_bf16x2(__uint_as_float(v[8 * m + 4]), __uint_as_float(v[8 * m + 5])),
                                  pack_bf16x2(__uint_as_float(v[8 * m + 6]), __uint_as_float(v[8 * m + 7])));
            } else {
              uint4* d = reinterpret_cast<uint4*>(static_cast<float*>(a.y) + yoff + p0);
#pragma unroll
              for (int m = 0; m < 4; ++m) d[m] = make_uint4(v[4 * m], v[4 * m + 1], v[4 * m + 2], v[4 * m + 3]);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 16; ++k)
              store_any(a.y, yoff + (int64_t)(p0 + k) * a.y_sp, a.y_bf16, __uint_as_float(v[k]));
          }
        }
      }
      if (a.dot && t < L) a.dot[(int64_t)b * a.dot_sb + (int64_t)t * a.dot_st + (int64_t)h * a.dot_sh] = dot;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_Y_EMPTY0 + yb));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// z rows for the dot products: 16-byte aligned with unit column stride
static bool scan_tc_dot_supported(const SsdArgs& a) {
  if (!a.dot) return true;
  const int es = a.z_bf16 ? 8 : 4;   // elements per 16 bytes
  return aligned16(a.z) && a.z_sb % es == 0 && a.z_st % es == 0 && a.z_sh % es == 0;
}

bool scan_tc_supported(const SsdArgs& a) {
  if (a.mode != 1 || !a.x_bf16 || !a.bm_bf16 || !a.cm_bf16) return false;
  const bool dims = (a.P == 64 && (a.N == 64 || a.N == 128)) || (a.P == 128 && a.N == 64);
  if (!dims || a.bm_sn != 1 || a.cm_sn != 1) return false;
  if (!aligned16(a.x) || !aligned16(a.Bm) || !aligned16(a.Cm)) return false;
  // every 16-byte row chunk starts on a 16-byte boundary: strides in multiples of 8 elements
  for (int64_t s : {a.x_sb, a.x_st, a.x_sh, a.bm_sb, a.bm_st, a.bm_sg, a.cm_sb, a.cm_st, a.cm_sg})
    if (s % 8 != 0) return false;
  return a.B <= 65535 && a.H > 0 && a.L > 0 && scan_tc_dot_supported(a);
}

int scan_tc(const SsdArgs& a, cudaStream_t s) {
  const int es = a.y_bf16 ? 8 : 4;   // elements per 16 bytes
  const int y_vec = a.y && a.y_sp == 1 && aligned16(a.y) && a.y_sb % es == 0 && a.y_st % es == 0 &&
                    a.y_sh % es == 0;
  dim3 grid(a.H, a.B);
  auto launch = [&](auto kernel, uint32_t smem) -> int {
    ALLOY_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kernel<<<grid, kThreads, smem, s>>>(a, y_vec);
    return check_launch("scan_tc_kernel");
  };
  if (a.P == 64 && a.N == 64) return launch(scan_tc_kernel<64, 64>, Layout<64, 64>::kSmem);
  if (a.P == 64) return launch(scan_tc_kernel<64, 128>, Layout<64, 128>::kSmem);
  return launch(scan_tc_kernel<128, 64>, Layout<128, 64>::kSmem);
}

int scan_tc_take_error(cudaStream_t stream, unsigned int out[3]) {
  ALLOY_CUDA(cudaStreamSynchronize(stream));
  unsigned int zero[3] = {0, 0, 0};
  ALLOY_CUDA(cudaMemcpyFromSymbol(out, g_scan_tc_error, sizeof(zero)));
  if (out[0] != 0) ALLOY_CUDA(cudaMemcpyToSymbol(g_scan_tc_error, zero, sizeof(zero)));
  return ALLOY_OK;
}

}  // namespace alloy
