// Tensor-core (tcgen05) chunked scan on pre-discretised bf16 inputs: the
// scan of MambaBlock._selective_scan / _scan_chunk (alloy/models/
// mamba_block.py:206-366) when x (dt-scaled), B and C arrive as separate bf16
// tensors, as in the split mode and in the gradient scans of training.
//
//   h_t = exp(la_t) h_{t-1} + B_t x_t^T,   y_t = C_t h_t        (h: [N, P] fp32)
//
// One CTA per (batch row, head) walks chunks of Q = 128 steps in order with
// the fp32 state resident in tensor memory.  Per chunk (t, s < Q):
//   cum[t]   = sum_{u<=t} la_u                               (load warps)
//   CB       = C B^T                                         (tcgen05 -> TMEM)
//   S[t,s]   = CB[t,s] exp(cum[t] - cum[s]) for s <= t, else 0  (bf16 pairs, in place over CB)
//   C~[t,:]  = exp(cum[t]) C[t,:]                            (bf16 pairs, beside S)
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
// Warp roles (23 warps): 0-7 scores and C~ (row t = lane quadrant, two warps
// a quadrant splitting its columns); 8-11 and 20-21 state copy/decay (row n)
// and X' (row s); 12-15 output rows; 16-19 loads and the decay scan; 22 TMEM
// allocation and MMA issue.  CB is double-buffered in tensor memory, so
// the next chunk's C B^T runs while this chunk's scores are computed.  Every mbarrier wait is
// bounded: on timeout the CTA records an error word, drains its copies and
// MMAs, frees its tensor memory and exits.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

// Phase markers: no code unless a timing build defines ALLOY_SCAN_TRACE.
#ifndef ALLOY_SCAN_TRACE
#define ALLOY_SCAN_TRACE(id, chunk)
#endif

namespace alloy {

// error word written by a CTA whose bounded wait ran out (0 = none):
// [0] = 1 + site id, [1] = blockIdx.x, [2] = blockIdx.y
__device__ unsigned int g_scan_tc_error[3];

namespace {

using namespace tc;

constexpr int Q = 128;
constexpr int kWarps = 23;
constexpr int kThreads = kWarps * 32;
constexpr int kStateWarp0 = 8;
constexpr int kOutWarp0 = 12;
constexpr int kLoadWarp0 = 16;
constexpr int kStateWarpX0 = 20;   // two more state warps (lane quadrants 0 and 1)
constexpr int kMmaWarp = 22;
constexpr long long kWaitCycles = 4000000000LL;   // ~2 s at 1.9 GHz
constexpr int kL2Ahead = 3;                         // chunks prefetched into L2 ahead of their loads
constexpr float kLog2e = 1.4426950408889634f;

constexpr int kMaxBuf = 3;   // load buffers (3 for head_dim = d_state = 64, else 2)

enum {
  B_FULL0 = 0,                         // loads -> all: x, B, C, cum, column factors of buffer i (4 warps)
  B_EMPTY0 = B_FULL0 + kMaxBuf,        // MMA -> loads: buffer i read by every MMA
  B_CB_FULL0 = B_EMPTY0 + kMaxBuf,     // MMA -> score warps: CB in TMEM buffer j (2)
  B_CB_FREE0 = B_CB_FULL0 + 2,         // MMA -> MMA: Y that read TMEM buffer j completed (2)
  B_S_READY0 = B_CB_FREE0 + 2,         // score warps -> MMA: S and C~ in TMEM buffer j (2, 8 warps)
  B_ST_READY = B_S_READY0 + 2,         // state warps -> MMA: H written, state decayed
  B_XP_READY0,                         // X' warps -> MMA: X' buffer i written (2)
  B_Y_FULL0 = B_XP_READY0 + 2,         // MMA -> output warps (per output accumulator, 2)
  B_Y_EMPTY0 = B_Y_FULL0 + 2,          // output warps -> MMA (2, 4 warps)
  B_ST_DONE = B_Y_EMPTY0 + 2,          // MMA -> state warps: state update complete
  B_PWG,                               // loader warps: warp totals of the decay scan (4)
  B_DRAIN,
  NBAR
};

template <int PP, int NN, bool SPLIT = false>
struct Layout {
  static constexpr int NBUF = (PP == 64 && NN == 64 && !SPLIT) ? 3 : 2;
  static constexpr uint32_t kX = PP * 256;           // x tile of one buffer [PP/64][128][64]
  static constexpr uint32_t kB = NN * 256;           // B tile [NN/64][128][64]
  static constexpr uint32_t kC = NN * 256;
  static constexpr uint32_t kBuf = kX + kB + kC;
  static constexpr uint32_t OFF_BUF = 0;             // NBUF buffers [x | B | C]
  static constexpr uint32_t OFF_ZERO = NBUF * kBuf;  // 16 KB of zeros: the B tile's second block for NN = 64
  static constexpr int NXP = PP == 128 ? 1 : 2;      // X' buffers
  // SPLIT (precise mode, head_dim = d_state = 64): X' and H as bf16 pairs, a
  // high tile and the remainder's tile
  static constexpr uint32_t kXPB = kX * (SPLIT ? 2 : 1);
  static constexpr uint32_t OFF_XP = OFF_ZERO + (NN == 64 ? 16384 : 0);   // NXP x X' [hi | lo][PP/64][128][64]
  static constexpr int NH = (PP == 64 && NN == 128) ? 1 : 2;   // H buffers
  static constexpr uint32_t kH = PP * NN * 2;
  static constexpr uint32_t kHB = kH * (SPLIT ? 2 : 1);
  static constexpr uint32_t OFF_H = OFF_XP + NXP * kXPB;   // NH x H [hi | lo][PP/64][NN][64]
  static constexpr uint32_t OFF_CUM = OFF_H + NH * kHB;            // [NBUF][128] f32
  static constexpr uint32_t OFF_CF = OFF_CUM + NBUF * 512;         // [NBUF][128] f32 column factors
  static constexpr uint32_t OFF_DIAG = OFF_CF + NBUF * 512;        // [4 chunks][128] f32: S[t,t] as rounded
  static constexpr uint32_t OFF_WSUM = OFF_DIAG + 4 * 512;         // [NBUF][4] f32
  static constexpr uint32_t OFF_BAR = OFF_WSUM + 64;
  static constexpr uint32_t OFF_TMEMPTR = OFF_BAR + NBAR * 8;
  static constexpr uint32_t OFF_ABORT = OFF_TMEMPTR + 8;
  static constexpr uint32_t kSmem = OFF_ABORT + 16 + 1024;  // + alignment slack
  // tensor memory columns: two CB buffers (CB, then in place: K-step k of S in
  // columns [16k, 16k+8) and of C~ in [16k+8, 16k+16)), NYB output
  // accumulators, the state
  // With SPLIT the scores take a piece's 16 columns (hi, lo) and C~ moves to
  // its own columns after the state (two buffers of NN: hi, lo).
  static_assert(!SPLIT || (PP == 64 && NN == 64), "precise mode: head_dim = d_state = 64");
  static constexpr int NYB = (PP == 128 || SPLIT) ? 1 : 2;
  static constexpr uint32_t T_CB = 0;                // + 128 * (chunk & 1)
  static constexpr uint32_t T_Y = 256;               // + PP * (chunk % NYB)
  static constexpr uint32_t T_ST = 256 + NYB * PP;   // PP: state rows n
  static constexpr uint32_t T_CT = T_ST + PP;        // SPLIT: + NN * (chunk & 1); lo at + NN/2
  static_assert(T_ST + PP + (SPLIT ? 2 * NN : 0) <= 512, "tensor memory");
  static_assert(kSmem <= 227 * 1024, "shared memory");
  static_assert(NBUF <= kMaxBuf, "buffers");
};

__device__ __forceinline__ void signal_abort(volatile int* abort_flag, int site) {
  *abort_flag = 1;
  if (atomicCAS(&g_scan_tc_error[0], 0u, 1u + site) == 0u) {
    g_scan_tc_error[1] = blockIdx.x;
    g_scan_tc_error[2] = blockIdx.y;
  }
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

// non-blocking test of an mbarrier phase
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
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

template <int PP, int NN, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) scan_tc_kernel(const SsdArgs a, int y_vec) {
  using Lo = Layout<PP, NN, SPLIT>;
  constexpr int NBUF = Lo::NBUF, NYB = Lo::NYB;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);
  float* cum_s = reinterpret_cast<float*>(smem + Lo::OFF_CUM);
  float* cf_s = reinterpret_cast<float*>(smem + Lo::OFF_CF);
  float* diag_s = reinterpret_cast<float*>(smem + Lo::OFF_DIAG);
  float* wsum = reinterpret_cast<float*>(smem + Lo::OFF_WSUM);
  volatile uint32_t* tmem_ptr = reinterpret_cast<volatile uint32_t*>(smem + Lo::OFF_TMEMPTR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Lo::OFF_ABORT);
  auto bar = [&](int i) { return base + Lo::OFF_BAR + 8u * i; };
  auto xt = [&](int lb) { return base + Lo::OFF_BUF + lb * Lo::kBuf; };
  auto bt = [&](int lb) { return xt(lb) + Lo::kX; };
  auto ct = [&](int lb) { return bt(lb) + Lo::kB; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, b = blockIdx.y;
  const int L = a.L;
  const int nk = (L + Q - 1) / Q;
  const int g = h / (a.H / a.Gbc);

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    int counts[NBAR];
    for (int i = 0; i < NBAR; ++i) counts[i] = 1;
    for (int i = 0; i < kMaxBuf; ++i) counts[B_FULL0 + i] = 4;
    counts[B_S_READY0] = counts[B_S_READY0 + 1] = 8;
    counts[B_Y_EMPTY0] = counts[B_Y_EMPTY0 + 1] = counts[B_PWG] = 4;
    // four warps copy the state, two write X'
    counts[B_ST_READY] = 4;
    counts[B_XP_READY0] = counts[B_XP_READY0 + 1] = 2;
    for (int i = 0; i < NBAR; ++i) mbar_init(bar(i), counts[i]);
    mbar_fence_init();
  }
  if (NN == 64) {
    for (int i = threadIdx.x; i < 1024; i += kThreads)
      st_shared_v4(base + Lo::OFF_ZERO + i * 16, make_uint4(0u, 0u, 0u, 0u));
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
    // One thread polls the barriers and issues whichever MMA group is ready:
    // CB of chunk `ncb` (at most one chunk ahead of the Y / state group), or
    // Y and the state update of chunk `ny`.
    if (lane == 0) {
      constexpr uint32_t ID_CB = idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t ID_Y = idesc_bf16(128, PP, 0, 1);
      constexpr uint32_t ID_ST = idesc_bf16(128, PP, 1, 1);
      // With two H buffers the state update of chunk c runs as soon as the
      // state is decayed and X' written, ahead of Y (which reads H); with one,
      // after Y.  The load buffer is released once both were issued.
      constexpr int NH = Lo::NH;
      int ncb = 0, ny = 0, nst = 0;
      long long t0 = clock64();
      while (ny < nk || nst < nk) {
        bool progress = false;
        if (ncb < nk && ncb <= ny + 1) {
          const int lb = ncb % NBUF, j = ncb & 1;
          if (mbar_test(bar(B_FULL0 + lb), (ncb / NBUF) & 1) &&
              (ncb < 2 || mbar_test(bar(B_CB_FREE0 + j), ((ncb >> 1) - 1) & 1))) {
            ALLOY_SCAN_TRACE(2, ncb);
            tc_fence_after();
            // K = d_state in 64-column swizzle blocks of 4 K16 steps (32 bytes apart)
#pragma unroll
            for (int kb = 0; kb < NN / 64; ++kb)
              umma_bf16_chain4<2, 2, sw128_hi(1024), sw128_hi(1024)>(
                  tmem + Lo::T_CB + 128 * j, sw128_lo(ct(lb) + kb * 16384, 16), sw128_lo(bt(lb) + kb * 16384, 16),
                  ID_CB, kb != 0);
            umma_commit(bar(B_CB_FULL0 + j));
            ++ncb;
            progress = true;
          }
        }
        if (nst < nk && (NH == 2 || ny > nst)) {
          const int c = nst, lb = c % NBUF, xb = c % Lo::NXP;
          if (mbar_test(bar(B_ST_READY), c & 1) && mbar_test(bar(B_XP_READY0 + xb), (c / Lo::NXP) & 1)) {
            tc_fence_after();
            // state[n, p] += sum_s B[s, n] X'[s, p]; rows n >= NN of A read the zero block
            const uint32_t lbo = NN == 64 ? Lo::OFF_ZERO - (bt(lb) - base) : 16384;
            const uint32_t sxp = base + Lo::OFF_XP + xb * Lo::kXPB;
            umma_bf16_chain8<128, 128, sw128_hi(1024), sw128_hi(1024)>(tmem + Lo::T_ST, sw128_lo(bt(lb), lbo),
                                                                        sw128_lo(sxp, 16384), ID_ST, 1);
            if (SPLIT)
              umma_bf16_chain8<128, 128, sw128_hi(1024), sw128_hi(1024)>(tmem + Lo::T_ST, sw128_lo(bt(lb), lbo),
                                                                          sw128_lo(sxp + Lo::kX, 16384), ID_ST, 1);
            umma_commit(bar(B_ST_DONE));
            if (ny > c) umma_commit(bar(B_EMPTY0 + lb));
            ++nst;
            progress = true;
          }
        }
        if (ny < ncb && (NH == 1 || nst > ny)) {
          const int c = ny, lb = c % NBUF, j = c & 1, yb = c % NYB;
          if (mbar_test(bar(B_S_READY0 + j), (c >> 1) & 1) &&
              (NH == 2 || mbar_test(bar(B_ST_READY), c & 1)) &&
              (c < NYB || mbar_test(bar(B_Y_EMPTY0 + yb), ((c / NYB) - 1) & 1))) {
            ALLOY_SCAN_TRACE(3, c);
            tc_fence_after();
            // Y = S x + C~ H
            const uint32_t ty = tmem + Lo::T_Y + yb * PP, tcb = tmem + Lo::T_CB + 128 * j;
            const uint32_t sh = base + Lo::OFF_H + (c % NH) * Lo::kHB;
            umma_bf16_ta_chain8<16, 128, sw128_hi(1024)>(ty, tcb, sw128_lo(xt(lb), 16384), ID_Y, 0);
            if (SPLIT) umma_bf16_ta_chain8<16, 128, sw128_hi(1024)>(ty, tcb + 8, sw128_lo(xt(lb), 16384), ID_Y, 1);
            const uint32_t tct = SPLIT ? tmem + Lo::T_CT + NN * j : tcb + 8;
            constexpr int CT_COLS = SPLIT ? 8 : 16;
            if (NN == 128) {
              umma_bf16_ta_chain8<CT_COLS, 128, sw128_hi(1024)>(ty, tct, sw128_lo(sh, NN * 128), ID_Y, 1);
            } else {
              umma_bf16_ta_chain4<CT_COLS, 128, sw128_hi(1024)>(ty, tct, sw128_lo(sh, NN * 128), ID_Y, 1);
              if (SPLIT) {
                // C~_lo H_hi + C~_hi H_lo (the lo x lo product is below the fp32 sums' precision)
                umma_bf16_ta_chain4<8, 128, sw128_hi(1024)>(ty, tct + NN / 2, sw128_lo(sh, NN * 128), ID_Y, 1);
                umma_bf16_ta_chain4<8, 128, sw128_hi(1024)>(ty, tct, sw128_lo(sh + Lo::kH, NN * 128), ID_Y, 1);
              }
            }
            umma_commit(bar(B_Y_FULL0 + yb));
            umma_commit(bar(B_CB_FREE0 + j));
            if (nst > c) umma_commit(bar(B_EMPTY0 + lb));
            ALLOY_SCAN_TRACE(5, c);
            ++ny;
            progress = true;
          }
        }
        if (progress) {
          t0 = clock64();
        } else {
          if (*abort_flag) break;
          if (clock64() - t0 > kWaitCycles) {
            signal_abort(abort_flag, 1);
            break;
          }
          __nanosleep(32);
        }
      }
      // wait (bounded) for every MMA this thread issued
      umma_commit(bar(B_DRAIN));
      const long long t1 = clock64();
      while (!mbar_try_wait(bar(B_DRAIN), 0) && clock64() - t1 < kWaitCycles) {
      }
    }
  } else if (warp >= kLoadWarp0 && warp < kLoadWarp0 + 4) {
    // ------------------------------------------------------------------ loads
    const int i = threadIdx.x - 32 * kLoadWarp0;
    const int xh = a.x_hpg > 1 ? h / a.x_hpg : h;
    const __nv_bfloat16* xs = static_cast<const __nv_bfloat16*>(a.x) + (int64_t)b * a.x_sb + (int64_t)xh * a.x_sh;
    const __nv_bfloat16* bs = static_cast<const __nv_bfloat16*>(a.Bm) + (int64_t)b * a.bm_sb + (int64_t)g * a.bm_sg;
    const __nv_bfloat16* cs = static_cast<const __nv_bfloat16*>(a.Cm) + (int64_t)b * a.cm_sb + (int64_t)g * a.cm_sg;
    // rows of a chunk a few chunks ahead into L2, so that the loads of a
    // buffer, which wait for that buffer's last MMA, find them there
    auto prefetch = [&](int cc) {
      const int t = cc * Q + i;
      if (cc >= nk || t >= L) return;
      const char* rows[3] = {reinterpret_cast<const char*>(xs + (int64_t)t * a.x_st),
                             reinterpret_cast<const char*>(bs + (int64_t)t * a.bm_st),
                             reinterpret_cast<const char*>(cs + (int64_t)t * a.cm_st)};
      const int bytes[3] = {PP * 2, NN * 2, NN * 2};
#pragma unroll
      for (int m = 0; m < 3; ++m)
        for (int o = 0; o < bytes[m] + 127; o += 128) prefetch_l2(rows[m] + min(o, bytes[m] - 1));
      if (a.log_a) prefetch_l2(a.log_a + (int64_t)b * a.la_sb + (int64_t)t * a.la_st + (int64_t)h * a.la_sh);
    };
    for (int cc = 1; cc < kL2Ahead; ++cc) prefetch(cc);
    for (int c = 0; c < nk; ++c) {
      const int lb = c % NBUF;
      prefetch(c + kL2Ahead);
      if (c >= NBUF && !waitw(bar(B_EMPTY0 + lb), ((c / NBUF) - 1) & 1, abort_flag, 10)) break;
      if (warp == kLoadWarp0) ALLOY_SCAN_TRACE(0, c);
      const int row0 = c * Q;
      load_rows<PP>(xt(lb), xs, a.x_st, row0, L, i);
      load_rows<NN>(bt(lb), bs, a.bm_st, row0, L, i);
      load_rows<NN>(ct(lb), cs, a.cm_st, row0, L, i);
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
        // cum[t] = inclusive sum of la over the chunk, while the copies fly
        float v = la;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float u = __shfl_up_sync(0xffffffffu, v, o);
          if (lane >= o) v += u;
        }
        // warp totals: wsum[lb] for chunk c+NBUF is written only after every
        // loader warp passed the PWG wait of chunk c+1, which follows its reads
        const int ql = warp - kLoadWarp0;
        if (lane == 31) wsum[lb * 4 + ql] = v;
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_PWG));
        if (!waitw(bar(B_PWG), c & 1, abort_flag, 11)) break;
        float pre = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) pre += k < ql ? wsum[lb * 4 + k] : 0.f;
        const float cum = v + pre;
        // column factor of source s = i inside its 16-column piece: exp(cum[m] -
        // cum[s]) <= 1, m the piece's last column (decays <= 1)
        const float cum_m = __shfl_sync(0xffffffffu, cum, lane | 15);
        cum_s[lb * 128 + i] = cum;
        cf_s[lb * 128 + i] = ex2_approx((cum_m - cum) * kLog2e);
      }
      cp_async_wait_all();
      fence_async_smem();
      __syncwarp();
      if (warp == kLoadWarp0) ALLOY_SCAN_TRACE(1, c);
      if (lane == 0) mbar_arrive(bar(B_FULL0 + lb));
    }
    cp_async_wait_all();
  } else if (warp < kStateWarp0) {
    // ------------------------------------------------------------------ scores
    // Two warps a lane quadrant: `half` 0 (warps 0-3) takes the even
    // 16-column pieces of the row, half 1 the odd ones, and each stores its S
    // and C~ K-steps inside pieces it read itself.
    const int t = r, half = warp >> 2;
    for (int c = 0; c < nk; ++c) {
      const int lb = c % NBUF, j = c & 1;
      if (!waitw(bar(B_FULL0 + lb), (c / NBUF) & 1, abort_flag, 22)) break;
      if (warp == 3) ALLOY_SCAN_TRACE(6, c);
      if (!waitw(bar(B_CB_FULL0 + j), (c >> 1) & 1, abort_flag, 23)) break;
      if (warp == 3) ALLOY_SCAN_TRACE(7, c);
      tc_fence_after();
      const float* cm = cum_s + lb * 128;
      const float* cf = cf_s + lb * 128;
      const float ct2 = cm[t] * kLog2e;
      const uint32_t tcb = lane_base + Lo::T_CB + 128 * j;
      // S[t, s] = CB[t, s] exp(cum[t] - cum[s]) (s <= t) for piece k -> columns [16k, 16k+8)
      auto score = [&](int k, const uint32_t (&rv)[16]) {
        float v[16];
        float own = 0.f;   // S[t,t] before rounding
        if (k < 2 * q) {
          // left of the quadrant's diagonal block: exp(cum[t] - cum[s]) = R cf[s],
          // R = exp(cum[t] - cum[m]) <= 1
          const uint64_t R2 = f2_splat(ex2_approx(fmaf(-cm[16 * k + 15], kLog2e, ct2)));
          const float4* cf4 = reinterpret_cast<const float4*>(cf + 16 * k);
#pragma unroll
          for (int i4 = 0; i4 < 4; ++i4) {
            const float4 f = cf4[i4];
            f2_unpack(f2_mul(f2_mul(f2_pack(__uint_as_float(rv[4 * i4]), __uint_as_float(rv[4 * i4 + 1])), R2),
                             f2_pack(f.x, f.y)), v[4 * i4], v[4 * i4 + 1]);
            f2_unpack(f2_mul(f2_mul(f2_pack(__uint_as_float(rv[4 * i4 + 2]), __uint_as_float(rv[4 * i4 + 3])), R2),
                             f2_pack(f.z, f.w)), v[4 * i4 + 2], v[4 * i4 + 3]);
          }
        } else {
          // the diagonal block: exact factors, zero right of the diagonal
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int s = 16 * k + e;
            const float f = __uint_as_float(rv[e]) * ex2_approx(fmaf(-cm[s], kLog2e, ct2));
            v[e] = s <= t ? f : 0.f;
            if (s == t) own = f;
          }
        }
        uint32_t o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
        // S[t,t] as rounded, for the output rows (slot c % 4: the rows of chunk c
        // are read out before the scores of chunk c + 4 start)
        if (!SPLIT && k >= 2 * q && (t >> 4) == k)
          diag_s[(c & 3) * 128 + t] = __bfloat162float(__float2bfloat16_rn(own));
        tmem_st8(tcb + 16 * k, o);
        if (SPLIT) {
          // the remainder, v - bf16(v), as a second bf16 K-step
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = pack_bf16x2(v[2 * e] - bf16_lo(o[e]), v[2 * e + 1] - bf16_hi(o[e]));
          tmem_st8(tcb + 16 * k + 8, o);
        }
      };
      // this warp's pieces at or left of the quadrant's diagonal: k = half, half + 2, .., 2q + half
      uint32_t ra[16], rb[16];
      tmem_ld16(tcb + 16 * half, ra);
#pragma unroll 1
      for (int jj = 0; jj <= q; jj += 2) {
        const int k = 2 * jj + half;
        tmem_ld_wait_regs(ra);
        if (jj + 1 <= q) tmem_ld16(tcb + 16 * (k + 2), rb);
        score(k, ra);
        if (jj + 1 > q) break;
        tmem_ld_wait_regs(rb);
        if (jj + 2 <= q) tmem_ld16(tcb + 16 * (k + 4), ra);
        score(k + 2, rb);
      }
      {
        uint32_t z[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) z[e] = 0u;
#pragma unroll 1
        for (int k = 2 * (q + 1) + half; k < 8; k += 2) {
          tmem_st8(tcb + 16 * k, z);
          if (SPLIT) tmem_st8(tcb + 16 * k + 8, z);
        }
      }
      // C~ = exp(cum[t]) C[t, :]: K-step k of the C~ H product -> columns [16k+8, 16k+16)
      {
        const uint64_t e2 = f2_splat(ex2_approx(ct2));
        const uint32_t crow = ct(lb);
#pragma unroll 1
        for (int k = half; k < NN / 16; k += 2) {
          uint32_t o[8], ol[8];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int jc = 2 * k + hh;   // 16-byte chunk of the row
            const uint4 w = ld_shared_v4(crow + (jc >> 3) * 16384 + sw_off(t, jc & 7));
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int m = 0; m < 4; ++m) {
              float lo, hi;
              f2_unpack(f2_mul(f2_from_bf2(ww[m]), e2), lo, hi);
              o[4 * hh + m] = pack_bf16x2(lo, hi);
              if (SPLIT) ol[4 * hh + m] = pack_bf16x2(lo - bf16_lo(o[4 * hh + m]), hi - bf16_hi(o[4 * hh + m]));
            }
          }
          if (SPLIT) {
            tmem_st8(lane_base + Lo::T_CT + NN * j + 8 * k, o);
            tmem_st8(lane_base + Lo::T_CT + NN * j + NN / 2 + 8 * k, ol);
          } else {
            tmem_st8(tcb + 16 * k + 8, o);
          }
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (warp == 3) ALLOY_SCAN_TRACE(8, c);
      if (warp == 7) ALLOY_SCAN_TRACE(9, c);
      if (warp == 0) ALLOY_SCAN_TRACE(14, c);
      if (lane == 0) mbar_arrive(bar(B_S_READY0 + j));
    }
  } else if (warp < kOutWarp0 || warp >= kStateWarpX0) {
    // ------------------------------------------------------------------ state and X'
    // Four warps copy and decay the state, two write X'.  d_state 64 (state
    // rows in lanes 0-63): warps 8 and 20 (quadrant 0) and 9 and 21 (quadrant 1)
    // take half of the columns each, warps 10-11 write X'.  d_state 128: warps
    // 8-11 take whole rows, warps 20-21 write X'.  X' rows: two a thread.
    const bool extra = warp >= kStateWarpX0;
    const bool h_role = NN == 64 ? (q < 2) : !extra;
    const bool xp_role = !h_role;
    const int p_lo = NN == 64 ? (extra ? PP / 2 : 0) : 0;
    const int p_hi = NN == 64 ? (extra ? PP : PP / 2) : PP;
    const int xq = NN == 64 ? q - 2 : q;   // X' warps: quadrants 2-3 (d_state 64) or 0-1 (128)
    // initial state: each copy warp its own columns; for d_state 64 warps
    // 10-11 zero the unused rows 64-127 (ordered before the first state update
    // by their X' barrier)
    if (h_role || (NN == 64 && !extra)) {
#pragma unroll 1
      for (int p0 = h_role ? p_lo : 0; p0 < (h_role ? p_hi : PP); p0 += 16) {
        uint32_t v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          float f = 0.f;
          if (r < NN && a.ssm_in)
            f = a.ssm_in[(int64_t)b * a.si_sb + (int64_t)h * a.si_sh + (int64_t)r * a.si_sn + (int64_t)(p0 + k) * a.si_sp];
          v[k] = __float_as_uint(f);
        }
        tmem_st16(lane_base + Lo::T_ST + p0, v);
      }
      tmem_st_wait();
    }
    for (int c = 0; c < nk; ++c) {
      const int lb = c % NBUF, xb = c % Lo::NXP;
      if (!waitw(bar(B_FULL0 + lb), (c / NBUF) & 1, abort_flag, 31)) break;
      const float* cm = cum_s + lb * 128;
      const float last = cm[127];
      if (xp_role) {
        // X'[s, :] = exp(cum[Q-1] - cum[s]) x[s, :] into buffer c % NXP, once the
        // state update that read that buffer (chunk c - NXP) has completed
        if (c >= Lo::NXP &&
            !waitw(bar(B_EMPTY0 + (c - Lo::NXP) % NBUF), ((c - Lo::NXP) / NBUF) & 1, abort_flag, 33))
          break;
        const uint32_t src = xt(lb), dst = base + Lo::OFF_XP + xb * Lo::kXPB;
#pragma unroll 1
        for (int rr = 0; rr < 2; ++rr) {
          const int s = xq * 32 + lane + 64 * rr;
          const uint64_t w2 = f2_splat(ex2_approx((last - cm[s]) * kLog2e));
#pragma unroll
          for (int jc = 0; jc < PP / 8; ++jc) {
            const uint32_t off = (jc >> 3) * 16384 + sw_off(s, jc & 7);
            const uint4 u = ld_shared_v4(src + off);
            const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
              float lo, hi;
              f2_unpack(f2_mul(f2_from_bf2(uw[m]), w2), lo, hi);
              hw[m] = pack_bf16x2(lo, hi);
              if (SPLIT) lw[m] = pack_bf16x2(lo - bf16_lo(hw[m]), hi - bf16_hi(hw[m]));
            }
            st_shared_v4(dst + off, make_uint4(hw[0], hw[1], hw[2], hw[3]));
            if (SPLIT) st_shared_v4(dst + Lo::kX + off, make_uint4(lw[0], lw[1], lw[2], lw[3]));
          }
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_XP_READY0 + xb));
      } else {
        // the previous state update has completed, and (two H buffers) the Y
        // that read this chunk's H buffer (chunk c - 2)
        if (c > 0 && !waitw(bar(B_ST_DONE), (c - 1) & 1, abort_flag, 32)) break;
        if (Lo::NH == 2 && c >= 2 && !waitw(bar(B_CB_FREE0 + (c & 1)), ((c - 2) >> 1) & 1, abort_flag, 35)) break;
        if (warp == kStateWarp0) ALLOY_SCAN_TRACE(10, c);
        tc_fence_after();
        const float e = ex2_approx(last * kLog2e);
        const uint32_t hrow = base + Lo::OFF_H + (c % Lo::NH) * Lo::kHB;
        auto copy = [&](int p0, uint32_t (&v)[16]) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int jc = p0 / 8 + hh;   // 16-byte chunk of the state row (8 p)
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
              const float lo = __uint_as_float(v[8 * hh + 2 * m]), hi = __uint_as_float(v[8 * hh + 2 * m + 1]);
              hw[m] = pack_bf16x2(lo, hi);
              if (SPLIT) lw[m] = pack_bf16x2(lo - bf16_lo(hw[m]), hi - bf16_hi(hw[m]));
            }
            const uint32_t off = (jc >> 3) * (NN * 128) + sw_off(r, jc & 7);
            st_shared_v4(hrow + off, make_uint4(hw[0], hw[1], hw[2], hw[3]));
            if (SPLIT) st_shared_v4(hrow + Lo::kH + off, make_uint4(lw[0], lw[1], lw[2], lw[3]));
          }
#pragma unroll
          for (int k = 0; k < 16; ++k) v[k] = __float_as_uint(e * __uint_as_float(v[k]));
          tmem_st16(lane_base + Lo::T_ST + p0, v);
        };
        // two 16-column pieces in flight
#pragma unroll 1
        for (int p0 = p_lo; p0 < p_hi; p0 += 32) {
          uint32_t va[16], vb[16];
          tmem_ld16(lane_base + Lo::T_ST + p0, va);
          tmem_ld16(lane_base + Lo::T_ST + p0 + 16, vb);
          tmem_ld_wait_regs(va);
          tmem_ld_wait_regs(vb);
          copy(p0, va);
          copy(p0 + 16, vb);
        }
        fence_async_smem();
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (warp == kStateWarp0) ALLOY_SCAN_TRACE(11, c);
        if (lane == 0) mbar_arrive(bar(B_ST_READY));
      }
    }
    // the final state
    if (h_role && !*abort_flag && a.ssm_out && nk > 0 && waitw(bar(B_ST_DONE), (nk - 1) & 1, abort_flag, 34)) {
      tc_fence_after();
      {
#pragma unroll 1
        for (int p0 = p_lo; p0 < p_hi; p0 += 16) {
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
      const int yb = c % Lo::NYB;
      if (!waitw(bar(B_Y_FULL0 + yb), (c / Lo::NYB) & 1, abort_flag, 40)) break;
      if (warp == kOutWarp0) ALLOY_SCAN_TRACE(12, c);
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
      if (a.dot && t < L) {
        if (a.dot_nodiag) {
          // leave out S[t,t] (x_t . z_t), the step's own term as the MMA saw it
          const int xh = a.x_hpg > 1 ? h / a.x_hpg : h;
          const uint4* xp = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.x) + (int64_t)b * a.x_sb +
                                                           (int64_t)t * a.x_st + (int64_t)xh * a.x_sh);
          float xz = 0.f;
#pragma unroll 2
          for (int m = 0; m < PP / 8; ++m) {
            const uint4 xx = __ldg(xp + m);
            const uint32_t xw[4] = {xx.x, xx.y, xx.z, xx.w};
            float zf[8];
            if (a.z_bf16) {
              const uint4 zz = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.z) + zoff) + m);
              const uint32_t zw[4] = {zz.x, zz.y, zz.z, zz.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) { zf[2 * e] = bf16_lo(zw[e]); zf[2 * e + 1] = bf16_hi(zw[e]); }
            } else {
              const float4* zp = reinterpret_cast<const float4*>(static_cast<const float*>(a.z) + zoff) + 2 * m;
              const float4 z0 = __ldg(zp), z1 = __ldg(zp + 1);
              zf[0] = z0.x; zf[1] = z0.y; zf[2] = z0.z; zf[3] = z0.w;
              zf[4] = z1.x; zf[5] = z1.y; zf[6] = z1.z; zf[7] = z1.w;
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              xz = fmaf(bf16_lo(xw[e]), zf[2 * e], xz);
              xz = fmaf(bf16_hi(xw[e]), zf[2 * e + 1], xz);
            }
          }
          dot = fmaf(-diag_s[(c & 3) * 128 + r], xz, dot);
        }
        a.dot[(int64_t)b * a.dot_sb + (int64_t)t * a.dot_st + (int64_t)h * a.dot_sh] = dot;
      }
      tc_fence_before();
      __syncwarp();
      if (warp == kOutWarp0) ALLOY_SCAN_TRACE(13, c);
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
  if (a.precise_scores && (a.P != 64 || a.N != 64)) return false;
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
  if (a.precise_scores) return launch(scan_tc_kernel<64, 64, true>, Layout<64, 64, true>::kSmem);
  if (a.P == 64 && a.N == 64) return launch(scan_tc_kernel<64, 64, false>, Layout<64, 64>::kSmem);
  if (a.P == 64) return launch(scan_tc_kernel<64, 128, false>, Layout<64, 128>::kSmem);
  return launch(scan_tc_kernel<128, 64, false>, Layout<128, 64>::kSmem);
}

int scan_tc_take_error(cudaStream_t stream, unsigned int out[3]) {
  ALLOY_CUDA(cudaStreamSynchronize(stream));
  unsigned int zero[3] = {0, 0, 0};
  ALLOY_CUDA(cudaMemcpyFromSymbol(out, g_scan_tc_error, sizeof(zero)));
  if (out[0] != 0) ALLOY_CUDA(cudaMemcpyToSymbol(g_scan_tc_error, zero, sizeof(zero)));
  return ALLOY_OK;
}

}  // namespace alloy
