// Tensor-core (tcgen05) chunked SSD for bf16 activations: the fused prefill
// of alloy/models/mamba_block.py:446-493 (conv + SiLU, discretisation,
// _selective_scan / _scan_chunk :206-366, D skip).
//
// Two launches per call:
//  1. bc_conv_kernel: conv1d + SiLU of the B and C columns of the selected
//     head groups -> bf16 workspace of 16 KB tiles, each a [128 rows][64
//     columns] half of B or C of one (batch row, chunk, group) laid out as the
//     SSD kernel's shared memory holds it (128-byte swizzle), so the kernel
//     fetches a chunk's B/C with plain bulk copies.  Every head of a group
//     reads the same B/C, so they are produced once instead of once per head
//     pair.
//  2. ssd_tc_kernel: one CTA per (batch row, pair of heads of one group),
//     walking chunks of Q = 128 steps in order with the fp32 state resident in
//     tensor memory.  Per chunk (t, s in [0, Q); p < P = 64; n < N):
//        cum[t]  = sum_{u<=t} A dt_u                      (fp32, per head)
//        CB      = C B^T                                  (tcgen05, TMEM)
//        S[t,s]  = CB[t,s] exp(cum[t]-cum[s]) dt_s  (s<=t), + D on s==t
//        Y       = S X                                    (tcgen05)
//        Yi      = C H^T,  H = bf16(state) before this chunk
//        y[t]    = Y[t] + exp(cum[t]) Yi[t]               (epilogue, bf16)
//        state   = exp(cum[Q-1]) state + X'^T B,  X'[s] = X[s] dt_s exp(cum[Q-1]-cum[s])
//     X is the unscaled conv+SiLU output of the pair's x channels (bf16,
//     produced in the CTA); B/C tiles arrive by bulk copy into a
//     two-stage ring of 64-column halves; raw x rows (with the 3-row conv
//     halo) arrive by TMA per head.  The state of both heads is one 128 x N
//     fp32 TMEM accumulator with rows (head, p): its update is a single
//     M = 128, N = d_state MMA chain.
//
// Warp roles: two consumer warpgroups (state copy, X', scores), two producer
// warpgroups (dt/cumsum, x conv, epilogue), a B/C TMA warp and an MMA warp;
// see the kernel.  Every mbarrier wait is bounded: on timeout the CTA records
// an error word, drains its in-flight copies and MMAs, frees its tensor memory
// and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <utility>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

// Phase markers: no code unless a timing build defines ALLOY_TRACE_POINT.
#ifndef ALLOY_TRACE_POINT
#define ALLOY_TRACE_POINT(role, chunk, id)
#endif
#ifndef ALLOY_TRACE_SPIN
#define ALLOY_TRACE_SPIN()
#endif
#ifndef ALLOY_TRACE_COPY_DONE
#define ALLOY_TRACE_COPY_DONE(bar, parity, role, chunk, id)
#endif
#ifndef ALLOY_TRACE_CTA_BEGIN
#define ALLOY_TRACE_CTA_BEGIN()
#define ALLOY_TRACE_CTA_END()
#endif

namespace alloy {

// error word written by a CTA whose bounded wait ran out (0 = none):
// [0] = 1 + site id, [1] = blockIdx.x, [2] = blockIdx.y
__device__ unsigned int g_ssd_tc_error[3];

namespace {

using namespace tc;

constexpr int Q = 128;                 // chunk length (UMMA M)
constexpr int P = 64;                  // head dim
constexpr int kThreads = 640;          // 20 warps: 4 compute warpgroups + 1 role warpgroup
// registers per thread after the split (launch: 640 x 96, i.e. 480 a thread
// summed over one thread of each of the five warpgroups): the full pass gives
// 2 x 120 to the producers, 2 x 88 to the consumers, 64 to the role warps; the
// state-only pass (producers: the conv alone, two chunks of x rows in
// registers; consumers: the dt scan) 2 x 144, 2 x 64 and 56
constexpr int kProducerRegs = 120;
constexpr int kConsumerRegs = 88;
constexpr int kRoleRegs = 64;
constexpr int kProducerRegsS = 144;
constexpr int kConsumerRegsS = 64;
constexpr int kRoleRegsS = 56;
// x conv + SiLU on packed f32x2 pairs: in the state-only pass (144 producer
// registers); the full pass keeps the scalar form, which fits its 120
#ifdef ALLOY_CONV_PACKED_ALL
constexpr bool kPackedConvAll = true;
#else
constexpr bool kPackedConvAll = false;
#endif
constexpr int kTmaWarp = 16;           // B/C half tiles
constexpr int kMmaWarp = 17;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kL2Ahead = 2;            // chunks of x and B/C prefetched into L2
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 1.9 GHz

// shared-memory map (bytes from the 1024-aligned base)
constexpr uint32_t kStageBytes = 32768;             // B half [128][64] + C half [128][64] bf16
constexpr uint32_t OFF_STAGE = 0;                   // 2 stages
constexpr uint32_t OFF_X = 65536;                   // X [2 buffers][2 heads][128 s][64 p] bf16
constexpr uint32_t OFF_H = 131072;                  // H [N/64 blocks][2 heads][64 p][64 n] bf16
constexpr uint32_t OFF_XP = 163840;                 // X' [2 heads][128 s][64 p] bf16
constexpr uint32_t OFF_MISC = 196608;
constexpr uint32_t OFF_CUM = OFF_MISC;              // [2 buffers][2 heads][128] f32
constexpr uint32_t OFF_DT = OFF_CUM + 2048;         // [2][2][128]
constexpr uint32_t OFF_CF = OFF_DT + 2048;          // [2][2][128] column factors
constexpr uint32_t OFF_WSUM = OFF_CF + 2048;        // [2 buffers][2 heads][4 warps]
constexpr uint32_t OFF_CW = OFF_WSUM + 64;          // x conv weights [2][4][16][4] + bias [2][16][4]
constexpr uint32_t OFF_XF = OFF_CW + 2560;          // X' row factors [2 heads][128]
constexpr uint32_t OFF_BAR = OFF_XF + 1024;         // mbarriers (8 bytes each)
constexpr int NBAR = 18;
constexpr uint32_t OFF_TMEMPTR = OFF_BAR + NBAR * 8;
constexpr uint32_t OFF_ABORT = OFF_TMEMPTR + 8;
constexpr uint32_t kSmemBytes = OFF_ABORT + 16 + 1024;  // + alignment slack

// barrier ids (counts in the kernel's init table)
enum {
  B_FULL0 = 0, B_FULL1, B_EMPTY0, B_EMPTY1,   // B/C stage ring (copies <-> MMA)
  B_X_READY0, B_X_READY1,                     // producers -> consumers, MMA: X, X', cum, dt, cf (per buffer)
  B_CB_FULL,                                  // MMA -> consumers: CB in TMEM
  B_HBF_READY,                                // consumers -> MMA: H written, state scaled
  B_S_READY,                                  // consumers -> MMA: scores in TMEM
  B_Y_FULL,                                   // MMA -> producers: Y and Yi complete
  B_ST_DONE,                                  // MMA -> producers: state update done (X' reusable)
  B_YI_DONE,                                  // MMA -> consumers: Yi done (H reusable; state update done)
  B_Y_EMPTY0, B_Y_EMPTY1,                     // producers -> MMA: y read out (per buffer)
  B_PWG0, B_PWG1,                             // producer warpgroup syncs
  B_DRAIN,
  B_NEVER                                     // nothing arrives: the wait-expiry test hook waits here
};
static_assert(B_NEVER + 1 == NBAR, "barrier table");
// the state-only pass reuses barriers only the full pass needs otherwise
constexpr int B_XF_FULL0 = B_HBF_READY;   // consumers -> producers: X' row factors of a chunk (per buffer)
constexpr int B_XF_EMPTY0 = B_ST_DONE;    // producers -> consumers: row factors read (per buffer)
constexpr int B_XP_FREE0 = B_Y_EMPTY0;    // MMA -> producers: X' buffer read (per buffer)
constexpr int B_ST_FINAL = B_Y_FULL;      // MMA -> consumers: the segment's end state complete
static_assert(B_XF_FULL0 + 1 == B_S_READY && B_XF_EMPTY0 + 1 == B_YI_DONE && B_XP_FREE0 + 1 == B_Y_EMPTY1,
              "paired barriers");

// TMEM columns
constexpr uint32_t T_CB = 0;      // CB [128 t][128 s] f32, overwritten in place by the scores
constexpr uint32_t T_ST = 128;    // state [128 (h,p)][N] f32
constexpr uint32_t T_Y = 256;     // + 64 h
constexpr uint32_t T_YI = 384;    // + 64 h

struct TcArgs {
  int B, L, H, N, G, K;
  int head_begin, group_begin, group_count;
  const __nv_bfloat16* xbc; int64_t x_sb, x_st;
  const void* dt; int dt_bf16; int64_t dt_sb, dt_st, dt_sh;
  const float* conv_w; int64_t cw_sc, cw_sk;
  const float* conv_b; int64_t cb_s;
  const float* dt_bias; int64_t dtb_s;
  const float* A_log; int64_t al_s;
  const float* Dp; int64_t d_s;
  const __nv_bfloat16* conv_in; int64_t ci_sb, ci_sk, ci_sc;
  const float* ssm_in; int64_t si_sb, si_sh, si_sn, si_sp;
  float* ssm_out; int64_t so_sb, so_sh, so_sn, so_sp;
  __nv_bfloat16* y; int64_t y_sb, y_st, y_sh;
  const __nv_bfloat16* bc;   // B/C tile workspace
  // sequence segments (gridDim.z of the full kernel): segment s of a (batch
  // row, head pair) covers chunks [s nchunks / nseg, (s+1) nchunks / nseg)
  int nseg;
  // [B][head pairs][nseg][128 (h,p)][N]: the state-only pass writes record
  // s + 1 = the end state of segment s walked from zero (s < nseg - 1);
  // seg_carry_kernel then turns record s into the state carried into
  // segment s (record 0 the call's initial state)
  float* seg_state;
  float* seg_logdecay;       // [B][head pairs][nseg][2]: sum of A dt over segment s, per head
  // split walk (split_units > 0): the nseg segments of every (batch row, head
  // pair) unit are walked one after another by successive launches, each CTA
  // of a launch one (unit, segment) task: task split_base + blockIdx.x is
  // segment tau / split_units of unit tau % split_units (unit = b * pairs +
  // pair).  Segment s > 0 starts from the end state of segment s - 1, handed
  // over exactly (fp32) in the unit's record [128 (h,p)][N] of seg_state.
  int split_units, split_base, pairs;
  // state-only pieces: each of segments 0..nseg-2 is walked by `pieces` CTAs of
  // the state-only pass (piece p: part p % pieces of segment p / pieces), so
  // that pass fills more SMs; a unit then has nrec = (nseg - 1) pieces + 1
  // records, the carry scans over pieces and the full pass's segment s starts
  // from record s * pieces
  int pieces, nrec;
  // > 0 only in a test of the bounded-wait error path: the consumer warps
  // first wait this many cycles on B_NEVER, which nothing completes
  long long stall_cycles;
};

#ifdef ALLOY_SOFTPLUS_LIB
#define ALLOY_SOFTPLUS softplus_f32
#else
#define ALLOY_SOFTPLUS softplus_fast
#endif
// softplus(x) = max(x, 0) + ln(1 + e^-|x|) from the hardware base-2
// exponential and logarithm (relative error ~1e-7 where the result is not
// tiny; for x < -17 the e^x term is below fp32 resolution next to 1 and the
// result is 0 instead of ~e^x, an absolute error below 4e-8)
__device__ __forceinline__ float softplus_fast(float x) {
  float l;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(l) : "f"(1.f + ex2_approx(-fabsf(x) * 1.4426950408889634f)));
  return fmaxf(x, 0.f) + 0.6931471805599453f * l;
}

// ----------------------------------------------------------------------------
// bounded waits
// ----------------------------------------------------------------------------
__device__ __forceinline__ void signal_abort(volatile int* abort_flag, int site) {
  *abort_flag = 1;
  if (atomicCAS(&g_ssd_tc_error[0], 0u, 1u + site) == 0u) {
    g_ssd_tc_error[1] = blockIdx.x;
    g_ssd_tc_error[2] = blockIdx.y;
  }
}

// single-thread wait (TMA / MMA roles)
__device__ __forceinline__ bool wait1(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                      int site) {
  const long long t0 = clock64();
  for (uint32_t it = 0; it < (1u << 30); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    ALLOY_TRACE_SPIN();
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) break;
  }
  signal_abort(abort_flag, site);
  return false;
}

// warp-uniform wait: every lane polls (bounded by the clock limit and the
// CTA's abort flag), then one vote makes the outcome the same on all lanes
__device__ __forceinline__ bool waitw(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                      int site, long long limit = kWaitCycles) {
  const long long t0 = clock64();
  bool ok;
  while (!(ok = mbar_try_wait(bar, parity) != 0)) {
    ALLOY_TRACE_SPIN();
    if (*abort_flag || clock64() - t0 > limit) break;
  }
  ok = __all_sync(0xffffffffu, ok);
  if (!ok && (threadIdx.x & 31) == 0 && !*abort_flag) signal_abort(abort_flag, site);
  __syncwarp();
  return ok;
}

// 16-byte chunk `chunk` (0..7) of row `row` in a 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// ----------------------------------------------------------------------------
// B/C conv + SiLU pre-pass
// ----------------------------------------------------------------------------
// Workspace: tiles bc[b][chunk][gl][k][part] of [128 rows][64 columns] bf16
// (16 KB), part 0 = B, 1 = C, k = 64-column half of the state index n,
// element (r, j) at byte r*128 + ((j/8 ^ r%8) * 16) + (j%8)*2 (the 128-byte
// swizzle of a K-major UMMA operand tile).  Rows past L are zeros.  Source
// column of (part, gl, n): H*P + part*G*N + (group_begin + gl)*N + n.
//
// One CTA per (run of a.bc_chunks consecutive chunks, W-column tile, batch row).
// Chunk i's rows [t0 - 3, t0 + kBcTileRows) of the tile's columns arrive by one
// tensor copy into one of two shared-memory buffers (rows outside [0, L) as
// zeros; rows before 0 are then taken from the conv cache): the copy of chunk
// i + 1 is in flight while chunk i is convolved.  Each thread convolves 8
// adjacent columns over a strip of rows with the last 3 inputs kept in
// registers.
constexpr int kBcTileRows = 128;   // one chunk

template <int W>   // tile width in columns: 128 or 64
__global__ void __launch_bounds__(256, 2)
bc_conv_kernel(const __grid_constant__ CUtensorMap src_map, const TcArgs a, __nv_bfloat16* __restrict__ bc,
               int ncols, int run) {
  constexpr int CG = W / 8;            // column groups of 8
  constexpr int R = kBcTileRows * CG / 256;   // rows per thread
  constexpr uint32_t kBuf = ((kBcTileRows + 3) * W * 2 + 1023) & ~1023u;   // buffers 1 KB aligned
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[2];
  __shared__ float4 taps_s[W];     // the tile's conv taps and bias, halved (silu(2h) = h + h tanh h)
  __shared__ float bias_s[W];
  const uint32_t stile = static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw));
  // the SSD kernel, launched programmatically after this one, may start its
  // prologue while this grid finishes (it waits before reading the workspace)
  pdl_trigger();
  const int b = blockIdx.z;
  const int j0 = blockIdx.y * W;
  const int span = a.group_count * a.N;
  const int part = j0 / span;
  const int src0 = a.H * P + part * a.G * a.N + a.group_begin * a.N + (j0 - part * span);
  const int nchunks = (a.L + Q - 1) / Q;
  const int chunk0 = blockIdx.x * run;
  const int nck = min(run, nchunks - chunk0);
  auto bar = [&](int i) { return static_cast<uint32_t>(__cvta_generic_to_shared(&full_bar[i])); };
  auto issue = [&](int i) {   // chunk chunk0 + i into buffer i & 1
    mbar_arrive_expect_tx(bar(i & 1), (kBcTileRows + 3) * W * 2);
    tma_load_3d(stile + (i & 1) * kBuf, &src_map, bar(i & 1), src0, (chunk0 + i) * kBcTileRows - 3, b);
  };
  if (threadIdx.x == 0) {
    mbar_init(bar(0), 1);
    mbar_init(bar(1), 1);
    mbar_fence_init();
    issue(0);
  }
  if (threadIdx.x < W) {   // one column each, consecutive threads on consecutive columns
    const int64_t ch = src0 + threadIdx.x;
    taps_s[threadIdx.x] = make_float4(0.5f * a.conv_w[ch * a.cw_sc], 0.5f * a.conv_w[ch * a.cw_sc + a.cw_sk],
                                      0.5f * a.conv_w[ch * a.cw_sc + 2 * a.cw_sk],
                                      0.5f * a.conv_w[ch * a.cw_sc + 3 * a.cw_sk]);
    bias_s[threadIdx.x] = a.conv_b ? 0.5f * a.conv_b[ch * a.cb_s] : 0.f;
  }
  __syncthreads();
  const int cg = threadIdx.x % CG, strip = threadIdx.x / CG;
  const int c = src0 + cg * 8;
  // this thread's 8 columns in the tile layout
  const int rem = j0 - part * span + cg * 8;   // gl * N + n
  const int gl = rem / a.N, n = rem % a.N;
  const int nn8 = (n % 64) / 8;   // 16-byte chunk of the row
  // halved taps and bias of this thread's 8 columns, as channel pairs
  uint64_t w2[4][4], b2[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 t0v = taps_s[cg * 8 + 2 * i], t1v = taps_s[cg * 8 + 2 * i + 1];
    w2[0][i] = f2_pack(t0v.x, t1v.x);
    w2[1][i] = f2_pack(t0v.y, t1v.y);
    w2[2][i] = f2_pack(t0v.z, t1v.z);
    w2[3][i] = f2_pack(t0v.w, t1v.w);
    b2[i] = f2_pack(bias_s[cg * 8 + 2 * i], bias_s[cg * 8 + 2 * i + 1]);
  }
  const int r0 = strip * R;            // first output row of this thread (tile-relative)
#pragma unroll 1
  for (int i = 0; i < nck; ++i) {
    const int chunk = chunk0 + i;
    const int t0 = chunk * kBcTileRows;
    // the next chunk's copy, into the buffer every thread finished reading
    // before the barrier that ended the previous iteration
    if (threadIdx.x == 0 && i + 1 < nck) {
      fence_async_smem();
      issue(i + 1);
    }
    // bounded wait for this chunk's tile; on timeout record the error and give
    // the copies in flight a second bounded period before the CTA leaves
    {
      const long long start = clock64();
      bool ok = false;
      while (!(ok = mbar_try_wait(bar(i & 1), (i >> 1) & 1)) && clock64() - start < kWaitCycles) {
      }
      if (!__syncthreads_and(ok)) {
        if (threadIdx.x == 0) {
          if (atomicCAS(&g_ssd_tc_error[0], 0u, 1u + 40u) == 0u) {
            g_ssd_tc_error[1] = blockIdx.x;
            g_ssd_tc_error[2] = blockIdx.y;
          }
          for (int k = i; k < min(i + 2, nck); ++k) {
            const long long again = clock64();
            while (!mbar_try_wait(bar(k & 1), (k >> 1) & 1) && clock64() - again < kWaitCycles) {
            }
          }
        }
        __syncthreads();
        return;
      }
    }
    const uint32_t col = stile + (i & 1) * kBuf + cg * 16;
    uint64_t win[3][4];
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      const int t = t0 + r0 - 3 + r;
      if (t >= 0) {
        uint32_t w0, w1, w2v, w3;
        asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(w0), "=r"(w1), "=r"(w2v), "=r"(w3) : "r"(col + (r0 + r) * (W * 2)));
        win[r][0] = f2_from_bf2(w0); win[r][1] = f2_from_bf2(w1);
        win[r][2] = f2_from_bf2(w2v); win[r][3] = f2_from_bf2(w3);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float f[2];
#pragma unroll
          for (int e = 0; e < 2; ++e)
            f[e] = a.conv_in ? __bfloat162float(a.conv_in[(int64_t)b * a.ci_sb + (int64_t)(a.K - 1 + t) * a.ci_sk +
                                                         (int64_t)(c + 2 * q + e) * a.ci_sc])
                             : 0.f;
          win[r][q] = f2_pack(f[0], f[1]);
        }
      }
    }
    const int64_t tile = ((((int64_t)b * nchunks + chunk) * a.group_count + gl) * (a.N / 64) + n / 64) * 2 + part;
    unsigned char* dst = reinterpret_cast<unsigned char*>(bc) + tile * 16384;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      uint32_t u0, u1, u2, u3;
      asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(u0), "=r"(u1), "=r"(u2), "=r"(u3) : "r"(col + (r0 + r + 3) * (W * 2)));
      const uint64_t x[4] = {f2_from_bf2(u0), f2_from_bf2(u1), f2_from_bf2(u2), f2_from_bf2(u3)};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint64_t acc = f2_fma(win[0][q], w2[0][q], b2[q]);
        acc = f2_fma(win[1][q], w2[1][q], acc);
        acc = f2_fma(win[2][q], w2[2][q], acc);
        acc = f2_fma(x[q], w2[3][q], acc);
        // acc = h = x/2: silu(x) = h + h tanh(h)
        float hl, hh;
        f2_unpack(acc, hl, hh);
        o[q] = t0 + r0 + r < a.L ? pack_bf16x2(fmaf(hl, tanh_approx(hl), hl), fmaf(hh, tanh_approx(hh), hh)) : 0u;
        win[0][q] = win[1][q];
        win[1][q] = win[2][q];
        win[2][q] = x[q];
      }
      const int row = r0 + r;
      *reinterpret_cast<uint4*>(dst + row * 128 + ((nn8 ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    __syncthreads();   // buffer i & 1 is free for chunk i + 2
  }
}

// ----------------------------------------------------------------------------
// state carried into each sequence segment
// ----------------------------------------------------------------------------
// Runs between the state-only pass and the full pass of a segmented call.
// Record 0 of a (batch row, head pair) becomes the call's initial state
// (ssm_in, zeros without one); record s, the end state of segment s-1 walked
// from zero, becomes the state carried into segment s:
//   rec[s] = exp(sum of A dt over segment s-1) rec[s-1] + rec[s],  s = 1 .. nseg-1,
// the chunk recurrence of alloy/models/mamba_block.py:340-357 at segment
// granularity, computed as an fp32 associative scan over the segments with
// warp shuffles.  Segment s contributes the affine map h -> d_s h + r_s
// (d_0 = 0, r_0 = the initial state; d_s = exp(log decay of segment s-1),
// r_s = record s); composing (d2, r2) o (d1, r1) = (d2 d1, d2 r1 + r2) is
// associative, so a Hillis-Steele scan over S lanes (S the power of two >=
// the segment count, at most 32) gives every segment's carried state at once.
// A warp scans G = 32 / S groups of 4 consecutive (h,p,n) elements: lane
// j G + g holds segment j of group g, so the lanes holding one segment read
// G consecutive groups (coalesced) and the scan shuffles by multiples of G.
// More than 32 segments take passes of 32, each chained to the last state of
// the one before.
constexpr int kCarryQuads = 4;   // groups of 4 state elements a carry thread
__global__ void __launch_bounds__(256) seg_carry_kernel(const TcArgs a, int pairs, int S) {
  pdl_trigger();
  // the records and log decays of the state-only pass
  pdl_wait();
  const int N = a.N;
  const int quads = 128 * N / 4;
  const int G = 32 / S, lane = threadIdx.x & 31;
  const int j = lane / G, sub = (threadIdx.x >> 5) * G + lane % G;
  const int pair = blockIdx.y, b = blockIdx.z;
  const size_t slot = ((size_t)b * pairs + pair) * a.nrec;
  const size_t rstride = (size_t)128 * N / 4;   // float4s between consecutive records
  // kCarryQuads groups of quads a thread, every load of a pass issued before
  // the scans (the kernel is bound by memory latency, not bandwidth)
  int e[kCarryQuads];
  bool valid[kCarryQuads];
#pragma unroll
  for (int u = 0; u < kCarryQuads; ++u) {
    const int eq = (blockIdx.x * kCarryQuads + u) * (256 / S) + sub;
    valid[u] = eq < quads;   // uniform over a sub-warp
    e[u] = (valid[u] ? eq : 0) * 4;
  }
  float4* rec = reinterpret_cast<float4*>(a.seg_state + slot * 128 * N);
  float4 carry[kCarryQuads];
#pragma unroll
  for (int u = 0; u < kCarryQuads; ++u) carry[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
  for (int p0 = 0; p0 < a.nrec; p0 += S) {
    const int sg = p0 + j;
    float d[kCarryQuads];
    float4 r[kCarryQuads];
#pragma unroll
    for (int u = 0; u < kCarryQuads; ++u) {
      const int t = e[u] / N, n = e[u] % N, hr = t >> 6, pr = t & 63;
      d[u] = 1.f;                                   // identity for lanes past the last piece
      r[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (valid[u] && sg < a.nrec) {
        if (sg == 0) {
          d[u] = 0.f;
          if (a.ssm_in) {
            const float* src = a.ssm_in + (int64_t)b * a.si_sb + (int64_t)(a.head_begin + 2 * pair + hr) * a.si_sh +
                               (int64_t)pr * a.si_sp + (int64_t)n * a.si_sn;
            r[u] = make_float4(src[0], src[a.si_sn], src[2 * a.si_sn], src[3 * a.si_sn]);
          }
        } else {
          d[u] = ex2_approx(a.seg_logdecay[(slot + sg - 1) * 2 + hr] * kLog2e);
          r[u] = rec[(size_t)sg * rstride + e[u] / 4];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kCarryQuads; ++u) {
      if (j == 0 && p0 > 0) {   // chain to the last state of the previous pass
        r[u] = make_float4(fmaf(d[u], carry[u].x, r[u].x), fmaf(d[u], carry[u].y, r[u].y),
                           fmaf(d[u], carry[u].z, r[u].z), fmaf(d[u], carry[u].w, r[u].w));
        d[u] = 0.f;
      }
#pragma unroll 1
      for (int o = 1; o < S; o <<= 1) {
        const int og = o * G;
        const float dp = __shfl_up_sync(0xffffffffu, d[u], og);
        const float rx = __shfl_up_sync(0xffffffffu, r[u].x, og), ry = __shfl_up_sync(0xffffffffu, r[u].y, og);
        const float rz = __shfl_up_sync(0xffffffffu, r[u].z, og), rw = __shfl_up_sync(0xffffffffu, r[u].w, og);
        if (j >= o) {
          r[u] = make_float4(fmaf(d[u], rx, r[u].x), fmaf(d[u], ry, r[u].y), fmaf(d[u], rz, r[u].z),
                             fmaf(d[u], rw, r[u].w));
          d[u] *= dp;
        }
      }
      if (valid[u] && sg < a.nrec) rec[(size_t)sg * rstride + e[u] / 4] = r[u];
      const int last = (S - 1) * G + lane % G;   // piece p0 + S - 1 of this group
      carry[u] = make_float4(__shfl_sync(0xffffffffu, r[u].x, last), __shfl_sync(0xffffffffu, r[u].y, last),
                             __shfl_sync(0xffffffffu, r[u].z, last), __shfl_sync(0xffffffffu, r[u].w, last));
    }
  }
}

// ----------------------------------------------------------------------------
// the SSD kernel
// ----------------------------------------------------------------------------
// Roles (20 warps, launched with 96 registers a thread; the role and consumer
// warpgroups hand registers to the producers with setmaxnreg):
//   warps 0-7   consumers, warpgroup cw = 0/1.  Per chunk: the bf16 copy H of
//               the state and its decay (state columns split by warpgroup),
//               then the scores S of both heads for the 32-column blocks
//               j = cw, cw + 2, written in place over CB in tensor memory.
//   warps 8-15  producers, warpgroup hh = 0/1 for head hh of the pair.  Per
//               chunk: dt, cumulative log decay and column factors; the conv +
//               SiLU of the head's x channels from x rows loaded into
//               registers (a chunk ahead), written as X (double-buffered) and
//               X' = X dt exp(cum[Q-1] - cum[s]); then the epilogue (y) of the
//               previous chunk.  They run up to one chunk ahead of the
//               consumers.
//   warp 16     bulk copies of the B/C tiles.
//   warp 17     TMEM allocation and the MMA issue (one thread).
//   warps 18-19 no work (they complete the role warpgroup).
// Per chunk the MMA thread issues CB, the state update (after the state copy
// and X'), Yi (after the previous epilogue), then Y (after the scores).
template <int N, bool kStateOnly>
__global__ void __launch_bounds__(kThreads, 1) ssd_tc_kernel(const TcArgs a) {
  constexpr bool kPackedConv = kStateOnly || kPackedConvAll;
  constexpr int NK = N / 64;            // 64-column halves of B/C per chunk
  constexpr int NHALF = N / 2;          // state columns per consumer warpgroup
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);

  float* cum_s = reinterpret_cast<float*>(smem + OFF_CUM);   // [buf][head][128]
  float* dt_s = reinterpret_cast<float*>(smem + OFF_DT);
  float* cf_s = reinterpret_cast<float*>(smem + OFF_CF);
  float* wsum = reinterpret_cast<float*>(smem + OFF_WSUM);
  float* cw_all = reinterpret_cast<float*>(smem + OFF_CW);   // [2][4][16][4], then bias [2][16][4]
  float* xf_s = reinterpret_cast<float*>(smem + OFF_XF);     // [head][128]
  volatile uint32_t* tmem_ptr = reinterpret_cast<volatile uint32_t*>(smem + OFF_TMEMPTR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_ABORT);
  auto bar = [&](int i) { return base + OFF_BAR + 8u * i; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // this CTA's (batch row, head pair, segment)
  const bool split = a.split_units > 0;
  const int task = a.split_base + (int)blockIdx.x;
  const int seg = split ? task / a.split_units : (int)blockIdx.z;
  const int unit = split ? task - seg * a.split_units : 0;
  const int b = split ? unit / a.pairs : (int)blockIdx.y;
  const int pair = split ? unit - b * a.pairs : (int)blockIdx.x;
  const int h0 = a.head_begin + 2 * pair;   // first head of the pair
  const int hpg = a.H / a.G;
  const int gl = h0 / hpg - a.group_begin;        // group index inside the workspace
  const int L = a.L;
  const int nchunks = (L + Q - 1) / Q;
  // this CTA's segment: chunks [c_lo, c_lo + nk); the loops below count c from 0
  // (32-bit unsigned: nseg <= the SM count and nchunks < 2^24 keep the products in range)
  // (the state-only pass: seg is a piece, part seg % pieces of segment seg / pieces)
  const int sg_of = kStateOnly ? seg / a.pieces : seg, part = kStateOnly ? seg - sg_of * a.pieces : 0;
  const int parts = kStateOnly ? a.pieces : 1;
  const int s_lo = (int)((unsigned)sg_of * (unsigned)nchunks / (unsigned)a.nseg);
  const int s_len = (int)((unsigned)(sg_of + 1) * (unsigned)nchunks / (unsigned)a.nseg) - s_lo;
  const int c_lo = s_lo + part * s_len / parts;
  const int nk = s_lo + (part + 1) * s_len / parts - c_lo;
  // the chunk of walk step c: the full pass walks its segment forward, the
  // state-only pass backward, so that each chunk's contribution to the
  // segment's end state carries its decay to that end (the sum of A dt over
  // the chunks already walked) and nothing rescales the state per chunk
  auto chunk_at = [&](int c) { return kStateOnly ? c_lo + nk - 1 - c : c_lo + c; };

  if constexpr (!kStateOnly) ALLOY_TRACE_CTA_BEGIN();
  // launched programmatically after the previous kernel of the call: every
  // thread that reads what an earlier kernel of this call wrote (the B/C
  // tiles, the segment records) first waits for it with pdl_wait(); the
  // rest of the prologue (TMEM, barriers, weights, the first chunk's x rows
  // and dt) overlaps that kernel's tail
  pdl_trigger();
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    // FULL0/1 EMPTY0/1 X_READY0/1 CB_FULL HBF_READY S_READY Y_FULL ST_DONE YI_DONE Y_EMPTY0/1 PWG0/1 DRAIN NEVER
    // (the state-only pass: XF_EMPTY0/1 in place of ST_DONE / YI_DONE,
    // XP_FREE0/1 in place of Y_EMPTY0/1)
    const int s8 = kStateOnly ? 8 : 1, s1 = kStateOnly ? 1 : 8;
    const int counts[NBAR] = {1, 1, 1, 1, 8, 8, 1, 8, 8, 1, s8, s8, s1, s1, 4, 4, 1, 1};
    for (int i = 0; i < NBAR; ++i) mbar_init(bar(i), counts[i]);
    mbar_fence_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(base + OFF_TMEMPTR, 512);
    tmem_relinquish();
  }
  // x conv weights of both heads, [head][tap][channel], and bias
  // [head][channel], halved: the conv then gives h = x/2 and silu(x) = h +
  // h tanh(h).  A producer thread reads its 4 channels of a tap as one float4,
  // the 16 channel groups of a warp in consecutive banks.
  if (threadIdx.x < 128) {
    const int hh = threadIdx.x >> 6, ch = threadIdx.x & 63;
    const int64_t c = (int64_t)(h0 + hh) * P + ch;
#pragma unroll
    for (int k = 0; k < 4; ++k) cw_all[(hh * 4 + k) * 64 + ch] = 0.5f * a.conv_w[c * a.cw_sc + k * a.cw_sk];
    cw_all[512 + hh * 64 + ch] = a.conv_b ? 0.5f * a.conv_b[c * a.cb_s] : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_ptr;

  if (warp >= 16) {
    // role warpgroup: hand registers to the compute warpgroups
    reg_dealloc<kStateOnly ? kRoleRegsS : kRoleRegs>();
    if (warp == kTmaWarp) {
      // ------------------------------------------------------------ B/C copies
      if (lane == 0) {
        pdl_wait();   // the B/C tiles of the pre-pass
        // this pair's group: chunk c's B/C halves are NK consecutive 32 KB
        // stage images [B half k | C half k]
        const int64_t chunk_stride = (int64_t)a.group_count * NK * kStageBytes;
        const unsigned char* src0 = reinterpret_cast<const unsigned char*>(a.bc) +
                                    ((int64_t)b * nchunks * a.group_count + gl) * NK * kStageBytes;
        int issued = 0;   // stages (full pass) or chunks (state-only pass) sent
        if constexpr (kStateOnly) {
          // B halves alone (16 KB each), two chunks in flight: chunk buffer cb
          // holds half k at stage offset 32 KB k + 16 KB cb, so a chunk's
          // halves sit 32 KB apart as in the full pass
          auto prefetch = [&](int c) {
            for (int k = 0; k < NK; ++k) bulk_prefetch_l2(src0 + chunk_at(c) * chunk_stride + k * kStageBytes, 16384);
          };
          for (int c = 1; c <= kL2Ahead && c < nk; ++c) prefetch(c);
          for (int c = 0; c < nk; ++c) {
            if (c + kL2Ahead < nk) prefetch(c + kL2Ahead);
            const int cb = c & 1;
            if (c >= 2 && !wait1(bar(B_EMPTY0 + cb), ((c >> 1) - 1) & 1, abort_flag, 2)) goto bc_done;
            mbar_arrive_expect_tx(bar(B_FULL0 + cb), NK * 16384);
            for (int k = 0; k < NK; ++k)
              bulk_load(base + OFF_STAGE + k * 32768 + cb * 16384,
                        src0 + chunk_at(c) * chunk_stride + k * kStageBytes, 16384, bar(B_FULL0 + cb));
            ++issued;
          }
        } else {
          for (int c = 1; c <= kL2Ahead && c < nk; ++c) bulk_prefetch_l2(src0 + chunk_at(c) * chunk_stride, NK * kStageBytes);
          for (int c = 0; c < nk; ++c) {
            if (c + kL2Ahead < nk) bulk_prefetch_l2(src0 + chunk_at(c + kL2Ahead) * chunk_stride, NK * kStageBytes);
            for (int k = 0; k < NK; ++k) {
              const int i = c * NK + k, slot = i & 1;
              if (i >= 2 && !wait1(bar(B_EMPTY0 + slot), ((i >> 1) - 1) & 1, abort_flag, 2)) goto bc_done;
              ALLOY_TRACE_POINT(2, c, k);
              mbar_arrive_expect_tx(bar(B_FULL0 + slot), kStageBytes);
              bulk_load(base + OFF_STAGE + slot * kStageBytes, src0 + chunk_at(c) * chunk_stride + k * kStageBytes,
                        kStageBytes, bar(B_FULL0 + slot));
              ALLOY_TRACE_COPY_DONE(bar(B_FULL0 + slot), (i >> 1) & 1, 2, c, 2 + k);
              ++issued;
            }
          }
        }
      bc_done:
        // the copies in flight land before the CTA leaves
        for (int i = max(0, issued - 2); i < issued; ++i) {
          const long long t0 = clock64();
          while (!mbar_try_wait(bar(B_FULL0 + (i & 1)), (i >> 1) & 1) && clock64() - t0 < kWaitCycles) {
          }
        }
      }
    } else if (warp == kMmaWarp) {
      // ------------------------------------------------------------ MMA issuer
      if (lane == 0) {
        constexpr uint32_t ID_CB = idesc_bf16(128, 128, 0, 0);
        constexpr uint32_t ID_YI = idesc_bf16(128, 128, 0, 0);
        constexpr uint32_t ID_ST = idesc_bf16(128, N, 1, 1);
        constexpr uint32_t ID_Y = idesc_bf16(128, 64, 0, 1);
        if constexpr (kStateOnly) {
          // state[(h,p), n] = sum over the walk of X'^T B, X' carrying the
          // decay to the segment's end (the first MMA overwrites tensor memory)
          for (int c = 0; c < nk; ++c) {
            const int cb = c & 1;
            if (!wait1(bar(B_FULL0 + cb), (c >> 1) & 1, abort_flag, 3)) goto mma_done;
            ALLOY_TRACE_POINT(3, c, 5);
            if (!wait1(bar(B_X_READY0 + cb), (c >> 1) & 1, abort_flag, 8)) goto mma_done;
            ALLOY_TRACE_POINT(3, c, 9);
            tc_fence_after();
            const uint32_t sB = base + OFF_STAGE + cb * 16384;
            const uint32_t sXp = base + (cb ? OFF_X : OFF_XP);
            umma_bf16_chain8<128, 128, sw128_hi(1024), sw128_hi(1024)>(
                tmem + T_ST, sw128_lo(sXp, 16384), sw128_lo(sB, kStageBytes), ID_ST, c != 0);
            umma_commit(bar(B_EMPTY0 + cb));     // B halves of buffer cb free
            umma_commit(bar(B_XP_FREE0 + cb));   // X'[cb] free
          }
          umma_commit(bar(B_ST_FINAL));
        } else
        for (int c = 0; c < nk; ++c) {
          const uint32_t ph = c & 1, pph = (c - 1) & 1;
          const int buf = c & 1;
          // CB = C B^T over the N halves; the region held the previous scores,
          // so Y(c-1) must have completed
          for (int k = 0; k < NK; ++k) {
            const int i = c * NK + k, slot = i & 1;
            if (!wait1(bar(B_FULL0 + slot), (i >> 1) & 1, abort_flag, 3)) goto mma_done;
            ALLOY_TRACE_POINT(3, c, 5 + k);
            if (k == 0 && c > 0 && !wait1(bar(B_Y_FULL), pph, abort_flag, 4)) goto mma_done;
            tc_fence_after();
            const uint32_t sB = base + OFF_STAGE + slot * kStageBytes, sC = sB + 16384;
            umma_bf16_chain4<2, 2, sw128_hi(1024), sw128_hi(1024)>(tmem + T_CB, sw128_lo(sC, 16), sw128_lo(sB, 16),
                                                                    ID_CB, k != 0);
          }
          umma_commit(bar(B_CB_FULL));
          ALLOY_TRACE_POINT(3, c, 0);
          // state[(h,p), n] += X'^T B over s, once the state is scaled and
          // copied (HBF) and X' has arrived with X
          if (!wait1(bar(B_HBF_READY), ph, abort_flag, 6)) goto mma_done;
          if (!wait1(bar(B_X_READY0 + buf), (c >> 1) & 1, abort_flag, 8)) goto mma_done;
          ALLOY_TRACE_POINT(3, c, 9);
          tc_fence_after();
          {
            // N = d_state in one chain: for d_state 128 the two 64-column halves of B
            // sit in the two stage slots, 32 KB apart (the MN-atom stride)
            const uint32_t sB = base + OFF_STAGE + ((c * NK) & 1) * kStageBytes;
            const uint32_t sXp = base + OFF_XP;
            umma_bf16_chain8<128, 128, sw128_hi(1024), sw128_hi(1024)>(
                tmem + T_ST, sw128_lo(sXp, 16384), sw128_lo(sB, kStageBytes), ID_ST, 1);
          }
          umma_commit(bar(B_ST_DONE));
          ALLOY_TRACE_POINT(3, c, 10);
          // Yi = C [H_0; H_1]^T for both heads at once (N = 128 rows (h, p));
          // its columns and Y's held chunk c-1's output until its epilogue.
          // H is a copy, so the state update above does not disturb it.
          if (c > 0 && !wait1(bar(B_Y_EMPTY0 + (buf ^ 1)), ((c - 1) >> 1) & 1, abort_flag, 5)) goto mma_done;
          tc_fence_after();
          for (int k = 0; k < NK; ++k) {
            const uint32_t sC = base + OFF_STAGE + ((c * NK + k) & 1) * kStageBytes + 16384;
            const uint32_t sH = base + OFF_H + k * 16384;
            umma_bf16_chain4<2, 2, sw128_hi(1024), sw128_hi(1024)>(tmem + T_YI, sw128_lo(sC, 16), sw128_lo(sH, 16),
                                                                    ID_YI, k != 0);
          }
          // the last reads of this chunk's B/C stages and of H
          for (int k = 0; k < NK; ++k) umma_commit(bar(B_EMPTY0 + ((c * NK + k) & 1)));
          umma_commit(bar(B_YI_DONE));
          ALLOY_TRACE_POINT(3, c, 1);
          // Y_h = S_h X_h, S_h (bf16 pairs) read from tensor memory
          if (!wait1(bar(B_S_READY), ph, abort_flag, 7)) goto mma_done;
          ALLOY_TRACE_POINT(3, c, 8);
          tc_fence_after();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t sX = base + OFF_X + (buf * 2 + h) * 16384;
            umma_bf16_ta_chain8<16, 128, sw128_hi(1024)>(tmem + T_Y + 64 * h, tmem + T_CB + 8 * h, sw128_lo(sX, 16),
                                                          ID_Y, 0);
          }
          umma_commit(bar(B_Y_FULL));
          ALLOY_TRACE_POINT(3, c, 2);
        }
      mma_done:
        // wait (bounded) for every MMA this thread issued
        umma_commit(bar(B_DRAIN));
        {
          const long long t0 = clock64();
          while (!mbar_try_wait(bar(B_DRAIN), 0) && clock64() - t0 < kWaitCycles) {
          }
        }
      }
    }
  } else {
    const int q = warp & 3;               // TMEM lane quadrant
    const int t = q * 32 + lane;          // row of this thread (t, s or (h,p))
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    if (warp >= 8) {
      // ------------------------------------------------------------ producers (warps 8-15)
      reg_alloc<kStateOnly ? kProducerRegsS : kProducerRegs>();
      const int hh = (warp - 8) >> 2;     // head of the pair
      const int head = h0 + hh;
      const float A = -expf(a.A_log[(int64_t)head * a.al_s]);
      const float dtb = a.dt_bias[(int64_t)head * a.dtb_s];
      // this thread's conv work: 4 channels (4*vc4 .. 4*vc4+3) x 16 rows
      // [16 strip, 16 strip + 16), inside the warp's rows [32q, 32q + 32)
      const int vc4 = t & 15, strip = t >> 4;
      const int xch = head * P + vc4 * 4;
      const __nv_bfloat16* xsrc = a.xbc + (int64_t)b * a.x_sb + xch;
      const int64_t dt_row = (int64_t)b * a.dt_sb + (int64_t)head * a.dt_sh;
      uint32_t dt_bits = 0;   // raw dt of the chunk about to be produced (converted when used)
      auto load_dt = [&](int cc) {
        const int64_t di = dt_row + (int64_t)min(chunk_at(cc) * Q + t, L - 1) * a.dt_st;
        if (a.dt_bf16)
          asm volatile("ld.global.nc.u16 %0, [%1];" : "=r"(dt_bits)
                       : "l"(static_cast<const __nv_bfloat16*>(a.dt) + di));
        else
          asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(dt_bits)
                       : "l"(static_cast<const float*>(a.dt) + di));
      };
      // x rows [cc*Q + 16 strip - 3, cc*Q + 16 strip + 16) of this thread's
      // channels (clamped into [0, L); rows before 0 are replaced from the
      // conv cache, rows past L only feed masked outputs)
      uint32_t rw[19][2];
      auto load_rows = [&](int cc, uint32_t (&rr)[19][2]) {
        const int r0 = chunk_at(cc) * Q + strip * 16 - 3;
#pragma unroll
        for (int r = 0; r < 19; ++r) {
          const int tt = min(max(r0 + r, 0), L - 1);
          asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];"
                       : "=r"(rr[r][0]), "=r"(rr[r][1])
                       : "l"(xsrc + (int64_t)tt * a.x_st));
        }
      };
      // the x rows of chunk cc into L2, one row a thread (128 threads, 131 rows)
      const __nv_bfloat16* xhead = a.xbc + (int64_t)b * a.x_sb + head * P;
      auto prefetch_rows = [&](int cc) {
        if (cc >= nk) return;
        const int r0 = chunk_at(cc) * Q - 3 + t;
        if (r0 >= 0 && r0 < L) prefetch_l2(xhead + (int64_t)r0 * a.x_st);
        if (t < 3 && r0 + Q < L) prefetch_l2(xhead + (int64_t)(r0 + Q) * a.x_st);
      };
      // ---- epilogue of chunk cc (head hh): y = Y + exp(cum[t]) Yi -> global ----
      // Each warp stages its 32 rows in its own rows of X[cc&1][hh] (read by
      // Y(cc), complete once Y_FULL(cc) is), then stores 4 full 128-byte rows
      // per instruction.
      auto epilogue = [&](int cc) -> bool {
        const int ebuf = cc & 1;
        if (!waitw(bar(B_Y_FULL), cc & 1, abort_flag, 34)) return false;
        ALLOY_TRACE_POINT(4 + hh, cc + 1, 5);
        tc_fence_after();
        const uint64_t e2 = f2_splat(ex2_approx(cum_s[(ebuf * 2 + hh) * 128 + t] * kLog2e));
        const uint32_t stage = base + OFF_X + (ebuf * 2 + hh) * 16384 + q * 4096;
        const uint32_t ty = lane_base + T_Y + 64 * hh, ti = lane_base + T_YI + 64 * hh;
        // 16-column pieces, the next pair read while this one is combined
        uint32_t ya[8], ia[8], yb[8], ib[8];
        auto combine = [&](int piece, uint32_t (&ry)[8], uint32_t (&ri)[8]) {
          uint32_t o4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o4[i] = f2_to_bf2(f2_fma(f2_pack(__uint_as_float(ri[2 * i]), __uint_as_float(ri[2 * i + 1])), e2,
                                     f2_pack(__uint_as_float(ry[2 * i]), __uint_as_float(ry[2 * i + 1]))));
          st_shared_v4(stage + sw_off(lane, piece), o4[0], o4[1], o4[2], o4[3]);
        };
        tmem_ld8(ty, ya);
        tmem_ld8(ti, ia);
#pragma unroll 1
        for (int pc = 0; pc < 8; pc += 2) {
          tmem_ld_wait_regs(ya, ia);
          tmem_ld8(ty + 8 * (pc + 1), yb);
          tmem_ld8(ti + 8 * (pc + 1), ib);
          combine(pc, ya, ia);
          tmem_ld_wait_regs(yb, ib);
          if (pc + 2 < 8) {
            tmem_ld8(ty + 8 * (pc + 2), ya);
            tmem_ld8(ti + 8 * (pc + 2), ia);
          }
          combine(pc + 1, yb, ib);
        }
        __syncwarp();
        const int t0 = chunk_at(cc) * Q;
        __nv_bfloat16* ybase = a.y + (int64_t)b * a.y_sb + (int64_t)head * a.y_sh + (lane & 7) * 8;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int row = 4 * k + (lane >> 3);
          const uint4 v = ld_shared_v4(stage + sw_off(row, lane & 7));
          const int tt = t0 + q * 32 + row;
          if (tt < L) *reinterpret_cast<uint4*>(ybase + (int64_t)tt * a.y_st) = v;
        }
        __syncwarp();
        tc_fence_before();
        if (lane == 0) mbar_arrive(bar(B_Y_EMPTY0 + ebuf));
        return true;
      };
      for (int cc = 1; cc <= kL2Ahead; ++cc) prefetch_rows(cc);
      if constexpr (!kStateOnly) load_dt(0);
      // ---- dt, warp-local scan and column factors of chunk cc; the warp's
      // total goes to wsum and the warp arrives on the group barrier, whose
      // wait (for the prefix over the warps) comes when the chunk is produced
      float v_c = 0.f, dt_c = 0.f, cf_c = 0.f;
      auto scan_chunk = [&](int cc) {
        const int cbuf = cc & 1;
        const float dt = chunk_at(cc) * Q + t < L
            ? ALLOY_SOFTPLUS((a.dt_bf16 ? __uint_as_float(dt_bits << 16) : __uint_as_float(dt_bits)) + dtb)
            : 0.f;
        if (cc + 1 < nk) load_dt(cc + 1);
        float v = A * dt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float u = __shfl_up_sync(0xffffffffu, v, o);
          if (lane >= o) v += u;
        }
        // column factor relative to the end of this row's 16-step piece
        const float vend = __shfl_sync(0xffffffffu, v, lane | 15);
        cf_c = ex2_approx((vend - v) * kLog2e) * dt;
        v_c = v;
        dt_c = dt;
        // (wsum is double-buffered by chunk parity: a warp writes it for chunk
        // cc+2 only after the wait for cc+1, which every warp's arrival for
        // cc+1 precedes, and each warp reads wsum(cc) before that arrival)
        if (lane == 31) wsum[(cbuf * 2 + hh) * 4 + q] = v;
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_PWG0 + hh));
      };
      // ---- chunk c from its rows rr: prefix over the warps, X (full pass) and X' ----
      auto produce = [&](int c, uint32_t (&rr)[19][2]) -> bool {
        const int buf = c & 1;
        const float* xfp;   // X' row factors of this chunk (head hh)
        if constexpr (kStateOnly) {
          // the row factors (decay to the segment's end) come from the consumer
          // warps; X' is double-buffered
          if (!waitw(bar(B_XF_FULL0 + buf), (c >> 1) & 1, abort_flag, 22)) return false;
          ALLOY_TRACE_POINT(4 + hh, c, 1);
          if (c >= 2 && !waitw(bar(B_XP_FREE0 + buf), ((c >> 1) - 1) & 1, abort_flag, 23)) return false;
          xfp = cum_s + (buf * 2 + hh) * 128;
        } else {
          // X[buf] and cum/dt/cf[buf] held chunk c-2, whose epilogue this
          // warpgroup finished last iteration (after Y(c-2), and so after the
          // scores and the state copy of c-2)
          ALLOY_TRACE_POINT(4 + hh, c, 0);
          // ---- prefix over the warps -> cumulative log decay ----
          if (!waitw(bar(B_PWG0 + hh), c & 1, abort_flag, 22)) return false;
          float pre = 0.f, tot = 0.f;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float w = wsum[(buf * 2 + hh) * 4 + i];
            pre += i < q ? w : 0.f;
            tot += w;
          }
          const float cum = v_c + pre;
          cum_s[(buf * 2 + hh) * 128 + t] = cum;
          dt_s[(buf * 2 + hh) * 128 + t] = dt_c;
          cf_s[(buf * 2 + hh) * 128 + t] = cf_c;
          // X' factor of row t, read back below by the lanes of this warp that convolve the row
          xf_s[hh * 128 + t] = ex2_approx((tot - cum) * kLog2e) * dt_c;
          __syncwarp();
          ALLOY_TRACE_POINT(4 + hh, c, 1);
          // X' is single-buffered: the state update of chunk c-1 read it
          if (c > 0 && !waitw(bar(B_ST_DONE), (c - 1) & 1, abort_flag, 23)) return false;
          xfp = xf_s + hh * 128;
        }
        // ---- conv + SiLU -> X[buf][hh] (bf16) and X'[hh] = X * xf ----
        {
          float w[4][4], bias[4];   // [tap][channel]
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 wk = *reinterpret_cast<const float4*>(cw_all + (hh * 4 + k) * 64 + vc4 * 4);
            w[k][0] = wk.x; w[k][1] = wk.y; w[k][2] = wk.z; w[k][3] = wk.w;
          }
          {
            const float4 bk = *reinterpret_cast<const float4*>(cw_all + 512 + hh * 64 + vc4 * 4);
            bias[0] = bk.x; bias[1] = bk.y; bias[2] = bk.z; bias[3] = bk.w;
          }
          if (chunk_at(c) == 0 && strip == 0) {
            // rows before t = 0 come from the conv cache (zeros without one)
#pragma unroll
            for (int r = 0; r < 3; ++r) {
              float f[4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
                f[i] = a.conv_in ? __bfloat162float(a.conv_in[(int64_t)b * a.ci_sb +
                                                             (int64_t)(a.K - 4 + r) * a.ci_sk +
                                                             (int64_t)(xch + i) * a.ci_sc])
                                 : 0.f;
              rr[r][0] = pack_bf16x2(f[0], f[1]);
              rr[r][1] = pack_bf16x2(f[2], f[3]);
            }
          }
          const uint32_t sX = base + OFF_X + (buf * 2 + hh) * 16384;
          const uint32_t sXp = base + (kStateOnly && buf ? OFF_X : OFF_XP) + hh * 16384;
          const float4* xf4 = reinterpret_cast<const float4*>(xfp + strip * 16);
          float4 fq;
          if constexpr (kPackedConv) {
          // the two channel pairs (0,1), (2,3) one after the other, as f32x2:
          // a pair's taps and bias, and a window of its last three input rows
          // (each row unpacked once)
          const uint32_t sxf = smem_u32(xfp + strip * 16);
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            uint64_t w2[4], b2, win[3];
#pragma unroll
            for (int k = 0; k < 4; ++k) w2[k] = f2_pack(w[k][2 * i], w[k][2 * i + 1]);
            b2 = f2_pack(bias[2 * i], bias[2 * i + 1]);
#pragma unroll
            for (int r = 0; r < 3; ++r) win[r] = f2_from_bf2(rr[r][i]);
#pragma unroll
            for (int r = 3; r < 19; ++r) {
              const int srow = strip * 16 + r - 3;
              // (volatile: the factor loads stay in row order instead of all
              // 16 factors being live at once)
              if (((r - 3) & 3) == 0)
                asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                             : "=f"(fq.x), "=f"(fq.y), "=f"(fq.z), "=f"(fq.w) : "r"(sxf + 4 * (r - 3)));
              const float fx = ((r - 3) & 3) == 0 ? fq.x : ((r - 3) & 3) == 1 ? fq.y : ((r - 3) & 3) == 2 ? fq.z : fq.w;
              const uint64_t xin = f2_from_bf2(rr[r][i]);
              uint64_t acc = f2_fma(win[0], w2[0], b2);
              acc = f2_fma(win[1], w2[1], acc);
              acc = f2_fma(win[2], w2[2], acc);
              acc = f2_fma(xin, w2[3], acc);
              // acc = h = x/2 (halved taps): silu(x) = h + h tanh(h)
              float hl, hh2;
              f2_unpack(acc, hl, hh2);
              const uint64_t y2 = f2_fma(acc, f2_pack(tanh_approx(hl), tanh_approx(hh2)), acc);
              const uint32_t off = srow * 128 + (((vc4 >> 1) ^ (srow & 7)) << 4) + ((vc4 & 1) << 3) + 4 * i;
              if constexpr (!kStateOnly)   // (the state-only pass needs X' alone)
                asm volatile("st.shared.b32 [%0], %1;" ::"r"(sX + off), "r"(f2_to_bf2(y2)) : "memory");
              asm volatile("st.shared.b32 [%0], %1;" ::"r"(sXp + off), "r"(f2_to_bf2(f2_mul(y2, f2_splat(fx))))
                           : "memory");
              win[0] = win[1];
              win[1] = win[2];
              win[2] = xin;
            }
          }
          } else {
#pragma unroll
          for (int r = 3; r < 19; ++r) {
            const int srow = strip * 16 + r - 3;
            if (((r - 3) & 3) == 0) fq = xf4[(r - 3) >> 2];
            const float fx = ((r - 3) & 3) == 0 ? fq.x : ((r - 3) & 3) == 1 ? fq.y : ((r - 3) & 3) == 2 ? fq.z : fq.w;
            // (rows past L need no masking: X and X' there only meet dt = 0
            // or outputs that are not stored)
            float y4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float acc = bias[i];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint32_t wd = rr[r - 3 + k][i >> 1];
                acc = fmaf((i & 1) ? bf16_hi(wd) : bf16_lo(wd), w[k][i], acc);
              }
              y4[i] = fmaf(acc, tanh_approx(acc), acc);   // silu of 2 acc
            }
            uint32_t o[2], ox[2];
            o[0] = pack_bf16x2(y4[0], y4[1]);
            o[1] = pack_bf16x2(y4[2], y4[3]);
            ox[0] = pack_bf16x2(y4[0] * fx, y4[1] * fx);
            ox[1] = pack_bf16x2(y4[2] * fx, y4[3] * fx);
            const uint32_t off = srow * 128 + (((vc4 >> 1) ^ (srow & 7)) << 4) + ((vc4 & 1) << 3);
            if constexpr (!kStateOnly)   // (the state-only pass needs X' alone)
              asm volatile("st.shared.v2.b32 [%0], {%1,%2};" ::"r"(sX + off), "r"(o[0]), "r"(o[1]) : "memory");
            asm volatile("st.shared.v2.b32 [%0], {%1,%2};" ::"r"(sXp + off), "r"(ox[0]), "r"(ox[1]) : "memory");
          }
          }
        }
        prefetch_rows(c + 1 + kL2Ahead);
        // X, X', cum, dt, cf of chunk c are ready
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar(B_X_READY0 + buf));
          if (kStateOnly) mbar_arrive(bar(B_XF_EMPTY0 + buf));
        }
        ALLOY_TRACE_POINT(4 + hh, c, 3);
        return true;
      };
      if constexpr (!kStateOnly) {
        // iteration c: chunk c (c >= 0); the rows and the scan of chunk c+1; the epilogue of c-1
        for (int c = -1; c <= nk; ++c) {
          if (c >= 0 && c < nk && !produce(c, rw)) break;
          // the next chunk's rows (in flight during the epilogue below) and its scan
          if (c + 1 < nk) {
            load_rows(c + 1, rw);
            ALLOY_TRACE_POINT(4 + hh, c + 1, 6);
            scan_chunk(c + 1);
            ALLOY_TRACE_POINT(4 + hh, c + 1, 7);
          }
          // the previous chunk's output, while the tensor cores and consumers work on this one
          if (c > 0 && !epilogue(c - 1)) break;
          ALLOY_TRACE_POINT(4 + hh, c, 4);
        }
      } else {
        // the conv alone (the consumer warps scan dt): the rows of chunk c+2
        // are in flight while chunk c+1 is produced (two register sets)
        uint32_t rw2[19][2];
        load_rows(0, rw);
        if (nk > 1) load_rows(1, rw2);
        for (int c = 0; c < nk; c += 2) {
          if (!produce(c, rw)) break;
          if (c + 2 < nk) load_rows(c + 2, rw);
          if (c + 1 >= nk || !produce(c + 1, rw2)) break;
          if (c + 3 < nk) load_rows(c + 3, rw2);
        }
      }
    } else {
      // ------------------------------------------------------------ consumers
      reg_dealloc<kStateOnly ? kConsumerRegsS : kConsumerRegs>();
      const int cw = warp >> 2;           // consumer warpgroup
      const float D0 = a.Dp ? a.Dp[(int64_t)h0 * a.d_s] : 0.f;
      const float D1 = a.Dp ? a.Dp[(int64_t)(h0 + 1) * a.d_s] : 0.f;
      // state rows: r = t -> head hr = t / 64, p = t % 64; this warpgroup owns
      // state columns [cw * N/2, (cw+1) * N/2)
      const int hr = t >> 6, pr = t & 63;

      // segment records of this (batch row, head pair): record 0 the call's
      // initial state, record j + 1 the end state of segment j from zero (a
      // split walk: one record, the state handed from segment to segment)
      const size_t seg_slot = split ? (size_t)unit : ((size_t)b * a.pairs + pair) * a.nrec;
      auto record = [&](int j, int n8) {
        return reinterpret_cast<float4*>(a.seg_state + ((seg_slot + j) * 128 + t) * N + cw * NHALF + n8 * 8);
      };
      if constexpr (kStateOnly) {
        // ---- per chunk of the walk: dt, its scan and the X' row factors ----
        // Warpgroup cw scans head h0 + cw, warp q rows [32q, 32q + 32).  The
        // factor of row t is exp(the sum of A dt after row t to the segment's
        // end) dt_t: the rest of its chunk (tot - cum_t) and the chunks walked
        // before it (suffix).  Double-buffered in the cum region, which the
        // state-only pass does not use otherwise.
        {
          const int head = h0 + cw;
          const float A = -expf(a.A_log[(int64_t)head * a.al_s]);
          const float dtb = a.dt_bias[(int64_t)head * a.dtb_s];
          const int64_t dt_row = (int64_t)b * a.dt_sb + (int64_t)head * a.dt_sh;
          auto load_dt = [&](int cc) {
            uint32_t bits;
            const int64_t di = dt_row + (int64_t)min(chunk_at(cc) * Q + t, L - 1) * a.dt_st;
            if (a.dt_bf16)
              asm volatile("ld.global.nc.u16 %0, [%1];" : "=r"(bits)
                           : "l"(static_cast<const __nv_bfloat16*>(a.dt) + di));
            else
              asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(bits)
                           : "l"(static_cast<const float*>(a.dt) + di));
            return bits;
          };
          uint32_t dt_bits = load_dt(0);
          float suffix = 0.f;
          for (int c = 0; c < nk; ++c) {
            const int buf = c & 1;
            const float dt = chunk_at(c) * Q + t < L
                ? ALLOY_SOFTPLUS((a.dt_bf16 ? __uint_as_float(dt_bits << 16) : __uint_as_float(dt_bits)) + dtb)
                : 0.f;
            if (c + 1 < nk) dt_bits = load_dt(c + 1);
            float v = A * dt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const float u = __shfl_up_sync(0xffffffffu, v, o);
              if (lane >= o) v += u;
            }
            // warp totals -> wsum[buf]: a warp writes it for chunk c+2 only after
            // the wait for c+1, which every warp's arrival for c+1 precedes, and
            // each warp reads wsum(c) before that arrival
            if (lane == 31) wsum[(buf * 2 + cw) * 4 + q] = v;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_PWG0 + cw));
            if (!waitw(bar(B_PWG0 + cw), c & 1, abort_flag, 24)) break;
            ALLOY_TRACE_POINT(cw, c, 0);
            float pre = 0.f, tot = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float w = wsum[(buf * 2 + cw) * 4 + i];
              pre += i < q ? w : 0.f;
              tot += w;
            }
            // the producers have read the factors of chunk c-2
            if (c >= 2 && !waitw(bar(B_XF_EMPTY0 + buf), ((c >> 1) - 1) & 1, abort_flag, 25)) break;
            cum_s[(buf * 2 + cw) * 128 + t] = ex2_approx((suffix + tot - (v + pre)) * kLog2e) * dt;
            suffix += tot;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_XF_FULL0 + buf));
            ALLOY_TRACE_POINT(cw, c, 1);
          }
          // the segment's log decay (head h0 + cw), for the full pass's carry
          if (t == 0) a.seg_logdecay[(seg_slot + seg) * 2 + cw] = suffix;
        }
        // the segment's end state from zero -> record seg + 1
        if (waitw(bar(B_ST_FINAL), 0, abort_flag, 36)) {
          tc_fence_after();
#pragma unroll 1
          for (int n8 = 0; n8 < NHALF / 8; ++n8) {
            uint32_t r[8];
            tmem_ld8(lane_base + T_ST + cw * NHALF + n8 * 8, r);
            tmem_ld_wait();
            record(seg + 1, n8)[0] = make_float4(__uint_as_float(r[0]), __uint_as_float(r[1]),
                                                 __uint_as_float(r[2]), __uint_as_float(r[3]));
            record(seg + 1, n8)[1] = make_float4(__uint_as_float(r[4]), __uint_as_float(r[5]),
                                                 __uint_as_float(r[6]), __uint_as_float(r[7]));
          }
        }
      } else {
      pdl_wait();   // the segment records (segmented calls)
      // initial state -> TMEM: the call's initial state (unsegmented), else
      // record seg, the state carried into this segment (seg_carry_kernel's
      // associative scan over the segments).
      // sp: a strided view of ssm_in, or the record (n stride 1), or none
      // (zero).  32 values a batch, every load of a batch issued before the
      // first use (one memory round trip a batch).
      const float* sp = nullptr;
      int64_t sn = 1;
      if (split ? seg > 0 : a.nseg > 1) {
        sp = reinterpret_cast<const float*>(record(split ? 0 : seg * a.pieces, 0));
      } else if (a.ssm_in) {
        sp = a.ssm_in + (int64_t)b * a.si_sb + (int64_t)(h0 + hr) * a.si_sh + (int64_t)pr * a.si_sp +
             (int64_t)(cw * NHALF) * a.si_sn;
        sn = a.si_sn;
      }
#pragma unroll 1
      for (int h32 = 0; h32 < NHALF / 32; ++h32) {
        uint32_t r[32];
        if (sp == nullptr) {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        } else if (sn == 1) {
          const float4* s4 = reinterpret_cast<const float4*>(sp + h32 * 32);
          float4 w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = s4[i];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            r[4 * i] = __float_as_uint(w[i].x); r[4 * i + 1] = __float_as_uint(w[i].y);
            r[4 * i + 2] = __float_as_uint(w[i].z); r[4 * i + 3] = __float_as_uint(w[i].w);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(sp[(int64_t)(h32 * 32 + i) * sn]);
        }
        tmem_st32(lane_base + T_ST + cw * NHALF + h32 * 32, r);
      }
      tmem_st_wait();

      // score pieces of this warp: 16-column halves g of the 32-column blocks
      // j = cw, cw + 2 (K-steps 2j + g of the Y MMA); blocks right of the
      // warp's rows (j > q) are zero
      const int npieces = q >= cw + 2 ? 4 : (q >= cw ? 2 : 0);
      auto piece_col = [&](int i) { return 32 * (cw + 2 * (i >> 1)) + 16 * (i & 1); };

      // test of the bounded-wait error path: a wait nothing completes runs
      // out (site 50), the CTA takes its abort path and the chunk loop is
      // skipped
      const bool stalled = a.stall_cycles > 0 && !waitw(bar(B_NEVER), 0, abort_flag, 50, a.stall_cycles);
      for (int c = 0; c < nk && !stalled; ++c) {
        const int buf = c & 1;
        if (!waitw(bar(B_X_READY0 + buf), (c >> 1) & 1, abort_flag, 30)) break;
        ALLOY_TRACE_POINT(cw, c, 0);
        // ---- state: H = bf16(state) -> smem; state *= exp(cum[Q-1]) ----
        // (Yi(c-1), the last reader of H, follows the state update of c-1)
        if (c > 0 && !waitw(bar(B_YI_DONE), (c - 1) & 1, abort_flag, 31)) break;
        tc_fence_after();
        {
          const float lg_end = cum_s[(buf * 2 + hr) * 128 + 127];
          const float e_end = ex2_approx(lg_end * kLog2e);
          const uint32_t sH = base + OFF_H + hr * 8192;   // [n block][head][64 p][64 n]
          const uint64_t e2 = f2_splat(e_end);
          // 16-column pieces of this warpgroup's state columns, the next piece
          // read from tensor memory while this one is copied and scaled
          auto copy_piece = [&](int i, uint32_t (&r)[16]) {
            const int n0 = cw * NHALF + 16 * i;
#pragma unroll
            for (int g4 = 0; g4 < 2; ++g4) {
              const int n = n0 + g4 * 8;
              st_shared_v4(sH + (n >> 6) * 16384 + sw_off(pr, (n & 63) >> 3),
                           pack_bf16x2(__uint_as_float(r[g4 * 8 + 0]), __uint_as_float(r[g4 * 8 + 1])),
                           pack_bf16x2(__uint_as_float(r[g4 * 8 + 2]), __uint_as_float(r[g4 * 8 + 3])),
                           pack_bf16x2(__uint_as_float(r[g4 * 8 + 4]), __uint_as_float(r[g4 * 8 + 5])),
                           pack_bf16x2(__uint_as_float(r[g4 * 8 + 6]), __uint_as_float(r[g4 * 8 + 7])));
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              float lo, hi;
              f2_unpack(f2_mul(f2_pack(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1])), e2), lo, hi);
              r[2 * k] = __float_as_uint(lo);
              r[2 * k + 1] = __float_as_uint(hi);
            }
            tmem_st16(lane_base + T_ST + n0, r);
          };
          uint32_t ra[16], rb[16];
          tmem_ld16(lane_base + T_ST + cw * NHALF, ra);
#pragma unroll 1
          for (int i = 0; i < NHALF / 16; i += 2) {
            tmem_ld_wait_regs(ra);
            tmem_ld16(lane_base + T_ST + cw * NHALF + 16 * (i + 1), rb);
            copy_piece(i, ra);
            tmem_ld_wait_regs(rb);
            if (i + 2 < NHALF / 16) tmem_ld16(lane_base + T_ST + cw * NHALF + 16 * (i + 2), ra);
            copy_piece(i + 1, rb);
          }
          tmem_st_wait();
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_HBF_READY));
        ALLOY_TRACE_POINT(cw, c, 1);
        // ---- scores of both heads, in place over CB ----
        // S_h[t, s] = CB[t, s] exp(cum_h[t] - cum_h[s]) dt_h[s] for s <= t (+ D_h on
        // s == t); K-step k (sources 16k .. 16k+15) of S_h stored as bf16 pairs
        // in columns [16k + 8h, 16k + 8h + 8), inside the piece it was read from
        if (!waitw(bar(B_CB_FULL), c & 1, abort_flag, 32)) break;
        ALLOY_TRACE_POINT(cw, c, 2);
        tc_fence_after();
        auto score_piece = [&](int i, const uint32_t (&r)[16]) {
          const int j = cw + 2 * (i >> 1);
          const int s0 = piece_col(i);
#ifdef ALLOY_SCORE_UNROLL
#pragma unroll
#else
#pragma unroll 1
#endif
          for (int h = 0; h < 2; ++h) {
            const float* cm = cum_s + (buf * 2 + h) * 128;
            const float cum_t = cm[t];
            uint32_t o[8];
            if (j < q) {
              // left of the diagonal block: exp(cum_t - cum_s) dt_s = R cf[s] with
              // R = exp(cum_t - cum[s0+15]) <= 1 and cf[s] = exp(cum[s0+15] - cum_s) dt_s <= dt_s
              const uint64_t R2 = f2_splat(ex2_approx((cum_t - cm[s0 + 15]) * kLog2e));
              const float4* cf4 = reinterpret_cast<const float4*>(cf_s + (buf * 2 + h) * 128 + s0);
#pragma unroll
              for (int i4 = 0; i4 < 4; ++i4) {
                const float4 f = cf4[i4];
                o[2 * i4] = f2_to_bf2(
                    f2_mul(f2_mul(f2_pack(__uint_as_float(r[4 * i4]), __uint_as_float(r[4 * i4 + 1])), R2),
                           f2_pack(f.x, f.y)));
                o[2 * i4 + 1] = f2_to_bf2(
                    f2_mul(f2_mul(f2_pack(__uint_as_float(r[4 * i4 + 2]), __uint_as_float(r[4 * i4 + 3])), R2),
                           f2_pack(f.z, f.w)));
              }
            } else if (cm[32 * q] - cm[32 * q + 31] < 64.f) {
              // the diagonal block with a decay range below e^64 over its 32
              // rows (uniform across the warp): factored like the pieces left of
              // it, R = exp(cum_t - cum[s0+15]) <= e^64; zero right of the
              // diagonal, D on it
              const uint64_t R2 = f2_splat(ex2_approx((cum_t - cm[s0 + 15]) * kLog2e));
              const float4* cf4 = reinterpret_cast<const float4*>(cf_s + (buf * 2 + h) * 128 + s0);
              const float Dh = h ? D1 : D0;
#ifdef ALLOY_DIAG_SAT
              // mask and D as factors: m_u = [s0 + u <= t] = sat(t - s0 + 1 - u),
              // d_u = [s0 + u == t] = m_u - m_{u+1}; S = CB R (cf m) + D d
              const uint64_t D2 = f2_splat(Dh);
              const float fdd = static_cast<float>(t - s0 + 1);
#pragma unroll
              for (int i4 = 0; i4 < 4; ++i4) {
                const float4 f = cf4[i4];
                float m[5];
#pragma unroll
                for (int u = 0; u < 5; ++u) {
                  const float v = fdd - static_cast<float>(4 * i4 + u);
                  asm("cvt.sat.f32.f32 %0, %1;" : "=f"(m[u]) : "f"(v));
                }
                const uint64_t m01 = f2_pack(m[0], m[1]), m23 = f2_pack(m[2], m[3]);
                const uint64_t d01 = f2_pack(m[0] - m[1], m[1] - m[2]), d23 = f2_pack(m[2] - m[3], m[3] - m[4]);
                o[2 * i4] = f2_to_bf2(f2_fma(
                    f2_mul(f2_pack(__uint_as_float(r[4 * i4]), __uint_as_float(r[4 * i4 + 1])), R2),
                    f2_mul(f2_pack(f.x, f.y), m01), f2_mul(d01, D2)));
                o[2 * i4 + 1] = f2_to_bf2(f2_fma(
                    f2_mul(f2_pack(__uint_as_float(r[4 * i4 + 2]), __uint_as_float(r[4 * i4 + 3])), R2),
                    f2_mul(f2_pack(f.z, f.w), m23), f2_mul(d23, D2)));
              }
#else
#pragma unroll
              for (int i4 = 0; i4 < 4; ++i4) {
                const float4 f = cf4[i4];
                float x[4];
                f2_unpack(f2_mul(f2_mul(f2_pack(__uint_as_float(r[4 * i4]), __uint_as_float(r[4 * i4 + 1])), R2),
                                 f2_pack(f.x, f.y)), x[0], x[1]);
                f2_unpack(f2_mul(f2_mul(f2_pack(__uint_as_float(r[4 * i4 + 2]), __uint_as_float(r[4 * i4 + 3])), R2),
                                 f2_pack(f.z, f.w)), x[2], x[3]);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const int s = s0 + 4 * i4 + u;
                  x[u] = s < t ? x[u] : (s == t ? x[u] + Dh : 0.f);
                }
                o[2 * i4] = pack_bf16x2(x[0], x[1]);
                o[2 * i4 + 1] = pack_bf16x2(x[2], x[3]);
              }
#endif
            } else {
              // the diagonal block at a larger decay range: exact factors (<= 1
              // for s <= t, at any range), zero right of the diagonal, D on it
              const float4* cm4 = reinterpret_cast<const float4*>(cm + s0);
              const float4* dv4 = reinterpret_cast<const float4*>(dt_s + (buf * 2 + h) * 128 + s0);
              const float Dh = h ? D1 : D0;
#pragma unroll
              for (int i4 = 0; i4 < 4; ++i4) {
                const float4 c4 = cm4[i4], d4 = dv4[i4];
                const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, ds[4] = {d4.x, d4.y, d4.z, d4.w};
                float x[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const int s = s0 + 4 * i4 + u;
                  const float xv = __uint_as_float(r[4 * i4 + u]) * (ex2_approx((cum_t - cs[u]) * kLog2e) * ds[u]);
                  x[u] = s < t ? xv : (s == t ? xv + Dh : 0.f);
                }
                o[2 * i4] = pack_bf16x2(x[0], x[1]);
                o[2 * i4 + 1] = pack_bf16x2(x[2], x[3]);
              }
            }
            tmem_st8(lane_base + T_CB + s0 + 8 * h, o);
          }
        };
        {
          uint32_t ra[16], rb[16];
          if (npieces > 0) tmem_ld16(lane_base + T_CB + piece_col(0), ra);
#pragma unroll 1
          for (int i = 0; i < npieces; i += 2) {
            tmem_ld_wait_regs(ra);
            if (i == 0) ALLOY_TRACE_POINT(cw, c, 8);
            tmem_ld16(lane_base + T_CB + piece_col(i + 1), rb);
            score_piece(i, ra);
            if (i == 0) ALLOY_TRACE_POINT(cw, c, 9);
            tmem_ld_wait_regs(rb);
            if (i + 2 < npieces) tmem_ld16(lane_base + T_CB + piece_col(i + 2), ra);
            score_piece(i + 1, rb);
            if (i == 0) ALLOY_TRACE_POINT(cw, c, 10);
          }
          uint32_t z[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) z[k] = 0u;
#pragma unroll 1
          for (int i = npieces; i < 4; ++i) {
            tmem_st8(lane_base + T_CB + piece_col(i), z);
            tmem_st8(lane_base + T_CB + piece_col(i) + 8, z);
          }
        }
        ALLOY_TRACE_POINT(cw, c, 11);
        tmem_st_wait();
        ALLOY_TRACE_POINT(cw, c, 12);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_S_READY));
        ALLOY_TRACE_POINT(cw, c, 3);
      }
      // ---- the final state: the last segment's end state -> ssm_out ----
      if (!*abort_flag && a.ssm_out && seg == a.nseg - 1 && waitw(bar(B_YI_DONE), (nk - 1) & 1, abort_flag, 35)) {
        tc_fence_after();
#pragma unroll 1
        for (int n8 = 0; n8 < NHALF / 8; ++n8) {
          const int n0 = cw * NHALF + n8 * 8;
          uint32_t r[8];
          tmem_ld8(lane_base + T_ST + n0, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            a.ssm_out[(int64_t)b * a.so_sb + (int64_t)(h0 + hr) * a.so_sh + (int64_t)(n0 + i) * a.so_sn +
                      (int64_t)pr * a.so_sp] = __uint_as_float(r[i]);
        }
      }
      // ---- a split walk: this segment's end state -> the unit's record ----
      if (!*abort_flag && split && seg < a.nseg - 1 && waitw(bar(B_YI_DONE), (nk - 1) & 1, abort_flag, 37)) {
        tc_fence_after();
#pragma unroll 1
        for (int n8 = 0; n8 < NHALF / 8; ++n8) {
          uint32_t r[8];
          tmem_ld8(lane_base + T_ST + cw * NHALF + n8 * 8, r);
          tmem_ld_wait();
          record(0, n8)[0] = make_float4(__uint_as_float(r[0]), __uint_as_float(r[1]), __uint_as_float(r[2]),
                                         __uint_as_float(r[3]));
          record(0, n8)[1] = make_float4(__uint_as_float(r[4]), __uint_as_float(r[5]), __uint_as_float(r[6]),
                                         __uint_as_float(r[7]));
        }
      }
      }   // full pass
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if constexpr (!kStateOnly) ALLOY_TRACE_CTA_END();
}

// ----------------------------------------------------------------------------
// host side
// ----------------------------------------------------------------------------

// Launches `kernel` on `stream` with programmatic stream serialization: it may
// start while the previous kernel on the stream finishes (once every CTA of
// that kernel has executed pdl_trigger); its threads that read the previous
// kernel's results wait for them with pdl_wait().
template <typename... KArgs, typename... Args>
int launch_after_previous(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ALLOY_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  return ALLOY_OK;
}

int group_range(const SsdArgs& a, int* g0, int* gs) {
  const int hpg = a.H / a.G;
  *g0 = a.head_begin / hpg;
  *gs = (a.head_begin + a.head_count - 1) / hpg - *g0 + 1;
  return ALLOY_OK;
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool ssd_tc_supported(const SsdArgs& a) {
  if (a.mode != 0 || !a.xbc_bf16 || !a.y_bf16) return false;
  if (a.P != 64 || !(a.N == 64 || a.N == 128) || a.K != 4) return false;
  if ((a.H / a.G) % 2 != 0 || a.head_begin % 2 != 0 || a.head_count % 2 != 0) return false;
  if (a.conv_in && !a.ci_bf16) return false;
  if ((reinterpret_cast<uintptr_t>(a.xBC) & 15) || (a.xbc_sb & 7) || (a.xbc_st & 7)) return false;
  if ((reinterpret_cast<uintptr_t>(a.y) & 15) || a.y_sp != 1 || (a.y_sb & 7) || (a.y_st & 7) ||
      (a.y_sh & 7))
    return false;
  if (a.L < 1 || a.B < 1 || a.B > 65535) return false;
  return true;
}

// A (batch row, head pair) is walked chunk after chunk by one CTA.  When the
// call has fewer pairs than the GPU has SMs, each pair's chunks are cut into
// nseg segments walked by nseg CTAs at once: a state-only pass first gives
// every segment but the last its end state (conv, X' and the state update
// alone; segment 0 from the call's initial state, the others from zero), and
// the full pass then starts segment s from the state carried over segments
// 0..s-1.  Segments keep at least kMinSegChunks chunks.
constexpr int kMinSegChunks = 4;

int sm_count_of_current_device() {
  static int counts[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    counts[dev] = n;
  }
  return counts[dev];
}

struct TcLayout {
  int nseg;
  int pieces, nrec;                               // state-only pieces a segment, records a unit
  bool split;                                     // segments walked in order (split walk)
  size_t tiles, seg_state, seg_logdecay, total;   // byte offsets / sizes in the workspace
};

// The split walk: with at least as many (batch row, head pair) units as SMs,
// one CTA per unit runs in ceil(units / SMs) waves of the whole sequence (256
// units on 148 SMs: 2 waves where 1.73 would do).  Cutting every unit into k
// segments walked one after another, the k * units (unit, segment) tasks run
// as ceil(k * units / SMs) launches ("slots") of at most one CTA per SM,
// segment s + 1 of a unit in a later slot than segment s (task s * units + u
// sits in slot (s * units + u) / SMs, and units >= SMs), each starting from
// the exact state its predecessor handed over.  Estimated cost in chunk walks
// (fitted to the Nemotron and Zamba2 layer shapes at 256 units: one wave of
// 64 / 32 chunks costs ~1.5 chunks more, a slot of 16 / 8 chunks ~4.4 / 2.6
// more, as a slot ends with its slowest CTA and the next starts cold):
// waves * (chunks + 1.5) unsplit, slots * (1.1 * chunks per segment + 2.3)
// split; k is taken when it beats the others by 3 %.
constexpr double kWaveOverheadChunks = 1.5, kSlotOverheadChunks = 2.3, kSlotSpread = 1.1;

int split_segments(int units, int nchunks, int sms) {
  if (units < sms || sms <= 0) return 1;
  auto cost = [&](int k) {
    const double slots = (double)(((int64_t)k * units + sms - 1) / sms);
    return k == 1 ? slots * (nchunks + kWaveOverheadChunks)
                  : slots * (kSlotSpread * nchunks / k + kSlotOverheadChunks);
  };
  int best = 1;
  double best_cost = cost(1);
  for (int k = 2; k <= 8 && nchunks / k >= kMinSegChunks; ++k) {
    const double c = cost(k);
    if (c < 0.97 * best_cost) {
      best = k;
      best_cost = c;
    }
  }
  return best;
}

TcLayout tc_layout(const SsdArgs& a) {
  int g0, gs;
  group_range(a, &g0, &gs);
  TcLayout l;
  const int nchunks = (a.L + Q - 1) / Q;
  const int units = a.B * (a.head_count / 2);
  const int sms = sm_count_of_current_device();
  l.nseg = 1;
  l.pieces = 1;
  l.split = false;
  if (units > 0 && sms > units) {
    l.nseg = std::max(1, std::min(sms / units, nchunks / kMinSegChunks));
    // the state-only pass over segments 0..nseg-2 in as many pieces a segment
    // as the SMs take (pieces of at least kMinSegChunks chunks)
    if (l.nseg > 1)
      l.pieces = std::max(1, std::min(sms / ((l.nseg - 1) * units), nchunks / l.nseg / kMinSegChunks));
  } else if (units > 0) {
    l.nseg = split_segments(units, nchunks, sms);
    l.split = l.nseg > 1;
  }
  // B/C tiles of every chunk, the last one padded to Q rows
  l.tiles = (size_t)a.B * nchunks * Q * 2 * gs * a.N * sizeof(__nv_bfloat16);
  // segment records: nseg a unit (segmented), one a unit (split walk)
  l.nrec = l.split ? 1 : l.nseg > 1 ? (l.nseg - 1) * l.pieces + 1 : 1;
  const size_t nslots = (size_t)units * l.nrec;
  l.seg_state = (l.tiles + 255) & ~size_t(255);
  l.seg_logdecay = l.seg_state + nslots * 128 * a.N * sizeof(float);
  l.total = l.split ? l.seg_logdecay : l.nseg > 1 ? l.seg_logdecay + nslots * 2 * sizeof(float) : l.tiles;
  return l;
}

size_t ssd_tc_workspace_bytes(const SsdArgs& a) { return tc_layout(a).total; }
size_t ssd_tc_workspace_min_bytes(const SsdArgs& a) { return tc_layout(a).tiles; }

int ssd_tc(const SsdArgs& s, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!ssd_tc_supported(s)) return fail(ALLOY_ERR_UNSUPPORTED, "ssd_tc: unsupported sizes/layout");
  const TcLayout lay = tc_layout(s);
  const size_t need = lay.tiles;
  if (workspace == nullptr || workspace_bytes < need)
    return fail(ALLOY_ERR_INVALID_ARG, "ssd_tc: workspace of %zu bytes required, got %zu", need,
                workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) & 15)
    return fail(ALLOY_ERR_ALIGNMENT, "ssd_tc: workspace must be 16-byte aligned");
  int g0, gs;
  group_range(s, &g0, &gs);

  TcArgs a;
  memset(&a, 0, sizeof(a));
  a.B = s.B; a.L = s.L; a.H = s.H; a.N = s.N; a.G = s.G; a.K = s.K;
  a.head_begin = s.head_begin; a.group_begin = g0; a.group_count = gs;
  a.xbc = static_cast<const __nv_bfloat16*>(s.xBC); a.x_sb = s.xbc_sb; a.x_st = s.xbc_st;
  a.dt = s.dt_raw; a.dt_bf16 = s.dt_bf16; a.dt_sb = s.dt_sb; a.dt_st = s.dt_st; a.dt_sh = s.dt_sh;
  a.conv_w = s.conv_w; a.cw_sc = s.cw_sc; a.cw_sk = s.cw_sk;
  a.conv_b = s.conv_b; a.cb_s = s.cb_s;
  a.dt_bias = s.dt_bias; a.dtb_s = s.dtb_s;
  a.A_log = s.A_log; a.al_s = s.al_s;
  a.Dp = s.Dp; a.d_s = s.d_s;
  a.conv_in = static_cast<const __nv_bfloat16*>(s.conv_in);
  a.ci_sb = s.ci_sb; a.ci_sk = s.ci_sk; a.ci_sc = s.ci_sc;
  a.ssm_in = s.ssm_in; a.si_sb = s.si_sb; a.si_sh = s.si_sh; a.si_sn = s.si_sn; a.si_sp = s.si_sp;
  a.ssm_out = s.ssm_out; a.so_sb = s.so_sb; a.so_sh = s.so_sh; a.so_sn = s.so_sn; a.so_sp = s.so_sp;
  a.y = static_cast<__nv_bfloat16*>(s.y); a.y_sb = s.y_sb; a.y_st = s.y_st; a.y_sh = s.y_sh;
  a.stall_cycles = ssd_tc_stall_cycles().load(std::memory_order_relaxed);

  // 1. B/C conv pre-pass into the workspace
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encode_fn();
  if (!encode) return fail(ALLOY_ERR_CUDA, "ssd_tc: cuTensorMapEncodeTiled unavailable");
  const cuuint32_t estride[3] = {1, 1, 1};
  const cuuint64_t xd[3] = {(cuuint64_t)(s.H * 64 + 2 * s.G * s.N), (cuuint64_t)s.L, (cuuint64_t)s.B};
  const cuuint64_t xs[2] = {(cuuint64_t)s.xbc_st * 2, (cuuint64_t)s.xbc_sb * 2};
  const int ncols = 2 * gs * s.N;
  __nv_bfloat16* bc = static_cast<__nv_bfloat16*>(workspace);
  {
    // 128-column tiles where they divide a B / C block (gs * N is a multiple of 64)
    const int span = gs * s.N;
    const int W = span % 128 == 0 ? 128 : 64;
    CUtensorMap smap;
    const cuuint32_t sbox[3] = {(cuuint32_t)W, (cuuint32_t)(kBcTileRows + 3), 1};
    CUresult r = encode(&smap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(s.xBC), xd, xs, sbox,
                        estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(ALLOY_ERR_CUDA, "ssd_tc: cuTensorMapEncodeTiled (B/C tile) failed (%d)", (int)r);
    // every row of every chunk, the padded rows past L included (written as
    // zeros); runs of chunks per CTA long enough to double-buffer, short enough
    // to leave about four CTAs per SM
    const int nchunks = (s.L + Q - 1) / Q;
    const int tiles = nchunks * (ncols / W) * s.B;
    const int run = std::max(1, std::min(8, tiles / (4 * std::max(1, sm_count_of_current_device()))));
    dim3 grid((nchunks + run - 1) / run, ncols / W, s.B);
    const int smem = 2 * (((kBcTileRows + 3) * W * 2 + 1023) & ~1023);
    if (W == 128) {
      ALLOY_CUDA(cudaFuncSetAttribute(bc_conv_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      bc_conv_kernel<128><<<grid, 256, smem, stream>>>(smap, a, bc, ncols, run);
    } else {
      ALLOY_CUDA(cudaFuncSetAttribute(bc_conv_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      bc_conv_kernel<64><<<grid, 256, smem, stream>>>(smap, a, bc, ncols, run);
    }
    ALLOY_TRY(check_launch("bc_conv_kernel"));
  }
  a.bc = bc;
  // segments: only with the workspace for their states (a workspace of the
  // B/C tiles alone runs one CTA per head pair)
  a.nseg = workspace_bytes >= lay.total ? lay.nseg : 1;
  a.pieces = a.nseg > 1 ? lay.pieces : 1;
  a.nrec = a.nseg > 1 ? lay.nrec : 1;
  a.seg_state = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + lay.seg_state);
  a.seg_logdecay = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + lay.seg_logdecay);
  a.pairs = s.head_count / 2;
  // 4. the SSD kernel: the state-only pass over all segments but the last,
  // then the full pass over all
  // An unsegmented call's SSD kernel is launched with programmatic stream
  // serialization after the pre-pass: its prologue (TMEM, barriers, weights,
  // the first chunk's x rows and dt) overlaps the pre-pass's tail (measured:
  // -0.8 % at the Nemotron layer, -1.3 % at the Zamba2 layer).  In the
  // segmented chain (state-only pass, carry, full pass) the carry and the
  // full pass use ordinary launches: there the early start measured slower
  // (+6 % for the 131k-token sequence).  The
  // pre-pass itself is always an ordinary launch, so a call never overlaps
  // the previous one, which used the same workspace.
  auto launch = [&](auto kernel, int nz, bool after_prepass) -> int {
    ALLOY_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    const dim3 grid(s.head_count / 2, s.B, nz);
    if (after_prepass) {
      ALLOY_TRY(launch_after_previous(kernel, grid, dim3(kThreads), kSmemBytes, stream, a));
    } else {
      kernel<<<grid, kThreads, kSmemBytes, stream>>>(a);
    }
    return check_launch("ssd_tc_kernel");
  };
  // The state-only pass of short segments (at most 64 chunks: the 4- and 8-GPU
  // shards) is launched programmatically after the pre-pass too, its prologue
  // overlapping the pre-pass's tail (-1.1 % at both shards); with long
  // segments (one 131k-token sequence: 256 chunks) that measured +0.5 %.
  const bool pdl_state_only = (s.L + Q - 1) / Q <= 64 * a.nseg;
  // the states carried into the segments, from the state-only pass's records
  auto carry = [&]() -> int {
    const int pairs = s.head_count / 2;
    int S = 1;
    while (S < a.nrec && S < 32) S <<= 1;   // lanes a sub-warp: a piece each
    const int quads = 128 * s.N / 4;
    const int per_cta = 256 / S * kCarryQuads;
    seg_carry_kernel<<<dim3((quads + per_cta - 1) / per_cta, pairs, s.B), 256, 0, stream>>>(a, pairs, S);
    return check_launch("seg_carry_kernel");
  };
  // the split walk: slots of at most one CTA per SM, the first after the pre-pass
  auto split_walk = [&](auto kernel) -> int {
    ALLOY_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    a.split_units = s.B * a.pairs;
    const int tasks = a.split_units * a.nseg;
    const int slot = std::max(1, sm_count_of_current_device());
    for (int first = 0; first < tasks; first += slot) {
      a.split_base = first;
      const dim3 grid(std::min(slot, tasks - first));
      if (first == 0) {
        ALLOY_TRY(launch_after_previous(kernel, grid, dim3(kThreads), kSmemBytes, stream, a));
      } else {
        kernel<<<grid, kThreads, kSmemBytes, stream>>>(a);
      }
      ALLOY_TRY(check_launch("ssd_tc_kernel"));
    }
    return ALLOY_OK;
  };
  if (lay.split && a.nseg > 1)
    return s.N == 128 ? split_walk(ssd_tc_kernel<128, false>) : split_walk(ssd_tc_kernel<64, false>);
  if (s.N == 128) {
    if (a.nseg > 1) {
      ALLOY_TRY(launch(ssd_tc_kernel<128, true>, (a.nseg - 1) * a.pieces, pdl_state_only));
      ALLOY_TRY(carry());
    }
    return launch(ssd_tc_kernel<128, false>, a.nseg, a.nseg == 1);
  }
  if (a.nseg > 1) {
    ALLOY_TRY(launch(ssd_tc_kernel<64, true>, (a.nseg - 1) * a.pieces, pdl_state_only));
    ALLOY_TRY(carry());
  }
  return launch(ssd_tc_kernel<64, false>, a.nseg, a.nseg == 1);
}

std::atomic<long long>& ssd_tc_stall_cycles() {
  static std::atomic<long long> v{0};
  return v;
}

int ssd_tc_take_error(cudaStream_t stream, unsigned int out[3]) {
  ALLOY_CUDA(cudaStreamSynchronize(stream));
  unsigned int zero[3] = {0, 0, 0};
  ALLOY_CUDA(cudaMemcpyFromSymbol(out, g_ssd_tc_error, sizeof(zero)));
  if (out[0] != 0) ALLOY_CUDA(cudaMemcpyToSymbol(g_ssd_tc_error, zero, sizeof(zero)));
  return ALLOY_OK;
}

}  // namespace alloy
