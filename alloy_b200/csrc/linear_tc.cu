// Tensor-core (tcgen05) GEMM for the projections of a prefill:
//   y [M, N] = x [M, K] W^T (+ bias),  W [N, K] as nn.Linear holds it,
// MambaBlock's in_proj and out_proj (alloy/models/mamba_block.py:438, :501)
// over all B x L tokens of a call.  bf16 operands, fp32 accumulation in tensor
// memory, bf16 result.
//
// One persistent CTA per SM walks output tiles of 256 x 256 (tile t, t + grid,
// ...), raster-ordered in bands of 16 row tiles so that the CTAs running at
// the same time share their x rows and W rows in L2.  Warp roles (12 warps):
//   warp 0     TMA: a K-step (64 columns) of the tile's x rows and W rows per
//              stage, 128-byte swizzled, into a 3-stage ring (64 KB a stage);
//   warp 1     tensor memory allocation and MMA issue: per stage two chains of
//              four M128 x N256 x K16 MMAs (rows 0-127 and 128-255 of the tile)
//              into the two accumulators (512 columns: the whole tensor memory);
//   warps 2-3  idle (they complete warpgroup 0 for the register split);
//   warps 4-11 epilogue: warp w reads lane quadrant w % 4 of accumulator
//              (w - 4) / 4, adds the bias, rounds to bf16 and writes 32 x 64
//              pieces through a swizzled shared-memory buffer with TMA stores.
// The accumulators are released as soon as the epilogue has read them into
// registers, so the next tile's MMAs overlap the conversion and the stores;
// the TMA warp runs up to three stages ahead of the MMAs across tiles.
// Every mbarrier wait is bounded: on timeout the CTA records an error word,
// waits (bounded) for its copies and MMAs in flight, frees its tensor memory
// and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace alloy {

// error word written by a CTA whose bounded wait ran out (0 = none):
// [0] = 1 + site id, [1] = blockIdx.x, [2] = the tile it was on
__device__ unsigned int g_linear_tc_error[3];

namespace {

using namespace tc;

constexpr int BM = 256, BN = 256, BK = 64, STAGES = 3;
constexpr int kEpiWarps = 8;
constexpr int kEpiWarp0 = 4;                          // epilogue: warpgroups 1 and 2
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;
// register split: warpgroup 0 (TMA, MMA, two idle warps) gives up registers
// to the epilogue, which holds a tile's 256 columns as bf16 pairs
constexpr int kRegsLaunch = 168, kRegsRole = 56, kRegsEpi = 224;
static_assert(4 * kRegsRole + kEpiWarps * kRegsEpi <= (4 + kEpiWarps) * kRegsLaunch, "register split");
constexpr int kBandRows = 16;                         // row tiles per raster band
constexpr long long kWaitCycles = 4000000000LL;       // ~2 s at 1.9 GHz
constexpr uint32_t kATile = BM * BK * 2;              // 32 KB
constexpr uint32_t kBTile = BN * BK * 2;              // 32 KB
constexpr uint32_t kStage = kATile + kBTile;
constexpr uint32_t kOutPiece = 32 * 64 * 2;           // one epilogue warp's 32 rows x 64 columns
constexpr uint32_t OFF_OUT = STAGES * kStage;
constexpr uint32_t OFF_BAR = OFF_OUT + kEpiWarps * kOutPiece;
enum { B_FULL0 = 0, B_EMPTY0 = B_FULL0 + STAGES, B_TFULL = B_EMPTY0 + STAGES, B_TEMPTY, B_DRAIN, NBAR };
constexpr uint32_t OFF_TMEMPTR = OFF_BAR + 8 * NBAR;
constexpr uint32_t OFF_ABORT = OFF_TMEMPTR + 8;
constexpr uint32_t kSmemUsed = OFF_ABORT + 8;
constexpr uint32_t kSmem = kSmemUsed + 1024;          // + slack to align the base to 1024 bytes
static_assert(kSmem <= 232448, "shared memory per CTA");
// M = 128 (one accumulator = the tile's rows 0-127 or 128-255), N = 256, both K-major
constexpr uint32_t kIdesc = idesc_bf16(128, BN, 0, 0);

enum { SITE_LOAD = 0, SITE_MMA_FULL = 1, SITE_MMA_TEMPTY = 2, SITE_EPI = 3 };

__device__ __forceinline__ void signal_abort(volatile int* abort_flag, int site, int tile) {
  *abort_flag = 1;
  if (atomicCAS(&g_linear_tc_error[0], 0u, 1u + site) == 0u) {
    g_linear_tc_error[1] = blockIdx.x;
    g_linear_tc_error[2] = (unsigned)tile;
  }
}

// single-thread wait (TMA / MMA lanes)
__device__ __forceinline__ bool wait1(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site, int tile) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      signal_abort(abort_flag, site, tile);
      return false;
    }
  }
  return true;
}

// warp-uniform wait (epilogue warps)
__device__ __forceinline__ bool waitw(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site, int tile) {
  const long long t0 = clock64();
  bool ok;
  while (!(ok = mbar_try_wait(bar, parity) != 0)) {
    if (*abort_flag || clock64() - t0 > kWaitCycles) break;
  }
  ok = __all_sync(0xffffffffu, ok);
  if (!ok && (threadIdx.x & 31) == 0 && !*abort_flag) signal_abort(abort_flag, site, tile);
  __syncwarp();
  return ok;
}

// row and column tile of tile t: bands of kBandRows row tiles, columns outer
// within a band, so consecutive tiles (the CTAs of one wave) share x and W rows
__device__ __forceinline__ void tile_of(int t, int m_tiles, int n_tiles, int& mt, int& nt) {
  const int per_band = kBandRows * n_tiles;
  const int band = t / per_band, in = t - band * per_band;
  const int m0 = band * kBandRows;
  const int rows = min(kBandRows, m_tiles - m0);
  mt = m0 + in % rows;
  nt = in / rows;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

template <bool HAS_BIAS>
__global__ void __launch_bounds__(kThreads, 1)
linear_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                 const __grid_constant__ CUtensorMap ymap, const __nv_bfloat16* __restrict__ bias, int M, int N,
                 int K) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);
  volatile uint32_t* tmem_ptr = reinterpret_cast<volatile uint32_t*>(smem + OFF_TMEMPTR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_ABORT);
  auto bar = [&](int i) { return base + OFF_BAR + 8u * i; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;
  const int nk = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int i = 0; i < NBAR; ++i) mbar_init(bar(i), i == B_TEMPTY ? kEpiWarps : 1);
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&xmap);
    prefetch_tmap(&wmap);
    prefetch_tmap(&ymap);
  }
  if (warp == 1) {
    tmem_alloc(base + OFF_TMEMPTR, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_ptr;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA
    reg_dealloc<kRegsRole>();
    if (lane == 0) {
      uint32_t it = 0;   // stage uses so far
      for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x) {
        int mt, nt;
        tile_of(t, m_tiles, n_tiles, mt, nt);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait1(bar(B_EMPTY0 + s), ph ^ 1, abort_flag, SITE_LOAD, t)) break;
          const uint32_t dst = base + s * kStage;
          mbar_arrive_expect_tx(bar(B_FULL0 + s), kStage);
          tma_load_2d(dst, &xmap, bar(B_FULL0 + s), kb * BK, mt * BM);
          tma_load_2d(dst + kATile, &wmap, bar(B_FULL0 + s), kb * BK, nt * BN);
        }
      }
      // on abort: wait (bounded) for the copies still in flight
      if (*abort_flag) {
        const uint32_t first = it > (uint32_t)STAGES ? it - STAGES : 0u;
        for (uint32_t j = first; j < it; ++j) {
          const long long t0 = clock64();
          while (!mbar_try_wait(bar(B_FULL0 + j % STAGES), (j / STAGES) & 1) && clock64() - t0 < kWaitCycles) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issue
    reg_dealloc<kRegsRole>();
    if (lane == 0) {
      uint32_t it = 0;
      int n_done = 0;
      for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++n_done) {
        // the epilogue has read the previous tile's accumulators
        if (n_done > 0 && !wait1(bar(B_TEMPTY), (n_done - 1) & 1, abort_flag, SITE_MMA_TEMPTY, t)) break;
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (!(ok = wait1(bar(B_FULL0 + s), (it / STAGES) & 1, abort_flag, SITE_MMA_FULL, t))) break;
          tc_fence_after();
          const uint32_t a = base + s * kStage, b = a + kATile;
          // 4 K16 steps 32 bytes apart inside the 128-byte swizzled rows
          umma_bf16_chain4<2, 2, sw128_hi(1024), sw128_hi(1024)>(tmem, sw128_lo(a, 16), sw128_lo(b, 16), kIdesc,
                                                                  kb > 0);
          umma_bf16_chain4<2, 2, sw128_hi(1024), sw128_hi(1024)>(tmem + 256, sw128_lo(a + kATile / 2, 16),
                                                                  sw128_lo(b, 16), kIdesc, kb > 0);
          umma_commit(bar(B_EMPTY0 + s));
        }
        if (!ok) break;
        umma_commit(bar(B_TFULL));
      }
      if (*abort_flag) {
        // wait (bounded) for every MMA issued so far before the memory is freed
        umma_commit(bar(B_DRAIN));
        const long long t0 = clock64();
        while (!mbar_try_wait(bar(B_DRAIN), 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    reg_dealloc<kRegsRole>();
  } else {
    // ------------------------------------------------------------------ epilogue
    reg_alloc<kRegsEpi>();
    const int q = warp & 3;                    // lane quadrant this warp may read
    const int half = (warp - kEpiWarp0) >> 2;  // accumulator: tile rows 0-127 or 128-255
    const uint32_t acc = tmem + 256u * half + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t piece = base + OFF_OUT + (warp - kEpiWarp0) * kOutPiece;
    int n_done = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++n_done) {
      int mt, nt;
      tile_of(t, m_tiles, n_tiles, mt, nt);
      if (!waitw(bar(B_TFULL), n_done & 1, abort_flag, SITE_EPI, t)) break;
      tc_fence_after();
      // the tile's 256 columns of this warp's 32 rows into registers as bf16
      // pairs (bias added), then release the accumulators to the next tile
      uint32_t pk[4][32];
      const int row0 = mt * BM + 128 * half + 32 * q;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t r[32];
        tmem_ld32(acc + 32 * j, r);
        tmem_ld_wait();
        const int col0 = nt * BN + 32 * j;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          float a0 = __uint_as_float(r[2 * c]), a1 = __uint_as_float(r[2 * c + 1]);
          if (HAS_BIAS) {
            // bias pairs past N read as zero (N is a multiple of 8, so a pair is all in or all out)
            const uint32_t bw = col0 + 2 * c < N ? __ldg(reinterpret_cast<const unsigned int*>(bias + col0) + c) : 0u;
            a0 += bf16_lo(bw);
            a1 += bf16_hi(bw);
          }
          pk[j >> 1][16 * (j & 1) + c] = pack_bf16x2(a0, a1);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_TEMPTY));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col0 = nt * BN + 64 * j;
        // the previous piece's store has finished reading the buffer
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_shared_v4(piece + lane * 128 + ((c ^ (lane & 7)) << 4), pk[j][4 * c], pk[j][4 * c + 1],
                       pk[j][4 * c + 2], pk[j][4 * c + 3]);
        fence_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < M && col0 < N) {
          tma_store_2d(&ymap, piece, col0, row0);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

bool linear_tc_supported(const alloy_tensor_t* x, const alloy_tensor_t* w, const alloy_tensor_t* y) {
  const int64_t K = x->shape[1];
  return x->dtype == ALLOY_BF16 && w->dtype == ALLOY_BF16 && y->dtype == ALLOY_BF16 && x->stride[1] == 1 &&
         w->stride[1] == 1 && y->stride[1] == 1 && K % 8 == 0 && x->stride[0] % 8 == 0 && w->stride[0] % 8 == 0 &&
         y->stride[0] % 8 == 0 && aligned16(x->data) && aligned16(w->data) && aligned16(y->data);
}

int linear_tc(const alloy_tensor_t* x, const alloy_tensor_t* w, const alloy_tensor_t* bias, alloy_tensor_t* y,
              cudaStream_t stream) {
  const int64_t M = x->shape[0], K = x->shape[1], N = w->shape[0];
  if (M == 0 || N == 0) return ALLOY_OK;
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encode_fn();
  if (!encode) return fail(ALLOY_ERR_CUDA, "linear_tc: cuTensorMapEncodeTiled unavailable");
  const cuuint32_t estride[2] = {1, 1};
  auto make = [&](CUtensorMap* map, const void* p, int64_t rows, int64_t cols, int64_t ld, uint32_t box_cols,
                  uint32_t box_rows, const char* what) -> int {
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {box_cols, box_rows};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(p), dims, strides, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ALLOY_ERR_CUDA, "linear_tc: cuTensorMapEncodeTiled (%s) failed (%d)", what, (int)r);
    return ALLOY_OK;
  };
  CUtensorMap xmap, wmap, ymap;
  ALLOY_TRY(make(&xmap, x->data, M, K, x->stride[0], BK, BM, "x"));
  ALLOY_TRY(make(&wmap, w->data, N, K, w->stride[0], BK, BN, "weight"));
  ALLOY_TRY(make(&ymap, y->data, M, N, y->stride[0], 64, 32, "y"));
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = (int)std::min<int64_t>(tiles, std::max(1, sm_count_of_current_device()));
  auto launch = [&](auto kernel) -> int {
    // the register split hands out exactly what the launch provides: a build
    // with another register count would leave the epilogue's increase waiting
    cudaFuncAttributes fa;
    ALLOY_CUDA(cudaFuncGetAttributes(&fa, kernel));
    if (fa.numRegs != kRegsLaunch)
      return fail(ALLOY_ERR_CUDA, "linear_tc: kernel built with %d registers a thread, the split assumes %d",
                  fa.numRegs, kRegsLaunch);
    ALLOY_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
    kernel<<<grid, kThreads, kSmem, stream>>>(
        xmap, wmap, ymap, present(bias) ? static_cast<const __nv_bfloat16*>(bias->data) : nullptr, (int)M, (int)N,
        (int)K);
    return ALLOY_OK;
  };
  ALLOY_TRY(present(bias) ? launch(linear_tc_kernel<true>) : launch(linear_tc_kernel<false>));
  return check_launch("linear_tc_kernel");
}

int linear_tc_take_error(cudaStream_t s, unsigned int out[3]) {
  const unsigned int zero[3] = {0, 0, 0};
  ALLOY_CUDA(cudaStreamSynchronize(s));
  ALLOY_CUDA(cudaMemcpyFromSymbol(out, g_linear_tc_error, sizeof(zero)));
  if (out[0] != 0) ALLOY_CUDA(cudaMemcpyToSymbol(g_linear_tc_error, zero, sizeof(zero)));
  return ALLOY_OK;
}

}  // namespace alloy
