// Internal launch interfaces of liballoy_ssd (host side).  Arguments have been
// validated by capi.cu before any of these is called.
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"

namespace alloy {

// conv.cu
int conv1d_silu(const alloy_tensor_t* x_padded, const alloy_tensor_t* w,
                const alloy_tensor_t* bias, alloy_tensor_t* out, bool silu, cudaStream_t s);

// conv_bwd.cu: VJP of conv1d + SiLU (dx_padded, dweight, dbias from dy);
// the workspace holds per-CTA partial sums of dweight / dbias
size_t conv1d_silu_backward_workspace(int64_t B, int64_t Lp, int64_t C, int64_t K);
int conv1d_silu_backward(const alloy_tensor_t* x_padded, const alloy_tensor_t* w,
                         const alloy_tensor_t* bias, const alloy_tensor_t* dy, alloy_tensor_t* dx,
                         alloy_tensor_t* dw, alloy_tensor_t* db, void* workspace, int B, int L, int C,
                         int K, cudaStream_t s);

// linear.cu: y [NB, out] = x [NB, in] W^T for NB <= 4 bf16 tokens (decode projections)
int decode_linear(const alloy_tensor_t* x, const alloy_tensor_t* w, alloy_tensor_t* y, cudaStream_t s);

// linear_tc.cu: y [M, N] = x [M, K] W^T (+ bias) on the tensor cores (prefill
// projections).  Supported: bf16 throughout, unit inner strides, row strides
// and K multiples of 8 elements, 16-byte aligned data.
bool linear_tc_supported(const alloy_tensor_t* x, const alloy_tensor_t* w, const alloy_tensor_t* y);
int linear_tc(const alloy_tensor_t* x, const alloy_tensor_t* w, const alloy_tensor_t* bias, alloy_tensor_t* y,
              cudaStream_t s);
// Synchronises the stream, then reads and clears the error word of the GEMM.
int linear_tc_take_error(cudaStream_t s, unsigned int out[3]);

// ssd_tc.cu: the driver's cuTensorMapEncodeTiled (null when unavailable)
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encode_fn();

// Flattened view of one SSD call, shared by the SSD kernels.  Strides are in
// elements.  mode 0: raw xBC (conv + discretisation fused); mode 1:
// pre-discretised inputs (x, log decay, B, C).
struct SsdArgs {
  int mode;
  int B, L, H, P, N, G, K;
  int head_begin, head_count;
  // mode 0 inputs
  const void* xBC; int xbc_bf16; int64_t xbc_sb, xbc_st;
  const void* dt_raw; int dt_bf16; int64_t dt_sb, dt_st, dt_sh;
  const float* conv_w; int64_t cw_sc, cw_sk;
  const float* conv_b; int64_t cb_s;
  const float* dt_bias; int64_t dtb_s;
  const float* A_log; int64_t al_s;
  const float* Dp; int64_t d_s;
  const void* conv_in; int ci_bf16; int64_t ci_sb, ci_sk, ci_sc;
  // mode 1 inputs
  const void* x; int x_bf16; int64_t x_sb, x_st, x_sh;
  const void* A_disc; int ad_bf16; int64_t ad_sb, ad_st, ad_sh;
  const float* log_a; int64_t la_sb, la_st, la_sh;
  const void* Bm; int bm_bf16; int64_t bm_sb, bm_st, bm_sg, bm_sn;
  const void* Cm; int cm_bf16; int64_t cm_sb, cm_st, cm_sg, cm_sn;
  int Gbc;
  // states and output
  const float* ssm_in; int64_t si_sb, si_sh, si_sn, si_sp;
  float* ssm_out; int64_t so_sb, so_sh, so_sn, so_sp;
  void* y; int y_bf16; int64_t y_sb, y_st, y_sh, y_sp;
  // tensor-core scan only: x indexed by head / x_hpg (x shared by x_hpg
  // consecutive heads; 1 = per head); optional row dot products
  // dot[b, t, h] = sum_p y[b, t, h, p] z[b, t, h / z_hpg, p] (y may then be null)
  int x_hpg;
  const void* z; int z_bf16; int64_t z_sb, z_st, z_sh; int z_hpg;
  float* dot; int64_t dot_sb, dot_st, dot_sh;
  // dot_nodiag: the dot products leave out the step's own term, S[t,t] (x_t . z_t)
  // with S[t,t] = C_t . B_t as the kernel rounds it
  int dot_nodiag;
  // precise_scores: the scores, exp(cum) C, the state copy and X' enter the
  // MMAs as bf16 pairs (hi + lo), ~16 bits instead of 8 (head_dim = d_state = 64)
  int precise_scores;
};

// scan_tc.cu: tcgen05 scan on pre-discretised bf16 inputs (mode 1: x, B, C
// bf16 with unit inner strides and 16-byte aligned rows; (P, N) = (64, 64),
// (64, 128) or (128, 64); log decays <= 0).
bool scan_tc_supported(const SsdArgs& a);
int scan_tc(const SsdArgs& a, cudaStream_t s);
// Synchronises the stream, then reads and clears the error word of the scan.
int scan_tc_take_error(cudaStream_t s, unsigned int out[3]);

// ssd_simt.cu: fp32 CUDA-core SSD (any sizes that fit shared memory).
int ssd_simt(const SsdArgs& a, cudaStream_t s);
size_t ssd_simt_smem_bytes(int P, int N);

// Rolls the conv cache after a prefill of L tokens: conv_out[b, j, c] =
// x_padded[b, L + j, c] for the channels of heads [h0, h0+hc) and of their
// groups' B and C columns.  Reads every source before writing, so conv_out
// may alias conv_in.
int conv_state_update(const alloy_tensor_t* xBC, const alloy_tensor_t* conv_in,
                      alloy_tensor_t* conv_out, int H, int P, int N, int G, int K,
                      int head_begin, int head_count, cudaStream_t s);

// decode.cu
struct DecodeArgs {
  int B, H, P, N, G, K, head_begin, head_count;
  const void* xbc; int x_bf16; int64_t x_sb;
  const void* dt; int dt_bf16; int64_t dt_sb, dt_sh;
  const float* conv_w; int64_t cw_sc, cw_sk;
  const float* conv_b; int64_t cb_s;
  const float* dt_bias; int64_t dtb_s;
  const float* A_log; int64_t al_s;
  const float* Dp; int64_t d_s;
  void* conv_state; int cs_bf16; int64_t cs_sb, cs_sk, cs_sc;
  float* state; int64_t st_sb, st_sh, st_row;   // row = the non-unit stride of (N, P)
  int state_pn;                                 // 1: [.., P, N] (N contiguous); 0: [.., N, P]
  void* y; int y_bf16; int64_t y_sb, y_sh;
};
int ssd_decode_step(const DecodeArgs& a, cudaStream_t s);

// norm.cu: out = rmsnorm(y * silu(gate)) * w over groups of `group` channels
// (w null: out = y * silu(gate)); y, gate, out [rows, D] with channel stride 1.
int gated_rmsnorm(const alloy_tensor_t* y, const alloy_tensor_t* gate, const alloy_tensor_t* w,
                  alloy_tensor_t* out, float eps, int group, cudaStream_t s);

// SMs of the current device (cached per device; 0 if the query fails).
int sm_count_of_current_device();

// ssd_tc.cu: tcgen05 tensor-core SSD for bf16 inputs (mode 0 only).
// Returns ALLOY_ERR_UNSUPPORTED (and launches nothing) for sizes it does not cover.
bool ssd_tc_supported(const SsdArgs& a);
size_t ssd_tc_workspace_bytes(const SsdArgs& a);       // with the sequence-segment states (fastest)
size_t ssd_tc_workspace_min_bytes(const SsdArgs& a);   // the B/C tiles alone (one CTA per head pair)
// workspace of alloy_ssd_combined for a layer: full size, or the smallest that
// runs (full == false); 0 when none is needed
size_t ssd_combined_workspace(int64_t batch, int64_t seqlen, int32_t dtype, const alloy_ssd_dims_t* dims,
                              bool full);
int ssd_tc(const SsdArgs& a, void* workspace, size_t workspace_bytes, cudaStream_t s);
// Synchronises the stream, then reads and clears the error word that a CTA
// of the tensor-core SSD writes when one of its bounded waits runs out.
int ssd_tc_take_error(cudaStream_t s, unsigned int out[3]);
// Cycles the consumer warps of every ssd_tc_kernel launched from now on first
// wait on a barrier nothing completes (0 = off; the bounded-wait test hook).
std::atomic<long long>& ssd_tc_stall_cycles();

}  // namespace alloy
