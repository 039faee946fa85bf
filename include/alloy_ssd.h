/*
 * alloy_ssd.h -- C ABI of liballoy_ssd.so, the B200 (sm_100a) kernels of the
 * Mamba-2 mixer hot path of gxcsoccer/alloy.
 *
 * The reference (alloy, Python + MLX) has no native library; its hot path is
 * the set of Python functions cited beside each entry point below.  Each entry
 * point is what a ctypes binding in the reference's kernel package
 * (alloy/kernels/__init__.py, currently an empty placeholder) would call in
 * place of those functions.
 *
 * Conventions
 *   - Every tensor is passed as an alloy_tensor_t: a device pointer, a dtype,
 *     a shape and element strides (like DLPack's DLTensor, without the device
 *     field).  The caller owns every buffer; the library allocates nothing.
 *   - Every call is asynchronous on the given cudaStream_t (passed as void*,
 *     NULL = legacy default stream) and returns ALLOY_OK or a negative
 *     status.  Argument errors are detected on the host before any launch.
 *     alloy_get_last_error() returns the calling thread's last message.
 *   - State tensors may be updated in place (state_in == state_out).
 *   - No call traps, asserts or spins without bound on the device.
 */
#ifndef ALLOY_SSD_H
#define ALLOY_SSD_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ALLOY_API __attribute__((visibility("default")))
#else
#define ALLOY_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define ALLOY_SSD_ABI_VERSION 1

/* status codes */
#define ALLOY_OK                0
#define ALLOY_ERR_INVALID_ARG  -1  /* null pointer, bad shape/stride/dtype      */
#define ALLOY_ERR_UNSUPPORTED  -2  /* valid but not implemented for these sizes */
#define ALLOY_ERR_ALIGNMENT    -3  /* pointer/stride alignment not met          */
#define ALLOY_ERR_CUDA         -4  /* a CUDA runtime call failed                */
#define ALLOY_ERR_DEVICE       -5  /* no usable sm_100 device                   */
#define ALLOY_ERR_TIMEOUT      -6  /* a bounded device-side wait ran out        */

/* element types */
#define ALLOY_F32   0
#define ALLOY_BF16  1

#define ALLOY_MAX_DIMS 5

typedef struct alloy_tensor {
    void*   data;                     /* device pointer (NULL = absent)  */
    int32_t dtype;                    /* ALLOY_F32 / ALLOY_BF16          */
    int32_t ndim;
    int64_t shape[ALLOY_MAX_DIMS];
    int64_t stride[ALLOY_MAX_DIMS];   /* in elements                     */
} alloy_tensor_t;

/* Sizes of one Mamba-2 mixer (MambaBlock constructor arguments,
 * alloy/models/mamba_block.py:76-102), plus the head range this call
 * computes (head_begin, head_count; head_count 0 = all heads).  The head
 * range lets a multi-GPU caller shard a layer by (batch, head-group) without
 * copying: tensors stay full-width and only the selected heads are read and
 * written. */
typedef struct alloy_ssd_dims {
    int64_t n_heads;      /* H */
    int64_t head_dim;     /* P */
    int64_t d_state;      /* N */
    int64_t n_groups;     /* G, H % G == 0; head h uses group h / (H/G) */
    int64_t d_conv;       /* K (4) */
    int64_t chunk_size;   /* the reference's scan chunk; results do not depend on it */
    int64_t head_begin;
    int64_t head_count;
} alloy_ssd_dims_t;

/* ABI version (ALLOY_SSD_ABI_VERSION) and a human-readable build string. */
ALLOY_API int         alloy_abi_version(void);
ALLOY_API const char* alloy_build_info(void);

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len); returns its full length. */
ALLOY_API size_t alloy_get_last_error(char* buf, size_t len);

/*
 * Causal depthwise conv1d + SiLU on a pre-padded input.
 * Replaces fused_conv1d_silu (alloy/models/mamba_kernels.py:39-50, Metal
 * kernel :17-36) and MambaBlock._depthwise_conv1d + nn.silu
 * (alloy/models/mamba_block.py:144-158, :454-455).
 *
 *   x_padded [B, L+K-1, C]  F32|BF16, channel stride 1
 *   weight   [C, K]         F32|BF16 (any strides)
 *   bias     [C]            F32|BF16 (data NULL = zero bias)
 *   out      [B, L, C]      dtype of x_padded, channel stride 1
 *   out[b,t,c] = silu(bias[c] + sum_k x_padded[b,t+k,c] * weight[c,k]),
 *   accumulated in fp32.
 */
ALLOY_API int alloy_conv1d_silu(const alloy_tensor_t* x_padded, const alloy_tensor_t* weight,
                      const alloy_tensor_t* bias, alloy_tensor_t* out, void* stream);

/*
 * The same causal depthwise conv without the SiLU.
 * Replaces MambaBlock._depthwise_conv1d (alloy/models/mamba_block.py:144-158).
 * Arguments as for alloy_conv1d_silu; out[b,t,c] = bias[c] + sum_k x_padded[b,t+k,c] * weight[c,k].
 */
ALLOY_API int alloy_depthwise_conv1d(const alloy_tensor_t* x_padded, const alloy_tensor_t* weight,
                                     const alloy_tensor_t* bias, alloy_tensor_t* out, void* stream);

/*
 * Backward of conv1d + SiLU (the VJP of alloy_conv1d_silu).
 * Replaces _metal_conv1d_silu_vjp (alloy/models/mamba_block.py:25-47), the
 * VJP alloy registers for its Metal conv kernel (used by _forward_split
 * :401 when training).
 *
 *   x_padded  [B, L+K-1, C]  F32|BF16 (the forward's input)
 *   weight    [C, K], bias [C] (data NULL = zero bias), F32|BF16
 *   dy        [B, L, C]      dtype of x_padded (cotangent of the output)
 *   dx_padded [B, L+K-1, C]  dtype of x_padded; must not overlap x_padded or dy
 *   dweight   [C, K]         F32|BF16;  dbias [C] F32|BF16 (data NULL = not wanted)
 *   pre = bias + sum_k x_padded[t+k] weight[:,k];  sig = sigmoid(pre)
 *   g = dy * sig * (1 + pre * (1 - sig))
 *   dx_padded[t'] = sum_k g[t'-k] weight[:,k];  dweight[:,k] = sum_{b,t} g[t] x_padded[t+k];
 *   dbias = sum_{b,t} g[t]
 * fp32 arithmetic; dweight / dbias are summed in a fixed order (the same
 * result on every call).  workspace: device memory of at least
 * alloy_conv1d_silu_backward_workspace_size(B, L+K-1, C, K) bytes, 4-byte
 * aligned, holding the per-CTA partial sums of dweight and dbias.
 */
ALLOY_API int alloy_conv1d_silu_backward(const alloy_tensor_t* x_padded, const alloy_tensor_t* weight,
                               const alloy_tensor_t* bias, const alloy_tensor_t* dy,
                               alloy_tensor_t* dx_padded, alloy_tensor_t* dweight,
                               alloy_tensor_t* dbias, void* workspace, size_t workspace_bytes,
                               void* stream);
ALLOY_API size_t alloy_conv1d_silu_backward_workspace_size(int64_t batch, int64_t padded_len,
                                                 int64_t channels, int64_t d_conv);

/*
 * The projections of a decode step for 1 to 4 tokens: y = x W^T.
 * Replaces MambaBlock's in_proj / out_proj (alloy/models/mamba_block.py:438,
 * :501, nn.Linear without bias) when a cached step runs one token per
 * sequence, where the product is a weight-streaming GEMV.
 *
 *   x      [NB, in]   BF16, 1 <= NB <= 4, last dim contiguous, rows 16-byte aligned
 *   weight [out, in]  BF16 (the nn.Linear weight), last dim contiguous, rows 16-byte aligned
 *   y      [NB, out]  BF16, last dim contiguous
 * in a multiple of 8; fp32 accumulation.
 */
ALLOY_API int alloy_decode_linear(const alloy_tensor_t* x, const alloy_tensor_t* weight,
                                  alloy_tensor_t* y, void* stream);

/*
 * The projections of a prefill or a training step: y = x W^T (+ bias) on the
 * tensor cores.  Replaces MambaBlock's in_proj / out_proj
 * (alloy/models/mamba_block.py:438, :501, nn.Linear) over all B x L tokens
 * of a call (x flattened to [B*L, in]).
 *
 *   x      [M, K]  BF16, last dim contiguous
 *   weight [N, K]  BF16 (the nn.Linear weight [out, in]), last dim contiguous
 *   bias   [N]     BF16, contiguous, or data NULL for none
 *   y      [M, N]  BF16, last dim contiguous; must not overlap x or weight
 * K and every row stride a multiple of 8 elements, N a multiple of 8, data
 * 16-byte aligned (ALLOY_ERR_ALIGNMENT otherwise); fp32 accumulation, one
 * bf16 rounding of the result.
 */
ALLOY_API int alloy_linear(const alloy_tensor_t* x, const alloy_tensor_t* weight,
                           const alloy_tensor_t* bias, alloy_tensor_t* y, void* stream);

/*
 * Fused Mamba-2 mixer core in combined (Zamba2 / Nemotron-H) mode, prefill of
 * L >= 1 tokens: conv1d+SiLU with the conv-cache prefix, split into x|B|C,
 * discretisation, chunked SSD scan with state carry, D skip.
 * Replaces the hot part of MambaBlock._forward_combined
 * (alloy/models/mamba_block.py:446-493): the conv-cache update (:446-452),
 * _depthwise_conv1d + silu (:454-455), the group split/repeat (:458-468),
 * discretisation (:471-486), _selective_scan (:287-366, with _scan_chunk
 * :206-285) and the D residual (:481-482, :492-493).
 *
 *   xBC        [B, L, conv_dim]  F32|BF16, conv_dim = H*P + 2*G*N, channel stride 1
 *   dt_raw     [B, L, H]         F32|BF16 (the in_proj dt slice, before softplus)
 *   conv_w     [conv_dim, K]     F32;  conv_b [conv_dim] F32 (data NULL = 0)
 *   dt_bias, A_log [H]           F32;  D [H] F32 (data NULL = no D skip)
 *   ssm_in     [B, H, N, P] or any permutation via strides, F32 (data NULL = zeros)
 *   conv_in    [B, K-1, conv_dim] (any strides), dtype of xBC (data NULL = zeros)
 *   y          [B, L, H, P]      dtype of xBC (head/P strides free, P stride 1 for BF16)
 *   ssm_out    like ssm_in, F32 (data NULL = not written); may alias ssm_in
 *   conv_out   like conv_in (data NULL = not written); may alias conv_in
 *   workspace  device scratch of alloy_ssd_combined_workspace_size() bytes, or
 *              of at least alloy_ssd_combined_min_workspace_size() (may be
 *              NULL when that size is 0)
 * y = scan(dt*x) + D*x, where x is the UNSCALED conv output.
 */
ALLOY_API int alloy_ssd_combined(const alloy_tensor_t* xBC, const alloy_tensor_t* dt_raw,
                       const alloy_tensor_t* conv_w, const alloy_tensor_t* conv_b,
                       const alloy_tensor_t* dt_bias, const alloy_tensor_t* A_log,
                       const alloy_tensor_t* D,
                       const alloy_tensor_t* ssm_in, const alloy_tensor_t* conv_in,
                       alloy_tensor_t* y, alloy_tensor_t* ssm_out,
                       alloy_tensor_t* conv_out,
                       void* workspace, size_t workspace_bytes,
                       const alloy_ssd_dims_t* dims, void* stream);

/*
 * Bytes of device workspace alloy_ssd_combined needs for a call with this
 * batch, sequence length, activation dtype and dims (0 = none), on the
 * current device.  The workspace holds the conv + SiLU of the B and C columns
 * (bf16), shared by all heads of a group, and, when the call has fewer
 * (batch row, head pair) units than the GPU has SMs, the end states of the
 * sequence segments the kernel then walks in parallel.  It must be 16-byte
 * aligned and may be reused across calls that do not overlap on the device.
 * No counterpart in the reference (its kernels allocate their outputs through
 * MLX).
 */
ALLOY_API size_t alloy_ssd_combined_workspace_size(int64_t batch, int64_t seqlen, int32_t dtype,
                                                   const alloy_ssd_dims_t* dims);

/*
 * The smallest workspace alloy_ssd_combined accepts for the same call: the B/C
 * tiles alone.  With it each (batch row, head pair) is walked by one CTA from
 * its first chunk to its last (results equal up to the fp32 rounding of the
 * state carried between segments).  No counterpart in the reference.
 */
ALLOY_API size_t alloy_ssd_combined_min_workspace_size(int64_t batch, int64_t seqlen, int32_t dtype,
                                                       const alloy_ssd_dims_t* dims);

/*
 * alloy_ssd_combined for callers that cannot allocate device memory.
 * No counterpart in the reference (MLX allocates every buffer itself).
 *
 * Who needs it: a process that gives all device memory to its own pool at
 * start-up and forbids allocation afterwards, or a host runtime that only has
 * raw device pointers from another framework and no CUDA allocator of its own
 * (for instance a Go or Java service calling in through FFI).
 * Same arguments and results as alloy_ssd_combined, without the workspace:
 * the scratch comes from one fixed 8 MiB array compiled into the library,
 * held by every device that loads it until the process exits.  Calls whose
 * smallest scratch (alloy_ssd_combined_min_workspace_size: the B/C tiles
 * alone) exceeds 8 MiB are rejected with ALLOY_ERR_UNSUPPORTED before
 * anything is launched.  The whole 8 MiB is handed to alloy_ssd_combined as
 * its workspace, so a call whose full workspace
 * (alloy_ssd_combined_workspace_size) also fits runs the segmented schedule
 * with its segment records in the array too; one whose full size does not
 * fit walks each (batch row, head pair) with one CTA.  The call allocates and
 * frees nothing.
 *  - The first call in a device's context looks up the array's device
 *    address (cudaGetSymbolAddress) with that device current and keeps it
 *    with the context's unique id; after the context is destroyed and created
 *    again (cudaDeviceReset) the next call looks it up anew.  Make the first
 *    call on each device (and the first after a reset) before any stream
 *    capture begins.
 *  - All calls on a device share the array, and it keeps the last call's
 *    contents: calls that may overlap on the device (different streams, or
 *    other host threads) race and must be serialised by the caller.  Nothing
 *    needs clearing between calls: the scan reads only what the same call's
 *    B/C pre-pass wrote.
 */
ALLOY_API int alloy_ssd_combined_noalloc(const alloy_tensor_t* xBC, const alloy_tensor_t* dt_raw,
                       const alloy_tensor_t* conv_w, const alloy_tensor_t* conv_b,
                       const alloy_tensor_t* dt_bias, const alloy_tensor_t* A_log,
                       const alloy_tensor_t* D,
                       const alloy_tensor_t* ssm_in, const alloy_tensor_t* conv_in,
                       alloy_tensor_t* y, alloy_tensor_t* ssm_out,
                       alloy_tensor_t* conv_out,
                       const alloy_ssd_dims_t* dims, void* stream);

/*
 * Synchronises `stream` and reports whether a kernel launched since the last
 * check gave up on a bounded device-side wait (ALLOY_ERR_TIMEOUT, with the
 * site in the last-error message); clears the record.  No counterpart in the
 * reference (MLX kernels have no device-side waits).
 */
ALLOY_API int alloy_check_device_status(void* stream);

/*
 * Test hook for the bounded-wait error path of the tensor-core prefill.
 * While cycles > 0, every ssd_tc_kernel launched afterwards (the bf16 path of
 * alloy_ssd_combined) makes its consumer warps first wait, for that many
 * clock cycles, on an mbarrier that nothing arrives on.  The wait runs out,
 * the CTA records site 50 in the device error word, drains its copies and
 * MMAs in flight, frees its tensor memory and returns, so the next
 * alloy_check_device_status reports ALLOY_ERR_TIMEOUT; y and the states of
 * such a call are not valid.  0 (the default) switches it off.  Process-wide;
 * cycles in [0, 2^32].  No counterpart in the reference (MLX kernels have no
 * device-side waits).
 */
ALLOY_API int alloy_debug_set_wait_stall(int64_t cycles);

/*
 * Gated RMS norm of the mixer output:
 *   g = y * silu(gate);  out = g * rsqrt(mean of g^2 over the group + eps) * weight
 * with the group the whole row (group_size 0) or consecutive runs of
 * group_size channels; math in fp32, out in the activation dtype.  With
 * weight NULL (data NULL) only the gate is applied: out = y * silu(gate).
 * Replaces step 7 of MambaBlock._forward_combined
 * (alloy/models/mamba_block.py:495-499: `y = y * nn.silu(gate)`, then
 * `self.norm(y)` with the nn.RMSNorm(d_inner) of :137, eps 1e-5).
 *   y, gate, out  [rows, D] BF16 or F32 (one dtype), channel stride 1, any row
 *                 stride; out may alias y (same element layout)
 *   weight        [D] F32, or NULL
 *   eps           >= 0, added to the mean of squares
 *   group_size    channels per norm group, dividing D (0 = D)
 * No counterpart kernel in the reference (MLX element-wise ops and
 * mx.fast.rms_norm).
 */
ALLOY_API int alloy_gated_rmsnorm(const alloy_tensor_t* y, const alloy_tensor_t* gate,
                                  const alloy_tensor_t* weight, alloy_tensor_t* out, float eps,
                                  int64_t group_size, void* stream);

/*
 * Number of kernels this library has launched in this process (every thread
 * and device), for counting the launches of a timed region: a segmented
 * prefill (alloy_ssd_combined with fewer (batch row, head pair) units than
 * SMs) launches two more than an unsegmented one (the state-only pass and
 * the segment carry); a split walk (at least as many units as SMs, each
 * unit's sequence walked in segments by successive launches of at most one
 * CTA per SM, when the workspace holds the units' handover states) launches
 * one SSD kernel per slot instead of one.  No counterpart in the reference.
 */
ALLOY_API uint64_t alloy_kernel_launch_count(void);

/*
 * Selective scan on pre-discretised inputs.
 * Replaces MambaBlock._selective_scan (alloy/models/mamba_block.py:287-366)
 * -- and, through it, _scan_chunk (:206-285), _selective_scan_sequential
 * (:160-204) and scan_chunk_metal / fused_parallel_scan_chunk
 * (alloy/models/mamba_kernels.py:193-224, :333-396), which compute the same
 * recurrence over one chunk.
 *
 *   x       [B, L, H, P]   F32|BF16 (already dt-scaled), P stride 1
 *   A_disc  [B, L, H]      F32|BF16, used as log(max(A_disc, 1e-10)) when log_a is absent
 *   log_a   [B, L, H]      F32 (data NULL = absent), mamba_block.py:246-249
 *   Bm, Cm  [B, L, G', N]  F32|BF16, G' divides H (G' = H for per-head B/C)
 *   ssm_in  [B, H, N, P]   F32 via strides (data NULL = zeros)
 *   y       [B, L, H, P]   F32|BF16
 *   ssm_out [B, H, N, P]   F32 via strides (data NULL = not written), may alias ssm_in
 * h_t = a_t h_{t-1} + B_t x_t^T;  y_t = C_t h_t  (fp32 state and accumulation).
 * Precondition for BF16 x, B and C at (P, N) = (64, 64), (64, 128), (128, 64)
 * (the tensor-core scan): every decay is at most 1 (A_disc <= 1, log_a <= 0),
 * as the reference's A_disc = exp(A dt) with A < 0 always is.  That scan
 * factors exp(cum_t - cum_s) into exp(cum_t) and exp(-cum_s) pieces bounded
 * only for non-increasing cumulative sums; larger decays overflow there
 * without an error.  F32 inputs and other sizes run the fp32 scan, which has
 * no such bound.
 */
ALLOY_API int alloy_selective_scan(const alloy_tensor_t* x, const alloy_tensor_t* A_disc,
                         const alloy_tensor_t* log_a, const alloy_tensor_t* Bm,
                         const alloy_tensor_t* Cm, const alloy_tensor_t* ssm_in,
                         alloy_tensor_t* y, alloy_tensor_t* ssm_out, void* stream);

/*
 * The scan of alloy_selective_scan on the tensor cores with operands shared
 * across heads and fused row dot products, for the gradient scans of
 * training (MLX autograd through MambaBlock._selective_scan,
 * alloy/models/mamba_block.py:287-366; no kernel counterpart in the
 * reference).  n_heads H is y's dim 2 (dot's when y is absent).
 *
 *   x       [B, L, Gx, P]  BF16, Gx divides H (head h reads x row h / (H/Gx)), P stride 1
 *   log_a   [B, L, H]      F32, <= 0 (a precondition the kernel does not check:
 *                          a positive log decay overflows its factored decays)
 *   Bm, Cm  [B, L, G', N]  BF16, G' divides H, N stride 1
 *   ssm_in  [B, H, N, P]   F32 via strides (data NULL = zeros)
 *   y       [B, L, H, P]   F32|BF16 (data NULL = not written)
 *   ssm_out [B, H, N, P]   F32 via strides (data NULL = not written)
 *   z       [B, L, Gz, P]  F32|BF16, Gz divides H, P stride 1, 16-byte aligned rows
 *   dot     [B, L, H]      F32 (data NULL = not written): dot[b,t,h] = sum_p y[b,t,h,p] z[b,t,h/(H/Gz),p]
 *   dot_mode bit 0: the dots without the step's own term S[t,t] (x_t . z_t), S[t,t] =
 *            C_t . B_t as the kernel rounds it; bit 1: precise mode -- the decayed
 *            scores, exp(cum) C, the state copy and X' enter the products as pairs
 *            of bf16 values (~16 bits instead of 8), for outputs whose differences
 *            cancel (head_dim = d_state = 64 only); the two bits are exclusive
 * (P, N) must be (64, 64), (64, 128) or (128, 64), the rows of x, Bm and Cm
 * 16-byte aligned; other calls return ALLOY_ERR_UNSUPPORTED.
 */
ALLOY_API int alloy_selective_scan_dot(const alloy_tensor_t* x, const alloy_tensor_t* log_a,
                                       const alloy_tensor_t* Bm, const alloy_tensor_t* Cm,
                                       const alloy_tensor_t* ssm_in, alloy_tensor_t* y,
                                       alloy_tensor_t* ssm_out, const alloy_tensor_t* z,
                                       alloy_tensor_t* dot, int32_t dot_mode, void* stream);

/*
 * One decode token through the conv cache and the SSM cache, in place.
 * Replaces the L = 1 path of MambaBlock._forward_combined: the conv-cache roll
 * (alloy/models/mamba_block.py:446-448), conv + silu (:454-455), split
 * (:458-468), discretisation (:471-486), _selective_scan_sequential
 * (:160-204) and the D residual (:492-493).
 *
 *   xBC_tok    [B, conv_dim]  F32|BF16, channel stride 1
 *   dt_tok     [B, H]         F32|BF16
 *   conv_w, conv_b, dt_bias, A_log, D   as in alloy_ssd_combined
 *   conv_state [B, K-1, conv_dim] or [B, conv_dim, K-1] via strides, dtype of
 *              xBC_tok; read and rolled in place
 *   ssm_state  [B, H, N, P] or [B, H, P, N] (one of N, P with stride 1), F32,
 *              updated in place
 *   y          [B, H, P]      dtype of xBC_tok, P stride 1
 */
ALLOY_API int alloy_ssd_decode_step(const alloy_tensor_t* xBC_tok, const alloy_tensor_t* dt_tok,
                          const alloy_tensor_t* conv_w, const alloy_tensor_t* conv_b,
                          const alloy_tensor_t* dt_bias, const alloy_tensor_t* A_log,
                          const alloy_tensor_t* D,
                          alloy_tensor_t* conv_state, alloy_tensor_t* ssm_state,
                          alloy_tensor_t* y, const alloy_ssd_dims_t* dims, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ALLOY_SSD_H */
