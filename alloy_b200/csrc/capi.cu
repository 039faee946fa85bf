// extern "C" entry points of liballoy_ssd (declared in include/alloy_ssd.h):
// argument validation on the host, then dispatch to the kernels.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace alloy {

std::string& last_error() {
  static thread_local std::string msg;
  return msg;
}

std::atomic<uint64_t>& launch_counter() {
  static std::atomic<uint64_t> n{0};
  return n;
}

int current_device_checked(int* dev) {
  // 0 = unchecked, 1 = sm_100, 2 = other architecture (per device, checked once)
  static int arch_ok[kMaxDevices] = {0};
  int d = 0;
  ALLOY_CUDA(cudaGetDevice(&d));
  if (d < 0 || d >= kMaxDevices) return fail(ALLOY_ERR_DEVICE, "device index %d out of range", d);
  if (arch_ok[d] == 0) {
    int major = 0, minor = 0;
    ALLOY_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d));
    ALLOY_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, d));
    arch_ok[d] = (major == 10 && minor == 0) ? 1 : 2;
    if (arch_ok[d] == 2)
      return fail(ALLOY_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", d,
                  major, minor);
  }
  if (arch_ok[d] == 2) return fail(ALLOY_ERR_DEVICE, "device %d is not sm_100", d);
  if (dev) *dev = d;
  return ALLOY_OK;
}

namespace {

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int check_vec(const alloy_tensor_t* t, const char* name, int64_t n, unsigned mask, bool optional) {
  if (optional && !present(t)) return ALLOY_OK;
  const int64_t shape[1] = {n};
  return check_tensor(t, name, 1, shape, mask);
}

int check_dims(const alloy_ssd_dims_t* d, int64_t* h0, int64_t* hc) {
  if (d == nullptr) return fail(ALLOY_ERR_INVALID_ARG, "dims: null");
  if (d->n_heads <= 0 || d->head_dim <= 0 || d->d_state <= 0 || d->n_groups <= 0)
    return fail(ALLOY_ERR_INVALID_ARG, "dims: n_heads, head_dim, d_state, n_groups must be > 0");
  if (d->n_heads % d->n_groups != 0)
    return fail(ALLOY_ERR_INVALID_ARG, "dims: n_heads (%lld) not divisible by n_groups (%lld)",
                (long long)d->n_heads, (long long)d->n_groups);
  if (d->d_conv < 2 || d->d_conv > 8)
    return fail(ALLOY_ERR_UNSUPPORTED, "dims: d_conv must be in [2, 8]");
  if (d->chunk_size <= 0) return fail(ALLOY_ERR_INVALID_ARG, "dims: chunk_size must be > 0");
  const int64_t count = d->head_count == 0 ? d->n_heads - d->head_begin : d->head_count;
  if (d->head_begin < 0 || count <= 0 || d->head_begin + count > d->n_heads)
    return fail(ALLOY_ERR_INVALID_ARG, "dims: head range [%lld, +%lld) outside [0, %lld)",
                (long long)d->head_begin, (long long)count, (long long)d->n_heads);
  if (d->n_heads * d->head_dim > (1 << 24) || d->d_state > 1024 || d->head_dim > 1024)
    return fail(ALLOY_ERR_UNSUPPORTED, "dims: sizes out of the supported range");
  *h0 = d->head_begin;
  *hc = count;
  return ALLOY_OK;
}

}  // namespace

size_t ssd_combined_workspace(int64_t batch, int64_t seqlen, int32_t dtype, const alloy_ssd_dims_t* dims,
                              bool full) {
  int64_t h0 = 0, hc = 0;
  if (check_dims(dims, &h0, &hc) != ALLOY_OK || batch < 0 || seqlen < 0) return 0;
  SsdArgs a;
  memset(&a, 0, sizeof(a));
  a.mode = 0;
  a.B = (int)batch; a.L = (int)seqlen; a.H = (int)dims->n_heads; a.P = (int)dims->head_dim;
  a.N = (int)dims->d_state; a.G = (int)dims->n_groups; a.K = (int)dims->d_conv;
  a.head_begin = (int)h0; a.head_count = (int)hc;
  a.xbc_bf16 = a.y_bf16 = (dtype == ALLOY_BF16);
  a.y_sp = 1;
  // layout conditions are checked per call; size the workspace by dims alone
  if (!a.xbc_bf16 || a.P != 64 || !(a.N == 64 || a.N == 128) || a.K != 4 ||
      (a.H / a.G) % 2 != 0 || a.head_begin % 2 != 0 || a.head_count % 2 != 0)
    return 0;
  return full ? ssd_tc_workspace_bytes(a) : ssd_tc_workspace_min_bytes(a);
}

}  // namespace alloy

using namespace alloy;

extern "C" {

int alloy_abi_version(void) { return ALLOY_SSD_ABI_VERSION; }

const char* alloy_build_info(void) {
  return "liballoy_ssd " __DATE__ " sm_100a (tcgen05 SSD, conv1d+SiLU, decode step)";
}

size_t alloy_get_last_error(char* buf, size_t len) {
  const std::string& m = last_error();
  if (buf && len) {
    const size_t n = std::min(len - 1, m.size());
    memcpy(buf, m.data(), n);
    buf[n] = '\0';
  }
  return m.size();
}

namespace {
int conv_entry(const alloy_tensor_t* x_padded, const alloy_tensor_t* weight,
               const alloy_tensor_t* bias, alloy_tensor_t* out, bool silu, void* stream) {
  last_error().clear();
  ALLOY_TRY(check_tensor(x_padded, "x_padded", 3, nullptr, kAnyFloat));
  ALLOY_TRY(check_tensor(weight, "weight", 2, nullptr, kAnyFloat));
  const int64_t B = x_padded->shape[0], Lp = x_padded->shape[1], C = x_padded->shape[2];
  const int64_t K = weight->shape[1];
  if (weight->shape[0] != C)
    return fail(ALLOY_ERR_INVALID_ARG, "weight: dim 0 is %lld, expected C = %lld",
                (long long)weight->shape[0], (long long)C);
  if (K < 1 || K > 8) return fail(ALLOY_ERR_UNSUPPORTED, "weight: K must be in [1, 8]");
  if (Lp < K - 1) return fail(ALLOY_ERR_INVALID_ARG, "x_padded: fewer than K-1 rows");
  ALLOY_TRY(check_vec(bias, "bias", C, kAnyFloat, true));
  const int64_t oshape[3] = {B, Lp - K + 1, C};
  ALLOY_TRY(check_tensor(out, "out", 3, oshape, 1u << x_padded->dtype));
  if (B * Lp * C >= (int64_t)1 << 40) return fail(ALLOY_ERR_UNSUPPORTED, "x_padded: too large");
  ALLOY_TRY(current_device_checked(nullptr));
  return conv1d_silu(x_padded, weight, bias, out, silu, as_stream(stream));
}
}  // namespace

int alloy_conv1d_silu(const alloy_tensor_t* x_padded, const alloy_tensor_t* weight,
                      const alloy_tensor_t* bias, alloy_tensor_t* out, void* stream) {
  return conv_entry(x_padded, weight, bias, out, true, stream);
}

int alloy_depthwise_conv1d(const alloy_tensor_t* x_padded, const alloy_tensor_t* weight,
                           const alloy_tensor_t* bias, alloy_tensor_t* out, void* stream) {
  return conv_entry(x_padded, weight, bias, out, false, stream);
}

size_t alloy_conv1d_silu_backward_workspace_size(int64_t batch, int64_t padded_len, int64_t channels,
                                                 int64_t d_conv) {
  if (batch < 0 || channels < 0 || d_conv < 1 || d_conv > 8 || padded_len < d_conv - 1) return 0;
  return conv1d_silu_backward_workspace(batch, padded_len, channels, d_conv);
}

int alloy_conv1d_silu_backward(const alloy_tensor_t* x_padded, const alloy_tensor_t* weight,
                               const alloy_tensor_t* bias, const alloy_tensor_t* dy,
                               alloy_tensor_t* dx_padded, alloy_tensor_t* dweight,
                               alloy_tensor_t* dbias, void* workspace, size_t workspace_bytes,
                               void* stream) {
  last_error().clear();
  ALLOY_TRY(check_tensor(x_padded, "x_padded", 3, nullptr, kAnyFloat));
  ALLOY_TRY(check_tensor(weight, "weight", 2, nullptr, kAnyFloat));
  const int64_t B = x_padded->shape[0], Lp = x_padded->shape[1], C = x_padded->shape[2];
  const int64_t K = weight->shape[1];
  if (weight->shape[0] != C)
    return fail(ALLOY_ERR_INVALID_ARG, "weight: dim 0 is %lld, expected C = %lld",
                (long long)weight->shape[0], (long long)C);
  if (K < 1 || K > 8) return fail(ALLOY_ERR_UNSUPPORTED, "weight: K must be in [1, 8]");
  if (Lp < K - 1) return fail(ALLOY_ERR_INVALID_ARG, "x_padded: fewer than K-1 rows");
  ALLOY_TRY(check_vec(bias, "bias", C, kAnyFloat, true));
  const unsigned act = 1u << x_padded->dtype;
  const int64_t yshape[3] = {B, Lp - K + 1, C};
  ALLOY_TRY(check_tensor(dy, "dy", 3, yshape, act));
  ALLOY_TRY(check_tensor(dx_padded, "dx_padded", 3, x_padded->shape, act));
  const int64_t wshape[2] = {C, K};
  ALLOY_TRY(check_tensor(dweight, "dweight", 2, wshape, kAnyFloat));
  ALLOY_TRY(check_vec(dbias, "dbias", C, kAnyFloat, true));
  if (B > 65535) return fail(ALLOY_ERR_UNSUPPORTED, "x_padded: batch above 65535");
  if (B * Lp * C >= (int64_t)1 << 40) return fail(ALLOY_ERR_UNSUPPORTED, "x_padded: too large");
  const size_t need = conv1d_silu_backward_workspace(B, Lp, C, K);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(ALLOY_ERR_INVALID_ARG, "conv1d_silu_backward: workspace of %zu bytes required, got %zu",
                need, workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) & 3)
    return fail(ALLOY_ERR_ALIGNMENT, "conv1d_silu_backward: workspace must be 4-byte aligned");
  ALLOY_TRY(current_device_checked(nullptr));
  return conv1d_silu_backward(x_padded, weight, bias, dy, dx_padded, dweight, dbias, workspace, (int)B,
                              (int)(Lp - K + 1), (int)C, (int)K, as_stream(stream));
}

int alloy_decode_linear(const alloy_tensor_t* x, const alloy_tensor_t* weight, alloy_tensor_t* y,
                        void* stream) {
  last_error().clear();
  ALLOY_TRY(check_tensor(x, "x", 2, nullptr, kBF16));
  ALLOY_TRY(check_tensor(weight, "weight", 2, nullptr, kBF16));
  const int64_t NB = x->shape[0], in = x->shape[1], out = weight->shape[0];
  if (weight->shape[1] != in)
    return fail(ALLOY_ERR_INVALID_ARG, "weight: dim 1 is %lld, expected in = %lld",
                (long long)weight->shape[1], (long long)in);
  const int64_t ys[2] = {NB, out};
  ALLOY_TRY(check_tensor(y, "y", 2, ys, kBF16));
  if (NB < 1 || NB > 4) return fail(ALLOY_ERR_UNSUPPORTED, "decode_linear: 1 to 4 rows, got %lld", (long long)NB);
  if (in % 8 != 0 || in * NB * 2 > 200 * 1024)
    return fail(ALLOY_ERR_UNSUPPORTED, "decode_linear: in must be a multiple of 8 and rows fit shared memory");
  if (x->stride[1] != 1 || weight->stride[1] != 1 || y->stride[1] != 1)
    return fail(ALLOY_ERR_INVALID_ARG, "decode_linear: the last dimension must be contiguous");
  if (!aligned16(x->data) || !aligned16(weight->data) || (x->stride[0] * 2) % 16 != 0 ||
      (weight->stride[0] * 2) % 16 != 0)
    return fail(ALLOY_ERR_ALIGNMENT, "decode_linear: x and weight rows must be 16-byte aligned");
  if (out > (int64_t)1 << 30) return fail(ALLOY_ERR_UNSUPPORTED, "decode_linear: too many outputs");
  ALLOY_TRY(current_device_checked(nullptr));
  return decode_linear(x, weight, y, as_stream(stream));
}

int alloy_linear(const alloy_tensor_t* x, const alloy_tensor_t* weight, const alloy_tensor_t* bias,
                 alloy_tensor_t* y, void* stream) {
  last_error().clear();
  ALLOY_TRY(check_tensor(x, "x", 2, nullptr, kBF16));
  ALLOY_TRY(check_tensor(weight, "weight", 2, nullptr, kBF16));
  const int64_t M = x->shape[0], K = x->shape[1], N = weight->shape[0];
  if (weight->shape[1] != K)
    return fail(ALLOY_ERR_INVALID_ARG, "weight: dim 1 is %lld, expected in = %lld", (long long)weight->shape[1],
                (long long)K);
  if (present(bias)) ALLOY_TRY(check_vec(bias, "bias", N, kBF16, false));
  if (present(bias) && bias->stride[0] != 1) return fail(ALLOY_ERR_INVALID_ARG, "linear: bias must be contiguous");
  const int64_t ys[2] = {M, N};
  ALLOY_TRY(check_tensor(y, "y", 2, ys, kBF16));
  if (x->stride[1] != 1 || weight->stride[1] != 1 || y->stride[1] != 1)
    return fail(ALLOY_ERR_INVALID_ARG, "linear: the last dimension must be contiguous");
  if (M >= ((int64_t)1 << 31) || N >= ((int64_t)1 << 31) || K >= ((int64_t)1 << 31))
    return fail(ALLOY_ERR_UNSUPPORTED, "linear: extents must be below 2^31");
  if (M == 0 || N == 0) return ALLOY_OK;
  if (K == 0) return fail(ALLOY_ERR_UNSUPPORTED, "linear: K = 0");
  if (K % 8 != 0 || N % 8 != 0 || x->stride[0] % 8 != 0 || weight->stride[0] % 8 != 0 || y->stride[0] % 8 != 0 ||
      !aligned16(x->data) || !aligned16(weight->data) || !aligned16(y->data) ||
      (present(bias) && (reinterpret_cast<uintptr_t>(bias->data) & 3u) != 0))
    return fail(ALLOY_ERR_ALIGNMENT,
                "linear: K, N and the row strides must be multiples of 8 elements and the data 16-byte aligned");
  ALLOY_TRY(current_device_checked(nullptr));
  return linear_tc(x, weight, bias, y, as_stream(stream));
}

int alloy_ssd_combined(const alloy_tensor_t* xBC, const alloy_tensor_t* dt_raw,
                       const alloy_tensor_t* conv_w, const alloy_tensor_t* conv_b,
                       const alloy_tensor_t* dt_bias, const alloy_tensor_t* A_log,
                       const alloy_tensor_t* D, const alloy_tensor_t* ssm_in,
                       const alloy_tensor_t* conv_in, alloy_tensor_t* y,
                       alloy_tensor_t* ssm_out, alloy_tensor_t* conv_out,
                       void* workspace, size_t workspace_bytes,
                       const alloy_ssd_dims_t* dims, void* stream) {
  last_error().clear();
  int64_t h0 = 0, hc = 0;
  ALLOY_TRY(check_dims(dims, &h0, &hc));
  const int64_t H = dims->n_heads, P = dims->head_dim, N = dims->d_state, G = dims->n_groups,
                K = dims->d_conv;
  const int64_t conv_dim = H * P + 2 * G * N;
  ALLOY_TRY(check_tensor(xBC, "xBC", 3, nullptr, kAnyFloat));
  const int64_t B = xBC->shape[0], L = xBC->shape[1];
  if (xBC->shape[2] != conv_dim)
    return fail(ALLOY_ERR_INVALID_ARG, "xBC: dim 2 is %lld, expected H*P + 2*G*N = %lld",
                (long long)xBC->shape[2], (long long)conv_dim);
  if (xBC->stride[2] != 1) return fail(ALLOY_ERR_INVALID_ARG, "xBC: channel stride must be 1");
  const unsigned act = 1u << xBC->dtype;
  const int64_t dts[3] = {B, L, H};
  ALLOY_TRY(check_tensor(dt_raw, "dt_raw", 3, dts, kAnyFloat));
  const int64_t cws[2] = {conv_dim, K};
  ALLOY_TRY(check_tensor(conv_w, "conv_w", 2, cws, kF32));
  ALLOY_TRY(check_vec(conv_b, "conv_b", conv_dim, kF32, true));
  ALLOY_TRY(check_vec(dt_bias, "dt_bias", H, kF32, false));
  ALLOY_TRY(check_vec(A_log, "A_log", H, kF32, false));
  ALLOY_TRY(check_vec(D, "D", H, kF32, true));
  // states: [B, H, N, P] in any axis order given through strides
  const int64_t ss[4] = {B, H, N, P};
  if (present(ssm_in)) ALLOY_TRY(check_tensor(ssm_in, "ssm_in", 4, ss, kF32));
  if (present(ssm_out)) ALLOY_TRY(check_tensor(ssm_out, "ssm_out", 4, ss, kF32));
  const int64_t cs[3] = {B, K - 1, conv_dim};
  if (present(conv_in)) ALLOY_TRY(check_tensor(conv_in, "conv_in", 3, cs, act));
  if (present(conv_out)) ALLOY_TRY(check_tensor(conv_out, "conv_out", 3, cs, act));
  const int64_t ys[4] = {B, L, H, P};
  ALLOY_TRY(check_tensor(y, "y", 4, ys, act));
  if (L == 0 && present(conv_out) == false && present(ssm_out) == false) return ALLOY_OK;
  ALLOY_TRY(current_device_checked(nullptr));
  const cudaStream_t s = as_stream(stream);

  SsdArgs a;
  memset(&a, 0, sizeof(a));
  a.mode = 0;
  a.B = (int)B; a.L = (int)L; a.H = (int)H; a.P = (int)P; a.N = (int)N; a.G = (int)G;
  a.K = (int)K; a.head_begin = (int)h0; a.head_count = (int)hc;
  a.xBC = xBC->data; a.xbc_bf16 = xBC->dtype == ALLOY_BF16;
  a.xbc_sb = xBC->stride[0]; a.xbc_st = xBC->stride[1];
  a.dt_raw = dt_raw->data; a.dt_bf16 = dt_raw->dtype == ALLOY_BF16;
  a.dt_sb = dt_raw->stride[0]; a.dt_st = dt_raw->stride[1]; a.dt_sh = dt_raw->stride[2];
  a.conv_w = static_cast<const float*>(conv_w->data);
  a.cw_sc = conv_w->stride[0]; a.cw_sk = conv_w->stride[1];
  if (present(conv_b)) { a.conv_b = static_cast<const float*>(conv_b->data); a.cb_s = conv_b->stride[0]; }
  a.dt_bias = static_cast<const float*>(dt_bias->data); a.dtb_s = dt_bias->stride[0];
  a.A_log = static_cast<const float*>(A_log->data); a.al_s = A_log->stride[0];
  if (present(D)) { a.Dp = static_cast<const float*>(D->data); a.d_s = D->stride[0]; }
  if (present(conv_in)) {
    a.conv_in = conv_in->data; a.ci_bf16 = conv_in->dtype == ALLOY_BF16;
    a.ci_sb = conv_in->stride[0]; a.ci_sk = conv_in->stride[1]; a.ci_sc = conv_in->stride[2];
  }
  if (present(ssm_in)) {
    a.ssm_in = static_cast<const float*>(ssm_in->data);
    a.si_sb = ssm_in->stride[0]; a.si_sh = ssm_in->stride[1];
    a.si_sn = ssm_in->stride[2]; a.si_sp = ssm_in->stride[3];
  }
  if (present(ssm_out)) {
    a.ssm_out = static_cast<float*>(ssm_out->data);
    a.so_sb = ssm_out->stride[0]; a.so_sh = ssm_out->stride[1];
    a.so_sn = ssm_out->stride[2]; a.so_sp = ssm_out->stride[3];
  }
  a.y = y->data; a.y_bf16 = y->dtype == ALLOY_BF16;
  a.y_sb = y->stride[0]; a.y_st = y->stride[1]; a.y_sh = y->stride[2]; a.y_sp = y->stride[3];

  if (L > 0) {
    if (ssd_tc_supported(a)) {
      ALLOY_TRY(ssd_tc(a, workspace, workspace_bytes, s));
    } else {
      ALLOY_TRY(ssd_simt(a, s));
    }
  } else if (present(ssm_out)) {
    // zero tokens: the state passes through unchanged
    return fail(ALLOY_ERR_UNSUPPORTED, "ssd_combined: L = 0 with ssm_out");
  }
  if (present(conv_out)) {
    // must run after the scan: the scan reads conv_in, which conv_out may alias
    ALLOY_TRY(conv_state_update(xBC, present(conv_in) ? conv_in : nullptr, conv_out, (int)H,
                                (int)P, (int)N, (int)G, (int)K, (int)h0, (int)hc, s));
  }
  return ALLOY_OK;
}


size_t alloy_ssd_combined_workspace_size(int64_t batch, int64_t seqlen, int32_t dtype,
                                         const alloy_ssd_dims_t* dims) {
  return ssd_combined_workspace(batch, seqlen, dtype, dims, true);
}

size_t alloy_ssd_combined_min_workspace_size(int64_t batch, int64_t seqlen, int32_t dtype,
                                             const alloy_ssd_dims_t* dims) {
  return ssd_combined_workspace(batch, seqlen, dtype, dims, false);
}

int alloy_gated_rmsnorm(const alloy_tensor_t* y, const alloy_tensor_t* gate,
                        const alloy_tensor_t* weight, alloy_tensor_t* out, float eps,
                        int64_t group_size, void* stream) {
  last_error().clear();
  ALLOY_TRY(check_tensor(y, "y", 2, nullptr, kAnyFloat));
  const int64_t rows = y->shape[0], D = y->shape[1];
  const int64_t s2[2] = {rows, D};
  const unsigned act = 1u << y->dtype;
  ALLOY_TRY(check_tensor(gate, "gate", 2, s2, act));
  ALLOY_TRY(check_tensor(out, "out", 2, s2, act));
  if (y->stride[1] != 1 || gate->stride[1] != 1 || out->stride[1] != 1)
    return fail(ALLOY_ERR_INVALID_ARG, "gated_rmsnorm: channel stride must be 1");
  ALLOY_TRY(check_vec(weight, "weight", D, kF32, true));
  const int64_t grp = group_size == 0 ? D : group_size;
  if (grp <= 0 || (D > 0 && D % grp != 0))
    return fail(ALLOY_ERR_INVALID_ARG, "gated_rmsnorm: group_size %lld does not divide %lld channels",
                (long long)group_size, (long long)D);
  if (!(eps >= 0.f)) return fail(ALLOY_ERR_INVALID_ARG, "gated_rmsnorm: eps must be >= 0");
  if (D > (1 << 24) || rows >= ((int64_t)1 << 31))
    return fail(ALLOY_ERR_UNSUPPORTED, "gated_rmsnorm: %lld rows x %lld channels too large",
                (long long)rows, (long long)D);
  if (rows == 0 || D == 0) return ALLOY_OK;
  ALLOY_TRY(current_device_checked(nullptr));
  return gated_rmsnorm(y, gate, present(weight) ? weight : nullptr, out, eps, (int)grp,
                       as_stream(stream));
}

uint64_t alloy_kernel_launch_count(void) { return launch_counter().load(std::memory_order_relaxed); }

int alloy_check_device_status(void* stream) {
  last_error().clear();
  unsigned int e[3] = {0, 0, 0};
  ALLOY_TRY(ssd_tc_take_error(as_stream(stream), e));
  if (e[0] != 0)
    return fail(ALLOY_ERR_TIMEOUT, "ssd_tc_kernel: bounded wait at site %u ran out (block %u, %u)",
                e[0] - 1, e[1], e[2]);
  ALLOY_TRY(scan_tc_take_error(as_stream(stream), e));
  if (e[0] != 0)
    return fail(ALLOY_ERR_TIMEOUT, "scan_tc_kernel: bounded wait at site %u ran out (block %u, %u)",
                e[0] - 1, e[1], e[2]);
  ALLOY_TRY(linear_tc_take_error(as_stream(stream), e));
  if (e[0] != 0)
    return fail(ALLOY_ERR_TIMEOUT, "linear_tc_kernel: bounded wait at site %u ran out (block %u, tile %u)",
                e[0] - 1, e[1], e[2]);
  return ALLOY_OK;
}

int alloy_debug_set_wait_stall(int64_t cycles) {
  last_error().clear();
  if (cycles < 0 || cycles > (int64_t(1) << 32))
    return fail(ALLOY_ERR_INVALID_ARG, "debug_set_wait_stall: cycles must be in [0, 2^32]");
  ssd_tc_stall_cycles().store(cycles, std::memory_order_relaxed);
  return ALLOY_OK;
}

int alloy_selective_scan(const alloy_tensor_t* x, const alloy_tensor_t* A_disc,
                         const alloy_tensor_t* log_a, const alloy_tensor_t* Bm,
                         const alloy_tensor_t* Cm, const alloy_tensor_t* ssm_in,
                         alloy_tensor_t* y, alloy_tensor_t* ssm_out, void* stream) {
  last_error().clear();
  ALLOY_TRY(check_tensor(x, "x", 4, nullptr, kAnyFloat));
  const int64_t B = x->shape[0], L = x->shape[1], H = x->shape[2], P = x->shape[3];
  const int64_t bh[3] = {B, L, H};
  if (present(log_a)) {
    ALLOY_TRY(check_tensor(log_a, "log_a", 3, bh, kF32));
  } else {
    ALLOY_TRY(check_tensor(A_disc, "A_disc", 3, bh, kAnyFloat));
  }
  ALLOY_TRY(check_tensor(Bm, "B", 4, nullptr, kAnyFloat));
  const int64_t Gb = Bm->shape[2], N = Bm->shape[3];
  const int64_t bs[4] = {B, L, Gb, N};
  ALLOY_TRY(check_tensor(Bm, "B", 4, bs, kAnyFloat));
  ALLOY_TRY(check_tensor(Cm, "C", 4, bs, kAnyFloat));
  if (Gb <= 0 || H % Gb != 0)
    return fail(ALLOY_ERR_INVALID_ARG, "B/C: group dim %lld does not divide n_heads %lld",
                (long long)Gb, (long long)H);
  const int64_t ss[4] = {B, H, N, P};
  if (present(ssm_in)) ALLOY_TRY(check_tensor(ssm_in, "ssm_in", 4, ss, kF32));
  if (present(ssm_out)) ALLOY_TRY(check_tensor(ssm_out, "ssm_out", 4, ss, kF32));
  const int64_t ys[4] = {B, L, H, P};
  ALLOY_TRY(check_tensor(y, "y", 4, ys, kAnyFloat));
  if (x->stride[3] != 1) return fail(ALLOY_ERR_INVALID_ARG, "x: head_dim stride must be 1");
  if (B == 0 || H == 0) return ALLOY_OK;
  if (L == 0) return fail(ALLOY_ERR_UNSUPPORTED, "selective_scan: L = 0");
  ALLOY_TRY(current_device_checked(nullptr));

  SsdArgs a;
  memset(&a, 0, sizeof(a));
  a.mode = 1;
  a.B = (int)B; a.L = (int)L; a.H = (int)H; a.P = (int)P; a.N = (int)N; a.G = 1; a.K = 1;
  a.head_begin = 0; a.head_count = (int)H; a.Gbc = (int)Gb;
  a.x = x->data; a.x_bf16 = x->dtype == ALLOY_BF16; a.x_hpg = 1;
  a.x_sb = x->stride[0]; a.x_st = x->stride[1]; a.x_sh = x->stride[2];
  if (present(log_a)) {
    a.log_a = static_cast<const float*>(log_a->data);
    a.la_sb = log_a->stride[0]; a.la_st = log_a->stride[1]; a.la_sh = log_a->stride[2];
  } else {
    a.A_disc = A_disc->data; a.ad_bf16 = A_disc->dtype == ALLOY_BF16;
    a.ad_sb = A_disc->stride[0]; a.ad_st = A_disc->stride[1]; a.ad_sh = A_disc->stride[2];
  }
  a.Bm = Bm->data; a.bm_bf16 = Bm->dtype == ALLOY_BF16;
  a.bm_sb = Bm->stride[0]; a.bm_st = Bm->stride[1]; a.bm_sg = Bm->stride[2]; a.bm_sn = Bm->stride[3];
  a.Cm = Cm->data; a.cm_bf16 = Cm->dtype == ALLOY_BF16;
  a.cm_sb = Cm->stride[0]; a.cm_st = Cm->stride[1]; a.cm_sg = Cm->stride[2]; a.cm_sn = Cm->stride[3];
  if (present(ssm_in)) {
    a.ssm_in = static_cast<const float*>(ssm_in->data);
    a.si_sb = ssm_in->stride[0]; a.si_sh = ssm_in->stride[1];
    a.si_sn = ssm_in->stride[2]; a.si_sp = ssm_in->stride[3];
  }
  if (present(ssm_out)) {
    a.ssm_out = static_cast<float*>(ssm_out->data);
    a.so_sb = ssm_out->stride[0]; a.so_sh = ssm_out->stride[1];
    a.so_sn = ssm_out->stride[2]; a.so_sp = ssm_out->stride[3];
  }
  a.y = y->data; a.y_bf16 = y->dtype == ALLOY_BF16;
  a.y_sb = y->stride[0]; a.y_st = y->stride[1]; a.y_sh = y->stride[2]; a.y_sp = y->stride[3];
  // bf16 operands of the tensor-core sizes: tcgen05 scan; otherwise the fp32 CUDA-core scan
  if (scan_tc_supported(a)) return scan_tc(a, as_stream(stream));
  return ssd_simt(a, as_stream(stream));
}

int alloy_selective_scan_dot(const alloy_tensor_t* x, const alloy_tensor_t* log_a,
                             const alloy_tensor_t* Bm, const alloy_tensor_t* Cm,
                             const alloy_tensor_t* ssm_in, alloy_tensor_t* y, alloy_tensor_t* ssm_out,
                             const alloy_tensor_t* z, alloy_tensor_t* dot, int32_t dot_mode, void* stream) {
  last_error().clear();
  if (!present(y) && !present(dot)) return fail(ALLOY_ERR_INVALID_ARG, "selective_scan_dot: neither y nor dot");
  if (dot_mode < 0 || dot_mode > 2)
    return fail(ALLOY_ERR_INVALID_ARG, "selective_scan_dot: dot_mode must be 0, 1 or 2 (the bits are exclusive)");
  ALLOY_TRY(check_tensor(x, "x", 4, nullptr, kBF16));
  const alloy_tensor_t* ref = present(y) ? y : dot;
  const int64_t B = x->shape[0], L = x->shape[1], P = x->shape[3];
  const int64_t H = ref->shape[2];
  if (present(y)) {
    ALLOY_TRY(check_tensor(y, "y", 4, nullptr, kAnyFloat));
    const int64_t ys[4] = {B, L, y->shape[2], P};
    ALLOY_TRY(check_tensor(y, "y", 4, ys, kAnyFloat));
  }
  const int64_t bh[3] = {B, L, H};
  if (present(dot)) ALLOY_TRY(check_tensor(dot, "dot", 3, bh, kF32));
  ALLOY_TRY(check_tensor(log_a, "log_a", 3, bh, kF32));
  auto divides = [&](int64_t g, const char* name) {
    return (g > 0 && H % g == 0) ? ALLOY_OK
                                 : fail(ALLOY_ERR_INVALID_ARG, "%s: dim 2 (%lld) does not divide n_heads %lld",
                                        name, (long long)g, (long long)H);
  };
  ALLOY_TRY(divides(x->shape[2], "x"));
  ALLOY_TRY(check_tensor(Bm, "B", 4, nullptr, kBF16));
  const int64_t Gb = Bm->shape[2], N = Bm->shape[3];
  const int64_t bs[4] = {B, L, Gb, N};
  ALLOY_TRY(check_tensor(Bm, "B", 4, bs, kBF16));
  ALLOY_TRY(check_tensor(Cm, "C", 4, bs, kBF16));
  ALLOY_TRY(divides(Gb, "B/C"));
  if (present(dot)) {
    ALLOY_TRY(check_tensor(z, "z", 4, nullptr, kAnyFloat));
    const int64_t zs[4] = {B, L, z->shape[2], P};
    ALLOY_TRY(check_tensor(z, "z", 4, zs, kAnyFloat));
    ALLOY_TRY(divides(z->shape[2], "z"));
    if (z->stride[3] != 1) return fail(ALLOY_ERR_INVALID_ARG, "z: head_dim stride must be 1");
  }
  const int64_t ss[4] = {B, H, N, P};
  if (present(ssm_in)) ALLOY_TRY(check_tensor(ssm_in, "ssm_in", 4, ss, kF32));
  if (present(ssm_out)) ALLOY_TRY(check_tensor(ssm_out, "ssm_out", 4, ss, kF32));
  if (x->stride[3] != 1) return fail(ALLOY_ERR_INVALID_ARG, "x: head_dim stride must be 1");
  if (B == 0 || H == 0) return ALLOY_OK;
  if (L == 0) return fail(ALLOY_ERR_UNSUPPORTED, "selective_scan_dot: L = 0");
  ALLOY_TRY(current_device_checked(nullptr));

  SsdArgs a;
  memset(&a, 0, sizeof(a));
  a.mode = 1;
  a.B = (int)B; a.L = (int)L; a.H = (int)H; a.P = (int)P; a.N = (int)N; a.G = 1; a.K = 1;
  a.head_begin = 0; a.head_count = (int)H; a.Gbc = (int)Gb;
  a.x = x->data; a.x_bf16 = 1; a.x_hpg = (int)(H / x->shape[2]);
  a.x_sb = x->stride[0]; a.x_st = x->stride[1]; a.x_sh = x->stride[2];
  a.log_a = static_cast<const float*>(log_a->data);
  a.la_sb = log_a->stride[0]; a.la_st = log_a->stride[1]; a.la_sh = log_a->stride[2];
  a.Bm = Bm->data; a.bm_bf16 = 1;
  a.bm_sb = Bm->stride[0]; a.bm_st = Bm->stride[1]; a.bm_sg = Bm->stride[2]; a.bm_sn = Bm->stride[3];
  a.Cm = Cm->data; a.cm_bf16 = 1;
  a.cm_sb = Cm->stride[0]; a.cm_st = Cm->stride[1]; a.cm_sg = Cm->stride[2]; a.cm_sn = Cm->stride[3];
  if (present(ssm_in)) {
    a.ssm_in = static_cast<const float*>(ssm_in->data);
    a.si_sb = ssm_in->stride[0]; a.si_sh = ssm_in->stride[1];
    a.si_sn = ssm_in->stride[2]; a.si_sp = ssm_in->stride[3];
  }
  if (present(ssm_out)) {
    a.ssm_out = static_cast<float*>(ssm_out->data);
    a.so_sb = ssm_out->stride[0]; a.so_sh = ssm_out->stride[1];
    a.so_sn = ssm_out->stride[2]; a.so_sp = ssm_out->stride[3];
  }
  if (present(y)) {
    if (y->shape[2] != H) return fail(ALLOY_ERR_INVALID_ARG, "y: dim 2 must be n_heads");
    a.y = y->data; a.y_bf16 = y->dtype == ALLOY_BF16;
    a.y_sb = y->stride[0]; a.y_st = y->stride[1]; a.y_sh = y->stride[2]; a.y_sp = y->stride[3];
  }
  if (present(dot)) {
    a.z = z->data; a.z_bf16 = z->dtype == ALLOY_BF16; a.z_hpg = (int)(H / z->shape[2]);
    a.z_sb = z->stride[0]; a.z_st = z->stride[1]; a.z_sh = z->stride[2];
    a.dot = static_cast<float*>(dot->data);
    a.dot_sb = dot->stride[0]; a.dot_st = dot->stride[1]; a.dot_sh = dot->stride[2];
    a.dot_nodiag = dot_mode & 1;
  }
  a.precise_scores = (dot_mode >> 1) & 1;
  if (!scan_tc_supported(a))
    return fail(ALLOY_ERR_UNSUPPORTED,
                "selective_scan_dot: needs (head_dim, d_state) of (64, 64), (64, 128) or (128, 64) (64, 64 "
                "in the precise mode), unit inner strides and 16-byte aligned rows");
  return scan_tc(a, as_stream(stream));
}

int alloy_ssd_decode_step(const alloy_tensor_t* xBC_tok, const alloy_tensor_t* dt_tok,
                          const alloy_tensor_t* conv_w, const alloy_tensor_t* conv_b,
                          const alloy_tensor_t* dt_bias, const alloy_tensor_t* A_log,
                          const alloy_tensor_t* D, alloy_tensor_t* conv_state,
                          alloy_tensor_t* ssm_state, alloy_tensor_t* y,
                          const alloy_ssd_dims_t* dims, void* stream) {
  last_error().clear();
  int64_t h0 = 0, hc = 0;
  ALLOY_TRY(check_dims(dims, &h0, &hc));
  const int64_t H = dims->n_heads, P = dims->head_dim, N = dims->d_state, G = dims->n_groups,
                K = dims->d_conv;
  const int64_t conv_dim = H * P + 2 * G * N;
  ALLOY_TRY(check_tensor(xBC_tok, "xBC_tok", 2, nullptr, kAnyFloat));
  const int64_t B = xBC_tok->shape[0];
  if (xBC_tok->shape[1] != conv_dim)
    return fail(ALLOY_ERR_INVALID_ARG, "xBC_tok: dim 1 is %lld, expected %lld",
                (long long)xBC_tok->shape[1], (long long)conv_dim);
  if (xBC_tok->stride[1] != 1) return fail(ALLOY_ERR_INVALID_ARG, "xBC_tok: channel stride must be 1");
  const unsigned act = 1u << xBC_tok->dtype;
  const int64_t dts[2] = {B, H};
  ALLOY_TRY(check_tensor(dt_tok, "dt_tok", 2, dts, kAnyFloat));
  const int64_t cws[2] = {conv_dim, K};
  ALLOY_TRY(check_tensor(conv_w, "conv_w", 2, cws, kF32));
  ALLOY_TRY(check_vec(conv_b, "conv_b", conv_dim, kF32, true));
  ALLOY_TRY(check_vec(dt_bias, "dt_bias", H, kF32, false));
  ALLOY_TRY(check_vec(A_log, "A_log", H, kF32, false));
  ALLOY_TRY(check_vec(D, "D", H, kF32, true));
  const int64_t cs[3] = {B, K - 1, conv_dim};
  ALLOY_TRY(check_tensor(conv_state, "conv_state", 3, cs, act));
  const int64_t ss[4] = {B, H, N, P};
  ALLOY_TRY(check_tensor(ssm_state, "ssm_state", 4, ss, kF32));
  const int64_t ys[3] = {B, H, P};
  ALLOY_TRY(check_tensor(y, "y", 3, ys, act));
  if (y->stride[2] != 1) return fail(ALLOY_ERR_INVALID_ARG, "y: head_dim stride must be 1");
  int state_pn;
  int64_t row;
  if (ssm_state->stride[2] == 1 && N > 1) {          // N contiguous: [.., P, N]
    state_pn = 1; row = ssm_state->stride[3];
  } else if (ssm_state->stride[3] == 1) {            // P contiguous: [.., N, P]
    state_pn = 0; row = ssm_state->stride[2];
  } else {
    return fail(ALLOY_ERR_INVALID_ARG, "ssm_state: one of the d_state / head_dim strides must be 1");
  }
  if (B == 0) return ALLOY_OK;
  ALLOY_TRY(current_device_checked(nullptr));

  DecodeArgs a;
  memset(&a, 0, sizeof(a));
  a.B = (int)B; a.H = (int)H; a.P = (int)P; a.N = (int)N; a.G = (int)G; a.K = (int)K;
  a.head_begin = (int)h0; a.head_count = (int)hc;
  a.xbc = xBC_tok->data; a.x_bf16 = xBC_tok->dtype == ALLOY_BF16; a.x_sb = xBC_tok->stride[0];
  a.dt = dt_tok->data; a.dt_bf16 = dt_tok->dtype == ALLOY_BF16;
  a.dt_sb = dt_tok->stride[0]; a.dt_sh = dt_tok->stride[1];
  a.conv_w = static_cast<const float*>(conv_w->data);
  a.cw_sc = conv_w->stride[0]; a.cw_sk = conv_w->stride[1];
  if (present(conv_b)) { a.conv_b = static_cast<const float*>(conv_b->data); a.cb_s = conv_b->stride[0]; }
  a.dt_bias = static_cast<const float*>(dt_bias->data); a.dtb_s = dt_bias->stride[0];
  a.A_log = static_cast<const float*>(A_log->data); a.al_s = A_log->stride[0];
  if (present(D)) { a.Dp = static_cast<const float*>(D->data); a.d_s = D->stride[0]; }
  a.conv_state = conv_state->data; a.cs_bf16 = conv_state->dtype == ALLOY_BF16;
  a.cs_sb = conv_state->stride[0]; a.cs_sk = conv_state->stride[1]; a.cs_sc = conv_state->stride[2];
  a.state = static_cast<float*>(ssm_state->data);
  a.st_sb = ssm_state->stride[0]; a.st_sh = ssm_state->stride[1]; a.st_row = row;
  a.state_pn = state_pn;
  a.y = y->data; a.y_bf16 = y->dtype == ALLOY_BF16; a.y_sb = y->stride[0]; a.y_sh = y->stride[1];
  return ssd_decode_step(a, as_stream(stream));
}

}  // extern "C"
