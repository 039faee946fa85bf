"""numpy restatement of alloy's Mamba-2 mixer hot path (oracle; test infrastructure).

Every function cites the reference lines it restates (paths relative to the
gxcsoccer/alloy project root).  Layouts follow the reference:

* ``xBC``          [B, L, conv_dim]   conv input, channels = [x | B | C]
* ``x``            [B, L, H, P]       per-head SSM input
* ``B``, ``C``     [B, L, G|H, N]     input-dependent SSM matrices
* ``ssm_state``    [B, H, N, P]       fp32 (``MambaCache.ssm_state``)
* ``conv_state``   [B, K-1, conv_dim] (``MambaCache.conv_state``)

All arithmetic is float32, like the reference's fp32 path, except the
``*_fp64`` functions, which are an independent float64 ground truth.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32

__all__ = [
    "softplus", "sigmoid", "silu", "depthwise_conv1d", "conv1d_silu", "conv1d_silu_vjp",
    "pad_conv_input", "discretize", "scan_chunk", "selective_scan",
    "selective_scan_sequential", "mixer_core", "mixer_core_fp64",
    "decode_step_fp64", "gated_rmsnorm", "make_inputs", "bf16_round", "rel_l2",
    "max_rel", "CONFIGS",
]


# ---------------------------------------------------------------------------
# element-wise activations (MLX nn.softplus / nn.silu semantics)
# ---------------------------------------------------------------------------

def softplus(x):
    """``nn.softplus`` = log(1 + exp(x)), computed as logaddexp(x, 0)."""
    return np.logaddexp(x, x.dtype.type(0)).astype(x.dtype, copy=False)


def sigmoid(x):
    one = x.dtype.type(1)
    return one / (one + np.exp(-x))


def silu(x):
    """``nn.silu`` (mamba_block.py:455) and the fused kernel's
    ``acc / (1 + exp(-acc))`` (mamba_kernels.py:33)."""
    return x * sigmoid(x)


# ---------------------------------------------------------------------------
# A1 / A2: causal depthwise conv1d (+ SiLU)
# ---------------------------------------------------------------------------

def depthwise_conv1d(x_padded, weight, bias, L):
    """Sliding-window depthwise conv, mamba_block.py:144-158.

    x_padded [B, L+K-1, C], weight [C, K], bias [C] -> [B, L, C].
    """
    out = np.zeros_like(x_padded[:, :L, :])
    for k in range(weight.shape[1]):
        out = out + x_padded[:, k:k + L, :] * weight[:, k]
    return out + bias


def conv1d_silu(x_padded, weight, bias, L):
    """Fused conv1d + SiLU, mamba_kernels.py:17-50 (K1) == mamba_block.py:454-455."""
    return silu(depthwise_conv1d(x_padded, weight, bias, L))


def conv1d_silu_vjp(x_padded, weight, bias, L, dy):
    """Backward of conv1d + SiLU, the VJP alloy attaches to its Metal kernel
    (``_metal_conv1d_silu_vjp``, mamba_block.py:25-47): the pre-activation is
    recomputed (:32-35), ``dsilu = sig (1 + pre (1 - sig))`` (:36-37),
    ``dconv = dy dsilu`` (:38), then per tap k ``dx_padded[k:k+L] += dconv w_k``
    and ``dweight[:, k] = sum(dconv x_padded[k:k+L])`` over batch and time
    (:39-45), ``dbias = sum(dconv)`` (:46).

    Returns (dx_padded [B, L+K-1, C], dweight [C, K], dbias [C]), fp32.
    """
    x_padded = np.asarray(x_padded, F32)
    weight = np.asarray(weight, F32)
    dy = np.asarray(dy, F32)
    K = weight.shape[1]
    pre = depthwise_conv1d(x_padded, weight, np.asarray(bias, F32), L)
    sig = sigmoid(pre)
    dconv = dy * (sig * (1 + pre * (1 - sig)))
    dx = np.zeros_like(x_padded)
    dw = np.zeros_like(weight)
    for k in range(K):
        dx[:, k:k + L, :] += dconv * weight[:, k]
        dw[:, k] += (dconv * x_padded[:, k:k + L, :]).sum(axis=(0, 1))
    return dx, dw, dconv.sum(axis=(0, 1))


def pad_conv_input(conv_input, K, conv_state=None):
    """Left padding / cache prefix of the conv input, mamba_block.py:446-452.

    Returns (x_padded, new_conv_state); new_conv_state is the last K-1 rows of
    x_padded, i.e. the raw (pre-conv) inputs, layout [B, K-1, C].
    """
    if conv_state is not None:
        x_padded = np.concatenate([conv_state, conv_input], axis=1)
    else:
        x_padded = np.pad(conv_input, [(0, 0), (K - 1, 0), (0, 0)])
    return x_padded, x_padded[:, -(K - 1):, :].copy()


# ---------------------------------------------------------------------------
# A3: discretisation (combined / Zamba2 / Nemotron-H mode)
# ---------------------------------------------------------------------------

def discretize(x_heads, dt_raw, dt_bias, A_log, D=None):
    """mamba_block.py:471-486, in the reference's order.

    Returns (x_scaled, A_disc, log_a, D_residual); D_residual uses the
    UNSCALED x (:481-482), x_scaled = x * dt (:484), log_a = A * dt (:485),
    A_disc = exp(log_a) (:486).
    """
    dt = softplus(dt_raw + dt_bias)
    A = -np.exp(A_log)
    D_res = None if D is None else D[None, None, :, None] * x_heads
    x_scaled = x_heads * dt[..., None]
    log_a = A * dt
    return x_scaled, np.exp(log_a), log_a, D_res


# ---------------------------------------------------------------------------
# A5: one chunk of the scan, state-space ("h_all") form
# ---------------------------------------------------------------------------

def scan_chunk(x_c, a_c, B_c, C_c, h, log_a_direct=None):
    """mamba_block.py:206-285 (== scan_chunk_pure_mlx, mamba_kernels.py:227-247).

    x_c [B,cs,H,P], a_c [B,cs,H], B_c/C_c [B,cs,H,N], h [B,H,N,P]
    -> (y_chunk [B,cs,H,P], h_new [B,H,N,P]).
    """
    Bsz, cs, H, P = x_c.shape
    N = B_c.shape[-1]
    x_c = x_c.astype(F32, copy=False)
    B_c = B_c.astype(F32, copy=False)
    C_c = C_c.astype(F32, copy=False)
    b_bar = B_c[..., None] * x_c[:, :, :, None, :]                      # :243
    if log_a_direct is not None:                                        # :246-249
        log_a = log_a_direct.astype(F32, copy=False)
    else:
        log_a = np.log(np.clip(a_c.astype(F32), F32(1e-10), None))
    lac = np.cumsum(log_a, axis=1).transpose(0, 2, 1)                   # :250, :254
    M_log = lac[:, :, :, None] - lac[:, :, None, :]                     # :256
    tril = np.tril(np.ones((cs, cs), dtype=F32)) > 0
    M = np.exp(np.where(tril, M_log, F32(-np.inf)))                     # :257-260 mask, then exp
    b_flat = b_bar.transpose(0, 2, 1, 3, 4).reshape(Bsz, H, cs, N * P)  # :264
    h_input = (M @ b_flat).reshape(Bsz, H, cs, N, P)                    # :265
    decay = np.exp(lac)                                                 # :269
    h_all = decay[:, :, :, None, None] * h[:, :, None, :, :] + h_input  # :270-273
    C_t = C_c.transpose(0, 2, 1, 3)
    y = (C_t[:, :, :, :, None] * h_all).sum(axis=3)                     # :276-277
    return y.transpose(0, 2, 1, 3), h_all[:, :, -1].copy()              # :280, :283


# ---------------------------------------------------------------------------
# A4 / A6: full scans
# ---------------------------------------------------------------------------

def selective_scan_sequential(x, A_disc, B, C, h0=None):
    """Step-by-step scan, mamba_block.py:160-204.

    x [B,L,H,P], A_disc [B,L,H], B/C [B,L,H,N], h0 [B,H,N,P] or None
    -> (y [B,L,H,P] fp32, h [B,H,N,P]).
    """
    x = x.astype(F32, copy=False)
    B = B.astype(F32, copy=False)
    C = C.astype(F32, copy=False)
    A_disc = A_disc.astype(F32, copy=False)
    Bsz, L, H, P = x.shape
    N = B.shape[-1]
    h = np.zeros((Bsz, H, N, P), F32) if h0 is None else h0.astype(F32)
    ys = []
    for t in range(L):                                                  # :194-199
        h = A_disc[:, t, :, None, None] * h + B[:, t, :, :, None] * x[:, t, :, None, :]
        ys.append((C[:, t, :, :, None] * h).sum(axis=2))
    return np.stack(ys, axis=1), h


def selective_scan(x, A_disc, B, C, h0=None, log_a=None, chunk_size=256):
    """Chunked scan with state carry, mamba_block.py:287-366.

    Returns (y [B,L,H,P] in x's dtype, h_final [B,H,N,P] fp32).
    """
    in_dtype = x.dtype
    Bsz, L, H, P = x.shape
    if L <= 1:                                                          # :322-323
        return selective_scan_sequential(x, A_disc, B, C, h0)
    N = B.shape[-1]
    h = np.zeros((Bsz, H, N, P), F32) if h0 is None else h0.astype(F32)
    outs = []
    for start in range(0, L, chunk_size):                               # :340-357
        end = min(start + chunk_size, L)
        y_c, h = scan_chunk(x[:, start:end], A_disc[:, start:end], B[:, start:end],
                            C[:, start:end], h,
                            None if log_a is None else log_a[:, start:end])
        outs.append(y_c)
    y = np.concatenate(outs, axis=1)
    return y.astype(in_dtype, copy=False), h                            # :362-365


# ---------------------------------------------------------------------------
# combined-mode mixer core (conv -> split -> discretise -> scan -> D skip)
# ---------------------------------------------------------------------------

def _split_groups(conv_out, H, P, N, G):
    """mamba_block.py:458-468: split [x | B | C] and repeat groups to heads."""
    Bsz, L, _ = conv_out.shape
    d_inner = H * P
    x = conv_out[..., :d_inner].reshape(Bsz, L, H, P)
    Bm = conv_out[..., d_inner:d_inner + G * N].reshape(Bsz, L, G, N)
    Cm = conv_out[..., d_inner + G * N:].reshape(Bsz, L, G, N)
    if G < H:
        Bm = np.repeat(Bm, H // G, axis=2)   # head h uses group h // (H/G)
        Cm = np.repeat(Cm, H // G, axis=2)
    return x, Bm, Cm


def mixer_core(xBC, dt_raw, conv_weight, conv_bias, dt_bias, A_log, D, *,
               n_heads, headdim, d_state, n_groups, chunk_size=256,
               ssm_state=None, conv_state=None):
    """The hot-path part of ``MambaBlock._forward_combined``, mamba_block.py:446-493.

    Everything between ``in_proj`` (:438) and the gate (:496): conv with the
    cache prefix, SiLU, split, discretisation, chunked (or, for L=1,
    sequential) scan with state carry, D residual.

    Returns (y [B,L,H,P] = scan + D*x, ssm_state [B,H,N,P], conv_state [B,K-1,C]).
    """
    K = conv_weight.shape[1]
    Bsz, L, _ = xBC.shape
    x_padded, new_conv_state = pad_conv_input(xBC, K, conv_state)
    conv_out = conv1d_silu(x_padded, conv_weight, conv_bias, L)
    x, Bm, Cm = _split_groups(conv_out, n_heads, headdim, d_state, n_groups)
    x_s, A_disc, log_a, D_res = discretize(x, dt_raw, dt_bias, A_log, D)
    y, h = selective_scan(x_s, A_disc, Bm, Cm, ssm_state, log_a, chunk_size)
    if D_res is not None:
        y = y + D_res
    return y, h, new_conv_state


def mixer_core_fp64(xBC, dt_raw, conv_weight, conv_bias, dt_bias, A_log, D, *,
                    n_heads, headdim, d_state, n_groups, ssm_state=None,
                    conv_state=None):
    """Independent float64 ground truth: the per-token recurrence
    h_t = exp(A dt_t) h_{t-1} + dt_t B_t x_t^T, y_t = C_t h_t + D x_t.

    Same inputs/outputs as :func:`mixer_core`, computed in float64 without
    chunking (vectorised over batch, heads and the state, looped over time).
    """
    f = np.float64
    K = conv_weight.shape[1]
    Bsz, L, Cdim = xBC.shape
    H, P, N, G = n_heads, headdim, d_state, n_groups
    xBC = xBC.astype(f)
    prefix = (np.zeros((Bsz, K - 1, Cdim), f) if conv_state is None
              else conv_state.astype(f))
    xp = np.concatenate([prefix, xBC], axis=1)
    w = conv_weight.astype(f)
    acc = np.zeros((Bsz, L, Cdim), f) + conv_bias.astype(f)
    for k in range(K):
        acc += xp[:, k:k + L, :] * w[:, k]
    u = acc / (1.0 + np.exp(-acc))
    x, Bm, Cm = _split_groups(u, H, P, N, G)
    dt = np.logaddexp(dt_raw.astype(f) + dt_bias.astype(f), 0.0)
    A = -np.exp(A_log.astype(f))
    dA = np.exp(A[None, None, :] * dt)
    h = np.zeros((Bsz, H, N, P), f) if ssm_state is None else ssm_state.astype(f)
    y = np.empty((Bsz, L, H, P), f)
    for t in range(L):
        h = dA[:, t, :, None, None] * h + (dt[:, t, :, None, None]
                                           * Bm[:, t, :, :, None] * x[:, t, :, None, :])
        y[:, t] = (Cm[:, t, :, :, None] * h).sum(axis=2)
    if D is not None:
        y += D.astype(f)[None, None, :, None] * x
    return y, h, xp[:, -(K - 1):, :]


def decode_step_fp64(xBC_tok, dt_tok, conv_weight, conv_bias, dt_bias, A_log, D,
                     ssm_state, conv_state, *, n_heads, headdim, d_state, n_groups):
    """One decode token (the L=1 branch of mamba_block.py:446-448 and :160-204)
    in float64.  xBC_tok [B, conv_dim], dt_tok [B, H]; returns
    (y [B,H,P], ssm_state, conv_state)."""
    y, h, cs = mixer_core_fp64(xBC_tok[:, None, :], dt_tok[:, None, :], conv_weight,
                               conv_bias, dt_bias, A_log, D, n_heads=n_heads,
                               headdim=headdim, d_state=d_state, n_groups=n_groups,
                               ssm_state=ssm_state, conv_state=conv_state)
    return y[:, 0], h, cs


# ---------------------------------------------------------------------------
# gate and inner norm after the scan
# ---------------------------------------------------------------------------

def gated_rmsnorm(y, gate, weight=None, eps=1e-5, group_size=0):
    """Step 7 of ``_forward_combined`` (mamba_block.py:495-499): the gate first,
    ``y * nn.silu(gate)``, then ``nn.RMSNorm(d_inner)`` (:137; MLX's
    ``x * rsqrt(mean(x^2, -1) + eps) * weight``, eps 1e-5) when a weight is
    given.  ``group_size`` > 0 normalises runs of that many channels instead of
    the whole row (the group-wise form of the same norm).  float32 on the given
    values."""
    y = np.asarray(y, F32)
    g = np.asarray(gate, F32)
    v = y * silu(g)
    if weight is None:
        return v
    D = v.shape[-1]
    gs = group_size or D
    vg = v.reshape(*v.shape[:-1], D // gs, gs)
    r = F32(1) / np.sqrt(np.mean(vg * vg, axis=-1, keepdims=True, dtype=F32) + F32(eps))
    return (vg * r).reshape(v.shape) * np.asarray(weight, F32)


# ---------------------------------------------------------------------------
# seeded synthetic inputs and the workload table
# ---------------------------------------------------------------------------

CONFIGS = {
    # toy fp32 mixer (parity config)
    "toy": dict(B=2, L=512, H=8, P=32, N=16, G=1, Q=64, dtype="fp32"),
    # Zamba2-1.2B-shaped layer prefill
    "zamba2": dict(B=8, L=4096, H=64, P=64, N=64, G=1, Q=256, dtype="bf16"),
    # Nemotron-H-8B-shaped layer prefill
    "nemotron": dict(B=4, L=8192, H=128, P=64, N=128, G=8, Q=256, dtype="bf16"),
    # Nemotron-H-8B-shaped decode, 64 steps
    "decode": dict(B=256, L=1, H=128, P=64, N=128, G=8, Q=256, dtype="bf16", steps=64),
    # long-context Zamba2-shaped prefill
    "long": dict(B=1, L=131072, H=64, P=64, N=64, G=1, Q=512, dtype="bf16"),
}


def bf16_round(a):
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    a = np.ascontiguousarray(a, dtype=F32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(F32)
    nan = np.isnan(a)
    if nan.any():
        out = np.where(nan, a, out)
    return out.reshape(a.shape)


def make_inputs(B, L, H, P, N, G, K=4, dtype="fp32", seed=0, with_state=False, **_):
    """Seeded synthetic inputs with the workload distributions:

    xBC ~ N(0,1); conv weight ~ N(0, 1/4) (std 0.5), bias 0; dt_raw ~ N(0,1);
    dt_bias = log(expm1(u)) with u log-uniform in [1e-3, 0.1] per head, so
    softplus(dt_bias) = u; A_log ~ U(log 1, log 16); D ~ N(0,1).  With
    ``with_state`` an initial ssm_state ~ N(0, 0.1) (variance) and conv_state ~
    N(0,1) are added.  For dtype "bf16" the activations and states that the
    kernels read as bf16 (xBC, dt_raw, conv_state) are rounded to bf16 values.
    """
    rng = np.random.default_rng(seed)
    conv_dim = H * P + 2 * G * N
    xBC = rng.standard_normal((B, L, conv_dim), dtype=F32)
    conv_w = (rng.standard_normal((conv_dim, K), dtype=F32) * F32(0.5)).astype(F32)
    conv_b = np.zeros((conv_dim,), F32)
    dt_raw = rng.standard_normal((B, L, H), dtype=F32)
    u = np.exp(rng.uniform(math.log(1e-3), math.log(0.1), size=H))
    dt_bias = np.log(np.expm1(u)).astype(F32)
    A_log = rng.uniform(0.0, math.log(16.0), size=H).astype(F32)
    D = rng.standard_normal(H, dtype=F32)
    out = dict(xBC=xBC, conv_weight=conv_w, conv_bias=conv_b, dt_raw=dt_raw,
               dt_bias=dt_bias, A_log=A_log, D=D)
    if with_state:
        out["ssm_state"] = (rng.standard_normal((B, H, N, P), dtype=F32)
                            * F32(math.sqrt(0.1))).astype(F32)
        out["conv_state"] = rng.standard_normal((B, K - 1, conv_dim), dtype=F32)
    if dtype == "bf16":
        for k in ("xBC", "dt_raw", "conv_state"):
            if k in out:
                out[k] = bf16_round(out[k])
    return out


# ---------------------------------------------------------------------------
# error metrics used by the parity tests
# ---------------------------------------------------------------------------

def rel_l2(got, ref):
    """||got - ref||_2 / ||ref||_2, in float64."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref.ravel())
    return float(np.linalg.norm((got - ref).ravel()) / (den if den > 0 else 1.0))


def max_rel(got, ref):
    """max |got - ref| / max |ref|, in float64."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.abs(ref).max() if ref.size else 1.0
    return float(np.abs(got - ref).max() / (den if den > 0 else 1.0)) if ref.size else 0.0
