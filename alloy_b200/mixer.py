"""Functional API of the Mamba-2 mixer hot path over torch CUDA tensors.

Each function validates devices on the host and calls one liballoy_ssd entry
point on torch's current CUDA stream.  Inputs must already be CUDA tensors,
except for ``ssd_combined_streamed``, which copies host activations in and
its results out around the same kernels; there is no CPU compute path and no
fallback.

Layouts follow gxcsoccer/alloy (alloy/models/mamba_block.py):
``xBC [B, L, H*P + 2*G*N]`` = conv input ``[x | B | C]``; ``dt_raw [B, L, H]``;
``ssm_state [B, H, N, P]`` fp32 and ``conv_state [B, K-1, conv_dim]``.
State arguments may be any permutation of those axes (given by strides), so
``[B, H, P, N]`` states are passed as ``state.transpose(2, 3)``.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = [
    "conv1d_silu", "depthwise_conv1d", "ssd_combined", "selective_scan",
    "ssd_decode_step", "gated_rmsnorm", "ssd_combined_streamed", "conv1d_silu_backward",
    "Conv1dSilu", "selective_scan_backward", "SelectiveScan", "decode_linear", "selective_scan_dot",
    "linear", "linear_fills_device",
]


def _cuda(name, t):
    if t is None:
        return None
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name}: expected a torch.Tensor, got {type(t).__name__}")
    if not t.is_cuda:
        raise ValueError(f"{name}: must be a CUDA tensor (liballoy_ssd has no CPU path)")
    return t


def _same_device(*named):
    dev = None
    for name, t in named:
        if t is None:
            continue
        _cuda(name, t)
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{name}: on {t.device}, expected {dev}")
    return dev


def _f32(t):
    return None if t is None else (t if t.dtype == torch.float32 else t.float())


def _dims(n_heads, head_dim, d_state, n_groups, d_conv, chunk_size, head_begin, head_count):
    d = _lib.Dims()
    d.n_heads, d.head_dim, d.d_state, d.n_groups = n_heads, head_dim, d_state, n_groups
    d.d_conv, d.chunk_size = d_conv, chunk_size
    d.head_begin, d.head_count = head_begin, head_count
    return d


def _conv(entry, x_padded, weight, bias, L, out):
    dev = _same_device(("x_padded", x_padded), ("weight", weight), ("bias", bias), ("out", out))
    Bsz, Lp, C = x_padded.shape
    K = weight.shape[1]
    if L is None:
        L = Lp - K + 1
    if L != Lp - K + 1:
        x_padded = x_padded[:, :L + K - 1]
    if out is None:
        out = torch.empty((Bsz, L, C), dtype=x_padded.dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.call(entry, *(_lib.ref(_lib.desc(t, n)) for t, n in (
            (x_padded, "x_padded"), (weight, "weight"), (bias, "bias"), (out, "out"))),
            _lib.stream_handle(dev))
    return out


def conv1d_silu(x_padded, weight, bias=None, L=None, out=None):
    """silu(causal depthwise conv) of a pre-padded input ``[B, L+K-1, C]``.

    Mirrors ``fused_conv1d_silu(x_padded, weight, bias, L)``
    (alloy/models/mamba_kernels.py:39-50).
    """
    return _conv("alloy_conv1d_silu", x_padded, weight, bias, L, out)


def depthwise_conv1d(x_padded, weight, bias=None, L=None, out=None):
    """Causal depthwise conv without activation, ``MambaBlock._depthwise_conv1d``
    (alloy/models/mamba_block.py:144-158)."""
    return _conv("alloy_depthwise_conv1d", x_padded, weight, bias, L, out)


def conv1d_silu_backward(x_padded, weight, bias, dy, L=None, dx_out=None):
    """Backward of ``conv1d_silu``: ``(dx_padded, dweight, dbias)`` from the
    output cotangent ``dy [B, L, C]``, as ``_metal_conv1d_silu_vjp``
    (alloy/models/mamba_block.py:25-47) computes them.  ``dx_padded`` has
    x_padded's shape (rows past L+K-1 get zero); ``dweight`` / ``dbias`` have
    the dtypes of weight / bias (``dbias`` is None without a bias).  Summed in
    fp32 in a fixed order: repeated calls give identical results.
    """
    dev = _same_device(("x_padded", x_padded), ("weight", weight), ("bias", bias), ("dy", dy),
                       ("dx_out", dx_out))
    Bsz, Lp, C = x_padded.shape
    K = weight.shape[1]
    if L is None:
        L = Lp - K + 1
    if dy.shape != (Bsz, L, C):
        raise ValueError(f"dy shape {tuple(dy.shape)} != {(Bsz, L, C)}")
    if dy.dtype != x_padded.dtype:
        dy = dy.to(x_padded.dtype)
    if dx_out is None:
        dx_out = (torch.empty_like(x_padded) if L + K - 1 == Lp
                  else torch.zeros_like(x_padded))
    x_used, dx_used = x_padded[:, :L + K - 1], dx_out[:, :L + K - 1]
    dweight = torch.empty(weight.shape, dtype=weight.dtype, device=dev)
    dbias = None if bias is None else torch.empty(bias.shape, dtype=bias.dtype, device=dev)
    ws_bytes = _lib.load().alloy_conv1d_silu_backward_workspace_size(Bsz, L + K - 1, C, K)
    ws = _workspace(dev, ws_bytes)
    descs = [_lib.desc(t, n) for t, n in ((x_used, "x_padded"), (weight, "weight"), (bias, "bias"),
                                          (dy, "dy"), (dx_used, "dx_padded"),
                                          (dweight, "dweight"), (dbias, "dbias"))]
    with torch.cuda.device(dev):
        _lib.call("alloy_conv1d_silu_backward", *(_lib.ref(d) for d in descs),
                  ws.data_ptr() if ws is not None else None, ws_bytes, _lib.stream_handle(dev))
    return dx_out, dweight, dbias


class Conv1dSilu(torch.autograd.Function):
    """``conv1d_silu`` with its VJP, the counterpart of alloy's
    ``@mx.custom_function _metal_conv1d_silu`` and its ``.vjp``
    (alloy/models/mamba_block.py:19-47)."""

    @staticmethod
    def forward(ctx, x_padded, weight, bias, L):
        ctx.save_for_backward(x_padded, weight, bias)
        ctx.L = L
        return conv1d_silu(x_padded, weight, bias, L)

    @staticmethod
    def backward(ctx, dy):
        x_padded, weight, bias = ctx.saved_tensors
        dx, dw, db = conv1d_silu_backward(x_padded, weight, bias, dy.contiguous(), ctx.L)
        return dx, dw, db, None


def ssd_combined(xBC, dt_raw, conv_weight, conv_bias, dt_bias, A_log, D, *, n_heads,
                 head_dim, d_state, n_groups, d_conv=4, chunk_size=256, ssm_state=None,
                 conv_state=None, out=None, ssm_state_out=None, conv_state_out=None,
                 write_ssm_state=True, write_conv_state=True, head_begin=0, head_count=0,
                 workspace="full"):
    """Fused conv + discretisation + chunked SSD scan + D skip (prefill).

    The hot part of ``MambaBlock._forward_combined``
    (alloy/models/mamba_block.py:446-493).  Returns
    ``(y [B, L, H, P], ssm_state_out [B, H, N, P] fp32, conv_state_out
    [B, K-1, conv_dim])``; the state outputs are new tensors unless given
    (they may alias the inputs for an in-place cache update).  ``head_begin``
    / ``head_count`` restrict the call to a head range (multi-GPU sharding):
    only those heads of ``y`` and of the states are written.  ``workspace``
    "full" sizes the scratch for the fastest schedule; "min" gives the
    library the smallest it accepts (each head pair walked by one CTA).
    """
    dev = _same_device(("xBC", xBC), ("dt_raw", dt_raw), ("conv_weight", conv_weight),
                       ("conv_bias", conv_bias), ("dt_bias", dt_bias), ("A_log", A_log),
                       ("D", D), ("ssm_state", ssm_state), ("conv_state", conv_state),
                       ("out", out), ("ssm_state_out", ssm_state_out),
                       ("conv_state_out", conv_state_out))
    Bsz, L, Cdim = xBC.shape
    H, P, N = n_heads, head_dim, d_state
    if out is None:
        out = torch.empty((Bsz, L, H, P), dtype=xBC.dtype, device=dev)
    if ssm_state_out is None and write_ssm_state:
        ssm_state_out = torch.empty((Bsz, H, N, P), dtype=torch.float32, device=dev)
    if conv_state_out is None and write_conv_state:
        conv_state_out = torch.empty((Bsz, d_conv - 1, Cdim), dtype=xBC.dtype, device=dev)
    if conv_state is not None and conv_state.dtype != xBC.dtype:
        conv_state = conv_state.to(xBC.dtype)
    dims = _dims(H, P, N, n_groups, d_conv, chunk_size, head_begin, head_count)
    if workspace not in ("full", "min"):
        raise ValueError(f"workspace must be 'full' or 'min', got {workspace!r}")
    size_fn = (_lib.load().alloy_ssd_combined_workspace_size if workspace == "full"
               else _lib.load().alloy_ssd_combined_min_workspace_size)
    ws_bytes = size_fn(Bsz, L, _lib.BF16 if xBC.dtype == torch.bfloat16 else _lib.F32, _lib.ref(dims))
    ws = _workspace(dev, ws_bytes)
    args = [(xBC, "xBC"), (dt_raw, "dt_raw"), (_f32(conv_weight), "conv_weight"),
            (_f32(conv_bias), "conv_bias"), (_f32(dt_bias), "dt_bias"), (_f32(A_log), "A_log"),
            (_f32(D), "D"), (ssm_state, "ssm_state"), (conv_state, "conv_state"), (out, "y"),
            (ssm_state_out, "ssm_state_out"), (conv_state_out, "conv_state_out")]
    descs = [_lib.desc(t, n) for t, n in args]
    with torch.cuda.device(dev):
        _lib.call("alloy_ssd_combined", *(_lib.ref(d) for d in descs),
                  ws.data_ptr() if ws is not None else None, ws_bytes, _lib.ref(dims),
                  _lib.stream_handle(dev))
    return out, ssm_state_out, conv_state_out


def ssd_combined_streamed(xBC, dt_raw, conv_weight, conv_bias, dt_bias, A_log, D, *, n_heads,
                          head_dim, d_state, n_groups, d_conv=4, chunk_size=256, ssm_state=None,
                          conv_state=None, out=None, ssm_state_out=None, conv_state_out=None,
                          piece_tokens=2048, slots=3):
    """``ssd_combined`` for activations that live in host memory.

    For a caller whose activations are host arrays: an MLX caller (unified
    memory, reached through ``mlx_bridge``'s numpy path), or a service that
    receives them over the network.  ``xBC`` [B, L, conv_dim] and ``dt_raw``
    [B, L, H] are pinned CPU tensors; the parameters are CUDA tensors and
    choose the device; ``ssm_state`` / ``conv_state`` (optional) are CPU
    tensors in the layouts ``ssd_combined`` takes.  Returns pinned CPU
    ``(y [B, L, H, P], ssm_state_out [B, H, N, P] fp32, conv_state_out
    [B, K-1, conv_dim])``, valid when the call returns.

    The sequence of each batch row is cut into pieces of ``piece_tokens``
    tokens.  Each piece is copied in on one stream, computed on a second and
    its y copied out on a third, through ``slots`` device buffers, so that the
    host->device copy of piece i+1, the kernels of piece i and the
    device->host copy of piece i-1 overlap; a row's states carry from piece
    to piece in device memory, in fp32 as inside one call.  Pieces start on
    multiples of ``chunk_size`` tokens when ``piece_tokens`` is one.
    """
    for name, t in (("xBC", xBC), ("dt_raw", dt_raw)):
        if not isinstance(t, torch.Tensor) or t.is_cuda:
            raise ValueError(f"{name}: expected a CPU tensor (use ssd_combined for CUDA tensors)")
        if not t.is_pinned():
            raise ValueError(f"{name}: must be in pinned host memory (torch.Tensor.pin_memory())")
        if not t.is_contiguous():
            raise ValueError(f"{name}: must be contiguous")
    dev = _same_device(("conv_weight", conv_weight), ("conv_bias", conv_bias),
                       ("dt_bias", dt_bias), ("A_log", A_log), ("D", D))
    if piece_tokens < 1 or slots < 2:
        raise ValueError("piece_tokens must be >= 1 and slots >= 2")
    Bsz, L, Cdim = xBC.shape
    H, P, N, K = n_heads, head_dim, d_state, d_conv
    if out is None:
        out = torch.empty((Bsz, L, H, P), dtype=xBC.dtype, pin_memory=True)
    if ssm_state_out is None:
        ssm_state_out = torch.empty((Bsz, H, N, P), dtype=torch.float32, pin_memory=True)
    if conv_state_out is None:
        conv_state_out = torch.empty((Bsz, K - 1, Cdim), dtype=xBC.dtype, pin_memory=True)
    kw = dict(n_heads=H, head_dim=P, d_state=N, n_groups=n_groups, d_conv=K,
              chunk_size=chunk_size)
    pieces = [(b, l0, min(L, l0 + piece_tokens)) for b in range(Bsz)
              for l0 in range(0, L, piece_tokens)]
    T = min(piece_tokens, L)
    main = torch.cuda.current_stream(dev)
    s_in, s_cmp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    with torch.cuda.device(dev):
        # every device buffer exists before the side streams start
        d_x = [torch.empty((1, T, Cdim), dtype=xBC.dtype, device=dev) for _ in range(slots)]
        d_dt = [torch.empty((1, T, H), dtype=dt_raw.dtype, device=dev) for _ in range(slots)]
        d_y = [torch.empty((1, T, H, P), dtype=xBC.dtype, device=dev) for _ in range(slots)]
        # the carried states, one set per row parity (a row's final states are
        # copied out while the next row runs on the other set)
        d_h = [torch.empty((1, H, N, P), dtype=torch.float32, device=dev) for _ in range(2)]
        d_cs = [torch.empty((1, K - 1, Cdim), dtype=xBC.dtype, device=dev) for _ in range(2)]
        states_out = [None, None]
        d_h0 = d_cs0 = None
        if ssm_state is not None:
            d_h0 = ssm_state.to(dev, torch.float32)
        if conv_state is not None:
            d_cs0 = conv_state.to(dev, xBC.dtype)
        ev = lambda: torch.cuda.Event()
        in_ready = [ev() for _ in range(slots)]
        consumed = [ev() for _ in range(slots)]
        copied_out = [ev() for _ in range(slots)]
        used = [False] * slots
        start = ev()
        start.record(main)
        for s in (s_in, s_cmp, s_out):
            s.wait_event(start)
        for i, (b, l0, l1) in enumerate(pieces):
            k, n = i % slots, l1 - l0
            # copy in: the slot's inputs were read by the piece that used it last
            if used[k]:
                s_in.wait_event(consumed[k])
            with torch.cuda.stream(s_in):
                d_x[k][:, :n].copy_(xBC[b:b + 1, l0:l1], non_blocking=True)
                d_dt[k][:, :n].copy_(dt_raw[b:b + 1, l0:l1], non_blocking=True)
                in_ready[k].record(s_in)
            # compute: inputs in, and the slot's previous y copied out
            s_cmp.wait_event(in_ready[k])
            if used[k]:
                s_cmp.wait_event(copied_out[k])
            st = b & 1
            first = l0 == 0
            if first and states_out[st] is not None:
                # this state set's previous row has been copied out
                s_cmp.wait_event(states_out[st])
            with torch.cuda.stream(s_cmp):
                h_in = (d_h0[b:b + 1] if d_h0 is not None else None) if first else d_h[st]
                cs_in = (d_cs0[b:b + 1] if d_cs0 is not None else None) if first else d_cs[st]
                ssd_combined(d_x[k][:, :n], d_dt[k][:, :n], conv_weight, conv_bias, dt_bias,
                             A_log, D, ssm_state=h_in, conv_state=cs_in, out=d_y[k][:, :n],
                             ssm_state_out=d_h[st], conv_state_out=d_cs[st], **kw)
                consumed[k].record(s_cmp)
            # copy out (the row's final states after its last piece)
            s_out.wait_event(consumed[k])
            with torch.cuda.stream(s_out):
                out[b:b + 1, l0:l1].copy_(d_y[k][:, :n], non_blocking=True)
                copied_out[k].record(s_out)
                if l1 == L:
                    ssm_state_out[b:b + 1].copy_(d_h[st], non_blocking=True)
                    conv_state_out[b:b + 1].copy_(d_cs[st], non_blocking=True)
                    states_out[st] = ev()
                    states_out[st].record(s_out)
            used[k] = True
        s_out.synchronize()
        main.wait_stream(s_out)
    return out, ssm_state_out, conv_state_out


def _workspace(dev, nbytes):
    """Device scratch for one call, from torch's caching allocator (freed when
    the last reference goes; the allocator orders reuse on the stream)."""
    if nbytes == 0:
        return None
    return torch.empty(nbytes, dtype=torch.uint8, device=dev)


def check_device_status(device=None):
    """Synchronise torch's current stream and raise AlloyError if a kernel gave
    up on a bounded device-side wait since the last check."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(dev):
        _lib.call("alloy_check_device_status", _lib.stream_handle(dev))


def selective_scan(x, A_disc, B, C, ssm_state=None, log_a=None, out=None, out_dtype=None,
                   ssm_state_out=None, write_ssm_state=True, reverse_time=False):
    """Scan on pre-discretised inputs (``MambaBlock._selective_scan``,
    alloy/models/mamba_block.py:287-366).

    x [B, L, H, P] (dt-scaled), A_disc [B, L, H], B/C [B, L, G', N] with G'
    dividing H (G' = H for the reference's per-head repeated B/C), ssm_state
    [B, H, N, P] fp32 or None.  ``log_a`` (fp32), when given, is used in
    place of log(A_disc).  Returns (y, ssm_state_out); y has ``out_dtype``
    (default: x's dtype).  ``reverse_time`` runs the scan from step L-1 down
    to step 0 (the library walks every time-indexed tensor with a negative
    time stride; y is still indexed by step), as the gradient scans need.
    """
    dev = _same_device(("x", x), ("A_disc", A_disc), ("B", B), ("C", C),
                       ("ssm_state", ssm_state), ("log_a", log_a), ("out", out),
                       ("ssm_state_out", ssm_state_out))
    Bsz, L, H, P = x.shape
    N = B.shape[-1]
    if x.stride(-1) != 1:
        x = x.contiguous()
    if out is None:
        out = torch.empty((Bsz, L, H, P), dtype=out_dtype or x.dtype, device=dev)
    if ssm_state_out is None and write_ssm_state:
        ssm_state_out = torch.empty((Bsz, H, N, P), dtype=torch.float32, device=dev)
    if ssm_state is not None and ssm_state.dtype != torch.float32:
        ssm_state = ssm_state.float()
    args = [(x, "x"), (A_disc, "A_disc"), (_f32(log_a), "log_a"), (B, "B"), (C, "C"),
            (ssm_state, "ssm_state"), (out, "y"), (ssm_state_out, "ssm_state_out")]
    descs = [_lib.desc(t, n) for t, n in args]
    if reverse_time and L > 1:
        for (t, name), d in zip(args, descs):
            if t is not None and name not in ("ssm_state", "ssm_state_out"):
                d.data += (L - 1) * t.stride(1) * t.element_size()
                d.stride[1] = -t.stride(1)
    with torch.cuda.device(dev):
        _lib.call("alloy_selective_scan", *(_lib.ref(d) for d in descs), _lib.stream_handle(dev))
    return out, ssm_state_out


def selective_scan_dot(x, B, C, log_a, *, z=None, ssm_state=None, y_dtype=torch.float32, write_y=True,
                       write_ssm_state=False, reverse_time=False, dot_without_own_term=False,
                       precise_scores=False):
    """The scan of ``selective_scan`` on the tensor cores (``alloy_selective_scan_dot``)
    for bf16 operands, with x and the dot operand shared across heads and the
    row dot products fused: the gradient scans of ``selective_scan_backward``.

    x [B, L, Gx, P] bf16 (Gx divides H: head h reads x row h // (H // Gx)),
    B/C [B, L, G', N] bf16, log_a [B, L, H] fp32 (<= 0; H is its dim 2),
    z [B, L, Gz, P] (optional).  Returns (y [B, L, H, P] of ``y_dtype`` or None,
    final state [B, H, N, P] fp32 or None, dot [B, L, H] fp32 or None) with
    dot[b, t, h] = sum_p y[b, t, h, p] z[b, t, h // (H // Gz), p]; with
    ``dot_without_own_term`` the step's own term S[t,t] (x_t . z_t), S[t,t] = C_t . B_t
    as the kernel rounds it, is left out.  ``precise_scores`` (head_dim = d_state
    = 64) feeds the decayed scores, exp(cum) C, the state copy and X' to the
    products as bf16 pairs (~16 bits) for outputs whose differences cancel; it
    excludes ``dot_without_own_term``.
    """
    dev = _same_device(("x", x), ("B", B), ("C", C), ("log_a", log_a), ("z", z),
                       ("ssm_state", ssm_state))
    Bsz, L, _, P = x.shape
    H, N = log_a.shape[2], B.shape[-1]
    y = torch.empty((Bsz, L, H, P), dtype=y_dtype, device=dev) if write_y else None
    h_out = torch.empty((Bsz, H, N, P), dtype=torch.float32, device=dev) if write_ssm_state else None
    dot = torch.empty((Bsz, L, H), dtype=torch.float32, device=dev) if z is not None else None
    args = [(x, "x"), (log_a, "log_a"), (B, "B"), (C, "C"), (ssm_state, "ssm_state"), (y, "y"),
            (h_out, "ssm_state_out"), (z, "z"), (dot, "dot")]
    descs = [_lib.desc(t, n) for t, n in args]
    if reverse_time and L > 1:
        for (t, name), d in zip(args, descs):
            if t is not None and name not in ("ssm_state", "ssm_state_out"):
                d.data += (L - 1) * t.stride(1) * t.element_size()
                d.stride[1] = -t.stride(1)
    with torch.cuda.device(dev):
        _lib.call("alloy_selective_scan_dot", *(_lib.ref(d) for d in descs),
                  int(dot_without_own_term) | (2 if precise_scores else 0), _lib.stream_handle(dev))
    return y, h_out, dot


# (head_dim, d_state) pairs whose forward and transposed gradient scans the tensor-core scan covers
_DOT_SCAN_DIMS = ((64, 64), (64, 128), (128, 64))


def selective_scan_backward(x, A_disc, B, C, dy, ssm_state=None, log_a=None, dssm_state_out=None,
                            tensor_core_log_decay=True):
    """Gradients of ``selective_scan``: ``(dx, dA_disc, dB, dC, dssm_state, dlog_a)``
    for the output cotangent ``dy [B, L, H, P]`` and (optional) the cotangent of
    the final state ``dssm_state_out [B, H, N, P]``.  What the reference gets
    from MLX autograd through ``_selective_scan`` (alloy/models/mamba_block.py:
    287-366); the reference has no custom kernel for it.

    The scan h_t = a_t h_{t-1} + B_t x_t^T, y_t = C_t h_t has the adjoint state
    g_t = a_{t+1} g_{t+1} + C_t dy_t^T (g_{L-1} also receives dssm_state_out),
    and every gradient is the output of a scan of the same form, run by the
    library's fp32 scan kernel on rearranged inputs:
      dx_t = g_t^T B_t   : time-reversed scan, x' = dy, B' = C, C' = B,
                           decay a'_u = a_{L-u} (a'_0 = 1), initial state dssm_state_out
      dB_t = g_t x_t     : the same reversed scan with x' = C, B' = dy, C' = x
      dC_t = h_t dy_t    : forward scan with x' = B, B' = x, C' = dy, initial state h0^T
      dssm_state = a_0 g_0
    and the log-decay gradient dla_t = <g_t, a_t h_{t-1}> telescopes (with
    <g_t, h_t> = <g_{t+1}, a_{t+1} h_t> + dy_t . y_t) into a reverse cumulative sum:
      dla_t = <dssm_state_out, h_{L-1}> + sum_{u >= t} (dy_u . y_u - B_u . dB_u).
    ``dlog_a`` is returned when ``log_a`` was given (the decay came from it),
    else ``dA_disc`` = dla / A_disc.  All arithmetic in fp32; the gradients have
    the dtypes of their inputs.  When x, B and C are bf16 (dy rounded to bf16)
    and the sizes suit the tensor-core scan, dB and dC run on it; the two scans
    that the log-decay gradient depends on run on the tensor-core scan with
    ~16-bit operands (``tensor_core_log_decay``, head_dim = d_state = 64) or on
    the fp32 scan (see ``_scan_backward_dot``); otherwise everything is fp32.
    """
    dev = _same_device(("x", x), ("A_disc", A_disc), ("B", B), ("C", C), ("dy", dy),
                       ("ssm_state", ssm_state), ("log_a", log_a),
                       ("dssm_state_out", dssm_state_out))

    def scan(xs, Bs, Cs, h0, la, want_state, reverse):
        return selective_scan(xs, None, Bs, Cs, ssm_state=h0, log_a=la, out_dtype=torch.float32,
                              write_ssm_state=want_state, reverse_time=reverse)

    la = log_a.float() if log_a is not None else torch.log(torch.clamp(A_disc.float(), min=1e-10))
    bf16 = all(t.dtype == torch.bfloat16 for t in (x, B, C))
    h0 = None if ssm_state is None else ssm_state.float()
    dhT = None if dssm_state_out is None else dssm_state_out.float()
    # the tensor-core log-decay scans (bf16 pairs throughout) cover head_dim = d_state = 64
    tensor_core_log_decay = tensor_core_log_decay and (x.shape[-1], B.shape[-1]) == (64, 64)
    if bf16 and (x.shape[-1], B.shape[-1]) in _DOT_SCAN_DIMS:
        bf = lambda t: t.to(torch.bfloat16).contiguous()   # noqa: E731
        dx, dla, dB, dC, dh0 = _scan_backward_dot(bf(x), la.contiguous(), bf(B), bf(C), bf(dy), h0, dhT,
                                                  dev, tensor_core_log_decay)
    else:
        op = (lambda t: t.to(torch.bfloat16).contiguous()) if bf16 else (lambda t: t.float().contiguous())
        dx, dla, dB, dC, dh0 = _scan_backward(scan, op(x), la, op(B), op(C), op(dy), h0, dhT, dev)
    dA = dla_out = None
    if log_a is not None:
        dla_out = dla.to(log_a.dtype)
    else:
        a = A_disc.float()
        dA = torch.where(a > 1e-10, dla / a, torch.zeros_like(dla)).to(A_disc.dtype)
    return (dx.to(x.dtype), dA, dB.to(B.dtype), dC.to(C.dtype),
            None if ssm_state is None else dh0.to(ssm_state.dtype), dla_out)


def _scan_backward(scan, x, la, B, C, dy, h0, dhT, device):
    """The gradient algebra of ``selective_scan_backward`` over a scan callable
    ``scan(x, B, C, h0, log_a, want_state, reverse) -> (y, final state or None)``
    (B/C per head or per group, states [B, H, N, P] in any axis order; with
    ``reverse`` the scan walks steps L-1 .. 0 of its step-indexed inputs)."""
    Bsz, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    r = H // G
    Bh = B.repeat_interleave(r, dim=2)          # per head [B, L, H, N]
    Ch = C.repeat_interleave(r, dim=2)
    if dhT is None:
        dhT = torch.zeros((Bsz, H, N, P), dtype=torch.float32, device=device)
    # the forward's outputs (y without D, and the final state)
    y, hT = scan(x, Bh, Ch, h0, la, True, False)
    # the reversed scans walk steps L-1 .. 0; the decay applied on reaching step
    # t is the one of step t+1 (none at the first step taken, t = L-1)
    la_next = torch.zeros_like(la)
    la_next[:, :-1] = la[:, 1:]
    dx, g0 = scan(dy, Ch, Bh, dhT, la_next, True, True)
    dBh, _ = scan(Ch, dy, x, dhT.transpose(2, 3), la_next, False, True)
    dCh, _ = scan(Bh, x, dy, None if h0 is None else h0.transpose(2, 3), la, False, False)
    # log-decay gradient: a reverse cumulative sum over the steps (along the
    # last dimension of a [B, H, L] copy)
    s = ((dy * y).sum(-1) - (Bh * dBh).sum(-1)).transpose(1, 2).contiguous()   # [B, H, L]
    dla = s.flip(-1).cumsum(-1).flip(-1).transpose(1, 2) + (dhT * hT).sum((-1, -2))[:, None, :]
    dh0 = torch.exp(la[:, 0])[:, :, None, None] * g0
    return (dx, dla, dBh.view(Bsz, L, G, r, N).sum(3), dCh.view(Bsz, L, G, r, N).sum(3), dh0)


def _scan_backward_dot(x, la, B, C, dy, h0, dhT, device, tensor_core_log_decay=False):
    """``_scan_backward`` for bf16 operands; dB and dC on the tensor-core scan
    (B/C kept per group, no per-head copies).  The log-decay gradient is a
    reverse cumulative sum of dy_t . y_t - B_t . dB_t (= x_t . dx_t), two terms
    that cancel nearly term by term at large decays, so the rounding of the
    scans that feed it -- the recomputed forward and the dx scan -- reaches it
    amplified.  With ``tensor_core_log_decay`` (the default; head_dim = d_state
    = 64) those two run on the tensor-core scan in its precise mode: the decayed
    scores, exp(cum) C, the state copy and X' all enter the products as bf16
    pairs (~16 bits).  Otherwise they run on the fp32 scan (on the bf16 values),
    about 5x slower.  (With single bf16 operands the A_log gradient of a test
    layer with decays up to exp(-2) a step was off by ~0.5 relative; with the
    scores alone as pairs, by ~7e-2.)"""
    Bsz, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    r = H // G
    if dhT is None:
        dhT = torch.zeros((Bsz, H, N, P), dtype=torch.float32, device=device)
    la_next = torch.zeros_like(la)
    la_next[:, :-1] = la[:, 1:]
    if tensor_core_log_decay:
        _, hT, dot_y = selective_scan_dot(x, B, C, la, z=dy, ssm_state=h0, write_y=False,
                                          write_ssm_state=True, precise_scores=True)
        dx, g0, dot_x = selective_scan_dot(dy, C, B, la_next, z=x, ssm_state=dhT, y_dtype=x.dtype,
                                           write_ssm_state=True, reverse_time=True, precise_scores=True)
    else:
        xf, Bf, Cf, dyf = x.float(), B.float(), C.float(), dy.float()
        y, hT = selective_scan(xf, None, Bf, Cf, ssm_state=h0, log_a=la, out_dtype=torch.float32)
        dx, g0 = selective_scan(dyf, None, Cf, Bf, ssm_state=dhT, log_a=la_next, out_dtype=torch.float32,
                                reverse_time=True)
        dot_y, dot_x = (dyf * y).sum(-1), (xf * dx).sum(-1)
    dBh, _, _ = selective_scan_dot(C, dy, x, la_next, ssm_state=dhT.transpose(2, 3), reverse_time=True)
    dCh, _, _ = selective_scan_dot(B, x, dy, la, ssm_state=None if h0 is None else h0.transpose(2, 3))
    s = (dot_y - dot_x).transpose(1, 2).contiguous()   # [B, H, L]
    dla = s.flip(-1).cumsum(-1).flip(-1).transpose(1, 2) + (dhT * hT).sum((-1, -2))[:, None, :]
    dh0 = torch.exp(la[:, 0])[:, :, None, None] * g0
    if r > 1:
        dBh, dCh = dBh.view(Bsz, L, G, r, N).sum(3), dCh.view(Bsz, L, G, r, N).sum(3)
    return dx, dla, dBh, dCh, dh0


class SelectiveScan(torch.autograd.Function):
    """``selective_scan`` with its gradient (``selective_scan_backward``), so
    that training differentiates the scan as the reference's MLX autograd
    differentiates ``_selective_scan`` (alloy/models/mamba_block.py:287-366).
    Returns (y in x's dtype, final state fp32)."""

    @staticmethod
    def forward(ctx, x, A_disc, B, C, ssm_state, log_a):
        y, h = selective_scan(x, A_disc, B, C, ssm_state=ssm_state, log_a=log_a)
        ctx.save_for_backward(x, A_disc, B, C, ssm_state, log_a)
        return y, h

    @staticmethod
    def backward(ctx, dy, dh):
        x, A_disc, B, C, ssm_state, log_a = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros(x.shape, dtype=x.dtype, device=x.device)
        dx, dA, dB, dC, dh0, dla = selective_scan_backward(
            x, A_disc if log_a is None else None, B, C, dy.contiguous(), ssm_state=ssm_state,
            log_a=log_a, dssm_state_out=dh)
        return dx, dA, dB, dC, dh0, dla


def decode_linear(x, weight, out=None):
    """``x @ weight.T`` for 1 to 4 bf16 rows (``x [NB, in]``, ``weight [out, in]``
    as an ``nn.Linear`` holds it): the in_proj / out_proj of a decode step
    (alloy/models/mamba_block.py:438, :501), a weight-streaming GEMV."""
    dev = _same_device(("x", x), ("weight", weight), ("out", out))
    if out is None:
        out = torch.empty((x.shape[0], weight.shape[0]), dtype=x.dtype, device=dev)
    descs = [_lib.desc(t, n) for t, n in ((x, "x"), (weight, "weight"), (out, "y"))]
    with torch.cuda.device(dev):
        _lib.call("alloy_decode_linear", *(_lib.ref(d) for d in descs), _lib.stream_handle(dev))
    return out


def linear_fills_device(rows, n_out, device):
    """Whether ``linear`` over ``rows`` x ``n_out`` outputs has at least one
    256 x 256 output tile per SM of ``device`` (the GEMM's persistent grid is
    one CTA per SM; with fewer tiles the weights stream through too few SMs)."""
    tiles = -(-rows // 256) * -(-n_out // 256)
    return tiles >= torch.cuda.get_device_properties(device).multi_processor_count


def linear(x, weight, bias=None, out=None):
    """``x @ weight.T (+ bias)`` on the tensor cores: the in_proj / out_proj of
    a prefill or training step (alloy/models/mamba_block.py:438, :501) over
    all tokens at once.  ``x [..., in]`` bf16 (leading dims flattened; a
    layout that does not flatten to one row stride is copied), ``weight
    [out, in]`` bf16 as an ``nn.Linear`` holds it, ``bias [out]`` bf16 or
    None; in, out and the row strides multiples of 8.  Returns ``[..., out]``
    bf16.  No autograd: the backward of a projection stays with torch."""
    dev = _same_device(("x", x), ("weight", weight), ("bias", bias), ("out", out))
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    n_out = weight.shape[0]
    if out is None:
        out = torch.empty((x2.shape[0], n_out), dtype=x.dtype, device=dev)
    descs = [_lib.desc(t, n) for t, n in ((x2, "x"), (weight, "weight"), (bias, "bias"), (out, "y"))]
    with torch.cuda.device(dev):
        _lib.call("alloy_linear", *(_lib.ref(d) for d in descs), _lib.stream_handle(dev))
    return out.reshape(*lead, n_out)


def ssd_decode_step(xBC_tok, dt_tok, conv_weight, conv_bias, dt_bias, A_log, D, conv_state,
                    ssm_state, *, n_heads, head_dim, d_state, n_groups, out=None, head_begin=0,
                    head_count=0):
    """One decode token, updating ``conv_state`` and ``ssm_state`` in place.

    The L = 1 path of ``MambaBlock._forward_combined`` (conv-cache roll,
    alloy/models/mamba_block.py:446-448; ``_selective_scan_sequential``
    :160-204; D residual :492-493).  xBC_tok [B, conv_dim], dt_tok [B, H],
    conv_state [B, K-1, conv_dim] (or its [B, conv_dim, K-1] transpose via
    strides), ssm_state [B, H, N, P] (or [B, H, P, N] via strides), fp32.
    Returns y [B, H, P].
    """
    dev = _same_device(("xBC_tok", xBC_tok), ("dt_tok", dt_tok), ("conv_weight", conv_weight),
                       ("conv_bias", conv_bias), ("dt_bias", dt_bias), ("A_log", A_log),
                       ("D", D), ("conv_state", conv_state), ("ssm_state", ssm_state),
                       ("out", out))
    Bsz = xBC_tok.shape[0]
    if out is None:
        out = torch.empty((Bsz, n_heads, head_dim), dtype=xBC_tok.dtype, device=dev)
    d_conv = conv_state.shape[1] + 1
    dims = _dims(n_heads, head_dim, d_state, n_groups, d_conv, 1, head_begin, head_count)
    args = [(xBC_tok, "xBC_tok"), (dt_tok, "dt_tok"), (_f32(conv_weight), "conv_weight"),
            (_f32(conv_bias), "conv_bias"), (_f32(dt_bias), "dt_bias"), (_f32(A_log), "A_log"),
            (_f32(D), "D"), (conv_state, "conv_state"), (ssm_state, "ssm_state"), (out, "y")]
    descs = [_lib.desc(t, n) for t, n in args]
    with torch.cuda.device(dev):
        _lib.call("alloy_ssd_decode_step", *(_lib.ref(d) for d in descs), _lib.ref(dims),
                  _lib.stream_handle(dev))
    return out


def gated_rmsnorm(y, gate, weight=None, *, eps=1e-5, group_size=0, out=None):
    """The gate and inner norm after the scan, ``MambaBlock._forward_combined``
    step 7 (alloy/models/mamba_block.py:495-499): ``g = y * silu(gate)``, then
    (when ``weight`` is given) ``g * rsqrt(mean(g^2) + eps) * weight`` over the
    last dimension (``nn.RMSNorm(d_inner)``, :137) or over runs of
    ``group_size`` channels of it.  ``y`` and ``gate`` [..., D] of one dtype
    (bf16 or fp32); fp32 math; returns ``out`` (y's shape and dtype; may be
    ``y`` itself).
    """
    dev = _same_device(("y", y), ("gate", gate), ("weight", weight), ("out", out))
    if gate.shape != y.shape:
        raise ValueError(f"gate shape {tuple(gate.shape)} != y shape {tuple(y.shape)}")
    D = y.shape[-1]
    if out is None:
        out = torch.empty(y.shape, dtype=y.dtype, device=dev)
    rows = lambda t: t.reshape(-1, D)   # a view for the usual layouts; a copy only for inputs
    try:
        out2 = out.view(-1, D)
    except RuntimeError as e:
        raise ValueError("out: its leading dimensions must flatten without a copy") from e
    args = [(rows(y), "y"), (rows(gate), "gate"), (_f32(weight), "weight"), (out2, "out")]
    descs = [_lib.desc(t, n) for t, n in args]
    with torch.cuda.device(dev):
        _lib.call("alloy_gated_rmsnorm", *(_lib.ref(d) for d in descs), float(eps), int(group_size),
                  _lib.stream_handle(dev))
    return out
