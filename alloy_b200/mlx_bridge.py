"""MLX arrays in and out of the CUDA hot path.

alloy's MambaBlock works on ``mlx.core.array``.  MLX runs on Apple silicon and
keeps arrays in unified host memory, so on a CUDA machine an MLX array is a
host buffer: it enters through DLPack when the array exports it, else through
numpy (bfloat16 arrays are widened to float32 on the MLX side first, since
numpy has no bfloat16), and is copied to the GPU.  Results return through
numpy.  ``patch_mamba_block`` swaps the hot-path methods of the reference's
MambaBlock class for bridging wrappers around ``alloy_b200.mamba_block``.
"""

from __future__ import annotations

import numpy as np
import torch

__all__ = ["to_torch", "to_mlx", "patch_mamba_block"]


def _is_mlx(a) -> bool:
    return type(a).__module__.startswith("mlx")


def to_torch(a, device="cuda", dtype=None) -> torch.Tensor:
    """An MLX array (or numpy array / torch tensor) as a torch tensor on ``device``."""
    if isinstance(a, torch.Tensor):
        t = a
    else:
        t = None
        if hasattr(a, "__dlpack__"):
            try:
                t = torch.from_dlpack(a)
            except Exception:  # exporter without a usable capsule for torch
                t = None
        if t is None:
            if _is_mlx(a) and "bfloat16" in str(getattr(a, "dtype", "")):
                import mlx.core as mx
                a = a.astype(mx.float32)
                dtype = dtype or torch.bfloat16
            t = torch.from_numpy(np.ascontiguousarray(np.asarray(a)))
    t = t.to(device)
    return t.to(dtype) if dtype is not None else t


def to_mlx(t: torch.Tensor):
    """A torch tensor as an ``mlx.core.array`` (bfloat16 stays bfloat16)."""
    import mlx.core as mx
    x = t.detach()
    if x.dtype == torch.bfloat16:
        return mx.array(x.float().cpu().numpy()).astype(mx.bfloat16)
    return mx.array(x.cpu().numpy())


def patch_mamba_block(cls, device="cuda"):
    """Route the hot-path methods of alloy's ``MambaBlock`` class (an MLX
    module) through liballoy_ssd.

    Replaced, with the reference's signatures (alloy/models/mamba_block.py):
    ``_depthwise_conv1d`` (:144), ``_scan_chunk`` (:206), ``_selective_scan``
    (:287), ``_selective_scan_sequential`` (:160).  Each wrapper moves its MLX
    arguments to ``device``, runs the CUDA kernel and returns MLX arrays; the
    cache's ``ssm_state`` is kept as an MLX array like the reference does.
    Returns the original methods so a caller can restore them.
    """
    from . import mixer

    saved = {n: getattr(cls, n) for n in ("_depthwise_conv1d", "_scan_chunk", "_selective_scan",
                                          "_selective_scan_sequential")}

    def _depthwise_conv1d(self, x_padded, L):
        out = mixer.depthwise_conv1d(to_torch(x_padded, device), to_torch(self.conv_weight, device),
                                     to_torch(self.conv_bias, device), L)
        return to_mlx(out)

    def _scan_chunk(self, x_c, a_c, B_c, C_c, h, cs, log_a_direct=None):
        y, hn = mixer.selective_scan(
            to_torch(x_c, device), to_torch(a_c, device), to_torch(B_c, device),
            to_torch(C_c, device), ssm_state=to_torch(h, device, torch.float32),
            log_a=None if log_a_direct is None else to_torch(log_a_direct, device, torch.float32),
            out_dtype=torch.float32)
        return to_mlx(y), to_mlx(hn)

    def _scan(self, x, A_disc, B, C, cache, log_a, out_dtype):
        h0 = None
        if cache is not None and cache.ssm_state is not None:
            h0 = to_torch(cache.ssm_state, device, torch.float32)
        y, h = mixer.selective_scan(
            to_torch(x, device), to_torch(A_disc, device), to_torch(B, device),
            to_torch(C, device), ssm_state=h0,
            log_a=None if log_a is None else to_torch(log_a, device, torch.float32),
            out_dtype=out_dtype)
        if cache is not None:
            cache.ssm_state = to_mlx(h)
        return to_mlx(y)

    def _selective_scan_sequential(self, x, A_disc, B, C, cache=None):
        return _scan(self, x, A_disc, B, C, cache, None, torch.float32)

    def _selective_scan(self, x, A_disc, B, C, cache=None, log_a=None):
        xt = to_torch(x, device)
        if xt.shape[1] <= 1:
            return _selective_scan_sequential(self, x, A_disc, B, C, cache)
        return _scan(self, x, A_disc, B, C, cache, log_a, xt.dtype)

    cls._depthwise_conv1d = _depthwise_conv1d
    cls._scan_chunk = _scan_chunk
    cls._selective_scan = _selective_scan
    cls._selective_scan_sequential = _selective_scan_sequential
    return saved
