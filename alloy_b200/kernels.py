"""Drop-in counterparts of alloy/models/mamba_kernels.py, over torch CUDA tensors.

Same names, arguments and return values as the reference module, backed by
liballoy_ssd instead of Metal:

* ``fused_conv1d_silu(x_padded, weight, bias, L)``        (mamba_kernels.py:39-50)
* ``scan_chunk_metal(x_c, a_c, B_c, C_c, h, n_heads, headdim, d_state)``
                                                           (mamba_kernels.py:193-224)
* ``fused_parallel_scan_chunk(...)``, same signature       (mamba_kernels.py:333-396)

The two scan-chunk functions run the same recurrence over one chunk:
``h_t = a_t h_{t-1} + B_t x_t^T``, ``y_t = C_t h_t`` with fp32 state and
outputs, and return ``(y_chunk [B, cs, H, P], h_new [B, H, N, P])``.  Unlike
the reference's parallel-scan kernel they are correct for any chunk length
(the reference's launches min(cs, 256) threads per group, :371).
The reference's materialising helpers ``flat_outer_product`` and
``c_contraction`` have no counterpart: the fused scan never forms B (x) x or
the per-step states.
"""

from __future__ import annotations

import torch

from . import mixer

__all__ = ["fused_conv1d_silu", "scan_chunk_metal", "fused_parallel_scan_chunk"]


def fused_conv1d_silu(x_padded, weight, bias, L):
    """Fused depthwise conv1d + SiLU: [B, L+d_conv-1, d_inner] -> [B, L, d_inner]."""
    return mixer.conv1d_silu(x_padded, weight, bias, L)


def scan_chunk_metal(x_c, a_c, B_c, C_c, h, n_heads, headdim, d_state):
    """One scan chunk: x_c [B,cs,H,P], a_c [B,cs,H] (decay factors), B_c/C_c
    [B,cs,H,N], h [B,H,N,P] -> (y_chunk fp32 [B,cs,H,P], h_new [B,H,N,P])."""
    if x_c.shape[2] != n_heads or x_c.shape[3] != headdim or B_c.shape[-1] != d_state:
        raise ValueError("scan_chunk_metal: n_heads/headdim/d_state do not match the inputs")
    return mixer.selective_scan(x_c, a_c, B_c, C_c, ssm_state=h, out_dtype=torch.float32)


def fused_parallel_scan_chunk(x_c, a_c, B_c, C_c, h, n_heads, headdim, d_state):
    """Same contract as :func:`scan_chunk_metal` (the reference's parallel-scan
    variant computes the same recurrence)."""
    return scan_chunk_metal(x_c, a_c, B_c, C_c, h, n_heads, headdim, d_state)
