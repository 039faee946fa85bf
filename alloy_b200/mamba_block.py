"""Mamba-2 block and its cache over torch CUDA tensors, with the hot path on
liballoy_ssd.

``MambaBlock`` keeps the reference's constructor (alloy/models/mamba_block.py:76-142)
and the signatures of its hot-path methods, so code written against the
reference's block reads the same:

* ``_depthwise_conv1d(x_padded, L)``                          (:144-158)
* ``_selective_scan_sequential(x, A_disc, B, C, cache=None)``  (:160-204)
* ``_scan_chunk(x_c, a_c, B_c, C_c, h, cs, log_a_direct=None)`` (:206-285)
* ``_selective_scan(x, A_disc, B, C, cache=None, log_a=None)`` (:287-366)
* ``__call__(x, cache=None)`` with the split (:385-426) and combined
  (:428-501) forward modes.

In combined mode the whole conv -> discretise -> scan -> D skip core is one
fused call (``mixer.ssd_combined``), and a cached single-token step is one
``mixer.ssd_decode_step`` that updates the cache tensors in place.  The
projections, gate and norm around the core (in_proj, out_proj, RMSNorm) are
plain torch modules: they are the caller of the hot path, not part of it.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from . import mixer

__all__ = ["MambaCache", "MambaBlock"]


def _needs_grad(*ts):
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ts)


def _metal_conv1d_silu(x_padded, weight, bias, L):
    """conv1d + SiLU that autograd differentiates with the library's backward
    kernel, as alloy's ``@mx.custom_function _metal_conv1d_silu`` with its
    ``.vjp`` (alloy/models/mamba_block.py:19-47)."""
    return mixer.Conv1dSilu.apply(x_padded, weight, bias, L)


@dataclass
class MambaCache:
    """Decode cache of one Mamba layer (alloy/models/cache.py:13-25).

    ssm_state:  [B, n_heads, d_state, headdim], fp32
    conv_state: [B, d_conv - 1, conv_dim], the activation dtype (raw conv inputs)
    """

    ssm_state: Optional[torch.Tensor] = None
    conv_state: Optional[torch.Tensor] = None


class MambaBlock(torch.nn.Module):
    """Mamba-2 selective state-space block (torch + liballoy_ssd)."""

    def __init__(self, d_model: int, d_state: int = 64, d_conv: int = 4, expand: int = 2,
                 headdim: int = 64, chunk_size: int = 256, combined_proj: bool = False,
                 n_groups: int = 1, use_D: bool = False, use_inner_norm: bool = False,
                 device=None, dtype=None):
        super().__init__()
        self.d_model = d_model
        self.d_state = d_state
        self.d_conv = d_conv
        self.expand = expand
        self.headdim = headdim
        self.chunk_size = chunk_size
        self.combined_proj = combined_proj
        self.n_groups = n_groups
        d_inner = d_model * expand
        self.d_inner = d_inner
        if d_inner % headdim != 0:
            raise ValueError("d_inner must be divisible by headdim")
        self.n_heads = d_inner // headdim
        fk = dict(device=device, dtype=dtype)
        if combined_proj:
            self.d_ssm = 2 * d_state * n_groups + self.n_heads
            self.in_proj = torch.nn.Linear(d_model, 2 * d_inner + self.d_ssm, bias=False, **fk)
            self.x_proj = None
            conv_dim = d_inner + 2 * d_state * n_groups
        else:
            self.in_proj = torch.nn.Linear(d_model, 2 * d_inner, bias=False, **fk)
            self.x_proj = torch.nn.Linear(d_inner, self.n_heads * (2 * d_state + 1), bias=False,
                                          **fk)
            conv_dim = d_inner
        self.conv_dim = conv_dim
        p32 = dict(device=device, dtype=torch.float32)
        self.conv_weight = torch.nn.Parameter(torch.randn(conv_dim, d_conv, **p32) * 0.02)
        self.conv_bias = torch.nn.Parameter(torch.zeros(conv_dim, **p32))
        self.A_log = torch.nn.Parameter(torch.zeros(self.n_heads, **p32))
        self.dt_bias = torch.nn.Parameter(torch.zeros(self.n_heads, **p32))
        self.D = torch.nn.Parameter(torch.zeros(self.n_heads, **p32)) if use_D else None
        # eps of the reference's nn.RMSNorm (MLX default 1e-5)
        self.norm = torch.nn.RMSNorm(d_inner, eps=1e-5, **fk) if use_inner_norm else None
        self.out_proj = torch.nn.Linear(d_inner, d_model, bias=False, **fk)

    # ------------------------------------------------------------------ hot path
    def _depthwise_conv1d(self, x_padded: torch.Tensor, L: int) -> torch.Tensor:
        """Causal depthwise conv (no activation): [B, L+K-1, C] -> [B, L, C]."""
        return mixer.depthwise_conv1d(x_padded, self.conv_weight, self.conv_bias, L)

    def _selective_scan_sequential(self, x, A_disc, B, C, cache=None):
        """Step-by-step scan; returns y [B, L, H, P] in fp32 like the reference
        (:181-184, :204) and stores the final state in ``cache``."""
        h0 = cache.ssm_state if cache is not None else None
        y, h = mixer.selective_scan(x, A_disc, B, C, ssm_state=h0, out_dtype=torch.float32)
        if cache is not None:
            cache.ssm_state = h
        return y

    def _scan_chunk(self, x_c, a_c, B_c, C_c, h, cs, log_a_direct=None):
        """One chunk: returns (y_chunk fp32 [B, cs, H, P], h_new [B, H, N, P])."""
        return mixer.selective_scan(x_c, a_c, B_c, C_c, ssm_state=h, log_a=log_a_direct,
                                    out_dtype=torch.float32)

    def _selective_scan(self, x, A_disc, B, C, cache=None, log_a=None):
        """Chunked scan with the cache's state; y in x's dtype (:364-365).
        Differentiable (``mixer.SelectiveScan``) when autograd needs it."""
        h0 = cache.ssm_state if cache is not None else None
        if _needs_grad(x, A_disc, B, C, log_a, h0):
            y, h = mixer.SelectiveScan.apply(x, A_disc if log_a is None else None, B, C, h0, log_a)
            if cache is not None:
                cache.ssm_state = h
            return y
        if x.shape[1] <= 1:
            return self._selective_scan_sequential(x, A_disc, B, C, cache)
        y, h = mixer.selective_scan(x, A_disc, B, C, ssm_state=h0, log_a=log_a,
                                    write_ssm_state=cache is not None)
        if cache is not None:
            cache.ssm_state = h
        return y

    def _forward_combined_train(self, gate, xBC, dt, Bsz, L):
        """Combined mode under autograd (training, no cache): the fused prefill has
        no backward, so the same steps run as differentiable pieces: the conv with
        its VJP (``_metal_conv1d_silu``), the split and discretisation of
        :458-486, the scan with its VJP (``mixer.SelectiveScan``), D on the
        unscaled x (:481-482), then the gate and the inner norm (:495-499)."""
        H, P, N, G, K = self.n_heads, self.headdim, self.d_state, self.n_groups, self.d_conv
        x_padded = F.pad(xBC, (0, 0, K - 1, 0))
        conv = _metal_conv1d_silu(x_padded, self.conv_weight, self.conv_bias, L)
        xs, Bm, Cm = conv.split([H * P, G * N, G * N], dim=-1)
        xh = xs.reshape(Bsz, L, H, P).float()
        dtv = F.softplus(dt.float() + self.dt_bias)
        log_a = dtv * -torch.exp(self.A_log.float())
        xin, Bin, Cin = xh * dtv[..., None], Bm.reshape(Bsz, L, G, N), Cm.reshape(Bsz, L, G, N)
        if xBC.dtype == torch.bfloat16:
            # bf16 operands, as the reference's bf16 arrays are: the scan and its
            # gradient run on the tensor-core scan (fp32 state and accumulation)
            xin = xin.to(torch.bfloat16)
        else:
            Bin, Cin = Bin.float(), Cin.float()
        y, _ = mixer.SelectiveScan.apply(xin, None, Bin, Cin, None, log_a)
        y = y.float()
        if self.D is not None:
            y = y + self.D.float()[:, None] * xh
        y = y.to(xBC.dtype).reshape(Bsz, L, self.d_inner)
        y = y * F.silu(gate)
        if self.norm is not None:
            y = self.norm(y)
        return self.out_proj(y)

    # ------------------------------------------------------------------ forward
    def forward(self, x: torch.Tensor, cache: Optional[MambaCache] = None) -> torch.Tensor:
        Bsz, L, _ = x.shape
        if self.combined_proj:
            return self._forward_combined(x, Bsz, L, cache)
        return self._forward_split(x, Bsz, L, cache)

    def _conv_input_padded(self, conv_input, cache):
        """mamba_block.py:392-398 / :446-452 (split mode keeps the padded copy)."""
        K = self.d_conv
        if cache is not None and cache.conv_state is not None:
            x_padded = torch.cat([cache.conv_state.to(conv_input.dtype), conv_input], dim=1)
        else:
            x_padded = F.pad(conv_input, (0, 0, K - 1, 0))
        if cache is not None:
            cache.conv_state = x_padded[:, -(K - 1):, :].contiguous()
        return x_padded

    def _forward_split(self, x, Bsz, L, cache):
        xz = self._project(self.in_proj, x)
        x_branch, z = xz[..., :self.d_inner], xz[..., self.d_inner:]
        x_padded = self._conv_input_padded(x_branch, cache)
        # (:399-404: the differentiable kernel without a cache, the plain one with)
        if cache is None:
            x_conv = _metal_conv1d_silu(x_padded, self.conv_weight, self.conv_bias, L)
        else:
            x_conv = mixer.conv1d_silu(x_padded, self.conv_weight, self.conv_bias, L)
        ssm = self.x_proj(x_conv).reshape(Bsz, L, self.n_heads, 2 * self.d_state + 1)
        B_param = ssm[..., :self.d_state]
        C_param = ssm[..., self.d_state:2 * self.d_state]
        dt = F.softplus(ssm[..., -1].float() + self.dt_bias)
        A_disc = torch.exp(dt * -torch.exp(self.A_log))
        y = self._selective_scan(x_conv.reshape(Bsz, L, self.n_heads, self.headdim), A_disc,
                                 B_param, C_param, cache)
        y = y.to(x.dtype).reshape(Bsz, L, self.d_inner) * F.silu(z)
        return self._project(self.out_proj, y)

    def _project(self, layer, t):
        """``layer(t)`` for an ``nn.Linear``.  Without autograd, bf16 on the GPU:
        a step of one token per sequence for up to 4 sequences (decoding) runs
        the library's GEMV, a product with at least one 256 x 256 output tile
        per SM its tensor-core GEMM; other sizes stay with torch (cuBLAS)."""
        w = layer.weight
        if (t.is_cuda and t.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
                and t.shape[-1] % 8 == 0 and w.shape[0] % 8 == 0 and w.stride(1) == 1
                and w.stride(0) % 8 == 0 and not _needs_grad(t, w, layer.bias)):
            if t.dim() == 3 and t.shape[1] == 1 and t.shape[0] <= 4 and layer.bias is None:
                return mixer.decode_linear(t.reshape(t.shape[0], t.shape[2]), w).unsqueeze(1)
            if ((layer.bias is None or layer.bias.dtype == torch.bfloat16)
                    and mixer.linear_fills_device(t.numel() // t.shape[-1], w.shape[0], t.device)):
                return mixer.linear(t, w, layer.bias)
        return layer(t)

    def _forward_combined(self, x, Bsz, L, cache):
        ng, N, K = self.n_groups, self.d_state, self.d_conv
        proj = self._project(self.in_proj, x)
        gate = proj[..., :self.d_inner]
        xBC = proj[..., self.d_inner:self.d_inner + self.conv_dim]
        dt = proj[..., self.d_inner + self.conv_dim:]
        kw = dict(n_heads=self.n_heads, head_dim=self.headdim, d_state=N, n_groups=ng)
        if cache is None and _needs_grad(xBC, dt, self.conv_weight, self.A_log, self.D):
            return self._forward_combined_train(gate, xBC, dt, Bsz, L)
        if (L == 1 and cache is not None and cache.ssm_state is not None
                and cache.conv_state is not None):
            y = mixer.ssd_decode_step(xBC[:, 0], dt[:, 0], self.conv_weight, self.conv_bias,
                                      self.dt_bias, self.A_log, self.D, cache.conv_state,
                                      cache.ssm_state, **kw)
            y = y.reshape(Bsz, 1, self.d_inner)
        else:
            h0 = cache.ssm_state if cache is not None else None
            c0 = cache.conv_state if cache is not None else None
            y, h, cs = mixer.ssd_combined(
                xBC, dt, self.conv_weight, self.conv_bias, self.dt_bias, self.A_log, self.D,
                d_conv=K, chunk_size=self.chunk_size, ssm_state=h0, conv_state=c0,
                write_ssm_state=cache is not None, write_conv_state=cache is not None, **kw)
            if cache is not None:
                cache.ssm_state, cache.conv_state = h, cs
            y = y.reshape(Bsz, L, self.d_inner)
        # gate first, then the inner norm (:495-499), fused in one kernel
        y = mixer.gated_rmsnorm(y, gate, self.norm.weight if self.norm is not None else None,
                                eps=self.norm.eps if self.norm is not None else 1e-5)
        return self._project(self.out_proj, y)
