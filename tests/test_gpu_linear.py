"""The tensor-core projection GEMM (``alloy_linear``, ``mixer.linear``)
against an fp32 torch product of the same bf16 operands.

MambaBlock's in_proj / out_proj (alloy/models/mamba_block.py:438, :501) are
``nn.Linear`` layers; the library computes y = x W^T (+ bias) with fp32
accumulation and one bf16 rounding, so the reference is the fp32 product of
the bf16 inputs and the bound is the bf16 rounding of the result
(relative error <= 2^-8 an element) plus the fp32 summation-order error.
"""

import pytest
import torch

from alloy_b200 import mixer

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL_REL_L2 = 3e-3


def _check(y, x, w, b=None, what=""):
    ref = x.float() @ w.float().t()
    if b is not None:
        ref = ref + b.float()
    got = y.float()
    err = (got - ref).norm() / ref.norm()
    bound = 2.0 ** -8 * ref.abs() + 1e-4 * ref.abs().max()
    worst = ((got - ref).abs() - bound).max().item()
    print(f"{what}: rel-L2 {err.item():.2e}")
    assert err.item() <= TOL_REL_L2, (what, err.item())
    assert worst <= 0, (what, worst)


def _rand(*shape, seed, scale=1.0):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,K,N", [
    (1, 8, 8),            # one row, one K step
    (300, 64, 136),       # partial row and column tiles
    (257, 200, 264),      # ragged K (zero-filled past K), one row past a tile
    (1000, 4096, 264),
    (4096, 512, 1024),    # more tiles than SMs: several tiles a CTA
])
def test_linear_vs_fp32(M, K, N):
    x = _rand(M, K, seed=1)
    w = _rand(N, K, seed=2, scale=K ** -0.5)
    _check(mixer.linear(x, w), x, w, what=f"M{M} K{K} N{N}")


def test_linear_bias_strided_rows_and_leading_dims():
    B, L, K, N = 2, 300, 256, 520
    big = _rand(B, L, K + 64, seed=3)
    x = big[..., 32:32 + K]                     # rows with a stride of K + 64
    w = _rand(N, K, seed=4, scale=K ** -0.5)
    b = _rand(N, seed=5)
    out = torch.full((B * L, N + 24), 7.0, dtype=torch.bfloat16, device=DEV)
    y = mixer.linear(x, w, b, out=out[:, :N])
    assert y.shape == (B, L, N)
    _check(y.reshape(B * L, N), x.reshape(B * L, K), w, b, what="bias, strided")
    # the padding columns of the output buffer are untouched
    assert torch.all(out[:, N:] == 7.0)


@pytest.mark.parametrize("which", ["in_proj", "out_proj"])
def test_linear_nemotron_projection_shapes(which):
    """The Nemotron-H-8B layer's projections (d_model 4096, in_proj to
    2*8192 + 2*8*128 + 128 = 18560, out_proj from 8192) on 4,096 tokens."""
    M = 4096
    K, N = (4096, 18560) if which == "in_proj" else (8192, 4096)
    x = _rand(M, K, seed=6)
    w = _rand(N, K, seed=7, scale=K ** -0.5)
    _check(mixer.linear(x, w), x, w, what=which)
    mixer.check_device_status()


@pytest.mark.parametrize("combined", [True, False])
def test_block_projections_use_the_gemm_and_match_torch(combined):
    """MambaBlock routes its bf16 in_proj / out_proj through the GEMM when no
    gradient is needed; the block's output matches the torch-projection path."""
    from alloy_b200.mamba_block import MambaBlock
    torch.manual_seed(0)
    blk = MambaBlock(d_model=256, d_state=64, d_conv=4, expand=2, headdim=64, chunk_size=128,
                     combined_proj=combined, n_groups=1, use_D=combined,
                     use_inner_norm=combined).to(DEV, torch.bfloat16)
    calls = []
    orig, orig_fills = mixer.linear, mixer.linear_fills_device
    mixer.linear = lambda *a, **k: (calls.append(1), orig(*a, **k))[1]
    # a toy layer has fewer output tiles than SMs: route it through the GEMM anyway
    mixer.linear_fills_device = lambda *a: True
    x = _rand(2, 300, 256, seed=8)
    with torch.no_grad():
        try:
            y = blk(x)
        finally:
            mixer.linear, mixer.linear_fills_device = orig, orig_fills
        assert len(calls) == 2, calls
        proj = blk._project
        blk._project = lambda layer, t: layer(t)
        try:
            y_ref = blk(x)
        finally:
            blk._project = proj
    err = ((y.float() - y_ref.float()).norm() / y_ref.float().norm()).item()
    print("block rel-L2 vs torch projections", err)
    assert err <= 1e-2, err


def test_small_products_stay_with_torch():
    """Products with fewer 256 x 256 output tiles than SMs (a short prefill)
    are left to torch; the Nemotron layer's projections over 4 x 8192 tokens
    fill the GPU."""
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    assert not mixer.linear_fills_device(64, 18560, torch.device(DEV))
    assert not mixer.linear_fills_device(2048, 4096, torch.device(DEV))
    assert mixer.linear_fills_device(32768, 4096, torch.device(DEV))
    assert mixer.linear_fills_device(256 * sms, 256, torch.device(DEV))
