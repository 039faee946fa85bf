"""The oracle against the reference's own outputs (golden vectors made by
tests/golden/make_golden.py) and against the invariants the reference's tests
hold.  CPU only."""

import numpy as np
import pytest

import oracle
from conftest import load_golden


def _core(g, with_state=True, **over):
    B, L, H, P, N, G, Q = (int(v) for v in g["dims"])
    kw = dict(n_heads=H, headdim=P, d_state=N, n_groups=G, chunk_size=Q)
    kw.update(over)
    return oracle.mixer_core(
        g["xBC"], g["dt_raw"], g["conv_weight"], g["conv_bias"], g["dt_bias"], g["A_log"],
        g["D"], ssm_state=g.get("ssm_state") if with_state else None,
        conv_state=g.get("conv_state") if with_state else None, **kw)


def _core64(g):
    B, L, H, P, N, G, Q = (int(v) for v in g["dims"])
    return oracle.mixer_core_fp64(
        g["xBC"], g["dt_raw"], g["conv_weight"], g["conv_bias"], g["dt_bias"], g["A_log"],
        g["D"], n_heads=H, headdim=P, d_state=N, n_groups=G,
        ssm_state=g.get("ssm_state"), conv_state=g.get("conv_state"))


def test_conv1d_silu_matches_reference():
    # reference tests/test_metal_kernels.py:18-35 (fused kernel == ops, atol 1e-5)
    g = load_golden("conv1d_silu")
    out = oracle.conv1d_silu(g["x_padded"], g["weight"], g["bias"], g["x_padded"].shape[1] - 3)
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=1e-6)


def test_conv1d_silu_vjp_matches_reference():
    # the reference's own _metal_conv1d_silu_vjp (mamba_block.py:25-47), executed
    g = load_golden("conv1d_silu_vjp")
    L = g["dy"].shape[1]
    dx, dw, db = oracle.conv1d_silu_vjp(g["x_padded"], g["weight"], g["bias"], L, g["dy"])
    np.testing.assert_allclose(dx, g["dx_padded"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(dw, g["dweight"], rtol=1e-6, atol=1e-5)
    np.testing.assert_allclose(db, g["dbias"], rtol=1e-6, atol=1e-5)


@pytest.mark.parametrize("K,L", [(4, 37), (2, 1), (3, 5)])
def test_conv1d_silu_vjp_is_the_gradient(K, L):
    # independent check: float64 autograd of conv + silu
    import torch
    rng = np.random.default_rng(K * 100 + L)
    B, C = 2, 24
    xp = rng.standard_normal((B, L + K - 1, C)).astype(np.float32)
    w = (rng.standard_normal((C, K)) * 0.5).astype(np.float32)
    b = (rng.standard_normal(C) * 0.1).astype(np.float32)
    dy = rng.standard_normal((B, L, C)).astype(np.float32)
    dx, dw, db = oracle.conv1d_silu_vjp(xp, w, b, L, dy)
    x_t, w_t, b_t = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (xp, w, b))
    pre = sum(x_t[:, k:k + L, :] * w_t[:, k] for k in range(K)) + b_t
    torch.nn.functional.silu(pre).backward(torch.tensor(dy, dtype=torch.float64))
    for got, ref in ((dx, x_t.grad), (dw, w_t.grad), (db, b_t.grad)):
        assert oracle.rel_l2(got, ref.numpy()) < 1e-6


def test_scan_chunk_matches_reference():
    # reference tests/test_metal_kernels.py:75-89 (chunk kernels == pure ops)
    g = load_golden("scan_chunk")
    y, h = oracle.scan_chunk(g["x"], g["a"], g["B"], g["C"], g["h"])
    assert oracle.rel_l2(y, g["y"]) < 1e-6
    assert oracle.rel_l2(h, g["h_new"]) < 1e-6


def test_scan_chunk_equals_sequential_scan():
    g = load_golden("scan_chunk")
    y_seq, _ = oracle.selective_scan_sequential(g["x"], g["a"], g["B"], g["C"], None)
    np.testing.assert_allclose(y_seq, g["y_seq_zero_h"], rtol=0, atol=1e-6)
    y_chunk, _ = oracle.scan_chunk(g["x"], g["a"], g["B"], g["C"],
                                   np.zeros_like(g["h"]))
    assert oracle.rel_l2(y_chunk, y_seq) < 1e-5


@pytest.mark.parametrize("name", ["toy_prefill", "groups_ragged_state", "short_state",
                                  "bf16_p64_n64", "bf16_p64_n128_g2"])
def test_mixer_core_matches_reference(name):
    g = load_golden(name)
    y, h, cs = _core(g)
    assert oracle.rel_l2(y, g["y"]) < 1e-6
    assert oracle.rel_l2(h, g["ssm_state_out"]) < 1e-6
    np.testing.assert_array_equal(cs, g["conv_state_out"])


@pytest.mark.parametrize("name", ["toy_prefill", "groups_ragged_state", "short_state",
                                  "bf16_p64_n128_g2"])
def test_reference_matches_fp64_recurrence(name):
    """Pins the reference algorithm itself to the SSM recurrence in float64."""
    g = load_golden(name)
    y64, h64, cs64 = _core64(g)
    assert oracle.rel_l2(g["y"], y64) < 2e-5
    assert oracle.rel_l2(g["ssm_state_out"], h64) < 2e-5
    np.testing.assert_array_equal(g["conv_state_out"], cs64.astype(np.float32))


def test_chunk_size_does_not_change_the_result():
    g = load_golden("toy_prefill")
    y64, _, _ = _core(g, chunk_size=64)
    for q in (16, 50, 512):
        y, _, _ = _core(g, chunk_size=q)
        assert oracle.rel_l2(y, y64) < 2e-6


def test_decode_steps_match_reference():
    """Prefill then single-token steps through the cache (reference
    tests/test_mamba_block.py:39-60: step-by-step == one pass)."""
    g = load_golden("decode_steps")
    B, L0, steps, H, P, N, G, Q = (int(v) for v in g["dims"])
    kw = dict(n_heads=H, headdim=P, d_state=N, n_groups=G, chunk_size=Q)
    args = [g[k] for k in ("conv_weight", "conv_bias", "dt_bias", "A_log", "D")]
    y0, h, cs = oracle.mixer_core(g["xBC"][:, :L0], g["dt_raw"][:, :L0], *args, **kw)
    assert oracle.rel_l2(y0, g["y_prefill"]) < 1e-6
    ys = []
    for t in range(L0, L0 + steps):
        y, h, cs = oracle.mixer_core(g["xBC"][:, t:t + 1], g["dt_raw"][:, t:t + 1], *args,
                                     ssm_state=h, conv_state=cs, **kw)
        ys.append(y[:, 0])
    assert oracle.rel_l2(np.stack(ys, 1), g["y_steps"]) < 1e-6
    assert oracle.rel_l2(h, g["ssm_state_out"]) < 1e-6
    np.testing.assert_array_equal(cs, g["conv_state_out"])
    # the reference's own invariant, on its own outputs
    y_cat = np.concatenate([g["y_prefill"], g["y_steps"]], axis=1)
    assert oracle.rel_l2(y_cat, g["y_full"]) < 1e-5


def test_bf16_round_is_round_to_nearest_even():
    import torch
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 100
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(oracle.bf16_round(x), ref)


def test_make_inputs_distributions():
    inp = oracle.make_inputs(B=2, L=64, H=32, P=8, N=4, G=2, seed=0)
    u = np.logaddexp(inp["dt_bias"], 0)   # softplus(dt_bias) = u
    assert (u > 0.99e-3).all() and (u < 0.101).all()
    A = np.exp(inp["A_log"])
    assert (A >= 1).all() and (A <= 16).all()
    assert abs(inp["conv_weight"].std() - 0.5) < 0.1
    assert inp["xBC"].shape == (2, 64, 32 * 8 + 2 * 2 * 4)


def test_gated_rmsnorm_matches_fp64():
    """Gate first, then RMS norm over the row or over channel groups
    (mamba_block.py:495-499), against a float64 restatement."""
    rng = np.random.default_rng(5)
    y = rng.standard_normal((4, 96)).astype(np.float32)
    g = rng.standard_normal((4, 96)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 96).astype(np.float32)
    v = y.astype(np.float64) * g / (1 + np.exp(-g.astype(np.float64)))
    for gs in (0, 32):
        n = gs or 96
        vv = v.reshape(4, 96 // n, n)
        ref = (vv / np.sqrt((vv ** 2).mean(-1, keepdims=True) + 1e-5)).reshape(4, 96) * w
        got = oracle.gated_rmsnorm(y, g, w, eps=1e-5, group_size=gs)
        assert got.dtype == np.float32
        assert oracle.rel_l2(got, ref) < 1e-6
    # no weight: the gate alone
    assert oracle.rel_l2(oracle.gated_rmsnorm(y, g), v) < 1e-6

