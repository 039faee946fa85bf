"""CUDA kernels (through the C ABI) against the oracle and the reference's
golden vectors.  Needs a B200."""

import numpy as np
import pytest
import torch

import oracle
from alloy_b200 import kernels, mixer
from alloy_b200.mamba_block import MambaBlock, MambaCache
from conftest import (TOL_BF16_MAX_REL, TOL_BF16_REL_L2, TOL_F32_REL_L2, load_golden)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def cu(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def np_(t):
    return t.detach().float().cpu().numpy()


def assert_close(got, ref, bf16):
    r = oracle.rel_l2(got, ref)
    if bf16:
        m = oracle.max_rel(got, ref)
        assert r <= TOL_BF16_REL_L2 and m <= TOL_BF16_MAX_REL, (r, m)
    else:
        assert r <= TOL_F32_REL_L2, r


def run_combined(g, dtype, *, with_state=True, state_layout="nP", conv_layout="kC", **kw):
    B, L, H, P, N, G, Q = (int(v) for v in g["dims"])
    ssm_in = conv_in = None
    if with_state and "ssm_state" in g:
        ssm_in = cu(g["ssm_state"])
        if state_layout == "pN":   # [B, H, P, N] storage passed as a strided view
            ssm_in = ssm_in.transpose(2, 3).contiguous().transpose(2, 3)
        conv_in = cu(g["conv_state"], dtype)
        if conv_layout == "Ck":    # [B, C, K-1] storage
            conv_in = conv_in.transpose(1, 2).contiguous().transpose(1, 2)
    y, h, cs = mixer.ssd_combined(
        cu(g["xBC"], dtype), cu(g["dt_raw"], dtype), cu(g["conv_weight"]), cu(g["conv_bias"]),
        cu(g["dt_bias"]), cu(g["A_log"]), cu(g["D"]), n_heads=H, head_dim=P, d_state=N,
        n_groups=G, chunk_size=Q, ssm_state=ssm_in, conv_state=conv_in, **kw)
    torch.cuda.synchronize()
    return y, h, cs


# --------------------------------------------------------------------------- conv
def test_conv1d_silu_golden():
    g = load_golden("conv1d_silu")
    out = kernels.fused_conv1d_silu(cu(g["x_padded"]), cu(g["weight"]), cu(g["bias"]),
                                    g["x_padded"].shape[1] - 3)
    np.testing.assert_allclose(np_(out), g["out"], rtol=0, atol=1e-5)


@pytest.mark.parametrize("B,L,C,dtype", [(1, 64, 128, torch.float32), (4, 2048, 1024, torch.bfloat16),
                                         (2, 512, 512, torch.float32), (3, 77, 4224, torch.bfloat16),
                                         (2, 5, 100, torch.bfloat16), (1, 1, 24, torch.float32)])
def test_conv1d_silu_sizes(B, L, C, dtype):
    # shapes of the reference's tests/test_metal_kernels.py:37-47 plus ragged ones
    rng = np.random.default_rng(B * 1000 + L)
    xp = rng.standard_normal((B, L + 3, C), dtype=np.float32)
    if dtype == torch.bfloat16:
        xp = oracle.bf16_round(xp)
    w = (rng.standard_normal((C, 4)) * 0.5).astype(np.float32)
    b = rng.standard_normal(C).astype(np.float32)
    ref = oracle.conv1d_silu(xp, w, b, L)
    out = mixer.conv1d_silu(cu(xp, dtype), cu(w), cu(b), L)
    assert out.shape == (B, L, C) and out.dtype == dtype
    assert_close(np_(out), ref, dtype == torch.bfloat16)
    out2 = mixer.depthwise_conv1d(cu(xp, dtype), cu(w), cu(b), L)
    assert_close(np_(out2), oracle.depthwise_conv1d(xp, w, b, L), dtype == torch.bfloat16)


def test_conv1d_silu_backward_golden():
    # the reference's own _metal_conv1d_silu_vjp (mamba_block.py:25-47) on fp32 inputs
    g = load_golden("conv1d_silu_vjp")
    dx, dw, db = mixer.conv1d_silu_backward(cu(g["x_padded"]), cu(g["weight"]), cu(g["bias"]),
                                            cu(g["dy"]))
    torch.cuda.synchronize()
    for got, ref in ((dx, "dx_padded"), (dw, "dweight"), (db, "dbias")):
        assert_close(np_(got), g[ref], False)


@pytest.mark.parametrize("B,L,C,K,dtype", [
    (4, 2048, 1024, 4, torch.bfloat16), (3, 77, 4224, 4, torch.bfloat16),
    (2, 600, 256, 4, torch.float32), (2, 5, 100, 4, torch.bfloat16),   # 4 does not divide C
    (1, 1, 24, 4, torch.float32), (2, 300, 64, 2, torch.float32), (1, 700, 128, 3, torch.bfloat16),
    (2, 0, 32, 4, torch.float32)])
def test_conv1d_silu_backward_vs_oracle(B, L, C, K, dtype):
    rng = np.random.default_rng(B * 1000 + L + K)
    xp = rng.standard_normal((B, L + K - 1, C), dtype=np.float32)
    dy = rng.standard_normal((B, L, C), dtype=np.float32)
    if dtype == torch.bfloat16:
        xp, dy = oracle.bf16_round(xp), oracle.bf16_round(dy)
    w = (rng.standard_normal((C, K)) * 0.5).astype(np.float32)
    b = (rng.standard_normal(C) * 0.1).astype(np.float32)
    ref = oracle.conv1d_silu_vjp(xp, w, b, L, dy)
    got = mixer.conv1d_silu_backward(cu(xp, dtype), cu(w), cu(b), cu(dy, dtype))
    torch.cuda.synchronize()
    assert got[0].dtype == dtype and got[0].shape == xp.shape
    for gt, rf in zip(got, ref):
        if np.abs(rf).max() == 0:
            assert np.abs(np_(gt)).max() == 0
        else:
            assert_close(np_(gt), rf, dtype == torch.bfloat16)


def test_conv1d_silu_backward_strided_deterministic_and_long_input():
    rng = np.random.default_rng(5)
    B, L, C = 2, 200, 512
    xp = rng.standard_normal((B, L + 3 + 10, C), dtype=np.float32)   # 10 rows past L+K-1
    w = (rng.standard_normal((C, 4)) * 0.5).astype(np.float32)
    dy = rng.standard_normal((B, L, C), dtype=np.float32)
    ref = oracle.conv1d_silu_vjp(xp[:, :L + 3], w, np.zeros(C, np.float32), L, dy)
    x_t = cu(xp)
    a = mixer.conv1d_silu_backward(x_t, cu(w), None, cu(dy), L=L)
    b2 = mixer.conv1d_silu_backward(x_t, cu(w), None, cu(dy), L=L)
    # channel-strided input (generic path)
    xs = cu(xp).transpose(1, 2).contiguous().transpose(1, 2)
    c = mixer.conv1d_silu_backward(xs, cu(w), None, cu(dy), L=L)
    torch.cuda.synchronize()
    assert a[2] is None
    assert torch.equal(a[0], b2[0]) and torch.equal(a[1], b2[1])   # fixed-order sums
    assert np.abs(np_(a[0])[:, L + 3:]).max() == 0                   # rows the conv never read
    for got in (a, c):
        assert_close(np_(got[0])[:, :L + 3], ref[0], False)
        assert_close(np_(got[1]), ref[1], False)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_conv1d_silu_autograd(dtype):
    # _metal_conv1d_silu's custom VJP (mamba_block.py:19-47) against float64 autograd
    from alloy_b200.mamba_block import _metal_conv1d_silu
    rng = np.random.default_rng(9)
    B, L, C = 2, 130, 192
    xp = oracle.bf16_round(rng.standard_normal((B, L + 3, C), dtype=np.float32))
    w = (rng.standard_normal((C, 4)) * 0.5).astype(np.float32)
    b = (rng.standard_normal(C) * 0.1).astype(np.float32)
    up = oracle.bf16_round(rng.standard_normal((B, L, C), dtype=np.float32))
    x_t = cu(xp, dtype).requires_grad_()
    w_t, b_t = cu(w).requires_grad_(), cu(b).requires_grad_()
    (_metal_conv1d_silu(x_t, w_t, b_t, L).float() * cu(up)).sum().backward()
    x64, w64, b64 = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (xp, w, b))
    pre = sum(x64[:, k:k + L, :] * w64[:, k] for k in range(4)) + b64
    (torch.nn.functional.silu(pre) * torch.tensor(up, dtype=torch.float64)).sum().backward()
    for got, ref in ((x_t.grad, x64.grad), (w_t.grad, w64.grad), (b_t.grad, b64.grad)):
        assert_close(np_(got), ref.numpy(), dtype == torch.bfloat16)


def test_conv1d_strided_input_uses_generic_path():
    rng = np.random.default_rng(7)
    xp = rng.standard_normal((2, 40, 64), dtype=np.float32)
    w = rng.standard_normal((32, 4), dtype=np.float32)
    ref = oracle.conv1d_silu(xp[:, :, ::2].copy(), w, np.zeros(32, np.float32), 37)
    out = mixer.conv1d_silu(cu(xp)[:, :, ::2], cu(w), None, 37)
    assert_close(np_(out), ref, False)


# --------------------------------------------------------------------- fused prefill
@pytest.mark.parametrize("name", ["toy_prefill", "groups_ragged_state", "short_state"])
def test_combined_fp32_golden(name):
    g = load_golden(name)
    y, h, cs = run_combined(g, torch.float32)
    assert_close(np_(y), g["y"], False)
    assert_close(np_(h), g["ssm_state_out"], False)
    np.testing.assert_array_equal(np_(cs), g["conv_state_out"])


@pytest.mark.parametrize("name", ["bf16_p64_n64", "bf16_p64_n128_g2"])
def test_combined_bf16_golden(name):
    g = load_golden(name)
    y, h, cs = run_combined(g, torch.bfloat16)
    assert y.dtype == torch.bfloat16
    assert_close(np_(y), g["y"], True)
    assert_close(np_(h), g["ssm_state_out"], True)
    np.testing.assert_array_equal(np_(cs), g["conv_state_out"])


def test_combined_state_layouts_and_in_place():
    g = load_golden("groups_ragged_state")
    y_ref, h_ref, cs_ref = run_combined(g, torch.float32)
    # [B,H,P,N] ssm state and [B,C,K-1] conv state storage, updated in place
    B, L, H, P, N, G, Q = (int(v) for v in g["dims"])
    ssm = cu(g["ssm_state"]).transpose(2, 3).contiguous()            # [B,H,P,N]
    conv = cu(g["conv_state"]).transpose(1, 2).contiguous()          # [B,C,K-1]
    ssm_v, conv_v = ssm.transpose(2, 3), conv.transpose(1, 2)
    y, _, _ = mixer.ssd_combined(
        cu(g["xBC"]), cu(g["dt_raw"]), cu(g["conv_weight"]), cu(g["conv_bias"]),
        cu(g["dt_bias"]), cu(g["A_log"]), cu(g["D"]), n_heads=H, head_dim=P, d_state=N,
        n_groups=G, ssm_state=ssm_v, conv_state=conv_v, ssm_state_out=ssm_v,
        conv_state_out=conv_v)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(np_(y), np_(y_ref))
    np.testing.assert_array_equal(np_(ssm.transpose(2, 3)), np_(h_ref))
    np.testing.assert_array_equal(np_(conv.transpose(1, 2)), np_(cs_ref))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_combined_head_ranges_partition_the_layer(dtype):
    """Sharding by head range (multi-GPU partitioning) computes exactly the
    heads of the full call."""
    g = load_golden("bf16_p64_n128_g2")
    B, L, H, P, N, G, Q = (int(v) for v in g["dims"])
    y_full, h_full, _ = run_combined(g, dtype)
    # ranges of whole head pairs run the same kernel as the full call: bit-exact
    y = torch.zeros_like(y_full)
    h = torch.zeros_like(h_full)
    for h0, hc in ((0, 2), (2, 2)):
        run_combined(g, dtype, out=y, ssm_state_out=h, head_begin=h0, head_count=hc,
                     write_conv_state=False)
    np.testing.assert_array_equal(np_(y), np_(y_full))
    np.testing.assert_array_equal(np_(h), np_(h_full))
    # odd ranges (computed by the fp32 kernel for bf16 inputs) within tolerance
    y2 = torch.zeros_like(y_full)
    h2 = torch.zeros_like(h_full)
    for h0, hc in ((0, 1), (1, 2), (3, 1)):
        run_combined(g, dtype, out=y2, ssm_state_out=h2, head_begin=h0, head_count=hc,
                     write_conv_state=False)
    assert_close(np_(y2), g["y"], dtype == torch.bfloat16)
    assert_close(np_(h2), g["ssm_state_out"], dtype == torch.bfloat16)


@pytest.mark.parametrize("cfg", [
    dict(B=2, L=700, H=8, P=64, N=64, G=1),
    dict(B=1, L=513, H=16, P=64, N=128, G=8),
    dict(B=1, L=129, H=4, P=32, N=16, G=2),
    dict(B=1, L=3, H=4, P=64, N=128, G=1),
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_combined_vs_fp64_recurrence(cfg, dtype):
    inp = oracle.make_inputs(**cfg, dtype="bf16" if dtype == torch.bfloat16 else "fp32",
                             seed=11, with_state=True)
    H, P, N, G = cfg["H"], cfg["P"], cfg["N"], cfg["G"]
    y64, h64, _ = oracle.mixer_core_fp64(
        inp["xBC"], inp["dt_raw"], inp["conv_weight"], inp["conv_bias"], inp["dt_bias"],
        inp["A_log"], inp["D"], n_heads=H, headdim=P, d_state=N, n_groups=G,
        ssm_state=inp["ssm_state"], conv_state=inp["conv_state"])
    y, h, _ = mixer.ssd_combined(
        cu(inp["xBC"], dtype), cu(inp["dt_raw"], dtype), cu(inp["conv_weight"]),
        cu(inp["conv_bias"]), cu(inp["dt_bias"]), cu(inp["A_log"]), cu(inp["D"]), n_heads=H,
        head_dim=P, d_state=N, n_groups=G, ssm_state=cu(inp["ssm_state"]),
        conv_state=cu(inp["conv_state"], dtype))
    torch.cuda.synchronize()
    assert_close(np_(y), y64, dtype == torch.bfloat16)
    assert_close(np_(h), h64, dtype == torch.bfloat16)


@pytest.mark.parametrize("cfg,piece", [
    (dict(B=2, L=700, H=8, P=64, N=128, G=2), 256),     # ragged last piece, tensor cores
    (dict(B=3, L=300, H=4, P=32, N=16, G=1), 128),      # CUDA-core path, odd row count
    (dict(B=1, L=1000, H=8, P=64, N=64, G=1), 4096),    # one piece per row
])
@pytest.mark.parametrize("with_state", [False, True])
def test_streamed_prefill_from_host_memory(cfg, piece, with_state):
    inp = oracle.make_inputs(**cfg, dtype="bf16", seed=17, with_state=True)
    H, P, N, G = cfg["H"], cfg["P"], cfg["N"], cfg["G"]
    ssm0 = inp["ssm_state"] if with_state else None
    cs0 = inp["conv_state"] if with_state else None
    y64, h64, cs64 = oracle.mixer_core_fp64(
        inp["xBC"], inp["dt_raw"], inp["conv_weight"], inp["conv_bias"], inp["dt_bias"],
        inp["A_log"], inp["D"], n_heads=H, headdim=P, d_state=N, n_groups=G,
        ssm_state=ssm0, conv_state=cs0)

    def host(a, dt=torch.float32):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dt).pin_memory()

    params = [cu(inp[k]) for k in ("conv_weight", "conv_bias", "dt_bias", "A_log", "D")]
    kw = dict(n_heads=H, head_dim=P, d_state=N, n_groups=G)
    y, h, cs = mixer.ssd_combined_streamed(
        host(inp["xBC"], torch.bfloat16), host(inp["dt_raw"], torch.bfloat16), *params,
        ssm_state=None if ssm0 is None else host(ssm0),
        conv_state=None if cs0 is None else host(cs0, torch.bfloat16), piece_tokens=piece, **kw)
    assert not y.is_cuda and y.shape == (cfg["B"], cfg["L"], H, P) and y.dtype == torch.bfloat16
    assert_close(y.float().numpy(), y64, True)
    assert_close(h.numpy(), h64, True)
    assert np.array_equal(cs.float().numpy(), cs64.astype(np.float32))
    # the same layer through the device API
    yd, hd, csd = mixer.ssd_combined(
        cu(inp["xBC"], torch.bfloat16), cu(inp["dt_raw"], torch.bfloat16), *params,
        ssm_state=None if ssm0 is None else cu(ssm0),
        conv_state=None if cs0 is None else cu(cs0, torch.bfloat16), **kw)
    torch.cuda.synchronize()
    assert_close(y.float().numpy(), np_(yd), True)
    assert torch.equal(cs, csd.cpu())


# ------------------------------------------------------------ pre-discretised scan
def test_scan_chunk_golden():
    g = load_golden("scan_chunk")
    H, P, N = 8, 64, 16
    y, h = kernels.scan_chunk_metal(cu(g["x"]), cu(g["a"]), cu(g["B"]), cu(g["C"]),
                                    cu(g["h"]), H, P, N)
    assert y.dtype == torch.float32
    assert_close(np_(y), g["y"], False)
    assert_close(np_(h), g["h_new"], False)
    y2, _ = kernels.fused_parallel_scan_chunk(cu(g["x"]), cu(g["a"]), cu(g["B"]), cu(g["C"]),
                                              cu(g["h"]) * 0, H, P, N)
    assert_close(np_(y2), g["y_seq_zero_h"], False)


def test_block_scan_methods_match_oracle():
    rng = np.random.default_rng(3)
    B, L, H, P, N = 2, 300, 4, 32, 16
    x = rng.standard_normal((B, L, H, P), dtype=np.float32)
    log_a = -rng.uniform(0.01, 0.5, size=(B, L, H)).astype(np.float32)
    Bm = rng.standard_normal((B, L, H, N), dtype=np.float32)
    Cm = rng.standard_normal((B, L, H, N), dtype=np.float32)
    y_ref, h_ref = oracle.selective_scan(x, np.exp(log_a), Bm, Cm, None, log_a, 64)
    blk = MambaBlock(d_model=H * P // 2, d_state=N, headdim=P, chunk_size=64, device=DEV)
    cache = MambaCache()
    y = blk._selective_scan(cu(x), cu(np.exp(log_a)), cu(Bm), cu(Cm), cache, cu(log_a))
    assert_close(np_(y), y_ref, False)
    assert_close(np_(cache.ssm_state), h_ref, False)
    y1 = blk._selective_scan_sequential(cu(x[:, :1]), cu(np.exp(log_a[:, :1])), cu(Bm[:, :1]),
                                        cu(Cm[:, :1]), None)
    y1_ref, _ = oracle.selective_scan_sequential(x[:, :1], np.exp(log_a[:, :1]), Bm[:, :1],
                                                 Cm[:, :1])
    assert_close(np_(y1), y1_ref, False)


# ---------------------------------------------------------------------- decode step
def test_decode_steps_golden():
    g = load_golden("decode_steps")
    B, L0, steps, H, P, N, G, Q = (int(v) for v in g["dims"])
    kw = dict(n_heads=H, head_dim=P, d_state=N, n_groups=G)
    p = [cu(g[k]) for k in ("conv_weight", "conv_bias", "dt_bias", "A_log", "D")]
    y0, h, cs = mixer.ssd_combined(cu(g["xBC"][:, :L0]), cu(g["dt_raw"][:, :L0]), *p,
                                   chunk_size=Q, **kw)
    assert_close(np_(y0), g["y_prefill"], False)
    ys = []
    for t in range(L0, L0 + steps):
        ys.append(mixer.ssd_decode_step(cu(g["xBC"][:, t]), cu(g["dt_raw"][:, t]), *p, cs, h,
                                        **kw))
    torch.cuda.synchronize()
    assert_close(np_(torch.stack(ys, 1)), g["y_steps"], False)
    assert_close(np_(h), g["ssm_state_out"], False)
    np.testing.assert_array_equal(np_(cs), g["conv_state_out"])


@pytest.mark.parametrize("state_layout", ["NP", "PN"])
@pytest.mark.parametrize("N,P,G,H", [(128, 64, 8, 32), (64, 64, 1, 8), (16, 32, 2, 4), (24, 20, 1, 2)])
def test_decode_step_vs_fp64(state_layout, N, P, G, H):
    B, K = 3, 4
    inp = oracle.make_inputs(B=B, L=1, H=H, P=P, N=N, G=G, dtype="bf16", seed=5,
                             with_state=True)
    y64, h64, cs64 = oracle.decode_step_fp64(
        inp["xBC"][:, 0], inp["dt_raw"][:, 0], inp["conv_weight"], inp["conv_bias"],
        inp["dt_bias"], inp["A_log"], inp["D"], inp["ssm_state"], inp["conv_state"],
        n_heads=H, headdim=P, d_state=N, n_groups=G)
    ssm = cu(inp["ssm_state"])
    if state_layout == "PN":
        store = ssm.transpose(2, 3).contiguous()      # [B, H, P, N]
        ssm = store.transpose(2, 3)
    conv_store = cu(inp["conv_state"], torch.bfloat16).transpose(1, 2).contiguous()  # [B, C, K-1]
    y = mixer.ssd_decode_step(
        cu(inp["xBC"][:, 0], torch.bfloat16), cu(inp["dt_raw"][:, 0], torch.bfloat16),
        cu(inp["conv_weight"]), cu(inp["conv_bias"]), cu(inp["dt_bias"]), cu(inp["A_log"]),
        cu(inp["D"]), conv_store.transpose(1, 2), ssm, n_heads=H, head_dim=P, d_state=N,
        n_groups=G)
    torch.cuda.synchronize()
    assert_close(np_(y), y64, True)
    assert_close(np_(ssm), h64, True)
    np.testing.assert_array_equal(np_(conv_store.transpose(1, 2)), cs64.astype(np.float32))


@pytest.mark.parametrize("B", [1, 2, 150])   # heads split over CTAs (1, 2); a CTA a group (150)
@pytest.mark.parametrize("ranges", [((0, 8),), ((0, 4), (4, 4))])
def test_decode_step_batch_and_head_ranges(B, ranges):
    """Small batches spread each group's heads over several CTAs (the B and C
    conv-cache channels rolled by a second launch), large batches give a CTA a
    whole group; a step taken as group-aligned head ranges, one call each,
    equals the whole step."""
    H, P, N, G = 8, 16, 16, 2
    inp = oracle.make_inputs(B=B, L=1, H=H, P=P, N=N, G=G, dtype="bf16", seed=B, with_state=True)
    y64, h64, cs64 = oracle.decode_step_fp64(
        inp["xBC"][:, 0], inp["dt_raw"][:, 0], inp["conv_weight"], inp["conv_bias"],
        inp["dt_bias"], inp["A_log"], inp["D"], inp["ssm_state"], inp["conv_state"],
        n_heads=H, headdim=P, d_state=N, n_groups=G)
    ssm = cu(inp["ssm_state"])
    conv = cu(inp["conv_state"], torch.bfloat16)
    y = torch.zeros(B, H, P, device=DEV, dtype=torch.bfloat16)
    for h0, hc in ranges:
        mixer.ssd_decode_step(
            cu(inp["xBC"][:, 0], torch.bfloat16), cu(inp["dt_raw"][:, 0], torch.bfloat16),
            cu(inp["conv_weight"]), cu(inp["conv_bias"]), cu(inp["dt_bias"]), cu(inp["A_log"]),
            cu(inp["D"]), conv, ssm, n_heads=H, head_dim=P, d_state=N, n_groups=G, out=y,
            head_begin=h0, head_count=hc)
    torch.cuda.synchronize()
    assert_close(np_(y), y64, True)
    assert_close(np_(ssm), h64, True)
    np.testing.assert_array_equal(np_(conv), cs64.astype(np.float32))


# ------------------------------------------------------------ gate + inner norm
@pytest.mark.parametrize("rows,D,group,dtype,with_w", [
    (64, 8192, 0, torch.bfloat16, True),      # Nemotron-H d_inner, full-width norm
    (33, 4096, 0, torch.bfloat16, True),      # Zamba2 d_inner
    (16, 8192, 1024, torch.bfloat16, True),   # group-wise: 8 groups of 1024 channels
    (40, 4096, 0, torch.float32, True),       # fp32 (4-wide vectors)
    (8, 8192, 0, torch.bfloat16, False),      # the gate alone
    (7, 100, 0, torch.bfloat16, True),        # 100 channels: the scalar kernel
    (5, 20000, 0, torch.float32, True),       # more than 8 vectors a thread: the scalar kernel
])
def test_gated_rmsnorm_vs_oracle(rows, D, group, dtype, with_w):
    rng = np.random.default_rng(rows + D)
    y = rng.standard_normal((rows, D)).astype(np.float32)
    g = rng.standard_normal((rows, D)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, D).astype(np.float32) if with_w else None
    yt, gt = cu(y, dtype), cu(g, dtype)
    out = mixer.gated_rmsnorm(yt, gt, cu(w) if with_w else None, eps=1e-5, group_size=group)
    torch.cuda.synchronize()
    assert out.dtype == dtype and out.shape == yt.shape
    ref = oracle.gated_rmsnorm(np_(yt), np_(gt), w, eps=1e-5, group_size=group)
    assert_close(np_(out), ref, dtype == torch.bfloat16)


@pytest.mark.parametrize("extra", [1280, 1283])   # row stride a multiple of 8 or not
def test_gated_rmsnorm_strided_gate_in_place(extra):
    """The gate as a column slice of the in-projection's output (row stride >
    D), y normalised in place."""
    proj = torch.randn(2, 50, 8192 + extra, device=DEV).to(torch.bfloat16)
    gate = proj[..., :8192]
    y = torch.randn(2, 50, 8192, device=DEV).to(torch.bfloat16)
    w = torch.rand(8192, device=DEV) + 0.5
    ref = oracle.gated_rmsnorm(np_(y), np_(gate), np_(w))
    out = mixer.gated_rmsnorm(y, gate, w, out=y)
    torch.cuda.synchronize()
    assert out.data_ptr() == y.data_ptr()
    assert_close(np_(out), ref, True)


# ------------------------------------------------------------------- block level
@pytest.mark.parametrize("combined", [True, False, "norm"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_block_autoregressive_matches_parallel(combined, dtype):
    """The reference's tests/test_mamba_block.py:39-60 invariant: step-by-step
    generation through the cache equals one parallel pass ("norm": the
    combined projection with the inner RMS norm, Zamba2's configuration)."""
    torch.manual_seed(42)
    kw = dict(combined_proj=True, n_groups=2, use_D=True) if combined else {}
    if combined == "norm":
        kw["use_inner_norm"] = True
    blk = MambaBlock(d_model=64, d_state=16, d_conv=4, expand=2, headdim=32, chunk_size=16,
                     device=DEV, dtype=dtype, **kw)
    with torch.no_grad():
        blk.A_log.uniform_(0, 2)
        blk.dt_bias.uniform_(-3, -1)
        if blk.D is not None:
            blk.D.normal_()
        blk.conv_weight.normal_(0, 0.5)
        x = torch.randn(2, 40, 64, device=DEV, dtype=dtype)
        y_par = blk(x)
        cache = MambaCache()
        y0 = blk(x[:, :24], cache=cache)
        outs = [y0] + [blk(x[:, t:t + 1], cache=cache) for t in range(24, 40)]
        y_seq = torch.cat(outs, dim=1)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-4
    assert oracle.rel_l2(np_(y_seq), np_(y_par)) < tol
    assert cache.ssm_state.shape == (2, 4, 16, 32)
    conv_dim = 128 + (2 * 2 * 16 if combined else 0)
    assert cache.conv_state.shape == (2, 3, conv_dim)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_graph_matches_eager(dtype):
    """Decode steps replayed from one captured CUDA graph (in-projection,
    in-place cache step, gate + inner norm, out-projection) equal the same
    steps run eagerly, outputs and cache."""
    from alloy_b200.decode_graph import MambaDecodeGraph
    torch.manual_seed(7)
    blk = MambaBlock(d_model=256, d_state=64, d_conv=4, expand=2, headdim=64, n_groups=2,
                     use_D=True, use_inner_norm=True, combined_proj=True, chunk_size=64,
                     device=DEV, dtype=dtype)
    with torch.no_grad():
        blk.A_log.uniform_(0, 2)
        blk.dt_bias.uniform_(-3, -1)
        blk.D.normal_()
        blk.conv_weight.normal_(0, 0.5)
        x = torch.randn(3, 20, 256, device=DEV, dtype=dtype)
        eager = MambaCache()
        blk(x[:, :12], cache=eager)
        graphed = MambaCache(ssm_state=eager.ssm_state.clone(), conv_state=eager.conv_state.clone())
        g = MambaDecodeGraph(blk, graphed, batch=3)
        assert torch.equal(graphed.ssm_state, eager.ssm_state)   # capture leaves the cache as it was
        for t in range(12, 20):
            ye = blk(x[:, t:t + 1], cache=eager)
            yg = g.step(x[:, t:t + 1]).clone()
            torch.testing.assert_close(yg, ye)
        torch.testing.assert_close(graphed.ssm_state, eager.ssm_state)
        torch.testing.assert_close(graphed.conv_state, eager.conv_state)


# ------------------------------------------------------- tensor-core path checks
def test_tensor_core_path_is_selected_for_bf16_layer_shapes():
    from alloy_b200 import _lib
    lib = _lib.load()
    for H, N, G in ((128, 128, 8), (64, 64, 1)):
        d = mixer._dims(H, 64, N, G, 4, 256, 0, 0)
        assert lib.alloy_ssd_combined_workspace_size(4, 1024, _lib.BF16, _lib.ref(d)) > 0
        assert lib.alloy_ssd_combined_workspace_size(4, 1024, _lib.F32, _lib.ref(d)) == 0


@pytest.mark.parametrize("cfg", [
    dict(B=2, L=1000, H=16, P=64, N=128, G=8),     # Nemotron-H head/state shape
    dict(B=1, L=1280, H=8, P=64, N=64, G=1),       # Zamba2 head/state shape, 10 chunks
    dict(B=3, L=128, H=2, P=64, N=64, G=1),        # exactly one chunk
    dict(B=1, L=257, H=4, P=64, N=128, G=2),       # one step into a third chunk
])
def test_tensor_core_ssd_vs_oracle(cfg):
    inp = oracle.make_inputs(**cfg, dtype="bf16", seed=21, with_state=True)
    H, P, N, G = cfg["H"], cfg["P"], cfg["N"], cfg["G"]
    y_ref, h_ref, cs_ref = oracle.mixer_core(
        inp["xBC"], inp["dt_raw"], inp["conv_weight"], inp["conv_bias"], inp["dt_bias"],
        inp["A_log"], inp["D"], n_heads=H, headdim=P, d_state=N, n_groups=G, chunk_size=256,
        ssm_state=inp["ssm_state"], conv_state=inp["conv_state"])
    y, h, cs = mixer.ssd_combined(
        cu(inp["xBC"], torch.bfloat16), cu(inp["dt_raw"], torch.bfloat16),
        cu(inp["conv_weight"]), cu(inp["conv_bias"]), cu(inp["dt_bias"]), cu(inp["A_log"]),
        cu(inp["D"]), n_heads=H, head_dim=P, d_state=N, n_groups=G,
        ssm_state=cu(inp["ssm_state"]), conv_state=cu(inp["conv_state"], torch.bfloat16))
    mixer.check_device_status()
    assert_close(np_(y), y_ref, True)
    assert_close(np_(h), h_ref, True)
    np.testing.assert_array_equal(np_(cs), cs_ref)


@pytest.mark.parametrize("dt_bias", [
    [8.0, 8.0, 8.0, 8.0],          # |A dt| of 8 to 128 a step: every 16-step piece spans > e^80
    [-3.0, 0.0, 1.5, 3.0],         # per-head ranges on both sides of that bound
])
def test_tensor_core_ssd_strong_decay(dt_bias):
    """Fast-decaying heads take the exact-exponent path on the diagonal pieces
    of the scores (a decay range over 16 steps beyond e^80); parity with the
    oracle holds there too."""
    cfg = dict(B=2, L=700, H=4, P=64, N=128, G=1)
    inp = oracle.make_inputs(**cfg, dtype="bf16", seed=23, with_state=True)
    inp["dt_bias"] = np.asarray(dt_bias, np.float32)
    y_ref, h_ref, _ = oracle.mixer_core(
        inp["xBC"], inp["dt_raw"], inp["conv_weight"], inp["conv_bias"], inp["dt_bias"],
        inp["A_log"], inp["D"], n_heads=4, headdim=64, d_state=128, n_groups=1, chunk_size=256,
        ssm_state=inp["ssm_state"], conv_state=inp["conv_state"])
    y, h, _ = mixer.ssd_combined(
        cu(inp["xBC"], torch.bfloat16), cu(inp["dt_raw"], torch.bfloat16),
        cu(inp["conv_weight"]), cu(inp["conv_bias"]), cu(inp["dt_bias"]), cu(inp["A_log"]),
        cu(inp["D"]), n_heads=4, head_dim=64, d_state=128, n_groups=1,
        ssm_state=cu(inp["ssm_state"]), conv_state=cu(inp["conv_state"], torch.bfloat16))
    mixer.check_device_status()
    assert np.isfinite(np_(y)).all() and np.isfinite(np_(h)).all()
    assert_close(np_(y), y_ref, True)
    assert_close(np_(h), h_ref, True)


@pytest.mark.parametrize("cfg", [
    dict(B=1, L=4096, H=4, P=64, N=128, G=1),      # 2 head pairs, 32 chunks: 8 segments each
    dict(B=2, L=2999, H=2, P=64, N=64, G=1),       # ragged last chunk, 24 chunks: 6 segments
])
def test_tensor_core_ssd_sequence_segments(cfg):
    """With fewer (batch row, head pair) units than SMs the chunks of a unit
    are cut into segments walked by several CTAs (a state-only pass, then the
    full pass from the carried state).  Parity with the oracle, agreement with
    the one-CTA-a-unit walk of the smallest workspace, and an in-place update
    of the state cache (ssm_state_out aliasing ssm_state)."""
    from alloy_b200 import _lib
    H, P, N, G, L = cfg["H"], cfg["P"], cfg["N"], cfg["G"], cfg["L"]
    lib = _lib.load()
    d = mixer._dims(H, P, N, G, 4, 256, 0, 0)
    full = lib.alloy_ssd_combined_workspace_size(cfg["B"], L, _lib.BF16, _lib.ref(d))
    small = lib.alloy_ssd_combined_min_workspace_size(cfg["B"], L, _lib.BF16, _lib.ref(d))
    assert full > small > 0       # the segment records only come with the full size
    inp = oracle.make_inputs(**cfg, dtype="bf16", seed=24, with_state=True)
    y_ref, h_ref, _ = oracle.mixer_core(
        inp["xBC"], inp["dt_raw"], inp["conv_weight"], inp["conv_bias"], inp["dt_bias"],
        inp["A_log"], inp["D"], n_heads=H, headdim=P, d_state=N, n_groups=G, chunk_size=256,
        ssm_state=inp["ssm_state"], conv_state=inp["conv_state"])
    args = (cu(inp["xBC"], torch.bfloat16), cu(inp["dt_raw"], torch.bfloat16),
            cu(inp["conv_weight"]), cu(inp["conv_bias"]), cu(inp["dt_bias"]),
            cu(inp["A_log"]), cu(inp["D"]))
    kw = dict(n_heads=H, head_dim=P, d_state=N, n_groups=G,
              conv_state=cu(inp["conv_state"], torch.bfloat16))
    state = cu(inp["ssm_state"])
    y_seg, h_seg, _ = mixer.ssd_combined(*args, ssm_state=state, ssm_state_out=state, **kw)
    y_one, h_one, _ = mixer.ssd_combined(*args, ssm_state=cu(inp["ssm_state"]), workspace="min",
                                         **kw)
    mixer.check_device_status()
    assert h_seg.data_ptr() == state.data_ptr()
    assert_close(np_(y_seg), y_ref, True)
    assert_close(np_(h_seg), h_ref, True)
    assert_close(np_(y_one), y_ref, True)
    assert_close(np_(h_one), h_ref, True)
    # the two walks differ only in the fp32 rounding of the carried state
    assert oracle.rel_l2(np_(y_seg), np_(y_one)) < 3e-3
    assert oracle.rel_l2(np_(h_seg), np_(h_one)) < 1e-4


def test_tensor_core_ssd_is_deterministic_and_chunk_independent():
    cfg = dict(B=1, L=600, H=4, P=64, N=128, G=1)
    inp = oracle.make_inputs(**cfg, dtype="bf16", seed=22)
    args = (cu(inp["xBC"], torch.bfloat16), cu(inp["dt_raw"], torch.bfloat16),
            cu(inp["conv_weight"]), cu(inp["conv_bias"]), cu(inp["dt_bias"]),
            cu(inp["A_log"]), cu(inp["D"]))
    kw = dict(n_heads=4, head_dim=64, d_state=128, n_groups=1)
    y1, h1, _ = mixer.ssd_combined(*args, chunk_size=256, **kw)
    y2, h2, _ = mixer.ssd_combined(*args, chunk_size=64, **kw)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2) and torch.equal(h1, h2)
    # a prefill split in two calls (state + conv cache carried) equals one call
    ya, ha, ca = mixer.ssd_combined(args[0][:, :384], args[1][:, :384], *args[2:], **kw)
    yb, hb, _ = mixer.ssd_combined(args[0][:, 384:], args[1][:, 384:], *args[2:],
                                   ssm_state=ha, conv_state=ca, **kw)
    torch.cuda.synchronize()
    y_cat = torch.cat([ya, yb], dim=1)
    assert oracle.rel_l2(np_(y_cat), np_(y1)) < 2e-3
    assert oracle.rel_l2(np_(hb), np_(h1)) < 2e-3


# ------------------------------------------------------------- training (backward)
def _scan64(x, A_log_decay, B, C, h0):
    """float64 per-step recurrence (mamba_block.py:160-204) with autograd."""
    b, L, H, _ = x.shape
    r = H // B.shape[2]
    Bh, Ch = B.repeat_interleave(r, 2), C.repeat_interleave(r, 2)
    h = h0
    ys = []
    for t in range(L):
        h = torch.exp(A_log_decay[:, t])[:, :, None, None] * h + Bh[:, t, :, :, None] * x[:, t, :, None, :]
        ys.append((Ch[:, t, :, :, None] * h).sum(2))
    return torch.stack(ys, 1), h


@pytest.mark.parametrize("cfg", [dict(b=2, L=70, H=4, P=16, N=8, G=2, log=False),
                                 dict(b=1, L=129, H=2, P=32, N=16, G=1, log=True)])
def test_selective_scan_backward_vs_fp64_autograd(cfg):
    g = torch.Generator().manual_seed(5)
    b, L, H, P, N, G = (cfg[k] for k in ("b", "L", "H", "P", "N", "G"))
    x = torch.randn(b, L, H, P, generator=g) * 0.5
    Bm, Cm = torch.randn(b, L, G, N, generator=g), torch.randn(b, L, G, N, generator=g)
    la = -torch.rand(b, L, H, generator=g) * 0.3
    h0 = torch.randn(b, H, N, P, generator=g) * 0.3
    U, V = torch.randn(b, L, H, P, generator=g), torch.randn(b, H, N, P, generator=g)
    # float64 reference
    leaves = [t.double().requires_grad_() for t in (x, la, Bm, Cm, h0)]
    y64, h64 = _scan64(leaves[0], leaves[1], leaves[2], leaves[3], leaves[4])
    ((y64 * U.double()).sum() + (h64 * V.double()).sum()).backward()
    # the library: A_disc or log_a input
    xs = [t.to(DEV).requires_grad_() for t in (x, la.exp() if not cfg["log"] else la, Bm, Cm, h0)]
    if cfg["log"]:
        y, h = mixer.SelectiveScan.apply(xs[0], None, xs[2], xs[3], xs[4], xs[1])
    else:
        y, h = mixer.SelectiveScan.apply(xs[0], xs[1], xs[2], xs[3], xs[4], None)
    ((y * U.to(DEV)).sum() + (h * V.to(DEV)).sum()).backward()
    assert_close(np_(y), y64.detach().numpy(), False)
    dla = xs[1].grad * (1.0 if cfg["log"] else xs[1].detach())   # d/dla = A d/dA
    for got, ref in ((xs[0].grad, leaves[0].grad), (dla, leaves[1].grad), (xs[2].grad, leaves[2].grad),
                     (xs[3].grad, leaves[3].grad), (xs[4].grad, leaves[4].grad)):
        assert_close(np_(got), ref.numpy(), False)


@pytest.mark.parametrize("P,N,G,H,L,reverse,with_h0,out,decay", [
    (64, 64, 1, 3, 300, False, True, torch.float32, 0.3),     # ragged last chunk, initial state
    (64, 128, 2, 4, 256, False, False, torch.bfloat16, 0.3),  # d_state 128, grouped B/C
    (128, 64, 4, 4, 200, True, True, torch.float32, 2.0),     # the dB / dC scan shape, reversed
    (64, 64, 2, 2, 77, True, False, torch.bfloat16, 2.0),     # one partial chunk, reversed
])
def test_tensor_core_scan_vs_fp64(P, N, G, H, L, reverse, with_h0, out, decay):
    """bf16 x, B, C on the tcgen05 scan: y and the final state against the
    float64 per-step recurrence on the same (bf16-rounded) values."""
    g = torch.Generator().manual_seed(P + N + L)
    b = 2
    x = (torch.randn(b, L, H, P, generator=g) * 0.5).bfloat16()
    Bm = torch.randn(b, L, G, N, generator=g).bfloat16()
    Cm = torch.randn(b, L, G, N, generator=g).bfloat16()
    la = -torch.rand(b, L, H, generator=g) * decay
    h0 = torch.randn(b, H, N, P, generator=g) * 0.3 if with_h0 else torch.zeros(b, H, N, P)
    y, h = mixer.selective_scan(x.to(DEV), None, Bm.to(DEV), Cm.to(DEV),
                                ssm_state=h0.to(DEV) if with_h0 else None, log_a=la.to(DEV),
                                out_dtype=out, reverse_time=reverse)
    torch.cuda.synchronize()
    f = (lambda t: t.flip(1)) if reverse else (lambda t: t)
    y64, h64 = _scan64(f(x).double(), f(la).double(), f(Bm).double(), f(Cm).double(), h0.double())
    assert y.dtype == out
    assert_close(np_(y), f(y64).numpy(), True)
    assert_close(np_(h), h64.numpy(), True)


@pytest.mark.parametrize("P,N,Gx,Gz,reverse", [(64, 64, 1, 2, False), (128, 64, 2, 4, True),
                                               (64, 128, 4, 1, False)])
def test_selective_scan_dot_shared_operands(P, N, Gx, Gz, reverse):
    """alloy_selective_scan_dot: x shared by groups of heads, the fused row dot
    products with a grouped z, y written or not, against the float64 recurrence."""
    g = torch.Generator().manual_seed(P + Gx)
    b, L, H, G = 2, 260, 4, 2
    x = (torch.randn(b, L, Gx, P, generator=g) * 0.5).bfloat16()
    Bm, Cm = torch.randn(b, L, G, N, generator=g).bfloat16(), torch.randn(b, L, G, N, generator=g).bfloat16()
    la = -torch.rand(b, L, H, generator=g) * 0.5
    z = torch.randn(b, L, Gz, P, generator=g).bfloat16()
    h0 = torch.randn(b, H, N, P, generator=g) * 0.3
    y, h, dot = mixer.selective_scan_dot(x.to(DEV), Bm.to(DEV), Cm.to(DEV), la.to(DEV), z=z.to(DEV),
                                         ssm_state=h0.to(DEV), write_ssm_state=True, reverse_time=reverse)
    _, h2, dot2 = mixer.selective_scan_dot(x.to(DEV), Bm.to(DEV), Cm.to(DEV), la.to(DEV), z=z.to(DEV),
                                           ssm_state=h0.to(DEV), write_y=False, write_ssm_state=True,
                                           reverse_time=reverse)
    torch.cuda.synchronize()
    f = (lambda t: t.flip(1)) if reverse else (lambda t: t)
    xh = x.repeat_interleave(H // Gx, 2)
    y64, h64 = _scan64(f(xh).double(), f(la).double(), f(Bm).double(), f(Cm).double(), h0.double())
    y64 = f(y64)
    dot64 = (y64 * z.repeat_interleave(H // Gz, 2).double()).sum(-1)
    assert_close(np_(y), y64.numpy(), True)
    assert_close(np_(h), h64.numpy(), True)
    assert_close(np_(dot), dot64.numpy(), True)
    assert torch.equal(dot, dot2) and torch.equal(h, h2)
    # without the step's own term (C_t . B_t)(x_t . z_t)
    _, _, dot3 = mixer.selective_scan_dot(x.to(DEV), Bm.to(DEV), Cm.to(DEV), la.to(DEV), z=z.to(DEV),
                                          ssm_state=h0.to(DEV), write_y=False, reverse_time=reverse,
                                          dot_without_own_term=True)
    r = H // G
    own = ((Cm.double() * Bm.double()).sum(-1).repeat_interleave(r, 2)
           * (xh.double() * z.repeat_interleave(H // Gz, 2).double()).sum(-1))
    err = (dot3.double().cpu() - (dot64 - own)).abs().max() / dot64.abs().max()
    assert err < 2e-2, float(err)
    if (P, N) == (64, 64):
        # the precise mode (operands as bf16 pairs): markedly closer to the float64 recurrence
        y4, _, dot4 = mixer.selective_scan_dot(x.to(DEV), Bm.to(DEV), Cm.to(DEV), la.to(DEV), z=z.to(DEV),
                                               ssm_state=h0.to(DEV), reverse_time=reverse, precise_scores=True)
        assert oracle.rel_l2(np_(y4), y64.numpy()) < 0.5 * oracle.rel_l2(np_(y), y64.numpy())
        assert oracle.rel_l2(np_(dot4), dot64.numpy()) < 0.5 * oracle.rel_l2(np_(dot), dot64.numpy())


@pytest.mark.parametrize("decay,tensor_core_log_decay,N", [(0.3, False, 64), (2.3, False, 64), (2.3, True, 64),
                                                          (2.3, True, 128)])
def test_selective_scan_backward_bf16_on_tensor_cores(decay, tensor_core_log_decay, N):
    """bf16 inputs: dB and dC on the tcgen05 scan with bf16 operands, the
    log-decay gradient's scans on the tcgen05 scan's precise mode (the default,
    through autograd) or in fp32; gradients against float64 autograd on the same bf16 values, within
    2e-2 relative L2 (bf16 operands, the cotangent rounded to bf16), at decays
    up to exp(-decay) a step.  d_state 128 (the Nemotron layer's shape): dB and
    dC on the (128, 64) tensor-core scan, the log-decay scans in fp32."""
    g = torch.Generator().manual_seed(11)
    b, L, H, P, G = 2, 300, 4, 64, 2
    x = (torch.randn(b, L, H, P, generator=g) * 0.5).bfloat16()
    Bm, Cm = torch.randn(b, L, G, N, generator=g).bfloat16(), torch.randn(b, L, G, N, generator=g).bfloat16()
    la = -torch.rand(b, L, H, generator=g) * decay
    h0 = torch.randn(b, H, N, P, generator=g) * 0.3
    U = torch.randn(b, L, H, P, generator=g).bfloat16()
    V = torch.randn(b, H, N, P, generator=g)
    leaves = [t.double().requires_grad_() for t in (x, la, Bm, Cm, h0)]
    y64, h64 = _scan64(*leaves)
    ((y64 * U.double()).sum() + (h64 * V.double()).sum()).backward()
    xs = [t.to(DEV).requires_grad_() for t in (x, la, Bm, Cm, h0)]
    if not tensor_core_log_decay:
        dx, _, dB, dC, dh0, dla = mixer.selective_scan_backward(
            xs[0].detach(), None, xs[2].detach(), xs[3].detach(), U.to(DEV), ssm_state=xs[4].detach(),
            log_a=xs[1].detach(), dssm_state_out=V.to(DEV), tensor_core_log_decay=False)
        grads = (dx, dla, dB, dC, dh0)
    else:
        y, h = mixer.SelectiveScan.apply(xs[0], None, xs[2], xs[3], xs[4], xs[1])
        ((y.float() * U.to(DEV).float()).sum() + (h * V.to(DEV)).sum()).backward()
        grads = (xs[0].grad, xs[1].grad, xs[2].grad, xs[3].grad, xs[4].grad)
    for got, ref in zip(grads, (leaf.grad for leaf in leaves)):
        assert got.dtype == (torch.bfloat16 if ref.shape in (x.shape, Bm.shape) else torch.float32)
        assert oracle.rel_l2(np_(got), ref.numpy()) < 2e-2


def test_combined_block_training_gradients_vs_fp64():
    """MambaBlock (combined projection, inner norm) under autograd: the forward
    equals the fused inference path, and every parameter's gradient matches a
    float64 torch restatement of the layer (conv, split, discretisation,
    per-step scan, D, gate, RMSNorm, projections)."""
    torch.manual_seed(7)
    blk = MambaBlock(d_model=64, d_state=16, d_conv=4, expand=2, headdim=32, chunk_size=16,
                     combined_proj=True, n_groups=2, use_D=True, use_inner_norm=True,
                     device=DEV, dtype=torch.float32)
    with torch.no_grad():
        blk.A_log.uniform_(0, 2)
        blk.dt_bias.uniform_(-3, -1)
        blk.D.normal_()
        blk.conv_weight.normal_(0, 0.5)
        blk.conv_bias.normal_(0, 0.1)
    x = torch.randn(2, 45, 64, device=DEV)
    U = torch.randn(2, 45, 64, device=DEV)
    with torch.no_grad():
        y_inf = blk(x)
    x_t = x.clone().requires_grad_()
    y = blk(x_t)
    assert_close(np_(y), np_(y_inf), False)
    (y * U).sum().backward()

    # float64 restatement
    p = {n: t.detach().double().cpu().requires_grad_() for n, t in blk.named_parameters()}
    x64 = x.detach().double().cpu().requires_grad_()
    H, P, N, G, K, Di = blk.n_heads, blk.headdim, blk.d_state, blk.n_groups, blk.d_conv, blk.d_inner
    proj = x64 @ p["in_proj.weight"].T
    gate, xBC, dt = proj[..., :Di], proj[..., Di:Di + blk.conv_dim], proj[..., Di + blk.conv_dim:]
    xp = torch.nn.functional.pad(xBC, (0, 0, K - 1, 0))
    L = x.shape[1]
    conv = sum(xp[:, k:k + L] * p["conv_weight"][:, k] for k in range(K)) + p["conv_bias"]
    conv = torch.nn.functional.silu(conv)
    xs, Bm, Cm = conv.split([H * P, G * N, G * N], dim=-1)
    xh = xs.reshape(2, L, H, P)
    dtv = torch.nn.functional.softplus(dt + p["dt_bias"])
    la = dtv * -torch.exp(p["A_log"])
    ys, _ = _scan64(xh * dtv[..., None], la, Bm.reshape(2, L, G, N), Cm.reshape(2, L, G, N),
                    torch.zeros(2, H, N, P, dtype=torch.float64))
    yy = (ys + p["D"][:, None] * xh).reshape(2, L, Di) * torch.nn.functional.silu(gate)
    yy = yy * torch.rsqrt((yy * yy).mean(-1, keepdim=True) + 1e-5) * p["norm.weight"]
    out = yy @ p["out_proj.weight"].T
    (out * U.double().cpu()).sum().backward()
    assert_close(np_(y), out.detach().numpy(), False)
    assert_close(np_(x_t.grad), x64.grad.numpy(), False)
    for n, t in blk.named_parameters():
        assert_close(np_(t.grad), p[n].grad.numpy(), False), n


def test_combined_block_training_bf16_on_tensor_cores():
    """A bf16 layer of tensor-core scan sizes (head_dim 64, d_state 64) under
    autograd: its scan forward and backward run on the tcgen05 scan with bf16
    operands; output and gradients against the same layer in fp32 (checked
    against float64 by the test above), within 3e-2 relative L2."""
    torch.manual_seed(3)
    kw = dict(d_model=128, d_state=64, d_conv=4, expand=2, headdim=64, chunk_size=64,
              combined_proj=True, n_groups=2, use_D=True, use_inner_norm=True, device=DEV)
    b16 = MambaBlock(dtype=torch.bfloat16, **kw)
    with torch.no_grad():
        b16.A_log.uniform_(0, 2)
        b16.dt_bias.uniform_(-3, -1)
        b16.D.normal_()
        b16.conv_weight.normal_(0, 0.5)
    f32 = MambaBlock(dtype=torch.float32, **kw)
    f32.load_state_dict({k: v.float() for k, v in b16.state_dict().items()})
    x = torch.randn(2, 300, 128, device=DEV).to(torch.bfloat16)
    U = torch.randn(2, 300, 128, device=DEV)
    outs = []
    for blk in (b16, f32):
        xt = x.to(blk.in_proj.weight.dtype).clone().requires_grad_()
        y = blk(xt)
        (y.float() * U).sum().backward()
        outs.append((y, xt.grad, {n: t.grad for n, t in blk.named_parameters()}))
    (y16, gx16, g16), (y32, gx32, g32) = outs
    assert y16.dtype == torch.bfloat16
    # (the default backward: the log-decay gradient's scans on the precise tensor-core mode)
    assert oracle.rel_l2(np_(y16), np_(y32)) < 3e-2
    assert oracle.rel_l2(np_(gx16), np_(gx32)) < 3e-2
    for n in g32:
        assert oracle.rel_l2(np_(g16[n]), np_(g32[n])) < 3e-2, n


@pytest.mark.parametrize("NB,inp,out", [(1, 4096, 18560), (1, 8192, 4096), (2, 64, 37), (3, 136, 250),
                                        (4, 4096, 4096)])
def test_decode_linear_vs_fp64(NB, inp, out):
    # the decode-step projections (mamba_block.py:438, :501) for 1-4 tokens
    g = torch.Generator(device=DEV).manual_seed(NB * 7 + out)
    x = torch.randn((NB, inp), generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn((out, inp), generator=g, device=DEV) / inp ** 0.5).to(torch.bfloat16)
    y = mixer.decode_linear(x, w)
    torch.cuda.synchronize()
    ref = (x.double() @ w.double().T).cpu().numpy()
    assert y.shape == (NB, out) and y.dtype == torch.bfloat16
    assert_close(np_(y), ref, True)


# ------------------------------------------------------- failure detection
def test_bounded_wait_expiry_is_reported_and_the_context_stays_usable():
    """A bounded device-side wait that runs out: with the test hook set, the
    consumer warps of every prefill CTA wait on an mbarrier that nothing
    completes; each CTA gives up after ~1 ms, drains its copies and MMAs,
    frees its tensor memory and returns.  The host then reads
    ALLOY_ERR_TIMEOUT with the site, and a normal call on the same stream
    afterwards passes parity (no fault, no trap, the context stays usable)."""
    from alloy_b200 import _lib
    lib = _lib.load()
    cfg = dict(B=1, L=512, H=4, P=64, N=64, G=1)
    inp = oracle.make_inputs(**cfg, dtype="bf16", seed=41, with_state=True)
    H, P, N, G = cfg["H"], cfg["P"], cfg["N"], cfg["G"]

    def run():
        return mixer.ssd_combined(
            cu(inp["xBC"], torch.bfloat16), cu(inp["dt_raw"], torch.bfloat16),
            cu(inp["conv_weight"]), cu(inp["conv_bias"]), cu(inp["dt_bias"]), cu(inp["A_log"]),
            cu(inp["D"]), n_heads=H, head_dim=P, d_state=N, n_groups=G,
            ssm_state=cu(inp["ssm_state"]), conv_state=cu(inp["conv_state"], torch.bfloat16))

    mixer.check_device_status()   # nothing pending from earlier tests
    assert lib.alloy_debug_set_wait_stall(2_000_000) == 0
    try:
        run()
        with pytest.raises(_lib.AlloyError) as err:
            mixer.check_device_status()
    finally:
        assert lib.alloy_debug_set_wait_stall(0) == 0
    assert err.value.status == -6
    assert "ssd_tc_kernel" in err.value.message and "site 50" in err.value.message
    mixer.check_device_status()   # the record was cleared by the check
    y_ref, h_ref, _ = oracle.mixer_core(
        inp["xBC"], inp["dt_raw"], inp["conv_weight"], inp["conv_bias"], inp["dt_bias"],
        inp["A_log"], inp["D"], n_heads=H, headdim=P, d_state=N, n_groups=G, chunk_size=256,
        ssm_state=inp["ssm_state"], conv_state=inp["conv_state"])
    y, h, _ = run()
    mixer.check_device_status()
    assert_close(np_(y), y_ref, True)
    assert_close(np_(h), h_ref, True)


def test_wait_stall_hook_rejects_out_of_range_values():
    from alloy_b200 import _lib
    lib = _lib.load()
    assert lib.alloy_debug_set_wait_stall(-1) == -1
    assert lib.alloy_debug_set_wait_stall((1 << 32) + 1) == -1
    assert lib.alloy_debug_set_wait_stall(0) == 0


# ------------------------------------------------- decode graph vs the oracle
def _layer_step_fp64(blk, x_tok, h, cs, bf16):
    """One decode token through a combined-mode layer in float64 on the
    layer's own (possibly bf16-valued) weights: in-projection, the mixer step
    (oracle.decode_step_fp64: mamba_block.py:446-448, :160-204, :492-493),
    gate + inner RMS norm (:495-499), out-projection (:501).  Where the layer
    stores an activation in bf16 (the projection's output, the mixer's y, the
    norm's output), the value is rounded to bf16 here too."""
    f = np.float64
    rnd = (lambda a: oracle.bf16_round(a.astype(np.float32)).astype(f)) if bf16 else (lambda a: a)
    W_in = np_(blk.in_proj.weight).astype(f)
    W_out = np_(blk.out_proj.weight).astype(f)
    di, cd = blk.d_inner, blk.conv_dim
    proj = rnd(x_tok.astype(f) @ W_in.T)
    gate, xBC, dt = proj[:, :di], proj[:, di:di + cd], proj[:, di + cd:]
    y, h, cs = oracle.decode_step_fp64(
        xBC, dt, np_(blk.conv_weight), np_(blk.conv_bias), np_(blk.dt_bias), np_(blk.A_log),
        np_(blk.D), h, cs, n_heads=blk.n_heads, headdim=blk.headdim, d_state=blk.d_state,
        n_groups=blk.n_groups)
    v = rnd(y.reshape(y.shape[0], di)) * (gate / (1.0 + np.exp(-gate)))
    v = v / np.sqrt((v * v).mean(axis=-1, keepdims=True) + blk.norm.eps) * np_(blk.norm.weight).astype(f)
    return rnd(v) @ W_out.T, h, cs


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_graph_steps_vs_oracle(dtype):
    """16 decode steps replayed from the captured CUDA graph (the generation
    loop of alloy/generate.py:84-94 with the cache in device memory) against
    the float64 layer step of the oracle: each step's output and, after the
    last, both caches."""
    from alloy_b200.decode_graph import MambaDecodeGraph
    torch.manual_seed(11)
    blk = MambaBlock(d_model=256, d_state=64, d_conv=4, expand=2, headdim=64, n_groups=2,
                     use_D=True, use_inner_norm=True, combined_proj=True, chunk_size=64,
                     device=DEV, dtype=dtype)
    bf16 = dtype == torch.bfloat16
    with torch.no_grad():
        blk.A_log.uniform_(0, 2)
        blk.dt_bias.uniform_(-3, -1)
        blk.D.normal_()
        blk.conv_weight.normal_(0, 0.5)
        blk.norm.weight.uniform_(0.5, 1.5)
        blk.in_proj.weight.normal_(0, 0.06)
        blk.out_proj.weight.normal_(0, 0.06)
        x = torch.randn(3, 30, 256, device=DEV, dtype=dtype)
        cache = MambaCache()
        blk(x[:, :14], cache=cache)
        h = np_(cache.ssm_state).astype(np.float64)
        cs = np_(cache.conv_state).astype(np.float64)
        g = MambaDecodeGraph(blk, cache, batch=3)
        got, ref = [], []
        for t in range(14, 30):
            got.append(np_(g.step(x[:, t:t + 1])))
            out, h, cs = _layer_step_fp64(blk, np_(x[:, t]), h, cs, bf16)
            ref.append(out)
        torch.cuda.synchronize()
    got, ref = np.stack(got)[:, :, 0], np.stack(ref)
    if bf16:
        assert_close(got, ref, True)
        assert_close(np_(cache.ssm_state), h, True)
        assert_close(np_(cache.conv_state), cs, True)
    else:
        assert oracle.rel_l2(got, ref) < 1e-4
        assert oracle.rel_l2(np_(cache.ssm_state), h) < 1e-4
        assert oracle.rel_l2(np_(cache.conv_state), cs) < 1e-4
