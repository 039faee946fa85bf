"""The workloads at their full sizes, through the C ABI, against the float64
recurrence of the oracle on slices the CPU can afford.

Each prefill layer runs whole on the GPU (every batch row and head, every
chunk of the carry); the oracle recomputes a few (batch row, head pair)
slices over the full sequence length: the chunk carry of
alloy/models/mamba_block.py:340-360 is checked across every chunk boundary of
the real length.  Head ranges of the 4- and 8-GPU shards run the segmented
walk (fewer (batch row, head pair) units than SMs).  The decode workload runs
64 sequential steps (mamba_block.py:160-204 with the conv-cache roll of
:446-448) at batch 256.  Inputs are seeded synthetic values with the
workloads' distributions, generated on the GPU.  The measured errors are
printed per case (`pytest -s` or `-rA` shows them).
"""

import math

import numpy as np
import pytest
import torch

import oracle
from alloy_b200 import mixer
from conftest import TOL_BF16_MAX_REL, TOL_BF16_REL_L2

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def gen_layer(B, L, H, P, N, G, seed, K=4):
    """Seeded inputs of one layer on the GPU: xBC ~ N(0,1) and dt_raw ~ N(0,1)
    rounded to bf16; conv weight ~ N(0, 1/4), bias 0; dt_bias = log(expm1(u)),
    u log-uniform in [1e-3, 0.1]; A_log ~ U(0, log 16); D ~ N(0,1)."""
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    C = H * P + 2 * G * N
    xBC = torch.randn((B, L, C), generator=g, device=DEV).to(torch.bfloat16)
    dt_raw = torch.randn((B, L, H), generator=g, device=DEV).to(torch.bfloat16)
    conv_w = torch.randn((C, K), generator=g, device=DEV) * 0.5
    conv_b = torch.zeros(C, device=DEV)
    u = torch.exp(torch.empty(H, device=DEV).uniform_(math.log(1e-3), math.log(0.1), generator=g))
    dt_bias = torch.log(torch.expm1(u))
    A_log = torch.empty(H, device=DEV).uniform_(0.0, math.log(16.0), generator=g)
    D = torch.randn(H, generator=g, device=DEV)
    return dict(xBC=xBC, dt_raw=dt_raw, conv_w=conv_w, conv_b=conv_b, dt_bias=dt_bias,
                A_log=A_log, D=D)


def np32(t):
    return t.detach().float().cpu().numpy()


def slice_layer(t, b, h0, nh, H, P, N, G):
    """Inputs of heads [h0, h0+nh) (inside one group) of batch row b as a
    one-group layer of nh heads, for the oracle."""
    hpg = H // G
    g = h0 // hpg
    assert (h0 + nh - 1) // hpg == g
    xc = list(range(h0 * P, (h0 + nh) * P))
    bc = list(range(H * P + g * N, H * P + (g + 1) * N))
    cc = list(range(H * P + G * N + g * N, H * P + G * N + (g + 1) * N))
    ch = torch.tensor(xc + bc + cc, device=DEV)
    return dict(xBC=np32(t["xBC"][b:b + 1].index_select(2, ch)),
                dt_raw=np32(t["dt_raw"][b:b + 1, :, h0:h0 + nh]),
                conv_weight=np32(t["conv_w"].index_select(0, ch)),
                conv_bias=np32(t["conv_b"].index_select(0, ch)),
                dt_bias=np32(t["dt_bias"][h0:h0 + nh]), A_log=np32(t["A_log"][h0:h0 + nh]),
                D=np32(t["D"][h0:h0 + nh]))


def check(name, got, ref):
    r, m = oracle.rel_l2(got, ref), oracle.max_rel(got, ref)
    print(f"{name}: rel-L2 {r:.3e}  max-rel {m:.3e}")
    assert r <= TOL_BF16_REL_L2 and m <= TOL_BF16_MAX_REL, (name, r, m)


def run_layer(t, H, P, N, G, chunk, **kw):
    y, h, cs = mixer.ssd_combined(t["xBC"], t["dt_raw"], t["conv_w"], t["conv_b"], t["dt_bias"],
                                  t["A_log"], t["D"], n_heads=H, head_dim=P, d_state=N,
                                  n_groups=G, chunk_size=chunk, **kw)
    mixer.check_device_status()
    return y, h, cs


def check_slices(tag, t, y, h, cfg, slices):
    B, L, H, P, N, G = (cfg[k] for k in ("B", "L", "H", "P", "N", "G"))
    for b, h0, nh in slices:
        s = slice_layer(t, b, h0, nh, H, P, N, G)
        y64, h64, _ = oracle.mixer_core_fp64(
            s["xBC"], s["dt_raw"], s["conv_weight"], s["conv_bias"], s["dt_bias"], s["A_log"],
            s["D"], n_heads=nh, headdim=P, d_state=N, n_groups=1)
        check(f"{tag} y[b={b}, heads {h0}-{h0 + nh - 1}]", np32(y[b:b + 1, :, h0:h0 + nh]), y64)
        check(f"{tag} state[b={b}, heads {h0}-{h0 + nh - 1}]", np32(h[b:b + 1, h0:h0 + nh]), h64)


def test_zamba2_layer_full_size():
    """Zamba2-1.2B layer prefill: B 8, L 4096, 64 heads x 64, d_state 64, 1 group."""
    cfg = dict(B=8, L=4096, H=64, P=64, N=64, G=1)
    t = gen_layer(**cfg, seed=101)
    y, h, _ = run_layer(t, 64, 64, 64, 1, 256)
    assert torch.isfinite(y.float()).all() and torch.isfinite(h).all()
    check_slices("zamba2", t, y, h, cfg, [(0, 0, 2), (7, 62, 2), (3, 30, 4)])


def test_nemotron_layer_full_size_and_shards():
    """Nemotron-H-8B layer prefill: B 4, L 8192, 128 heads x 64, d_state 128,
    8 groups; then the head ranges of a 4-GPU shard (32 heads: 64 units,
    segmented) and an 8-GPU shard (16 heads: 32 units, segmented)."""
    cfg = dict(B=4, L=8192, H=128, P=64, N=128, G=8)
    t = gen_layer(**cfg, seed=102)
    y, h, _ = run_layer(t, 128, 64, 128, 8, 256)
    assert torch.isfinite(y.float()).all() and torch.isfinite(h).all()
    check_slices("nemotron", t, y, h, cfg, [(0, 0, 4), (3, 124, 4), (2, 70, 2)])
    for shard_heads in (32, 16):
        for h0 in (0, 128 - shard_heads):
            ys = torch.zeros_like(y)
            hs = torch.zeros_like(h)
            run_layer(t, 128, 64, 128, 8, 256, out=ys, ssm_state_out=hs, head_begin=h0,
                      head_count=shard_heads, write_conv_state=False)
            sl = slice(h0, h0 + shard_heads)
            # the segmented walk differs from the whole-layer call only in the
            # fp32 rounding of the carried state
            ry = (ys[:, :, sl].float() - y[:, :, sl].float()).norm() / y[:, :, sl].float().norm()
            rh = (hs[:, sl] - h[:, sl]).norm() / h[:, sl].norm()
            print(f"nemotron {128 // shard_heads}-GPU shard heads {h0}-{h0 + shard_heads - 1} "
                  f"vs whole layer: y rel-L2 {ry:.3e}, state rel-L2 {rh:.3e}")
            assert ry < 3e-3 and rh < 1e-4
            check_slices(f"nemotron {128 // shard_heads}-GPU shard", t, ys, hs, cfg,
                         [(0, h0, 4), (3, h0 + shard_heads - 2, 2)])


def test_long_context_zamba2_full_size():
    """One 131,072-token Zamba2-shaped sequence (chunk 512): the whole layer
    (32 units, segmented), and the head range of an 8-GPU shard (8 heads: 4
    units in many segments)."""
    cfg = dict(B=1, L=131072, H=64, P=64, N=64, G=1)
    t = gen_layer(**cfg, seed=104)
    y, h, _ = run_layer(t, 64, 64, 64, 1, 512)
    assert torch.isfinite(y.float()).all() and torch.isfinite(h).all()
    check_slices("long", t, y, h, cfg, [(0, 0, 2), (0, 62, 2)])
    ys = torch.zeros_like(y)
    hs = torch.zeros_like(h)
    run_layer(t, 64, 64, 64, 1, 512, out=ys, ssm_state_out=hs, head_begin=0, head_count=8,
              write_conv_state=False)
    check_slices("long 8-GPU shard", t, ys, hs, cfg, [(0, 0, 2), (0, 6, 2)])


def test_nemotron_decode_64_steps_batch_256():
    """64 sequential decode steps at batch 256 (Nemotron-H shape), states in
    the [B, H, P, N] / [B, C, K-1] layouts, checked on batch rows 0 and 255
    against the float64 per-token step."""
    B, H, P, N, G, K, steps = 256, 128, 64, 128, 8, 4, 64
    C = H * P + 2 * G * N
    t = gen_layer(B=1, L=1, H=H, P=P, N=N, G=G, seed=103)
    g = torch.Generator(device=DEV)
    g.manual_seed(1103)
    xs = torch.randn((steps, B, C), generator=g, device=DEV).to(torch.bfloat16)
    dts = torch.randn((steps, B, H), generator=g, device=DEV).to(torch.bfloat16)
    ssm_store = torch.randn((B, H, P, N), generator=g, device=DEV) * math.sqrt(0.1)   # [B, H, P, N]
    conv_store = torch.randn((B, C, K - 1), generator=g, device=DEV).to(torch.bfloat16)
    rows = [0, 255]
    h64 = np.ascontiguousarray(np32(ssm_store[rows]).transpose(0, 1, 3, 2)).astype(np.float64)
    cs64 = np.ascontiguousarray(np32(conv_store[rows]).transpose(0, 2, 1)).astype(np.float64)
    p = dict(conv_weight=np32(t["conv_w"]), conv_bias=np32(t["conv_b"]),
             dt_bias=np32(t["dt_bias"]), A_log=np32(t["A_log"]), D=np32(t["D"]))
    ssm = ssm_store.transpose(2, 3)          # [B, H, N, P] view
    conv = conv_store.transpose(1, 2)        # [B, K-1, C] view
    ys = []
    for s in range(steps):
        ys.append(mixer.ssd_decode_step(xs[s], dts[s], t["conv_w"], t["conv_b"], t["dt_bias"],
                                        t["A_log"], t["D"], conv, ssm, n_heads=H, head_dim=P,
                                        d_state=N, n_groups=G)[rows].clone())
    torch.cuda.synchronize()
    xs_r, dts_r = np32(xs[:, rows]), np32(dts[:, rows])
    y_ref = []
    for s in range(steps):
        y64, h64, cs64 = oracle.decode_step_fp64(
            xs_r[s], dts_r[s], p["conv_weight"], p["conv_bias"], p["dt_bias"], p["A_log"], p["D"],
            h64, cs64, n_heads=H, headdim=P, d_state=N, n_groups=G)
        y_ref.append(y64)
    check("decode y (64 steps, rows 0 and 255)", np32(torch.stack(ys)), np.stack(y_ref))
    check("decode state after 64 steps (rows 0 and 255)", np32(ssm[rows]), h64)
    # the conv cache after 64 steps holds the last K-1 inputs, bit-exact
    np.testing.assert_array_equal(np32(conv[rows]), cs64.astype(np.float32))


def test_split_walk_between_one_and_two_waves():
    """Batch 3 of the Nemotron-H layer shape (L 2048): 192 (batch row, head
    pair) units, between one and two per SM, which the library walks split
    (each unit's chunks in segments run by successive launches of one CTA per
    SM, the state handed over exactly).  Checked against the oracle on slices
    whose units sit in different segments' launches, and against the same call
    with the smallest workspace (one CTA per unit, no split)."""
    from alloy_b200 import _lib
    cfg = dict(B=3, L=2048, H=128, P=64, N=128, G=8)
    t = gen_layer(**cfg, seed=104)
    lib = _lib.load()
    n0 = lib.alloy_kernel_launch_count()
    y, h, _ = run_layer(t, 128, 64, 128, 8, 256)
    split_launches = lib.alloy_kernel_launch_count() - n0
    n0 = lib.alloy_kernel_launch_count()
    y1, h1, _ = run_layer(t, 128, 64, 128, 8, 256, workspace="min")
    plain_launches = lib.alloy_kernel_launch_count() - n0
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    print(f"split walk: {split_launches} launches, one CTA per unit: {plain_launches}")
    if 3 * 64 >= sms:
        assert split_launches > plain_launches
    # the split walk hands the fp32 state over exactly: the same chunks in the same order
    ry = ((y.float() - y1.float()).norm() / y1.float().norm()).item()
    rh = ((h - h1).norm() / h1.norm()).item()
    print(f"split walk vs one CTA per unit: y rel-L2 {ry:.3e}, state rel-L2 {rh:.3e}")
    assert ry == 0.0 and rh == 0.0
    check_slices("split walk", t, y, h, cfg, [(0, 0, 2), (2, 126, 2), (1, 64, 4)])
