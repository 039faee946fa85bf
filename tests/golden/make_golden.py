"""Generate the golden vectors in this folder by running the reference itself.

The reference (gxcsoccer/alloy) is an MLX package; MLX cannot be installed
here, so this script registers ``mlx_numpy_standin`` as ``mlx`` and then
executes the reference's own, unmodified ``alloy/models/mamba_block.py`` and
``alloy/models/cache.py`` from the reference checkout.  ``mamba_kernels``
(Metal-only) is blocked, which takes the reference's own
``USE_METAL_KERNELS = False`` branch (mamba_block.py:49-50), i.e. its pure-op
conv and chunked/sequential scans.

``MambaBlock.__call__`` is driven end to end (combined / Zamba2 / Nemotron-H
mode, use_D=True) with ``in_proj`` replaced by a callable that returns a
prepared projection ``[gate | xBC | dt_raw]`` and ``out_proj`` by the
identity.  The gate is the constant 32: in float32 silu(32) == 32 exactly, so
the block's output divided by 32 is exactly the mixer output y (scan + D*x)
before gating.  The cache (``MambaCache``) carries ssm_state/conv_state.

Usage:  python tests/golden/make_golden.py [REFERENCE_ROOT]
Inputs come from ``oracle.make_inputs`` (numpy PCG64, seeded) and are stored
in the .npz next to the outputs, so the fixtures are self-contained.
"""

from __future__ import annotations

import importlib.util
import types
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

import mlx_numpy_standin  # noqa: E402

from oracle import make_inputs  # noqa: E402

GATE = np.float32(32.0)


def load_reference(root):
    mlx_numpy_standin.install()
    # The Metal kernels module cannot run here: make its import fail with
    # ImportError so mamba_block takes its own USE_METAL_KERNELS = False path.
    sys.modules["alloy.models.mamba_kernels"] = None
    mods = {}
    for name in ("cache", "mamba_block"):
        path = os.path.join(root, "alloy", "models", name + ".py")
        spec = importlib.util.spec_from_file_location("alloy_ref_" + name, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mods[name] = mod
    assert mods["mamba_block"].USE_METAL_KERNELS is False
    return mods["mamba_block"], mods["cache"]


def load_reference_conv_vjp(root):
    """mamba_block.py loaded with a stand-in for its Metal kernels module, so
    that its try-block (:17-50) defines ``_metal_conv1d_silu_vjp``; only the
    VJP body, which uses elementary MLX ops alone, is executed."""
    mlx_numpy_standin.install()
    kern = types.ModuleType("alloy.models.mamba_kernels")
    for fn in ("fused_conv1d_silu", "scan_chunk_metal", "fused_parallel_scan_chunk"):
        setattr(kern, fn, None)
    saved = sys.modules.get("alloy.models.mamba_kernels", "absent")
    sys.modules["alloy.models.mamba_kernels"] = kern
    try:
        path = os.path.join(root, "alloy", "models", "mamba_block.py")
        spec = importlib.util.spec_from_file_location("alloy_ref_mamba_block_vjp", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        if saved == "absent":
            del sys.modules["alloy.models.mamba_kernels"]
        else:
            sys.modules["alloy.models.mamba_kernels"] = saved
    assert mod.USE_METAL_KERNELS is True
    return mod


class _Proj:
    """Stands in for in_proj: returns the prepared projection for the next call."""

    def __init__(self):
        self.value = None

    def __call__(self, x):
        return self.value


def make_block(mb, H, P, N, G, Q, inp):
    d_inner = H * P
    blk = mb.MambaBlock(d_model=d_inner // 2, d_state=N, d_conv=4, expand=2,
                        headdim=P, chunk_size=Q, combined_proj=True, n_groups=G,
                        use_D=True, use_inner_norm=False)
    blk.conv_weight = inp["conv_weight"]
    blk.conv_bias = inp["conv_bias"]
    blk.dt_bias = inp["dt_bias"]
    blk.A_log = inp["A_log"]
    blk.D = inp["D"]
    blk.in_proj = _Proj()
    blk.out_proj = lambda y: y
    return blk


def run_block(blk, xBC, dt_raw, cache):
    Bsz, L, _ = xBC.shape
    gate = np.full((Bsz, L, blk.d_inner), GATE, np.float32)
    blk.in_proj.value = np.concatenate([gate, xBC, dt_raw], axis=-1).astype(np.float32)
    dummy = np.zeros((Bsz, L, blk.d_model), np.float32)
    out = blk(dummy, cache=cache)
    y = (out / GATE).reshape(Bsz, L, blk.n_heads, blk.headdim)
    return y.astype(np.float32)


def case_prefill(mb, cache_mod, name, B, L, H, P, N, G, Q, dtype="fp32", seed=0,
                 with_state=False):
    inp = make_inputs(B=B, L=L, H=H, P=P, N=N, G=G, dtype=dtype, seed=seed,
                      with_state=with_state)
    blk = make_block(mb, H, P, N, G, Q, inp)
    cache = cache_mod.MambaCache()
    if with_state:
        cache.ssm_state = inp["ssm_state"].copy()
        cache.conv_state = inp["conv_state"].copy()
    y = run_block(blk, inp["xBC"], inp["dt_raw"], cache)
    out = dict(inp)
    out.update(dims=np.array([B, L, H, P, N, G, Q]), y=y,
               ssm_state_out=np.asarray(cache.ssm_state, np.float32),
               conv_state_out=np.asarray(cache.conv_state, np.float32))
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
    print(f"{name}: y {y.shape}, |y|max {np.abs(y).max():.3g}")


def case_decode(mb, cache_mod, name, B, L0, steps, H, P, N, G, Q, seed=0):
    inp = make_inputs(B=B, L=L0 + steps, H=H, P=P, N=N, G=G, seed=seed)
    blk = make_block(mb, H, P, N, G, Q, inp)
    cache = cache_mod.MambaCache()
    y_pre = run_block(blk, inp["xBC"][:, :L0], inp["dt_raw"][:, :L0], cache)
    pre_ssm = np.asarray(cache.ssm_state, np.float32).copy()
    pre_conv = np.asarray(cache.conv_state, np.float32).copy()
    ys = []
    for t in range(L0, L0 + steps):
        ys.append(run_block(blk, inp["xBC"][:, t:t + 1], inp["dt_raw"][:, t:t + 1], cache)[:, 0])
    # the same tokens in one chunked prefill, for the prefill == decode invariant
    cache_full = cache_mod.MambaCache()
    y_full = run_block(blk, inp["xBC"], inp["dt_raw"], cache_full)
    out = dict(inp)
    out.update(dims=np.array([B, L0, steps, H, P, N, G, Q]), y_prefill=y_pre,
               ssm_state_prefill=pre_ssm, conv_state_prefill=pre_conv,
               y_steps=np.stack(ys, axis=1),
               ssm_state_out=np.asarray(cache.ssm_state, np.float32),
               conv_state_out=np.asarray(cache.conv_state, np.float32),
               y_full=y_full,
               ssm_state_full=np.asarray(cache_full.ssm_state, np.float32))
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
    print(f"{name}: steps {steps}")


def case_scan_chunk(mb, name, seed=42):
    """``_scan_chunk`` alone, shapes and value ranges of the reference's
    tests/test_metal_kernels.py:75-89 (B=2, cs=64, H=8, P=64, N=16)."""
    rng = np.random.default_rng(seed)
    B, cs, H, P, N = 2, 64, 8, 64, 16
    x = rng.standard_normal((B, cs, H, P), dtype=np.float32)
    a = (rng.uniform(size=(B, cs, H)) * 0.5 + 0.25).astype(np.float32)
    Bc = (rng.standard_normal((B, cs, H, N)) * 0.1).astype(np.float32)
    Cc = (rng.standard_normal((B, cs, H, N)) * 0.1).astype(np.float32)
    h = (rng.standard_normal((B, H, N, P)) * 0.1).astype(np.float32)
    blk = mb.MambaBlock(d_model=H * P // 2, d_state=N, expand=2, headdim=P, chunk_size=cs)
    y, h_new = blk._scan_chunk(x, a, Bc, Cc, h, cs)
    # the sequential scan on the same inputs (mamba_block.py:160-204)
    y_seq = blk._selective_scan_sequential(x, a, Bc, Cc, None)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), x=x, a=a, B=Bc, C=Cc, h=h,
                        y=np.asarray(y, np.float32), h_new=np.asarray(h_new, np.float32),
                        y_seq_zero_h=np.asarray(y_seq, np.float32))
    print(f"{name}: y {y.shape}")


def case_conv(mb, name, seed=42):
    """``_depthwise_conv1d`` + silu at the shapes of the reference's
    tests/test_metal_kernels.py:18-35 (B=2, L=128, D=256, K=4, w ~ N(0,1)*0.02)."""
    import mlx.nn as nn
    rng = np.random.default_rng(seed)
    B, L, D, K = 2, 128, 256, 4
    xp = rng.standard_normal((B, L + K - 1, D), dtype=np.float32)
    w = (rng.standard_normal((D, K)) * 0.02).astype(np.float32)
    b = np.zeros((D,), np.float32)
    blk = mb.MambaBlock(d_model=D // 2, d_state=16, expand=2, headdim=64)
    blk.conv_weight, blk.conv_bias = w, b
    out = nn.silu(blk._depthwise_conv1d(xp, L))
    np.savez_compressed(os.path.join(HERE, name + ".npz"), x_padded=xp, weight=w, bias=b,
                        out=np.asarray(out, np.float32))
    print(f"{name}: out {out.shape}")


def case_conv_vjp(root, name, seed=43):
    """The reference's own ``_metal_conv1d_silu_vjp`` (mamba_block.py:25-47)
    on the conv shapes of tests/test_metal_kernels.py:18-35 with a non-zero
    bias and a random cotangent."""
    mod = load_reference_conv_vjp(root)
    rng = np.random.default_rng(seed)
    B, L, D, K = 2, 128, 256, 4
    xp = rng.standard_normal((B, L + K - 1, D), dtype=np.float32).view(mlx_numpy_standin.AtArray)
    w = (rng.standard_normal((D, K)) * 0.5).astype(np.float32).view(mlx_numpy_standin.AtArray)
    b = (rng.standard_normal(D) * 0.1).astype(np.float32).view(mlx_numpy_standin.AtArray)
    dy = rng.standard_normal((B, L, D), dtype=np.float32).view(mlx_numpy_standin.AtArray)
    dx, dw, db, _ = mod._metal_conv1d_silu_vjp((xp, w, b, np.array(L)), dy, None)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), x_padded=np.asarray(xp), weight=np.asarray(w),
                        bias=np.asarray(b), dy=np.asarray(dy), dx_padded=np.asarray(dx, np.float32),
                        dweight=np.asarray(dw, np.float32), dbias=np.asarray(db, np.float32))
    print(f"{name}: dx {dx.shape}, dweight {dw.shape}")


HOT_PATH = ("_depthwise_conv1d", "_selective_scan", "_scan_chunk", "_selective_scan_sequential")


def case_bridge_trace(mb, cache_mod, name, seed=6):
    """Every hot-path call the reference's own ``MambaBlock.__call__`` makes,
    recorded with its arguments, its results and the cache's ssm_state before
    and after, in both modes: combined (Zamba2 / Nemotron-H: ``_forward_combined``,
    mamba_block.py:428-501) as a chunked prefill through a cache followed by
    single-token cached steps, and split (``_forward_split``, :385-426) as a
    prefill without a cache, a prefill with one and cached steps.  Nested
    calls (``_scan_chunk`` inside ``_selective_scan``, :340-357, and the L <= 1
    hand-off to ``_selective_scan_sequential``, :322-323) are recorded too.
    A GPU test replays each call through ``alloy_b200.mlx_bridge`` (the
    reference's source does not exist where the GPU tests run)."""
    calls = []
    saved = {n: getattr(mb.MambaBlock, n) for n in HOT_PATH}

    def recorder(nm, fn):
        def rec(self, *args, **kwargs):
            cache = kwargs.get("cache", args[4] if nm in ("_selective_scan", "_selective_scan_sequential")
                               and len(args) > 4 else None)
            h0 = None if cache is None or cache.ssm_state is None else np.array(cache.ssm_state)
            entry = dict(name=nm, args=[None if hasattr(a, "ssm_state") else a for a in args],
                         kwargs={k: v for k, v in kwargs.items() if k != "cache"}, cache=cache is not None,
                         h_before=h0, conv_weight=np.array(self.conv_weight), conv_bias=np.array(self.conv_bias),
                         dims=(self.n_heads, self.headdim, self.d_state, self.chunk_size))
            calls.append(entry)
            out = fn(self, *args, **kwargs)
            entry["out"] = out
            entry["h_after"] = None if cache is None or cache.ssm_state is None else np.array(cache.ssm_state)
            return out
        return rec

    for n_, f in saved.items():
        setattr(mb.MambaBlock, n_, recorder(n_, f))
    try:
        # combined mode: chunked prefill of 40 tokens (chunk 16, ragged last
        # chunk) with a cache, then 3 cached single-token steps
        H, P, N, G, Q = 4, 16, 8, 2, 16
        inp = make_inputs(B=2, L=43, H=H, P=P, N=N, G=G, seed=seed)
        blk = make_block(mb, H, P, N, G, Q, inp)
        cache = cache_mod.MambaCache()
        run_block(blk, inp["xBC"][:, :40], inp["dt_raw"][:, :40], cache)
        for t in range(40, 43):
            run_block(blk, inp["xBC"][:, t:t + 1], inp["dt_raw"][:, t:t + 1], cache)
        # split mode: in_proj returns a prepared [x | z], x_proj a fixed linear map
        d_model, Hs, Ps, Ns = 32, 4, 16, 8
        rng = np.random.default_rng(seed + 1)
        sblk = mb.MambaBlock(d_model=d_model, d_state=Ns, d_conv=4, expand=2, headdim=Ps, chunk_size=8)
        sblk.conv_weight = (rng.standard_normal((2 * d_model, 4)) * 0.5).astype(np.float32)
        sblk.conv_bias = (rng.standard_normal(2 * d_model) * 0.1).astype(np.float32)
        sblk.dt_bias = np.log(np.expm1(np.exp(rng.uniform(np.log(1e-3), np.log(0.1), Hs)))).astype(np.float32)
        sblk.A_log = rng.uniform(0, np.log(16), Hs).astype(np.float32)
        W = (rng.standard_normal((2 * d_model, Hs * (2 * Ns + 1))) * 0.2).astype(np.float32)
        sblk.x_proj = lambda v: v @ W
        sblk.in_proj = _Proj()
        sblk.out_proj = lambda y: y

        def run_split(L, cache):
            sblk.in_proj.value = rng.standard_normal((2, L, 4 * d_model)).astype(np.float32)
            return sblk(np.zeros((2, L, d_model), np.float32), cache=cache)

        run_split(20, None)
        scache = cache_mod.MambaCache()
        run_split(20, scache)
        for _ in range(2):
            run_split(1, scache)
    finally:
        for n_, f in saved.items():
            setattr(mb.MambaBlock, n_, f)

    # flatten into npz entries: c{i}_name, c{i}_a{k} (array arguments, k-th
    # positional), c{i}_L / c{i}_cs / c{i}_log_a, c{i}_out{k}, c{i}_h_before / _after
    out = {"n_calls": np.array(len(calls))}
    for i, c in enumerate(calls):
        out[f"c{i}_name"] = np.array(c["name"])
        out[f"c{i}_dims"] = np.array(c["dims"])
        out[f"c{i}_conv_weight"] = c["conv_weight"]
        out[f"c{i}_conv_bias"] = c["conv_bias"]
        out[f"c{i}_cache"] = np.array(c["cache"])
        for k, a in enumerate(c["args"]):
            if isinstance(a, np.ndarray):
                out[f"c{i}_a{k}"] = a
            elif isinstance(a, (int, np.integer)):
                out[f"c{i}_i{k}"] = np.array(int(a))
        if c["kwargs"].get("log_a") is not None:
            out[f"c{i}_log_a"] = c["kwargs"]["log_a"]
        if c["kwargs"].get("log_a_direct") is not None:
            out[f"c{i}_log_a"] = c["kwargs"]["log_a_direct"]
        res = c["out"] if isinstance(c["out"], tuple) else (c["out"],)
        for k, r in enumerate(res):
            out[f"c{i}_out{k}"] = np.asarray(r, np.float32)
        if c["h_before"] is not None:
            out[f"c{i}_h_before"] = c["h_before"].astype(np.float32)
        if c["h_after"] is not None:
            out[f"c{i}_h_after"] = c["h_after"].astype(np.float32)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
    print(f"{name}: {len(calls)} calls: " + ", ".join(sorted({c['name'] for c in calls})))


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    mb, cache_mod = load_reference(root)
    case_conv(mb, "conv1d_silu")
    case_conv_vjp(root, "conv1d_silu_vjp")
    case_scan_chunk(mb, "scan_chunk")
    # the toy fp32 mixer configuration, full size
    case_prefill(mb, cache_mod, "toy_prefill", B=2, L=512, H=8, P=32, N=16, G=1, Q=64)
    # ngroups > 1, L not a multiple of the chunk, carried ssm/conv state
    case_prefill(mb, cache_mod, "groups_ragged_state", B=1, L=100, H=4, P=16, N=8, G=2,
                 Q=32, seed=1, with_state=True)
    # L = 2 < K - 1: the new conv state mixes old state rows and new inputs
    case_prefill(mb, cache_mod, "short_state", B=2, L=2, H=4, P=16, N=8, G=2, Q=32,
                 seed=2, with_state=True)
    # bf16-rounded inputs at the tensor-core kernel's head/state sizes
    case_prefill(mb, cache_mod, "bf16_p64_n64", B=1, L=300, H=8, P=64, N=64, G=1, Q=128,
                 dtype="bf16", seed=3)
    case_prefill(mb, cache_mod, "bf16_p64_n128_g2", B=2, L=260, H=4, P=64, N=128, G=2,
                 Q=128, dtype="bf16", seed=4, with_state=True)
    # chunked prefill, then single-token decode steps through the cache
    case_decode(mb, cache_mod, "decode_steps", B=2, L0=40, steps=8, H=4, P=16, N=8, G=2,
                Q=16, seed=5)
    # the hot-path calls of the reference's MambaBlock, for the bridge's GPU test
    case_bridge_trace(mb, cache_mod, "bridge_trace", seed=6)


if __name__ == "__main__":
    main()
