"""The reference's own MambaBlock calls, routed through the MLX bridge to the GPU.

``tests/golden/bridge_trace.npz`` holds every hot-path call that alloy's
``MambaBlock.__call__`` made when ``tests/golden/make_golden.py`` drove the
reference's unmodified ``alloy/models/mamba_block.py`` (numpy MLX stand-in)
in combined mode (chunked prefill through a cache, then cached single-token
steps) and split mode (prefill without a cache, with one, cached steps):
``_depthwise_conv1d`` (mamba_block.py:144), ``_selective_scan`` (:287, with
its ``log_a`` keyword), the ``_scan_chunk`` calls it makes per chunk (:206)
and the ``_selective_scan_sequential`` hand-off for L <= 1 (:160, :322-323),
with their exact arguments, results and the cache's ssm_state before and
after.  This test installs the same numpy stand-in as ``mlx`` (MLX itself
does not exist on CUDA machines), patches a class with the reference's four
method names through ``mlx_bridge.patch_mamba_block`` and replays each call:
MLX-typed arguments in, the CUDA kernels, MLX-typed results and the cache
update out, compared with what the reference computed (fp32, rel-L2 <= 1e-4).
"""

import os
import sys
import types

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, TOL_F32_REL_L2, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bridged():
    sys.path.insert(0, GOLDEN)
    import mlx_numpy_standin
    saved = {k: sys.modules.get(k) for k in ("mlx", "mlx.core", "mlx.nn")}
    mlx_numpy_standin.install()
    from alloy_b200 import mlx_bridge

    class RefMethods:
        """Carries the four hot-path method names of alloy's MambaBlock."""
        def _depthwise_conv1d(self, x_padded, L):
            raise AssertionError("not patched")

        def _scan_chunk(self, x_c, a_c, B_c, C_c, h, cs, log_a_direct=None):
            raise AssertionError("not patched")

        def _selective_scan(self, x, A_disc, B, C, cache=None, log_a=None):
            raise AssertionError("not patched")

        def _selective_scan_sequential(self, x, A_disc, B, C, cache=None):
            raise AssertionError("not patched")

    mlx_bridge.patch_mamba_block(RefMethods, device="cuda")
    yield RefMethods
    for k, v in saved.items():
        if v is None:
            sys.modules.pop(k, None)
        else:
            sys.modules[k] = v


def _close(got, ref, what):
    got = np.asarray(got, np.float32)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    r = oracle.rel_l2(got, ref)
    assert r <= TOL_F32_REL_L2, (what, r)
    return r


def test_reference_block_calls_through_the_bridge(bridged):
    g = load_golden("bridge_trace")
    n = int(g["n_calls"])
    seen = {}
    for i in range(n):
        name = str(g[f"c{i}_name"])
        H, P, N, cs = (int(v) for v in g[f"c{i}_dims"])
        blk = bridged()
        blk.conv_weight, blk.conv_bias = g[f"c{i}_conv_weight"], g[f"c{i}_conv_bias"]
        blk.n_heads, blk.headdim, blk.d_state, blk.chunk_size = H, P, N, cs
        args = []
        cache = None
        for k in range(6):
            if f"c{i}_a{k}" in g:
                args.append(g[f"c{i}_a{k}"])
            elif f"c{i}_i{k}" in g:
                args.append(int(g[f"c{i}_i{k}"]))
            elif k == 4 and name in ("_selective_scan", "_selective_scan_sequential") and bool(g[f"c{i}_cache"]):
                cache = types.SimpleNamespace(
                    ssm_state=g[f"c{i}_h_before"] if f"c{i}_h_before" in g else None, conv_state=None)
                args.append(cache)
            else:
                break
        kwargs = {}
        if f"c{i}_log_a" in g:
            kwargs["log_a_direct" if name == "_scan_chunk" else "log_a"] = g[f"c{i}_log_a"]
        out = getattr(blk, name)(*args, **kwargs)
        outs = out if isinstance(out, tuple) else (out,)
        for k, o in enumerate(outs):
            _close(o, g[f"c{i}_out{k}"], f"call {i} {name} output {k}")
        if cache is not None and f"c{i}_h_after" in g:
            _close(cache.ssm_state, g[f"c{i}_h_after"], f"call {i} {name} cache.ssm_state")
        seen[name] = seen.get(name, 0) + 1
    # every hot-path method the reference routes through was exercised
    assert set(seen) == {"_depthwise_conv1d", "_selective_scan", "_scan_chunk", "_selective_scan_sequential"}, seen
    print("replayed", n, "reference calls:", seen)
