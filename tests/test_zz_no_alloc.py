"""alloy_ssd_combined_noalloc, the prefill entry point for callers that may not
allocate device memory (a process whose device memory all belongs to its own
pool, or an FFI caller holding only raw pointers from another framework).
It takes its scratch from a fixed 8 MiB array inside the library instead of a
caller workspace.  This file is collected last so that a run stopping at the
first failure has run every other test already; it also passes on its own in
a fresh process, where its first call sets up the array's device address."""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from alloy_b200 import _lib, mixer
from conftest import TOL_BF16_MAX_REL, TOL_BF16_REL_L2

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


# one walk per (batch row, head pair); and a long sequence over few head pairs,
# whose full workspace (B/C tiles and segment records) fits the 8 MiB array,
# so the call runs the segmented schedule with its records there too
CASES = {"unsegmented": dict(B=2, L=300, H=4, P=64, N=128, G=2),
         "segmented": dict(B=1, L=2048, H=4, P=64, N=64, G=2)}


def _inputs(seed, cfg):
    inp = oracle.make_inputs(**cfg, dtype="bf16", seed=seed, with_state=True)

    def cu(a, dt=torch.float32):
        return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dt)

    t = dict(xBC=cu(inp["xBC"], torch.bfloat16), dt_raw=cu(inp["dt_raw"], torch.bfloat16),
             conv_w=cu(inp["conv_weight"]), conv_b=cu(inp["conv_bias"]), dt_bias=cu(inp["dt_bias"]),
             A_log=cu(inp["A_log"]), D=cu(inp["D"]), ssm=cu(inp["ssm_state"]),
             conv=cu(inp["conv_state"], torch.bfloat16))
    return t


def _noalloc(cfg, t):
    B, L, H, P, N, G = (cfg[k] for k in ("B", "L", "H", "P", "N", "G"))
    y = torch.empty((B, L, H, P), dtype=torch.bfloat16, device=DEV)
    h = torch.empty((B, H, N, P), dtype=torch.float32, device=DEV)
    cs = torch.empty_like(t["conv"])
    dims = mixer._dims(H, P, N, G, 4, 256, 0, 0)
    args = [t["xBC"], t["dt_raw"], t["conv_w"], t["conv_b"], t["dt_bias"], t["A_log"], t["D"],
            t["ssm"], t["conv"], y, h, cs]
    descs = [_lib.desc(a) for a in args]
    _lib.call("alloy_ssd_combined_noalloc", *(_lib.ref(d) for d in descs), _lib.ref(dims),
              _lib.stream_handle(torch.device(DEV)))
    return y, h, cs


def _close(got, ref):
    got, ref = got.float().cpu().numpy(), ref.float().cpu().numpy()
    assert oracle.rel_l2(got, ref) <= TOL_BF16_REL_L2
    assert oracle.max_rel(got, ref) <= TOL_BF16_MAX_REL


@pytest.mark.parametrize("case", sorted(CASES))
def test_noalloc_matches_the_workspace_entry_point_on_two_calls(case):
    torch.cuda.set_device(0)
    cfg = CASES[case]
    d = mixer._dims(cfg["H"], cfg["P"], cfg["N"], cfg["G"], 4, 256, 0, 0)
    lib = _lib.load()
    full = lib.alloy_ssd_combined_workspace_size(cfg["B"], cfg["L"], _lib.BF16, _lib.ref(d))
    small = lib.alloy_ssd_combined_min_workspace_size(cfg["B"], cfg["L"], _lib.BF16, _lib.ref(d))
    if case == "segmented":
        assert small < full <= 8 << 20
    for seed in (31, 32):   # two calls in a row on the shared scratch array
        t = _inputs(seed, cfg)
        y_ref, h_ref, cs_ref = mixer.ssd_combined(
            t["xBC"], t["dt_raw"], t["conv_w"], t["conv_b"], t["dt_bias"], t["A_log"], t["D"],
            n_heads=cfg["H"], head_dim=cfg["P"], d_state=cfg["N"], n_groups=cfg["G"],
            ssm_state=t["ssm"], conv_state=t["conv"])
        y, h, cs = _noalloc(cfg, t)
        torch.cuda.synchronize()
        mixer.check_device_status()
        _close(y, y_ref)
        _close(h, h_ref)
        assert torch.equal(cs, cs_ref)


def test_noalloc_rejects_calls_beyond_the_fixed_scratch():
    # a Nemotron-H-sized layer needs ~134 MB of scratch: rejected before any launch
    B, L, H, P, N, G = 8, 4096, 128, 64, 128, 8
    C = H * P + 2 * G * N

    def fake(shape, dtype=_lib.BF16):
        d = _lib.Tensor()
        d.data, d.dtype, d.ndim = 0x1000, dtype, len(shape)
        acc = 1
        for i in reversed(range(len(shape))):
            d.shape[i], d.stride[i] = shape[i], acc
            acc *= shape[i]
        return d

    descs = [fake([B, L, C]), fake([B, L, H]), fake([C, 4], _lib.F32), _lib.Tensor(),
             fake([H], _lib.F32), fake([H], _lib.F32), _lib.Tensor(), _lib.Tensor(),
             _lib.Tensor(), fake([B, L, H, P]), _lib.Tensor(), _lib.Tensor()]
    dims = mixer._dims(H, P, N, G, 4, 256, 0, 0)
    st = _lib.load().alloy_ssd_combined_noalloc(*(ctypes.byref(d) for d in descs),
                                                ctypes.byref(dims), None)
    assert st == -2
    assert "fixed scratch holds" in _lib.last_error()
