"""The C ABI without a GPU: the library loads, exports every entry point the
header declares, and rejects bad arguments on the host before touching a
device."""

import ctypes
import os
import re

import pytest

from alloy_b200 import _lib
from conftest import REPO

HEADER = os.path.join(REPO, "include", "alloy_ssd.h")


def header_entry_points():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"ALLOY_API\s+[\w\s\*]+?\b(alloy_\w+)\s*\(", text)))


def test_header_declares_the_python_export_list():
    assert header_entry_points() == sorted(_lib.EXPORTS)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    for name in header_entry_points():
        assert hasattr(lib, name), name
    assert lib.alloy_abi_version() == _lib.ABI_VERSION
    assert b"sm_100a" in lib.alloy_build_info()


def _t(shape, dtype=_lib.F32, ptr=0x1000, strides=None):
    d = _lib.Tensor()
    d.data = ptr
    d.dtype = dtype
    d.ndim = len(shape)
    if strides is None:
        strides, acc = [], 1
        for s in reversed(shape):
            strides.insert(0, acc)
            acc *= s
    for i, (s, st) in enumerate(zip(shape, strides)):
        d.shape[i] = s
        d.stride[i] = st
    return d


def _dims(H=8, P=32, N=16, G=1, K=4, Q=64, h0=0, hc=0):
    d = _lib.Dims()
    d.n_heads, d.head_dim, d.d_state, d.n_groups, d.d_conv, d.chunk_size = H, P, N, G, K, Q
    d.head_begin, d.head_count = h0, hc
    return d


def _combined(**over):
    B, L, H, P, N, G, K = 2, 16, 8, 32, 16, 1, 4
    C = H * P + 2 * G * N
    t = dict(xBC=_t([B, L, C]), dt=_t([B, L, H]), w=_t([C, K]), b=_t([C]), dtb=_t([H]),
             alog=_t([H]), D=_t([H]), si=_lib.Tensor(), ci=_lib.Tensor(),
             y=_t([B, L, H, P]), so=_lib.Tensor(), co=_lib.Tensor())
    dims = over.pop("dims", _dims(H, P, N, G, K))
    t.update(over)
    lib = _lib.load()
    order = ["xBC", "dt", "w", "b", "dtb", "alog", "D", "si", "ci", "y", "so", "co"]
    st = lib.alloy_ssd_combined(*(ctypes.byref(t[k]) for k in order), None, 0,
                                ctypes.byref(dims), None)
    return st, _lib.last_error()


@pytest.mark.parametrize("over,needle", [
    (dict(xBC=_lib.Tensor()), "xBC: null"),
    (dict(xBC=_t([2, 16, 300])), "expected H*P + 2*G*N"),
    (dict(dt=_t([2, 15, 8])), "dt_raw: dim 1"),
    (dict(w=_t([288, 4], dtype=_lib.BF16)), "conv_w: unsupported dtype"),
    (dict(y=_t([2, 16, 8, 32], dtype=_lib.BF16)), "y: unsupported dtype"),
    (dict(dims=_dims(H=8, G=3)), "not divisible"),
    (dict(dims=_dims(h0=6, hc=4)), "head range"),
    (dict(dims=_dims(K=9)), "d_conv"),
    (dict(so=_t([2, 8, 16, 31])), "ssm_out: dim 3"),
    (dict(xBC=_t([2, 16, 288], strides=[16 * 288 * 2, 288 * 2, 2])), "channel stride"),
])
def test_combined_rejects_bad_arguments(over, needle):
    st, msg = _combined(**over)
    assert st in (-1, -2), (st, msg)
    assert needle in msg, msg


def test_conv_rejects_bad_arguments():
    lib = _lib.load()
    x, w, out = _t([2, 19, 64]), _t([64, 4]), _t([2, 15, 64])
    st = lib.alloy_conv1d_silu(ctypes.byref(x), ctypes.byref(w), None, ctypes.byref(out), None)
    assert st == -1 and "out: dim 1" in _lib.last_error()
    w9 = _t([64, 9])
    st = lib.alloy_depthwise_conv1d(ctypes.byref(x), ctypes.byref(w9), None, ctypes.byref(out), None)
    assert st == -2 and "K must be" in _lib.last_error()


def test_decode_rejects_bad_state_layout():
    lib = _lib.load()
    B, H, P, N, G, K = 2, 8, 32, 16, 1, 4
    C = H * P + 2 * G * N
    st_bad = _t([B, H, N, P], strides=[H * N * P * 2, N * P * 2, 2 * P, 2])
    args = [_t([B, C]), _t([B, H]), _t([C, K]), _lib.Tensor(), _t([H]), _t([H]),
            _lib.Tensor(), _t([B, K - 1, C]), st_bad, _t([B, H, P])]
    st = lib.alloy_ssd_decode_step(*(ctypes.byref(a) for a in args),
                                   ctypes.byref(_dims(H, P, N, G, K)), None)
    assert st == -1 and "ssm_state" in _lib.last_error()


def test_selective_scan_rejects_group_mismatch():
    lib = _lib.load()
    B, L, H, P, N = 1, 8, 6, 16, 8
    args = [_t([B, L, H, P]), _t([B, L, H]), _lib.Tensor(), _t([B, L, 4, N]),
            _t([B, L, 4, N]), _lib.Tensor(), _t([B, L, H, P]), _lib.Tensor()]
    st = lib.alloy_selective_scan(*(ctypes.byref(a) for a in args), None)
    assert st == -1 and "does not divide" in _lib.last_error()


def _scan_dot(**over):
    B, L, H, P, N = 2, 16, 8, 64, 64
    BF = _lib.BF16
    t = dict(x=_t([B, L, 2, P], BF), la=_t([B, L, H]), Bm=_t([B, L, 1, N], BF), Cm=_t([B, L, 1, N], BF),
             si=_lib.Tensor(), y=_t([B, L, H, P]), so=_lib.Tensor(), z=_t([B, L, H, P], BF),
             dot=_t([B, L, H]))
    t.update({k: v for k, v in over.items() if k != "mode"})
    lib = _lib.load()
    order = ["x", "la", "Bm", "Cm", "si", "y", "so", "z", "dot"]
    st = lib.alloy_selective_scan_dot(*(ctypes.byref(t[k]) for k in order), over.get("mode", 0), None)
    return st, _lib.last_error()


@pytest.mark.parametrize("over,needle", [
    (dict(y=_lib.Tensor(), dot=_lib.Tensor()), "neither y nor dot"),
    (dict(x=_t([2, 16, 2, 64])), "x: unsupported dtype"),
    (dict(x=_t([2, 16, 3, 64], _lib.BF16)), "x: dim 2 (3) does not divide"),
    (dict(la=_lib.Tensor()), "log_a: null"),
    (dict(Bm=_t([2, 16, 1, 64])), "B: unsupported dtype"),
    (dict(z=_lib.Tensor()), "z: null"),
    (dict(z=_t([2, 16, 8, 64], _lib.BF16, strides=[16 * 8 * 128, 8 * 128, 128, 2])), "z: head_dim stride"),
    (dict(dot=_t([2, 16, 4])), "dot: dim 2"),
    (dict(mode=4), "dot_mode"),
    (dict(mode=3), "exclusive"),
])
def test_selective_scan_dot_rejects_bad_arguments(over, needle):
    st, msg = _scan_dot(**over)
    assert st == -1, (st, msg)
    assert needle in msg, msg


def _linear(**over):
    BF = _lib.BF16
    t = dict(x=_t([300, 64], BF), w=_t([136, 64], BF), b=_lib.Tensor(), y=_t([300, 136], BF))
    t.update(over)
    lib = _lib.load()
    st = lib.alloy_linear(*(ctypes.byref(t[k]) for k in ("x", "w", "b", "y")), None)
    return st, _lib.last_error()


@pytest.mark.parametrize("over,needle,status", [
    (dict(x=_t([300, 64])), "x: unsupported dtype", -1),
    (dict(w=_t([136, 72], _lib.BF16)), "weight: dim 1 is 72", -1),
    (dict(y=_t([300, 128], _lib.BF16)), "y: dim 1 is 128", -1),
    (dict(b=_t([128], _lib.BF16)), "bias: dim 0 is 128", -1),
    (dict(x=_t([300, 64], _lib.BF16, strides=[64, 2])), "last dimension must be contiguous", -1),
    (dict(x=_t([300, 60], _lib.BF16), w=_t([136, 60], _lib.BF16)), "multiples of 8", -3),
    (dict(w=_t([132, 64], _lib.BF16), y=_t([300, 132], _lib.BF16)), "multiples of 8", -3),
    (dict(x=_t([300, 64], _lib.BF16, strides=[68, 1])), "multiples of 8", -3),
    (dict(x=_t([300, 64], _lib.BF16, ptr=0x1008)), "16-byte aligned", -3),
    (dict(x=_t([300, 0], _lib.BF16), w=_t([136, 0], _lib.BF16)), "K = 0", -2),
])
def test_linear_rejects_bad_arguments(over, needle, status):
    st, msg = _linear(**over)
    assert st == status, (st, msg)
    assert needle in msg, msg


def test_error_message_is_per_thread():
    import threading
    _combined(xBC=_lib.Tensor())
    seen = {}

    def other():
        seen["msg"] = _lib.last_error()

    th = threading.Thread(target=other)
    th.start()
    th.join()
    assert seen["msg"] == ""
    assert "xBC" in _lib.last_error()
