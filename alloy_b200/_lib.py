"""ctypes binding of liballoy_ssd.so (the C ABI in include/alloy_ssd.h).

The library is loaded from the package directory.  There is no fallback: if
the shared library is missing or was built for another ABI version, every
call raises :class:`AlloyLibraryError`.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liballoy_ssd.so")

ABI_VERSION = 1
MAX_DIMS = 5

F32 = 0
BF16 = 1

STATUS = {
    0: "ok",
    -1: "invalid argument",
    -2: "unsupported",
    -3: "alignment",
    -4: "cuda error",
    -5: "no usable device",
    -6: "device wait timed out",
}

# every entry point include/alloy_ssd.h declares
EXPORTS = (
    "alloy_abi_version",
    "alloy_build_info",
    "alloy_get_last_error",
    "alloy_conv1d_silu",
    "alloy_depthwise_conv1d",
    "alloy_ssd_combined",
    "alloy_selective_scan",
    "alloy_selective_scan_dot",
    "alloy_ssd_decode_step",
    "alloy_ssd_combined_workspace_size",
    "alloy_ssd_combined_min_workspace_size",
    "alloy_check_device_status",
    "alloy_ssd_combined_noalloc",
    "alloy_kernel_launch_count",
    "alloy_gated_rmsnorm",
    "alloy_conv1d_silu_backward",
    "alloy_conv1d_silu_backward_workspace_size",
    "alloy_decode_linear",
    "alloy_linear",
    "alloy_debug_set_wait_stall",
)


class AlloyLibraryError(RuntimeError):
    """liballoy_ssd.so could not be loaded."""


class AlloyError(RuntimeError):
    """A liballoy_ssd call returned a negative status."""

    def __init__(self, fn, status, message):
        self.status = status
        self.message = message
        super().__init__(f"{fn}: {STATUS.get(status, status)}: {message}")


class Tensor(ctypes.Structure):
    """alloy_tensor_t."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("stride", ctypes.c_int64 * MAX_DIMS),
    ]


class Dims(ctypes.Structure):
    """alloy_ssd_dims_t."""

    _fields_ = [(n, ctypes.c_int64) for n in (
        "n_heads", "head_dim", "d_state", "n_groups", "d_conv", "chunk_size",
        "head_begin", "head_count")]


_lock = threading.Lock()
_lib = None


def load():
    """Load (once) and return the ctypes handle of liballoy_ssd.so."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise AlloyLibraryError(
                f"{LIB_PATH} is missing; build it with `python -m alloy_b200.build`")
        try:
            lib = ctypes.CDLL(LIB_PATH)
        except OSError as e:  # pragma: no cover - broken build
            raise AlloyLibraryError(f"cannot load {LIB_PATH}: {e}") from e
        for name in EXPORTS:
            if not hasattr(lib, name):
                raise AlloyLibraryError(f"{LIB_PATH} does not export {name}")
        lib.alloy_abi_version.restype = ctypes.c_int
        lib.alloy_build_info.restype = ctypes.c_char_p
        lib.alloy_get_last_error.restype = ctypes.c_size_t
        lib.alloy_get_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
        P = ctypes.POINTER(Tensor)
        D = ctypes.POINTER(Dims)
        vp = ctypes.c_void_p
        lib.alloy_conv1d_silu.argtypes = [P, P, P, P, vp]
        lib.alloy_depthwise_conv1d.argtypes = [P, P, P, P, vp]
        lib.alloy_conv1d_silu_backward.argtypes = [P] * 7 + [vp, ctypes.c_size_t, vp]
        lib.alloy_conv1d_silu_backward_workspace_size.argtypes = [ctypes.c_int64] * 4
        lib.alloy_conv1d_silu_backward_workspace_size.restype = ctypes.c_size_t
        lib.alloy_decode_linear.argtypes = [P, P, P, vp]
        lib.alloy_decode_linear.restype = ctypes.c_int
        lib.alloy_linear.argtypes = [P, P, P, P, vp]
        lib.alloy_linear.restype = ctypes.c_int
        lib.alloy_ssd_combined.argtypes = [P] * 12 + [vp, ctypes.c_size_t, D, vp]
        lib.alloy_ssd_combined_workspace_size.argtypes = [ctypes.c_int64, ctypes.c_int64,
                                                          ctypes.c_int32, D]
        lib.alloy_ssd_combined_workspace_size.restype = ctypes.c_size_t
        lib.alloy_ssd_combined_min_workspace_size.argtypes = [ctypes.c_int64, ctypes.c_int64,
                                                          ctypes.c_int32, D]
        lib.alloy_ssd_combined_min_workspace_size.restype = ctypes.c_size_t
        lib.alloy_check_device_status.argtypes = [vp]
        lib.alloy_debug_set_wait_stall.argtypes = [ctypes.c_int64]
        lib.alloy_debug_set_wait_stall.restype = ctypes.c_int
        lib.alloy_gated_rmsnorm.argtypes = [P, P, P, P, ctypes.c_float, ctypes.c_int64, vp]
        lib.alloy_gated_rmsnorm.restype = ctypes.c_int
        lib.alloy_kernel_launch_count.argtypes = []
        lib.alloy_kernel_launch_count.restype = ctypes.c_uint64
        lib.alloy_ssd_combined_noalloc.argtypes = [P] * 12 + [D, vp]
        lib.alloy_selective_scan.argtypes = [P] * 8 + [vp]
        lib.alloy_selective_scan_dot.argtypes = [P] * 9 + [ctypes.c_int32, vp]
        lib.alloy_ssd_decode_step.argtypes = [P] * 10 + [D, vp]
        for name in ("alloy_conv1d_silu", "alloy_depthwise_conv1d", "alloy_conv1d_silu_backward",
                     "alloy_ssd_combined",
                     "alloy_selective_scan", "alloy_selective_scan_dot", "alloy_ssd_decode_step",
                     "alloy_check_device_status",
                     "alloy_ssd_combined_noalloc"):
            getattr(lib, name).restype = ctypes.c_int
        if lib.alloy_abi_version() != ABI_VERSION:
            raise AlloyLibraryError(
                f"{LIB_PATH} has ABI {lib.alloy_abi_version()}, expected {ABI_VERSION}")
        _lib = lib
        return lib


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(1024)
    lib.alloy_get_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def call(name, *args):
    """Call an entry point; raise AlloyError on a negative status."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != 0:
        raise AlloyError(name, status, last_error())
    return status


_DTYPES = {torch.float32: F32, torch.bfloat16: BF16}


def desc(t: torch.Tensor | None, name: str = "tensor") -> Tensor:
    """alloy_tensor_t describing a torch tensor (None -> an absent tensor)."""
    d = Tensor()
    if t is None:
        return d
    if t.dtype not in _DTYPES:
        raise TypeError(f"{name}: dtype {t.dtype} is not supported (float32 or bfloat16)")
    if t.dim() > MAX_DIMS:
        raise ValueError(f"{name}: at most {MAX_DIMS} dims")
    # empty tensors still need a non-null pointer to be "present" (nothing
    # dereferences it: every extent that indexes it is zero)
    d.data = t.data_ptr() if t.numel() > 0 else 16
    d.dtype = _DTYPES[t.dtype]
    d.ndim = t.dim()
    for i, (s, st) in enumerate(zip(t.shape, t.stride())):
        d.shape[i] = s
        d.stride[i] = st
    return d


def ref(d: Tensor):
    return ctypes.byref(d)


def stream_handle(device: torch.device | None = None) -> ctypes.c_void_p:
    """The raw cudaStream_t of torch's current stream on ``device``."""
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
