"""ctypes binding of the C ABI in include/momentum_scan_b200.h.

The shared library is built in-tree (``python -m momentummamba_b200.build``) and
loaded once per process.  There is no fallback: if the library is missing or a
tensor is not on a CUDA device the call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import build as _build

_c_i64 = ctypes.c_int64
_c_f = ctypes.c_float
_c_i32 = ctypes.c_int32
_c_p = ctypes.c_void_p
_c_size = ctypes.c_size_t

_lock = threading.Lock()
_lib = None


class MMScanDesc(ctypes.Structure):
    """mirror of struct mmb_mmscan_desc"""
    _fields_ = [
        ("batch", _c_i64), ("seqlen", _c_i64), ("dim", _c_i64), ("dstate", _c_i64),
        ("x_stride", _c_i64 * 2), ("delta_stride", _c_i64 * 2), ("z_stride", _c_i64 * 2),
        ("B_stride", _c_i64 * 2), ("C_stride", _c_i64 * 2),
        ("beta", _c_f), ("alpha", _c_f), ("delta_softplus", _c_i32), ("dtype", _c_i32),
        ("time_chunk", _c_i32), ("reserved", _c_i32),
    ]


MMB_F32, MMB_BF16 = 0, 1


class MMScanTensors(ctypes.Structure):
    """mirror of struct mmb_mmscan_tensors (device pointers; None = NULL)"""
    _fields_ = [(name, _c_p) for name in (
        "x", "delta", "z", "B", "C", "A", "D", "delta_bias", "state_in", "gstate_in", "dout",
        "out", "state_out", "ckpt", "dx", "ddelta", "dz", "dA", "dB", "dC", "dD",
        "ddelta_bias", "gstate_out")]


class StepDesc(ctypes.Structure):
    """mirror of struct mmb_step_desc"""
    _fields_ = [
        ("batch", _c_i64), ("dim", _c_i64), ("dstate", _c_i64),
        ("x_row_stride", _c_i64), ("delta_row_stride", _c_i64), ("z_row_stride", _c_i64),
        ("B_row_stride", _c_i64), ("C_row_stride", _c_i64), ("state_stride", _c_i64 * 2),
        ("beta", _c_f), ("alpha", _c_f), ("delta_softplus", _c_i32), ("reserved", _c_i32),
    ]


_DESC_P = ctypes.POINTER(MMScanDesc)
_TENS_P = ctypes.POINTER(MMScanTensors)
_I64_P = ctypes.POINTER(_c_i64)


# name -> (restype, argtypes)
_SIGNATURES = {
    "mmb_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "mmb_abi_version": (ctypes.c_int, []),
    "mmb_last_error": (ctypes.c_char_p, []),
    "mmb_device_status": (ctypes.c_int, [_c_p]),
    "mmb_selftest_device_wait": (ctypes.c_int, [_c_i32, _c_p]),
    "mmb_mmscan_ckpt_floats": (_c_size, [_c_i64, _c_i64, _c_i64, _c_i64]),
    "mmb_mmscan_workspace_floats": (_c_size, [_DESC_P]),
    "mmb_mmscan_fwd": (ctypes.c_int, [ctypes.POINTER(MMScanDesc)] + [_c_p] * 10 + [_c_p]),
    "mmb_mmscan_bwd": (ctypes.c_int, [ctypes.POINTER(MMScanDesc)] + [_c_p] * 18 + [_c_p]),
    "mmb_mmscan_forward": (ctypes.c_int, [_DESC_P, _TENS_P, _c_p]),
    "mmb_mmscan_backward": (ctypes.c_int, [_DESC_P, _TENS_P, _c_p]),
    "mmb_mmscan_fwd_summary": (ctypes.c_int, [_DESC_P, _TENS_P, _c_p, _c_p]),
    "mmb_mmscan_bwd_summary": (ctypes.c_int, [_DESC_P, _TENS_P, _c_p, _c_p]),
    "mmb_mmscan_carry_fwd": (ctypes.c_int, [_c_i64, _c_i64, _I64_P, _c_i64, _c_i64, _c_i64, _c_f,
                                            _c_p, _c_p, _c_p]),
    "mmb_mmscan_carry_bwd": (ctypes.c_int, [_c_i64, _c_i64, _I64_P, _c_i64, _c_i64, _c_i64, _c_f,
                                            _c_p, _c_p, _c_p, _c_p]),
    "mmb_conv1d_silu_fwd": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_i32, _c_p, _I64_P]
                            + [_c_p] * 6),
    "mmb_conv1d_silu_bwd": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_i32, _c_p, _I64_P]
                            + [_c_p] * 8),
    "mmb_conv1d_step": (ctypes.c_int, [_c_i64, _c_i64, _c_i32, _c_p, _c_i64] + [_c_p] * 6),
    "mmb_mmscan_step": (ctypes.c_int, [ctypes.POINTER(StepDesc)] + [_c_p] * 14),
    "mmb_linoss_sel_work_floats": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "mmb_linoss_sel_fwd": (ctypes.c_int, [_c_i32, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p,
                                          _I64_P, _c_p, _c_p, _I64_P, _c_p, _c_p, _c_p]),
    "mmb_linoss_sel_bwd": (ctypes.c_int, [_c_i32, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p,
                                          _I64_P, _c_p, _c_p, _I64_P] + [_c_p] * 9),
    "mmb_rows_fwd": (ctypes.c_int, [_c_i64, _c_i64, _c_p, _c_f, _c_p, _c_p, _c_p, _c_p]),
    "mmb_rows_bwd": (ctypes.c_int, [_c_i64, _c_i64, _c_p, _c_p, _c_f, _c_p, _c_p, _c_p, _c_p]),
    "mmb_pscan_fwd": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p]),
    "mmb_pscan_bwd": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p]),
    "mmb_scan2_work_floats": (_c_size, [_c_i64, _c_i64, _c_i64, _c_i32]),
    "mmb_scan2_fwd": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_i32] + [_c_p] * 6),
    "mmb_scan2_bwd": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_i32] + [_c_p] * 9),
    "mmb_gemm_f32": (ctypes.c_int, [_c_i32, _c_i32, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p,
                                    _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i32,
                                    _c_i32, _c_p]),
    "mmb_split_tf32": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_i64, _c_p]),
    "mmb_col_dot_f32": (ctypes.c_int, [_c_i64, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i32,
                                       _c_p]),
    "mmb_linoss_work_floats": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "mmb_linoss_fwd": (ctypes.c_int, [_c_i32, _c_i64, _c_i64, _c_i64] + [_c_p] * 6),
    "mmb_linoss_bwd": (ctypes.c_int, [_c_i32, _c_i64, _c_i64, _c_i64] + [_c_p] * 9),
}


def lib_path() -> str:
    return _build.LIB_PATH


def load():
    """Load (building first if the sources are newer) the C-ABI library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = _build.LIB_PATH
            if _build.is_stale():
                _build.build()
            if not os.path.exists(path):
                raise ImportError(f"momentummamba_b200: CUDA library not found at {path}")
            lib = ctypes.CDLL(path)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        lib = load()
        msg = lib.mmb_status_string(int(status)).decode()
        if status == 6:  # MMB_ERR_LAUNCH: add the CUDA runtime's own text
            msg += f" [{lib.mmb_last_error().decode()}]"
        raise RuntimeError(f"momentummamba_b200: {what} failed: {msg} (status {status})")


def require_cuda(*tensors) -> None:
    """Raise unless every given tensor lives on the same CUDA device."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("momentummamba_b200 kernels need CUDA tensors (no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("momentummamba_b200: all tensors must be on one CUDA device")


def ptr(t):
    """Device pointer of a CUDA tensor, or None."""
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("momentummamba_b200 kernels need CUDA tensors (no CPU path)")
    return ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)
