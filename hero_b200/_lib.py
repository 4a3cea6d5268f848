"""ctypes binding of libnmg.so (the C ABI in include/nmg.h).

The library is built in-tree (hero_b200/libnmg.so) by ``__graft_entry__.build()``
or ``make -C hero_b200/csrc``.  Loading fails loudly when it is missing: there is
no CPU fallback for anything in this package.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnmg.so")

OK, INVALID_ARGUMENT, OUT_OF_RANGE, RUNTIME_ERROR, LENGTH_ERROR, LOGIC_ERROR = 0, 1, 2, 3, 4, 5
CUDA_ERROR, DEVICE_TIMEOUT, COMM_ERROR, UNSUPPORTED, VALUE_OVERFLOW = 6, 7, 8, 9, 10
F32, F16, BF16, Q8_0 = 0, 1, 2, 3


class NmgError(Exception):
    """Base of every error raised from a non-zero nmg status."""

    status = -1


class InvalidArgument(NmgError, ValueError):
    """std::invalid_argument in the reference (e.g. attention.hpp:217, :322)."""

    status = INVALID_ARGUMENT


class OutOfRange(NmgError, IndexError):
    """std::out_of_range (attention.hpp:240-245, :380-385; recurrent.hpp:128)."""

    status = OUT_OF_RANGE


class NoVisibleKeys(NmgError, RuntimeError):
    """std::runtime_error: a query with no visible key (attention.hpp:224, :349)."""

    status = RUNTIME_ERROR


class LengthError(NmgError, OverflowError):
    """std::length_error (attention.hpp:325; device capacity exhausted)."""

    status = LENGTH_ERROR


class LogicError(NmgError, RuntimeError):
    """std::logic_error (attention.hpp:275, :295)."""

    status = LOGIC_ERROR


class CudaError(NmgError, RuntimeError):
    status = CUDA_ERROR


class DeviceTimeout(NmgError, RuntimeError):
    """A bounded device-side wait gave up (kernel returned early, flag raised)."""

    status = DEVICE_TIMEOUT


class CommError(NmgError, RuntimeError):
    status = COMM_ERROR


class Unsupported(NmgError, NotImplementedError):
    status = UNSUPPORTED


class ValueOverflow(NmgError, ArithmeticError):
    """A V value beyond fp16's range reached a bf16 cache (which keeps V as fp16)."""

    status = VALUE_OVERFLOW


_ERRORS = {c.status: c for c in (InvalidArgument, OutOfRange, NoVisibleKeys, LengthError, LogicError, CudaError,
                                 DeviceTimeout, CommError, Unsupported, ValueOverflow)}

_lock = threading.Lock()
_lib = None

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_i64p = ctypes.POINTER(ctypes.c_int64)

# name -> (argtypes)
SIGNATURES = {
    "nmg_device_status": [_i32, _vp],
    "nmg_selftest_wait_timeout": [_i32, _i32, _vp],
    "nmg_kv_create": [_i32, _i32, _i32, _i64, _i64, _i32, ctypes.POINTER(_vp)],
    "nmg_kv_destroy": [_vp],
    "nmg_kv_append": [_vp, _i64, _vp, _vp, _i64, _i32, _vp],
    "nmg_kv_size": [_vp, _i64p],
    "nmg_kv_position": [_vp, _i64, _i64p],
    "nmg_kv_window": [_vp, _i64p],
    "nmg_kv_can_append_without_eviction": [_vp, _i64, ctypes.POINTER(_i32)],
    "nmg_kv_visible_rows": [_vp, _i64, _i64p, _i64p],
    "nmg_kv_begin_batch_retention": [_vp, _i64],
    "nmg_kv_end_batch_retention": [_vp],
    "nmg_kv_read_row": [_vp, _i64, _i32, ctypes.POINTER(_f32), ctypes.POINTER(_f32), _vp],
    "nmg_kv_storage": [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _i64p],
    "nmg_kv_scales": [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _i64p],
    "nmg_kv_reset": [_vp],
    "nmg_attend": [_vp, _i32, _vp, _i32, _i64, _i64, _f32, _i32, _vp, _i32, _vp],
    "nmg_append_attend": [_vp, _i64, _vp, _vp, _i32, _i32, _vp, _i32, _i64, _f32, _i32, _vp, _i32, _vp],
    "nmg_attend_noalloc": [_vp, _i32, _vp, _i32, _i64, _i64, _f32, _i32, _vp, _i32, _vp],
    "nmg_attend_batch": [ctypes.POINTER(_vp), _i32, _i64p, _i32, _vp, _i32, _f32, _i32, _vp, _i32, _vp],
    "nmg_sdpa": [_i32, _i32, _vp, _vp, _vp, _i32, _i64, _i64, _f32, _vp, _i32, _vp],
    "nmg_delta_create": [_i32, _i32, _i32, _i32, ctypes.POINTER(_vp)],
    "nmg_delta_destroy": [_vp],
    "nmg_delta_clear": [_vp, _vp],
    "nmg_delta_head": [_vp, _i32, ctypes.POINTER(_vp)],
    "nmg_gated_delta_step": [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "nmg_delta_step": [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "nmg_delta_step_batch": [ctypes.POINTER(_vp), _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "nmg_delta_prefill": [_vp, _i32, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp],
    "nmg_conv_create": [_i32, _i32, _i32, ctypes.POINTER(_vp)],
    "nmg_conv_destroy": [_vp],
    "nmg_conv_clear": [_vp, _vp],
    "nmg_conv_history": [_vp, ctypes.POINTER(_vp)],
    "nmg_conv_step": [_vp, _vp, _vp, _i64, _vp, _i32, _vp],
    "nmg_delta_prologue": [_vp, _vp, _i32, _i32, _i32, _i32, _i64] + [_vp] * 10 + [_vp],
    "nmg_delta_epilogue": [_i32, _i32, _i64, _vp, _vp, _vp, ctypes.c_float, _vp, _vp],
    "nmg_delta_decode_token": [_vp, _vp, _vp, _i32] + [_vp] * 7 + [ctypes.c_float, _vp, _vp],
    "nmg_attn_prologue": [_vp, _i32, _i64, _i64, _vp, _i32, _vp, _vp, _vp, _vp, _i32, ctypes.c_float, ctypes.c_double,
                          _i32, _i32, _vp, _i32, _vp],
    "nmg_attn_prepare": [_i32, _i32, _i32, _i64, _i64, _vp, _i32, _vp, _vp, _vp, _vp, _i32, ctypes.c_float,
                         ctypes.c_double, _i32, _i32, _vp, _i32, _vp, _vp, _vp],
    "nmg_attn_gate": [_i64, _i32, _i32, _vp, _vp, _i32, _vp],
    "nmg_comm_unique_id": [_vp],
    "nmg_comm_init": [_vp, _i32, _i32, _i32, ctypes.POINTER(_vp)],
    "nmg_comm_destroy": [_vp],
    "nmg_allgather": [_vp, _vp, _vp, _i64, _vp],
    "nmg_gather_heads_to_rows": [_vp, _vp, _i32, _i64, _i64, _vp],
    "nmg_comm_barrier": [_vp, _vp],
    "nmg_shared_alloc": [_i64, _i32, ctypes.POINTER(_vp), _vp],
    "nmg_shared_free": [_vp],
    "nmg_ipc_open": [_vp, _i32, ctypes.POINTER(_vp)],
    "nmg_ipc_close": [_vp],
    "nmg_attend_fanout": [_vp, _i32, _vp, _i32, _i64, _i64, _f32, _i32, ctypes.POINTER(_vp), _i32, _i64, _i64, _i32,
                          _vp],
    "nmg_weight_row_bytes": [_i32, _i64, ctypes.POINTER(_i64)],
    "nmg_weight_create": [_i32, _i64, _i64, _vp, _i32, _i32, ctypes.POINTER(_vp)],
    "nmg_weight_destroy": [_vp],
    "nmg_weight_info": [_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i64), ctypes.POINTER(_i64)],
    "nmg_weight_matvec": [_vp, _vp, _vp, _i32, _vp],
    "nmg_weight_matmul": [_vp, _i64, _vp, _vp, _i32, _vp],
    "nmg_weight_gather_rows": [_vp, _vp, _i64, _vp, _vp],
    "nmg_quantize_activations": [_i32, _i64, _i64, _vp, _vp, _vp],
}


def lib():
    """The loaded libnmg.so; raises ImportError when it was never built."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is missing: run __graft_entry__.build() or make -C hero_b200/csrc")
            L = ctypes.CDLL(LIB_PATH)
            for name, argtypes in SIGNATURES.items():
                fn = getattr(L, name)
                fn.argtypes = argtypes
                fn.restype = ctypes.c_int
            L.nmg_last_error.restype = ctypes.c_char_p
            L.nmg_version.restype = ctypes.c_char_p
            _lib = L
    return _lib


def check(status: int) -> None:
    if status != OK:
        msg = lib().nmg_last_error().decode(errors="replace")
        raise _ERRORS.get(status, NmgError)(msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
