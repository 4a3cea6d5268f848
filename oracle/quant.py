"""CPU oracle for the quantised weight products (Weight<In,Out>::matvec / matmul).

TEST INFRASTRUCTURE ONLY.  Wraps ``nm_quant_oracle.c`` (the C restatement,
built into ``libnm_oracle.so``) and the reference's own quantised-weight code
instantiated by ``ref_shim.cpp`` (``_ref/libnmref.so``).  The product never
imports it.

Weights are GGUF block bytes, row-major with one row per output
(src/quant.hpp:465-487: ``qp_ + o * row_bytes``); activations are fp32
``[rows][in]``.  ``matmul`` returns ``[rows][out]`` as Weight::matmul does
(src/quant_i8.hpp:430-514); ``rows == 1`` is Weight::matvec (:351-428).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _fp, lib, normal, ref

# GGUF type codes (src/quant.hpp:18-27) plus ggml's Q8_K activation blocks.
F32, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K = 0, 2, 8, 12, 13, 14, 15
NAMES = {F32: "F32", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", Q8_K: "Q8_K"}
BLOCK = {F32: (1, 4), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
         Q8_K: (256, 292)}
I8_TYPES = (Q8_0, Q4_0, Q4_K, Q6_K)  # has_i8_kernel (src/quant_i8.hpp:325)

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_registered = set()


def _L():
    L = lib()
    if "o" not in _registered:
        L.nmq_row_bytes.argtypes = [ctypes.c_int, _i64]
        L.nmq_row_bytes.restype = _i64
        L.nmq_dequant_row.argtypes = [ctypes.c_int, _vp, _vp, _i64]
        L.nmq_dot_fp32.argtypes = [ctypes.c_int, _i64, _vp, _vp]
        L.nmq_dot_fp32.restype = ctypes.c_float
        L.nmq_quantize_row_q8_0.argtypes = [_vp, _i64, _vp]
        L.nmq_quantize_row_q8_K.argtypes = [_vp, _i64, _vp]
        L.nmq_vec_dot_i8.argtypes = [ctypes.c_int, _i64, _vp, _vp]
        L.nmq_vec_dot_i8.restype = ctypes.c_float
        L.nmq_matmul.argtypes = [ctypes.c_int, _i64, _i64, _vp, _i64, _vp, _vp, ctypes.c_int, ctypes.c_int]
        _registered.add("o")
    return L


def _R():
    R = ref()
    if R is not None and "r" not in _registered:
        R.nmref_quantize_row_q8_0_blocks.argtypes = [_vp, _i64, _vp]
        R.nmref_quantize_row_q8_K.argtypes = [_vp, _i64, _vp]
        R.nmref_quantize_q8_0_weights.argtypes = [_vp, _i64, _vp]
        R.nmref_quantize_q4_0_weights.argtypes = [_vp, _i64, _vp]
        R.nmref_vec_dot_i8.argtypes = [ctypes.c_int, _i64, _vp, _vp]
        R.nmref_vec_dot_i8.restype = ctypes.c_float
        R.nmref_dot_fp32.argtypes = [ctypes.c_int, _i64, _vp, _vp]
        R.nmref_dot_fp32.restype = ctypes.c_float
        R.nmref_dequant.argtypes = [ctypes.c_int, _vp, _vp, _i64]
        R.nmref_weight_product.argtypes = [ctypes.c_int, _i64, _i64, _vp, _i64, _vp, _vp]
        _registered.add("r")
    return R


def row_bytes(wtype: int, n: int) -> int:
    bl, bb = BLOCK[wtype]
    assert n % bl == 0, f"{NAMES[wtype]} rows hold whole blocks of {bl}"
    return n // bl * bb


def act_type(wtype: int) -> int:
    """The activation block type a weight type's integer dot takes."""
    return Q8_K if wtype in (Q4_K, Q6_K) else Q8_0


def _f32(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def quantize_act(x, atype: int, use_ref: bool = False) -> np.ndarray:
    """quantize_row_q8_0 / quantize_row_q8_K of each row of x: packed block bytes
    [rows][row_bytes].  use_ref runs the reference's own function."""
    x = _f32(np.atleast_2d(x))
    rows, n = x.shape
    out = np.empty((rows, row_bytes(atype, n)), np.uint8)
    if use_ref:
        fn = _R().nmref_quantize_row_q8_K if atype == Q8_K else _R().nmref_quantize_row_q8_0_blocks
    else:
        fn = _L().nmq_quantize_row_q8_K if atype == Q8_K else _L().nmq_quantize_row_q8_0
    for r in range(rows):
        fn(x[r].ctypes.data, n, out[r].ctypes.data)
    return out


def dequant(wtype: int, w, n: int, use_ref: bool = False) -> np.ndarray:
    """dequant_to_f32 of every row of w (GGUF bytes [out][row_bytes]) -> [out][n]."""
    w = np.ascontiguousarray(np.atleast_2d(w), dtype=np.uint8)
    out = np.empty((w.shape[0], n), np.float32)
    fn = _R().nmref_dequant if use_ref else _L().nmq_dequant_row
    for o in range(w.shape[0]):
        rc = fn(wtype, w[o].ctypes.data, out[o].ctypes.data, n)
        assert rc == 0, rc
    return out


def vec_dot_i8(wtype: int, n: int, wrow, act_row, use_ref: bool = False) -> float:
    wrow = np.ascontiguousarray(wrow, np.uint8)
    act_row = np.ascontiguousarray(act_row, np.uint8)
    fn = _R().nmref_vec_dot_i8 if use_ref else _L().nmq_vec_dot_i8
    return float(fn(wtype, n, wrow.ctypes.data, act_row.ctypes.data))


def dot_fp32(wtype: int, n: int, wrow, x, use_ref: bool = False) -> float:
    wrow = np.ascontiguousarray(wrow, np.uint8)
    x = _f32(x)
    fn = _R().nmref_dot_fp32 if use_ref else _L().nmq_dot_fp32
    return float(fn(wtype, n, wrow.ctypes.data, x.ctypes.data))


def matmul(wtype: int, w, x, fp32_act: bool = False, threads: int = 1) -> np.ndarray:
    """Weight::matmul of the oracle: y[rows][out] for x[rows][in] (1-D x: one row)."""
    w = np.ascontiguousarray(np.atleast_2d(w), dtype=np.uint8)
    x2 = _f32(np.atleast_2d(x))
    rows, n = x2.shape
    out = w.shape[0]
    assert w.shape[1] == row_bytes(wtype, n)
    y = np.empty((rows, out), np.float32)
    rc = _L().nmq_matmul(wtype, n, out, w.ctypes.data, rows, x2.ctypes.data, y.ctypes.data, int(bool(fp32_act)), threads)
    assert rc == 0, rc
    return y if np.ndim(x) == 2 else y[0]


def ref_product(wtype: int, w, x) -> np.ndarray | None:
    """The reference's own Weight<In,Out>::matvec (one row) / matmul, for the
    shapes ref_shim.cpp instantiates; None where the reference was not built."""
    R = _R()
    if R is None:
        return None
    w = np.ascontiguousarray(np.atleast_2d(w), dtype=np.uint8)
    x2 = _f32(np.atleast_2d(x))
    rows, n = x2.shape
    y = np.empty((rows, w.shape[0]), np.float32)
    rc = R.nmref_weight_product(wtype, n, w.shape[0], w.ctypes.data, rows, x2.ctypes.data, y.ctypes.data)
    assert rc == 0, f"nmref_weight_product: {rc}"
    return y if np.ndim(x) == 2 else y[0]


def _fp16_bits(v):
    from . import fp16_bits

    return fp16_bits(np.asarray(v, np.float32))


def random_weight(wtype: int, out: int, n: int, seed: int = 0) -> np.ndarray:
    """Synthetic GGUF bytes [out][row_bytes]: random quant bytes (as the
    reference's quant tests draw them, tests/quant_tests.cpp:31-38) with the fp16
    scale fields set so a weight's magnitude is about 1 / sqrt(n) and a product
    with N(0, 1) activations is O(1)."""
    rng = np.random.default_rng(seed)
    if wtype == F32:
        return (normal(seed, 101, out * n).reshape(out, n) / np.float32(np.sqrt(n))).view(np.uint8).reshape(out, 4 * n)
    bl, bb = BLOCK[wtype]
    nb = n // bl
    w = rng.integers(0, 256, size=(out, nb, bb), dtype=np.uint8)
    s = 1.0 / np.sqrt(n)
    u = lambda: rng.uniform(0.5, 1.5, size=(out, nb)).astype(np.float32)

    def put16(off, vals):
        b = _fp16_bits(vals)
        w[:, :, off] = (b & 0xFF).astype(np.uint8)
        w[:, :, off + 1] = (b >> 8).astype(np.uint8)

    if wtype == Q8_0:
        put16(0, s / 74 * u())
    elif wtype == Q4_0:
        put16(0, s / 4.6 * u())
    elif wtype in (Q4_K, Q5_K):
        d = (s / (36 * (8.8 if wtype == Q4_K else 18.0))) * u()
        put16(0, d)
        put16(2, d * (7.5 if wtype == Q4_K else 15.5) * u())
    elif wtype == Q6_K:
        put16(208, s / (74 * 18.5) * u())
    return w.reshape(out, nb * bb)
