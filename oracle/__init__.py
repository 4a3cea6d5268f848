"""CPU oracle for the nm attention / KV-cache / gated delta-rule hot path.

TEST INFRASTRUCTURE ONLY.  The product (hero_b200/) never imports this
package; tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm are the only callers, and only as the checker or the timed CPU baseline.

Two checkers live here:

* ``lib()`` -- ``nm_oracle.c``, a C restatement of the reference arithmetic
  (each function cites the reference file:line it follows).  Builds anywhere
  gcc is, including the GPU box.
* ``ref()`` -- ``_ref/libnmref.so``, the reference engine's own headers
  instantiated by ``ref_shim.cpp``.  Built only where the reference sources
  exist; the built library travels with the repository snapshot.

Plus ``CacheModel``, a Python restatement of the cache bookkeeping of
``FullAttentionCache`` / ``LocalAttentionCache`` (src/attention.hpp:201-395):
positions, sizes, ring eviction and batch retention, for exact comparison with
the device cache's position map.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libnm_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libnmref.so")

_lock = threading.Lock()
_lib = None
_ref = None
_ref_tried = False

OK, INVALID_ARGUMENT, OUT_OF_RANGE, RUNTIME_ERROR, LENGTH_ERROR, LOGIC_ERROR = 0, 1, 2, 3, 4, 5

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i64 = ctypes.c_int64


def build() -> None:
    """Compile the C oracle (and the reference shim where the sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def _fp(a):
    return a.ctypes.data_as(_f32p)


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(ORACLE_SO):
                subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
            L = ctypes.CDLL(ORACLE_SO)
            L.nmo_attend.argtypes = [_f32p, _f32p, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, _f32p, _i64,
                                     ctypes.c_int, _i64, ctypes.c_float, ctypes.c_int, _f32p, ctypes.c_int]
            L.nmo_attend.restype = ctypes.c_int
            L.nmo_visible_rows.argtypes = [_i64, _i64, _i64, _i64, _i64p, _i64p]
            L.nmo_contains.argtypes = [_i64, _i64, _i64]
            L.nmo_contains.restype = ctypes.c_int
            L.nmo_gated_delta_step.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_float, ctypes.c_float, _f32p,
                                               ctypes.c_int, ctypes.c_int, _f32p]
            L.nmo_delta_run.argtypes = [_f32p, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p,
                                        _f32p, _f32p, _f32p, _f32p, _f32p]
            L.nmo_softplus.argtypes = [ctypes.c_float]
            L.nmo_softplus.restype = ctypes.c_float
            L.nmo_sigmoid.argtypes = [ctypes.c_float]
            L.nmo_sigmoid.restype = ctypes.c_float
            L.nmo_l2_normalize.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_float]
            L.nmo_conv_run.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int64, _f32p, _f32p]
            L.nmo_silu.argtypes = [ctypes.c_float]
            L.nmo_silu.restype = ctypes.c_float
            L.nmo_delta_prologue.argtypes = ([_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int64] + [_f32p] * 11)
            L.nmo_delta_epilogue.argtypes = [ctypes.c_int64, ctypes.c_int, _f32p, _f32p, _f32p, ctypes.c_float, _f32p]
            L.nmo_rope_freqs.argtypes = [ctypes.c_int, ctypes.c_double, ctypes.c_int, ctypes.c_int, _f32p]
            L.nmo_rope.argtypes = [_f32p, ctypes.c_int, _f32p, ctypes.c_int64]
            L.nmo_rmsnorm.argtypes = [ctypes.c_int, _f32p, ctypes.c_float, _f32p, _f32p]
            L.nmo_attn_prologue.argtypes = ([ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                             _f32p, ctypes.c_int, _f32p, _f32p, _f32p, _f32p, ctypes.c_int,
                                             ctypes.c_float, ctypes.c_double, ctypes.c_int, ctypes.c_int,
                                             _f32p, _f32p, _f32p])
            L.nmo_attn_gate.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int, _f32p, _f32p]
            L.nmo_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _i64, _f32p]
            L.nmo_uniform_int.argtypes = [ctypes.c_uint64, ctypes.c_uint64, _i64, _i64, _i64, _i64p]
            L.nmo_round_bf16.argtypes = [_f32p, _i64]
            L.nmo_round_fp16.argtypes = [_f32p, _i64]
            L.nmo_to_bf16.argtypes = [_f32p, _u16p, _i64]
            L.nmo_to_fp16.argtypes = [_f32p, _u16p, _i64]
            L.nmo_fp32_to_bf16.argtypes = [ctypes.c_float]
            L.nmo_fp32_to_bf16.restype = ctypes.c_uint16
            L.nmo_fp32_to_fp16.argtypes = [ctypes.c_float]
            L.nmo_fp32_to_fp16.restype = ctypes.c_uint16
            L.nmo_bf16_to_fp32.argtypes = [ctypes.c_uint16]
            L.nmo_bf16_to_fp32.restype = ctypes.c_float
            L.nmo_fp16_to_fp32.argtypes = [ctypes.c_uint16]
            L.nmo_fp16_to_fp32.restype = ctypes.c_float
            L.nmo_quantize_q8_0.argtypes = [_f32p, _i64, ctypes.c_void_p, ctypes.c_void_p]
            _lib = L
    return _lib


def ref():
    """The reference engine's own code (ref_shim.cpp), or None where it was never built."""
    global _ref, _ref_tried
    with _lock:
        if not _ref_tried:
            _ref_tried = True
            if os.path.exists(REF_SO):
                R = ctypes.CDLL(REF_SO)
                R.nmref_attend_full.argtypes = [ctypes.c_int, ctypes.c_int, _f32p, _f32p, _i64, _i64, _f32p, _i64,
                                                ctypes.c_int, _i64, ctypes.c_float, ctypes.c_int, _f32p]
                R.nmref_attend_local.argtypes = [ctypes.c_int, ctypes.c_int, _i64, _f32p, _f32p, _i64, _i64, _f32p,
                                                 _i64, ctypes.c_int, ctypes.c_float, ctypes.c_int, _f32p]
                R.nmref_local_script.argtypes = [_i64, _i64p, _i64, _i64p, _i64p, _i64, _i64p]
                R.nmref_visible_rows.argtypes = [_i64, _i64, _i64, _i64, _i64p, _i64p]
                R.nmref_contains.argtypes = [_i64, _i64, _i64]
                R.nmref_delta_run.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p, _i64, ctypes.c_int,
                                              _f32p, _f32p, _f32p, _f32p, _f32p, _f32p]
                R.nmref_softplus.argtypes = [ctypes.c_float]
                R.nmref_softplus.restype = ctypes.c_float
                R.nmref_sigmoid.argtypes = [ctypes.c_float]
                R.nmref_sigmoid.restype = ctypes.c_float
                R.nmref_l2_normalize.argtypes = [ctypes.c_int, _f32p, _f32p]
                R.nmref_conv_run.argtypes = [ctypes.c_int, ctypes.c_int, _f32p, _f32p, _i64, _f32p]
                R.nmref_silu.argtypes = [_i64, _f32p, _f32p]
                R.nmref_rmsnorm.argtypes = [ctypes.c_int, _i64, _f32p, ctypes.c_float, _f32p, _f32p]
                R.nmref_rope.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i64,
                                         _i64, _f32p]
                R.nmref_head_norm.argtypes = [ctypes.c_int, ctypes.c_int, _i64, _f32p, ctypes.c_float, _f32p, _f32p]
                R.nmref_sigmoid_n.argtypes = [_i64, _f32p, _f32p]
                R.nmref_sdpa.argtypes = [ctypes.c_int, ctypes.c_int, _i64, _i64, _f32p, _f32p, _f32p, ctypes.c_float,
                                         _f32p]
                R.nmref_fp32_to_bf16.argtypes = [ctypes.c_float]
                R.nmref_fp32_to_bf16.restype = ctypes.c_uint16
                R.nmref_fp32_to_fp16.argtypes = [ctypes.c_float]
                R.nmref_fp32_to_fp16.restype = ctypes.c_uint16
                R.nmref_bf16_to_fp32.argtypes = [ctypes.c_uint16]
                R.nmref_bf16_to_fp32.restype = ctypes.c_float
                R.nmref_fp16_to_fp32.argtypes = [ctypes.c_uint16]
                R.nmref_fp16_to_fp32.restype = ctypes.c_float
                R.nmref_quantize_q8_0.argtypes = [_f32p, _i64, ctypes.c_void_p, ctypes.c_void_p]
                _ref = R
    return _ref


# ---- seeded inputs ----------------------------------------------------------

def normal(seed: int, stream: int, n: int, first: int = 0) -> np.ndarray:
    """n standard normals, element i a pure function of (seed, stream, first + i)."""
    out = np.empty(int(n), dtype=np.float32)
    lib().nmo_normal(seed, stream, first, int(n), _fp(out))
    return out


def uniform_int(seed: int, stream: int, n: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(int(n), dtype=np.int64)
    lib().nmo_uniform_int(seed, stream, int(n), lo, hi, out.ctypes.data_as(_i64p))
    return out


# ---- rounding (src/core.hpp:61-100), vectorised --------------------------------

def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round-nearest-even, NaN kept quiet (core.hpp:92-100)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((b >> 16) | 0x40).astype(np.uint16), r)


def from_bf16_bits(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return from_bf16_bits(bf16_bits(x)).reshape(np.shape(x))


def fp16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 bits exactly as core.hpp:61-79 (normal range: round half up on bit 12)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size, dtype=np.uint16)
    lib().nmo_to_fp16(_fp(x.reshape(-1)), out.ctypes.data_as(_u16p), x.size)
    return out.reshape(x.shape)


def from_fp16_bits(h: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def round_fp16(x: np.ndarray) -> np.ndarray:
    return from_fp16_bits(fp16_bits(x))


def quantize_q8_0(x, use_ref=False):
    """quantize_row_q8_0 (src/quant_i8.hpp:69-81) of each row of x (last axis a
    multiple of 32): returns (int8 quants, shape of x; fp16 scale bits, one per
    32 values).  use_ref runs the reference's own function (oracle/_ref)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    qs = np.empty(n, np.int8)
    d = np.empty(n // 32, np.uint16)
    fn = ref().nmref_quantize_q8_0 if use_ref else lib().nmo_quantize_q8_0
    fn(_fp(x.reshape(-1)), n, qs.ctypes.data, d.ctypes.data)
    return qs.reshape(x.shape), d.reshape(x.shape[:-1] + (x.shape[-1] // 32,))


def dequantize_q8_0(qs, d):
    """The values a Q8_0 block holds: fp16 scale (core.hpp:34-59) times each int8 quant."""
    scale = from_fp16_bits(np.asarray(d, np.uint16))
    q = np.asarray(qs, np.int8).astype(np.float32)
    return (q.reshape(q.shape[:-1] + (-1, 32)) * scale[..., None]).reshape(q.shape).astype(np.float32)


# ---- the arithmetic -------------------------------------------------------------

def visible_rows(width: int, query: int, oldest: int, rows: int) -> tuple[int, int]:
    f, e = ctypes.c_int64(), ctypes.c_int64()
    lib().nmo_visible_rows(width, query, oldest, rows, ctypes.byref(f), ctypes.byref(e))
    return f.value, e.value


def contains(width: int, key: int, query: int) -> bool:
    return bool(lib().nmo_contains(width, key, query))


class NoVisibleKeys(RuntimeError):
    """A query with no visible key is an error, never zeros (attention.hpp:224, :349)."""


def attend(keys, values, oldest, window, hkv, dh, q, hq, first_query, scale=1.0, use_scale=True, threads=None):
    """The reference reduction over chronological cache rows.

    keys/values: [rows, hkv*dh] fp32; q: [qrows, hq*dh] fp32; returns [qrows, hq*dh].
    """
    keys = np.ascontiguousarray(keys, dtype=np.float32).reshape(-1, hkv * dh)
    values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1, hkv * dh)
    q = np.ascontiguousarray(q, dtype=np.float32).reshape(-1, hq * dh)
    out = np.zeros_like(q)
    if threads is None:
        threads = os.cpu_count() or 1
    st = lib().nmo_attend(_fp(keys), _fp(values), keys.shape[0], oldest, window, hkv, dh, _fp(q), q.shape[0], hq,
                          first_query, float(scale), 1 if use_scale else 0, _fp(out), int(threads))
    if st == RUNTIME_ERROR:
        raise NoVisibleKeys("query has no visible keys")
    if st != OK:
        raise ValueError(f"nmo_attend status {st}")
    return out


def delta_run(state, q, k, v, g, beta, hk):
    """Sequential gated delta rule over T tokens; returns (out [T,hv,dv], new state)."""
    state = np.array(state, dtype=np.float32, copy=True, order="C")
    hv, dk, dv = state.shape
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    g = np.ascontiguousarray(g, dtype=np.float32)
    beta = np.ascontiguousarray(beta, dtype=np.float32)
    T = v.shape[0]
    out = np.zeros((T, hv, dv), dtype=np.float32)
    lib().nmo_delta_run(_fp(state), T, hk, hv, dk, dv, _fp(q), _fp(k), _fp(v), _fp(g), _fp(beta), _fp(out))
    return out, state


def l2_normalize(x, eps=1e-6):
    x = np.ascontiguousarray(x, dtype=np.float32)
    flat = x.reshape(-1, x.shape[-1])
    y = np.empty_like(flat)
    for r in range(flat.shape[0]):
        lib().nmo_l2_normalize(_fp(flat[r]), _fp(y[r]), flat.shape[1], eps)
    return y.reshape(x.shape)


def conv_run(weights, x, history=None):
    """CausalConv1dState::step over T tokens (src/recurrent.hpp:76-104).

    weights [C][W] (tap 0 oldest), x [T][C], history [W-1][C] oldest first (zero
    when None); returns (y [T][C], the advanced history)."""
    w = np.ascontiguousarray(weights, dtype=np.float32)
    C, W = w.shape
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, C)
    hist = np.zeros((max(W - 1, 1), C), np.float32) if history is None else np.array(history, np.float32, order="C")
    y = np.empty_like(x)
    lib().nmo_conv_run(_fp(w), C, W, _fp(x), x.shape[0], _fp(hist), _fp(y))
    return y, hist


def silu(x):
    """x / (1 + e^-x) elementwise (src/components.hpp:102-105)."""
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore"):  # e^-x overflows to inf for x < -88: the result is -0, as in fp32
        return np.vectorize(lambda e: lib().nmo_silu(float(e)), otypes=[np.float32])(x).astype(np.float32)


def delta_prologue(weights, qkv, beta_raw, alpha_raw, dt_bias, decay_scale, hk, hv, dk, dv, history=None):
    """qwen35.hpp:396-446 for T tokens: returns (q [T,hk,dk], k, v [T,hv,dv], beta [T,hv], gate [T,hv], history)."""
    w = np.ascontiguousarray(weights, dtype=np.float32)
    C, W = w.shape
    qkv = np.ascontiguousarray(qkv, dtype=np.float32).reshape(-1, C)
    T = qkv.shape[0]
    hist = np.zeros((max(W - 1, 1), C), np.float32) if history is None else np.array(history, np.float32, order="C")
    f = lambda a: np.ascontiguousarray(a, dtype=np.float32)
    q = np.empty((T, hk, dk), np.float32)
    k = np.empty((T, hk, dk), np.float32)
    v = np.empty((T, hv, dv), np.float32)
    beta = np.empty((T, hv), np.float32)
    gate = np.empty((T, hv), np.float32)
    lib().nmo_delta_prologue(_fp(w), W, hk, hv, dk, dv, T, _fp(qkv), _fp(hist), _fp(f(beta_raw)), _fp(f(alpha_raw)),
                             _fp(f(dt_bias)), _fp(f(decay_scale)), _fp(q), _fp(k), _fp(v), _fp(beta), _fp(gate))
    return q, k, v, beta, gate, hist


def delta_epilogue(o, z, gamma, eps=1e-6):
    """RMSNorm per head then the SiLU(z) gate (qwen35.hpp:458-460); o, z [..., dv]."""
    o = np.ascontiguousarray(o, dtype=np.float32)
    z = np.ascontiguousarray(z, dtype=np.float32)
    dv = o.shape[-1]
    out = np.empty_like(o)
    lib().nmo_delta_epilogue(o.size // dv, dv, _fp(o), _fp(z), _fp(np.ascontiguousarray(gamma, dtype=np.float32)),
                             float(eps), _fp(out))
    return out


def rope_freqs(head_dim, base, num=1, den=1):
    """RotaryEmbedding<head_dim, base, num, den>'s inv_freq table (src/attention.hpp:76-80)."""
    out = np.empty(head_dim // 2, np.float32)
    lib().nmo_rope_freqs(int(head_dim), float(base), int(num), int(den), _fp(out))
    return out


def rope(x, first_position, base, num=1, den=1):
    """Half-split RoPE of every head of x [..., rows, heads, head_dim], row r at
    first_position + r (src/attention.hpp:82-101)."""
    x = np.array(x, dtype=np.float32, order="C")
    dh = x.shape[-1]
    freqs = rope_freqs(dh, base, num, den)
    rows = x.reshape(-1, x.shape[-2], dh)
    for r in range(rows.shape[0]):
        for h in range(rows.shape[1]):
            lib().nmo_rope(_fp(rows[r, h]), dh, _fp(freqs), int(first_position) + r)
    return x


def rmsnorm(x, gamma=None, eps=1e-6):
    """RMSNorm over the last axis (src/components.hpp:167-180), or RMSNormNoScale
    (:204-215) when gamma is None."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    flat, y = x.reshape(-1, n), np.empty(x.shape, np.float32).reshape(-1, n)
    g = None if gamma is None else np.ascontiguousarray(gamma, dtype=np.float32)
    for r in range(flat.shape[0]):
        lib().nmo_rmsnorm(n, None if g is None else _fp(g), float(eps), _fp(flat[r]), _fp(y[r]))
    return y.reshape(x.shape)


def attn_prologue(q, k, v, q_gamma, k_gamma, hq, hkv, head_dim, position, eps, base, num=1, den=1, *, gated=True,
                  v_norm=False):
    """Q, K, V of an attention layer (qwen35.hpp:343-352; gemma4.hpp:206-209, :676-680).

    q [T, (2 if gated) * hq * head_dim] (gated: head-major [q | gate] pairs),
    k, v [T, hkv * head_dim]; returns (Q [T, hq*dh], K [T, hkv*dh], V [T, hkv*dh])."""
    f = lambda a: np.ascontiguousarray(a, dtype=np.float32)
    q, k, v = f(q), f(k), f(v)
    T = q.shape[0]
    qo = np.empty((T, hq * head_dim), np.float32)
    ko = np.empty((T, hkv * head_dim), np.float32)
    vo = np.empty((T, hkv * head_dim), np.float32)
    lib().nmo_attn_prologue(T, hq, hkv, head_dim, int(position), _fp(q), int(bool(gated)), _fp(k), _fp(v),
                            _fp(f(q_gamma)), _fp(f(k_gamma)), int(bool(v_norm)), float(eps), float(base), int(num),
                            int(den), _fp(qo), _fp(ko), _fp(vo))
    return qo, ko, vo


def attn_gate(qg, a, head_dim):
    """a * sigmoid(gate) (qwen35.hpp:390-393); qg [T, 2*hq*dh] head-major [q | gate] pairs, a [T, hq*dh]."""
    out = np.array(a, dtype=np.float32, order="C")
    T = out.shape[0]
    lib().nmo_attn_gate(T, out.shape[1] // head_dim, int(head_dim), _fp(np.ascontiguousarray(qg, dtype=np.float32)),
                        _fp(out))
    return out


def softplus(x: float) -> float:
    return lib().nmo_softplus(x)


def sigmoid(x: float) -> float:
    return lib().nmo_sigmoid(x)


# ---- cache bookkeeping (src/attention.hpp:201-395) ------------------------------

class CacheModel:
    """Positions, size and retention state of a Full (window=0) or Local cache.

    Restates only the integer bookkeeping: ``append`` (:215-220, :320-345),
    ``visible_rows`` (:222-226, :347-351), ``position`` (:208-211, :264-267),
    ``can_append_without_eviction`` (:213, :315-318) and batch retention
    (:274-313), raising the same exception types.
    """

    def __init__(self, window: int = 0, local: bool = False):
        if local and window == 0:
            raise ValueError("LocalAttentionCache: window must be positive")
        self.local = local
        self.window = window if local else 0
        self.size = 0
        self.oldest = 0
        self.retaining = False
        self.batch_remaining = 0

    def position(self, row: int) -> int:
        if row >= self.size:
            raise IndexError("row out of range")
        return self.oldest + row

    def can_append_without_eviction(self, rows: int) -> bool:
        if not self.local:
            return True
        if self.retaining:
            return rows <= self.batch_remaining
        return rows <= self.window - self.size

    def append(self, position: int) -> None:
        if self.size == 0:
            self.oldest = position
        elif position != self.oldest + self.size:
            raise ValueError("positions must be consecutive")
        if not self.local:
            self.size += 1
            return
        if self.retaining:
            if self.batch_remaining == 0:
                raise OverflowError("retained batch received too many rows")
            self.size += 1
            self.batch_remaining -= 1
            return
        if self.size < self.window:
            self.size += 1
        else:
            self.oldest += 1

    def begin_batch_retention(self, rows: int) -> None:
        if self.retaining:
            raise RuntimeError("batch retention already active")
        if rows <= 1:
            return
        self.retaining = True
        self.batch_remaining = rows

    def end_batch_retention(self) -> None:
        if not self.retaining:
            return
        if self.batch_remaining != 0:
            raise RuntimeError("retained batch was not fully appended")
        kept = min(self.size, self.window)
        self.oldest += self.size - kept
        self.size = kept
        self.retaining = False

    def visible_rows(self, query: int) -> tuple[int, int]:
        f, e = visible_rows(self.window, query, self.oldest, self.size)
        if f == e:
            raise NoVisibleKeys("query has no visible keys")
        return f, e
