"""The reference's attention / KV-cache / delta-rule interface, device-resident.

Mirrors the nm engine's types and calls (paths relative to the nm/ project):

* ``FullAttentionCache`` / ``LocalAttentionCache`` -- src/attention.hpp:201-395
  (append, size, position, visible_rows, key, value, window,
  can_append_without_eviction, begin/end_batch_retention), same exceptions.
* ``attend`` -- the per-layer softmax reduction (src/qwen35.hpp:360-382 with a
  score scale; src/gemma4.hpp:211-235 et al. with none).
* ``append_attend`` -- a layer's append-then-reduce step with the Gemma local
  fallback (src/gemma4.hpp:237-253, :617-630).
* ``scaled_dot_product_attention`` -- src/attention.hpp:124-139.
* ``DeltaNetState`` / ``gated_delta_step`` -- src/recurrent.hpp:117-177, and
  ``delta_step`` / ``delta_prefill`` for the head loop of src/qwen35.hpp:436-456.
* ``attn_prologue`` / ``attn_prepare`` / ``attn_gate`` -- the steps either side
  of the attention reduction (src/qwen35.hpp:343-352, :390-393;
  src/gemma4.hpp:206-209, :676-680).
* ``ConvState`` / ``delta_prologue`` / ``delta_epilogue`` -- the steps either
  side of the delta rule (src/recurrent.hpp:63-110; src/qwen35.hpp:396-461).

Every call goes through libnmg.so's C ABI.  Tensors are torch CUDA tensors
(torch provides device memory and streams only); nothing here computes on the
host.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import BF16, F16, F32, Q8_0, call

_DT = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
_TORCH = {F32: torch.float32, F16: torch.float16, BF16: torch.bfloat16}


def dtype_code(dt) -> int:
    if isinstance(dt, int):
        return dt
    if isinstance(dt, str):
        return {"f32": F32, "fp32": F32, "f16": F16, "fp16": F16, "bf16": BF16, "q8_0": Q8_0}[dt]
    return _DT[dt]


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _dev(t: torch.Tensor) -> torch.Tensor:
    if not t.is_cuda:
        raise ValueError("device tensors expected")
    return t.contiguous()


def device_status(device: int = 0) -> None:
    """Synchronise; raise DeviceTimeout if a kernel gave up a bounded device-side wait, or
    ValueOverflow if a V value beyond fp16's range was appended to a bf16 cache."""
    call("nmg_device_status", int(device), _stream(device))


@dataclass(frozen=True)
class VisibleRows:
    """Half-open chronological row interval (src/attention.hpp:144-150)."""

    first: int
    end: int

    def empty(self) -> bool:
        return self.first == self.end

    def count(self) -> int:
        return self.end - self.first


class _Cache:
    def __init__(self, hkv: int, head_dim: int, window: int, capacity: int, dtype, device: int):
        self.hkv, self.head_dim = int(hkv), int(head_dim)
        self.dtype = dtype_code(dtype)
        self.device = int(device)
        h = ctypes.c_void_p()
        call("nmg_kv_create", self.hkv, self.head_dim, self.dtype, int(window), int(capacity), self.device,
             ctypes.byref(h))
        self._h = h

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.lib().nmg_kv_destroy(h)
            except Exception:
                pass
            self._h = None

    @property
    def width(self) -> int:
        return self.hkv * self.head_dim

    def size(self) -> int:
        v = ctypes.c_int64()
        call("nmg_kv_size", self._h, ctypes.byref(v))
        return v.value

    def window(self) -> int:
        v = ctypes.c_int64()
        call("nmg_kv_window", self._h, ctypes.byref(v))
        return v.value

    def position(self, chronological_row: int) -> int:
        v = ctypes.c_int64()
        call("nmg_kv_position", self._h, int(chronological_row), ctypes.byref(v))
        return v.value

    def can_append_without_eviction(self, rows: int) -> bool:
        v = ctypes.c_int()
        call("nmg_kv_can_append_without_eviction", self._h, int(rows), ctypes.byref(v))
        return bool(v.value)

    def append(self, position: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """Append one row ([hkv*head_dim]) or a batch of consecutive rows ([rows, hkv*head_dim])."""
        key, value = _dev(key), _dev(value)
        if key.shape != value.shape or key.shape[-1] != self.width:
            raise _lib.InvalidArgument("append: key/value rows must be [.., hkv*head_dim]")
        rows = 1 if key.dim() == 1 else key.shape[0]
        call("nmg_kv_append", self._h, int(position), _ptr(key), _ptr(value), rows, _DT[key.dtype],
             _stream(key.device))

    def visible_rows(self, query: int) -> VisibleRows:
        f, e = ctypes.c_int64(), ctypes.c_int64()
        call("nmg_kv_visible_rows", self._h, int(query), ctypes.byref(f), ctypes.byref(e))
        return VisibleRows(f.value, e.value)

    def _row(self, chronological_row: int, head: int):
        k = (ctypes.c_float * self.head_dim)()
        v = (ctypes.c_float * self.head_dim)()
        call("nmg_kv_read_row", self._h, int(chronological_row), int(head), k, v, _stream(self.device))
        return torch.tensor(list(k), dtype=torch.float32), torch.tensor(list(v), dtype=torch.float32)

    def key(self, chronological_row: int, head: int) -> torch.Tensor:
        """Host copy of one cached key (slow debug accessor; attention.hpp:228-232)."""
        return self._row(chronological_row, head)[0]

    def value(self, chronological_row: int, head: int) -> torch.Tensor:
        return self._row(chronological_row, head)[1]

    def reset(self) -> None:
        """Forget every row: a new sequence on the same device storage."""
        call("nmg_kv_reset", self._h)

    def storage(self):
        """(keys_ptr, values_ptr, slots) of the head-major device storage."""
        k, v, s = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_int64()
        call("nmg_kv_storage", self._h, ctypes.byref(k), ctypes.byref(v), ctypes.byref(s))
        return k.value, v.value, s.value

    def q8_blocks(self, head: int):
        """A Q8_0 cache's raw blocks of one K/V head, as host arrays: (K quants
        [slots, head_dim] int8, K scales [slots, head_dim/32] fp16 bits, V quants,
        V scales)."""
        kp, vp, slots = self.storage()
        ks, vs, sr = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_int64()
        call("nmg_kv_scales", self._h, ctypes.byref(ks), ctypes.byref(vs), ctypes.byref(sr))
        n, nb = slots * self.head_dim, slots * (self.head_dim // 32)
        nbs = sr.value * (self.head_dim // 32)  # scale rows per head: slots rounded up to 64

        def grab(ptr, count, dtype, off):
            t = _from_ptr(ptr + off * torch.tensor([], dtype=dtype).element_size(), count, self.device, dtype)
            return t.cpu().numpy().copy()

        h = int(head)
        return (grab(kp, n, torch.int8, h * n).reshape(slots, -1),
                grab(ks.value, nb, torch.int16, h * nbs).view("u2").reshape(slots, -1),
                grab(vp, n, torch.int8, h * n).reshape(slots, -1),
                grab(vs.value, nb, torch.int16, h * nbs).view("u2").reshape(slots, -1))


class FullAttentionCache(_Cache):
    """Append-only device K/V cache (src/attention.hpp:201-250) of `capacity` rows."""

    def __init__(self, hkv: int, head_dim: int, *, capacity: int, dtype="f32", device: int = 0):
        super().__init__(hkv, head_dim, 0, capacity, dtype, device)


class LocalAttentionCache(_Cache):
    """Fixed-window ring (src/attention.hpp:252-395).

    ``capacity`` physical rows (default: window rounded up to 128) bound how
    many rows one batch may append and still be attended as a whole and how
    large a retained batch may grow; ``append_attend`` chunks larger batches.
    """

    def __init__(self, hkv: int, head_dim: int, window: int, *, capacity: int | None = None, dtype="f32",
                 device: int = 0):
        if window <= 0:
            raise _lib.InvalidArgument("LocalAttentionCache: window must be positive")
        if capacity is None:
            capacity = (window + 127) // 128 * 128
        super().__init__(hkv, head_dim, window, capacity, dtype, device)

    def begin_batch_retention(self, appended_rows: int) -> None:
        call("nmg_kv_begin_batch_retention", self._h, int(appended_rows))

    def end_batch_retention(self) -> None:
        call("nmg_kv_end_batch_retention", self._h)


def _out(q: torch.Tensor, out, out_dtype):
    if out is not None:
        return out
    dt = _TORCH[dtype_code(out_dtype)] if out_dtype is not None else q.dtype
    return torch.empty(q.shape, dtype=dt, device=q.device)


def attend(cache: _Cache, q: torch.Tensor, at: int, scale: float | None = None, *, out=None, out_dtype=None):
    """Reduce query rows q [rows, hq*head_dim] at positions at.. over the cache.

    ``scale=None`` is the Gemma form (scores are plain dot products);
    otherwise scores are ``scale * dot`` (the Qwen form, scale 1/sqrt(head_dim)).
    """
    q = _dev(q)
    if q.dim() == 1:
        q = q.unsqueeze(0)
    if q.shape[-1] % cache.head_dim:
        raise _lib.InvalidArgument("attend: query width is not a whole number of heads")
    hq = q.shape[-1] // cache.head_dim
    out = _out(q, out, out_dtype)
    call("nmg_attend", cache.handle, hq, _ptr(q), _DT[q.dtype], q.shape[0], int(at),
         float(scale if scale is not None else 1.0), 0 if scale is None else 1, _ptr(out), _DT[out.dtype],
         _stream(q.device))
    return out


def append_attend(cache: _Cache, position: int, key: torch.Tensor, value: torch.Tensor, q: torch.Tensor,
                  scale: float | None = None, *, out=None, out_dtype=None):
    """Append rows at position.. then reduce the matching queries, as a layer does."""
    key, value, q = _dev(key), _dev(value), _dev(q)
    hq = q.shape[-1] // cache.head_dim
    out = _out(q, out, out_dtype)
    call("nmg_append_attend", cache.handle, int(position), _ptr(key), _ptr(value), _DT[key.dtype], hq, _ptr(q),
         _DT[q.dtype], q.shape[0], float(scale if scale is not None else 1.0), 0 if scale is None else 1, _ptr(out),
         _DT[out.dtype], _stream(q.device))
    return out


def attend_batch(caches, q: torch.Tensor, scale: float | None = None, *, queries_at=None, out=None, out_dtype=None):
    """One decode query per cache: q [batch, hq*head_dim]."""
    q = _dev(q)
    n = len(caches)
    arr = (ctypes.c_void_p * n)(*[c.handle.value for c in caches])
    qa = None
    if queries_at is not None:
        qa = (ctypes.c_int64 * n)(*[int(x) for x in queries_at])
    hq = q.shape[-1] // caches[0].head_dim
    out = _out(q, out, out_dtype)
    call("nmg_attend_batch", arr, n, qa, hq, _ptr(q), _DT[q.dtype], float(scale if scale is not None else 1.0),
         0 if scale is None else 1, _ptr(out), _DT[out.dtype], _stream(q.device))
    return out


def scaled_dot_product_attention(q, k, v, heads: int, scale: float, *, out=None, out_dtype=None):
    """softmax_rows(scale * Q K^T) V per head, no mask (src/attention.hpp:124-139)."""
    q, k, v = _dev(q), _dev(k), _dev(v)
    if k.shape[0] != v.shape[0]:
        raise _lib.InvalidArgument("scaled_dot_product_attention: K/V row mismatch")
    head_dim = q.shape[-1] // heads
    out = _out(q, out, out_dtype)
    call("nmg_sdpa", heads, head_dim, _ptr(q), _ptr(k), _ptr(v), _DT[q.dtype], q.shape[0], k.shape[0], float(scale),
         _ptr(out), _DT[out.dtype], _stream(q.device))
    return out


class DeltaNetState:
    """Device fp32 [heads][dk][dv] state, zero-initialised (src/recurrent.hpp:117-138)."""

    def __init__(self, heads: int, dk: int, dv: int, device: int = 0):
        self.heads, self.dk, self.dv, self.device = int(heads), int(dk), int(dv), int(device)
        h = ctypes.c_void_p()
        call("nmg_delta_create", self.heads, self.dk, self.dv, self.device, ctypes.byref(h))
        self._h = h
        p = ctypes.c_void_p()
        call("nmg_delta_head", self._h, 0, ctypes.byref(p))
        self._base = p.value

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.lib().nmg_delta_destroy(h)
            except Exception:
                pass
            self._h = None

    @property
    def handle(self):
        return self._h

    def clear(self) -> None:
        call("nmg_delta_clear", self._h, _stream(self.device))

    def head_ptr(self, h: int) -> int:
        p = ctypes.c_void_p()
        call("nmg_delta_head", self._h, int(h), ctypes.byref(p))
        return p.value

    def tensor(self) -> torch.Tensor:
        """A torch view of the whole device state (no copy)."""
        n = self.heads * self.dk * self.dv
        storage = _from_ptr(self._base, n, self.device)
        return storage.view(self.heads, self.dk, self.dv)

    def head(self, h: int) -> torch.Tensor:
        self.head_ptr(h)  # range check, OutOfRange like recurrent.hpp:128
        return self.tensor()[h]


def _from_ptr(ptr: int, n: int, device: int, dtype=torch.float32) -> torch.Tensor:
    """Wrap n device values at ptr as a tensor (the owner keeps them alive)."""
    typestr, view = {torch.float32: ("<f4", None), torch.float16: ("<f2", None),
                     torch.bfloat16: ("<i2", torch.bfloat16), torch.int8: ("|i1", None),
                     torch.int16: ("<i2", None)}[dtype]

    class _Holder:
        def __init__(self, p, n, dev):
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (p, False), "version": 3,
                                             "strides": None}
            self.dev = dev

    with torch.cuda.device(device):
        t = torch.as_tensor(_Holder(ptr, n, device), device=f"cuda:{device}")
    return t.view(view) if view is not None else t


def gated_delta_step(state_head: torch.Tensor, q, k, v, gate, beta) -> torch.Tensor:
    """One head, one token (src/recurrent.hpp:146-177); state_head [dk, dv] updated in place.

    gate/beta are device tensors of one element (so a CUDA graph can replay the step).
    """
    dk, dv = state_head.shape
    out = torch.empty(dv, dtype=torch.float32, device=state_head.device)
    gate = torch.as_tensor(gate, dtype=torch.float32, device=state_head.device).reshape(1)
    beta = torch.as_tensor(beta, dtype=torch.float32, device=state_head.device).reshape(1)
    call("nmg_gated_delta_step", ctypes.c_void_p(state_head.data_ptr()), dk, dv, _ptr(_dev(q)), _ptr(_dev(k)),
         _ptr(_dev(v)), _ptr(gate), _ptr(beta), _ptr(out), _stream(state_head.device))
    return out


def delta_step(state: DeltaNetState, q, k, v, gate, beta, hk: int, *, out=None) -> torch.Tensor:
    """One token through every value head (src/qwen35.hpp:449-454)."""
    if out is None:
        out = torch.empty(state.heads, state.dv, dtype=torch.float32, device=q.device)
    call("nmg_delta_step", state.handle, int(hk), _ptr(_dev(q)), _ptr(_dev(k)), _ptr(_dev(v)), _ptr(_dev(gate)),
         _ptr(_dev(beta)), _ptr(out), _stream(q.device))
    return out


def delta_step_batch(states, q, k, v, gate, beta, hk: int, *, out=None) -> torch.Tensor:
    """One decode token for each sequence of a batch, each with its own state:
    q,k [B,hk,dk], v [B,heads,dv], gate/beta [B,heads]; returns [B,heads,dv]."""
    n = len(states)
    s0 = states[0]
    if out is None:
        out = torch.empty(n, s0.heads, s0.dv, dtype=torch.float32, device=v.device)
    arr = (ctypes.c_void_p * n)(*[st.handle.value for st in states])
    call("nmg_delta_step_batch", arr, n, int(hk), _ptr(_dev(q)), _ptr(_dev(k)), _ptr(_dev(v)), _ptr(_dev(gate)),
         _ptr(_dev(beta)), _ptr(out), _stream(v.device))
    return out


def delta_prefill(state: DeltaNetState, q, k, v, gate, beta, hk: int, *, chunk: int = 64, out=None) -> torch.Tensor:
    """T tokens of the recurrence: q,k [T,hk,dk], v [T,heads,dv], gate/beta [T,heads]."""
    T = v.shape[0]
    if out is None:
        out = torch.empty(T, state.heads, state.dv, dtype=torch.float32, device=v.device)
    call("nmg_delta_prefill", state.handle, int(hk), T, _ptr(_dev(q)), _ptr(_dev(k)), _ptr(_dev(v)), _ptr(_dev(gate)),
         _ptr(_dev(beta)), _ptr(out), int(chunk), _stream(v.device))
    return out


# ---- the steps either side of the attention reduction (src/qwen35.hpp:343-393)

def attn_prologue(cache: _Cache, position: int, q, k, v, q_gamma, k_gamma, eps: float, rope_base: float,
                  rotary_num: int = 1, rotary_den: int = 1, *, gated: bool = True, v_norm: bool = False,
                  q_dtype=None) -> torch.Tensor:
    """Prepare one attention layer's Q, K, V for the reduction and append K, V to the cache.

    Q = rope(rmsnorm_per_head(q)), K = rope(rmsnorm_per_head(k)); V as given, or
    rmsnorm_no_scale_per_head(v) with v_norm (Gemma 4).  With gated (Qwen 3.5),
    q is the [T, 2*hq*dh] query projection in head-major [q | gate] pairs;
    otherwise q is [T, hq*dh].  Returns Q [T, hq*dh] in q_dtype (default: the
    cache's dtype); the cache gains rows position .. position + T - 1."""
    q = _dev(q)
    T = q.shape[0]
    hq = q.shape[1] // ((2 if gated else 1) * cache.head_dim)
    q_dtype = q_dtype or _TORCH[cache.dtype]
    out = torch.empty(T, hq * cache.head_dim, dtype=q_dtype, device=q.device)
    call("nmg_attn_prologue", cache.handle, int(hq), int(position), T, _ptr(q), int(bool(gated)), _ptr(_dev(k)),
         _ptr(_dev(v)), _ptr(_dev(q_gamma)), _ptr(_dev(k_gamma)), int(bool(v_norm)), float(eps), float(rope_base),
         int(rotary_num), int(rotary_den), _ptr(out), _DT[q_dtype], _stream(q.device))
    return out


def attn_prepare(hkv: int, head_dim: int, position: int, q, k, v, q_gamma, k_gamma, eps: float, rope_base: float,
                 rotary_num: int = 1, rotary_den: int = 1, *, gated: bool = True, v_norm: bool = False,
                 q_dtype=torch.float32):
    """attn_prologue without a cache: returns (Q [T, hq*dh] in q_dtype, K [T, hkv*dh] fp32,
    V [T, hkv*dh] fp32 -- v itself unless v_norm), for nm.append_attend."""
    q, k, v = _dev(q), _dev(k), _dev(v)
    T = q.shape[0]
    hq = q.shape[1] // ((2 if gated else 1) * head_dim)
    qo = torch.empty(T, hq * head_dim, dtype=q_dtype, device=q.device)
    ko = torch.empty(T, hkv * head_dim, dtype=torch.float32, device=q.device)
    vo = torch.empty_like(ko) if v_norm else v
    call("nmg_attn_prepare", int(hq), int(hkv), int(head_dim), int(position), T, _ptr(q), int(bool(gated)), _ptr(k),
         _ptr(v), _ptr(_dev(q_gamma)), _ptr(_dev(k_gamma)), int(bool(v_norm)), float(eps), float(rope_base),
         int(rotary_num), int(rotary_den), _ptr(qo), _DT[q_dtype], _ptr(ko), _ptr(vo) if v_norm else None,
         _stream(q.device))
    return qo, ko, vo


def attn_gate(qg, a: torch.Tensor, head_dim: int) -> torch.Tensor:
    """a [T, hq*head_dim] *= sigmoid(gate) in place, the gates the second halves of qg's
    [T, 2*hq*head_dim] head pairs; returns a."""
    qg = _dev(qg)
    a2 = a.reshape(a.shape[0], -1) if a.is_contiguous() else None
    if a2 is None or not a.is_cuda or a2.shape[0] != qg.shape[0] or 2 * a2.shape[1] != qg.shape[1] \
            or a2.shape[1] % head_dim:
        raise ValueError("attn_gate: a must be a contiguous device tensor [T, hq*head_dim] beside qg [T, 2*hq*head_dim]")
    call("nmg_attn_gate", a2.shape[0], a2.shape[1] // head_dim, int(head_dim), _ptr(qg), _ptr(a2), _DT[a.dtype],
         _stream(a.device))
    return a


# ---- the steps either side of the recurrence (src/qwen35.hpp:420-461) -------

class ConvState:
    """Device CausalConv1dState<channels, width> (src/recurrent.hpp:63-110): the
    last width - 1 inputs of a depthwise causal conv, zero (the causal pad)."""

    def __init__(self, channels: int, width: int, device: int = 0):
        self.channels, self.width, self.device = int(channels), int(width), int(device)
        h = ctypes.c_void_p()
        call("nmg_conv_create", self.channels, self.width, self.device, ctypes.byref(h))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.lib().nmg_conv_destroy(h)
            except Exception:
                pass
            self._h = None

    @property
    def handle(self):
        return self._h

    def clear(self) -> None:
        call("nmg_conv_clear", self._h, _stream(self.device))

    def history(self) -> torch.Tensor:
        """A torch view [width - 1, channels] of the carried inputs, oldest first (no copy)."""
        p = ctypes.c_void_p()
        call("nmg_conv_history", self._h, ctypes.byref(p))
        rows = max(self.width - 1, 1)
        return _from_ptr(p.value, rows * self.channels, self.device).view(rows, self.channels)

    def step(self, weights, x, *, silu: bool = False, out=None) -> torch.Tensor:
        """step() over T tokens: x [T, channels] -> y [T, channels]; weights [channels, width]."""
        x = _dev(x)
        if x.dim() == 1:
            x = x.unsqueeze(0)
        if out is None:
            out = torch.empty_like(x, dtype=torch.float32)
        call("nmg_conv_step", self._h, _ptr(_dev(weights)), _ptr(x), x.shape[0], _ptr(out), 1 if silu else 0,
             _stream(x.device))
        return out


def delta_prologue(conv: ConvState, conv_weights, qkv, beta_raw, alpha_raw, dt_bias, decay_scale, hk: int, hv: int,
                   dk: int, dv: int):
    """The packed projection qkv [T, 2*hk*dk + hv*dv] -> (q [T,hk,dk], k [T,hk,dk],
    v [T,hv,dv], beta [T,hv], gate [T,hv]) as qwen35.hpp:396-446 builds them."""
    qkv = _dev(qkv)
    T, dev = qkv.shape[0], qkv.device
    q = torch.empty(T, hk, dk, dtype=torch.float32, device=dev)
    k = torch.empty(T, hk, dk, dtype=torch.float32, device=dev)
    v = torch.empty(T, hv, dv, dtype=torch.float32, device=dev)
    beta = torch.empty(T, hv, dtype=torch.float32, device=dev)
    gate = torch.empty(T, hv, dtype=torch.float32, device=dev)
    call("nmg_delta_prologue", conv.handle, _ptr(_dev(conv_weights)), int(hk), int(hv), int(dk), int(dv), T, _ptr(qkv),
         _ptr(_dev(beta_raw)), _ptr(_dev(alpha_raw)), _ptr(_dev(dt_bias)), _ptr(_dev(decay_scale)), _ptr(q), _ptr(k),
         _ptr(v), _ptr(beta), _ptr(gate), _stream(dev))
    return q, k, v, beta, gate


def delta_epilogue(o, z, gamma, eps: float = 1e-6, *, out=None) -> torch.Tensor:
    """RMSNorm per head then SiLU(z) gate (qwen35.hpp:458-460): o, z [T, hv, dv], gamma [dv]."""
    o, z = _dev(o), _dev(z)
    T, hv, dv = o.shape
    if out is None:
        out = torch.empty_like(o)
    call("nmg_delta_epilogue", int(hv), int(dv), T, _ptr(o), _ptr(z), _ptr(_dev(gamma)), float(eps), _ptr(out),
         _stream(o.device))
    return out


def delta_decode_token(state: DeltaNetState, conv: ConvState, conv_weights, qkv, beta_raw, alpha_raw, dt_bias,
                       decay_scale, hk: int, z, gamma, eps: float = 1e-6, *, out=None) -> torch.Tensor:
    """One decode token of the layer core in one launch (qwen35.hpp:396-461 at
    T = 1): delta_prologue, delta_step and delta_epilogue fused.  qkv
    [2*hk*dk + hv*dv], beta_raw/alpha_raw [hv], z [hv, dv]; returns [hv, dv]."""
    qkv = _dev(qkv)
    if out is None:
        out = torch.empty(state.heads, state.dv, dtype=torch.float32, device=qkv.device)
    call("nmg_delta_decode_token", state.handle, conv.handle, _ptr(_dev(conv_weights)), int(hk), _ptr(qkv),
         _ptr(_dev(beta_raw)), _ptr(_dev(alpha_raw)), _ptr(_dev(dt_bias)), _ptr(_dev(decay_scale)), _ptr(_dev(z)),
         _ptr(_dev(gamma)), float(eps), _ptr(out), _stream(qkv.device))
    return out


# ---- quantised projections (src/quant.hpp, src/quant_i8.hpp) -----------------

class GT:
    """GGUF tensor types (src/quant.hpp:18-27); Q8_K is the activation block type."""
    F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 0, 1, 2, 8, 12, 13, 14, 15, 30


def type_size_bytes(gt: int, nelem: int) -> int:
    """Bytes of `nelem` values stored as `gt` (src/quant.hpp:89-108)."""
    b = ctypes.c_int64()
    call("nmg_weight_row_bytes", int(gt), int(nelem), ctypes.byref(b))
    return b.value


def _fp32_act_default() -> bool:
    e = os.environ.get("NM_FP32_ACT", "")
    return bool(e) and e[0] != "0"


class Weight:
    """Weight<In,Out> over GGUF bytes (src/quant.hpp:439-487), held on the device.

    ``data``: ``out * type_size_bytes(gt, in_features)`` bytes, one row per
    output, as a numpy/bytes buffer (host) or a uint8 CUDA tensor.  Products
    follow the reference's activation handling: quantised Q8_0/Q8_K
    activations and integer block dots for Q8_0, Q4_0, Q4_K and Q6_K, fp32
    otherwise; ``fp32_act`` (default: the NM_FP32_ACT environment variable,
    src/quant_i8.hpp:343-349) selects the fp32-activation path for every type."""

    def __init__(self, gt: int, in_features: int, out_features: int, data, device: int = 0,
                 fp32_act: bool | None = None):
        self.gt, self.in_features, self.out_features, self.device = int(gt), int(in_features), int(out_features), int(device)
        self.fp32_act = _fp32_act_default() if fp32_act is None else bool(fp32_act)
        h = ctypes.c_void_p()
        if isinstance(data, torch.Tensor):
            if not data.is_cuda:
                data = data.contiguous().numpy()
            else:
                data = data.contiguous()
                call("nmg_weight_create", self.gt, self.in_features, self.out_features, ctypes.c_void_p(data.data_ptr()),
                     1, self.device, ctypes.byref(h))
        if not h.value:
            buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8) if isinstance(data, (bytes, bytearray))
                                       else np.asarray(data).view(np.uint8).reshape(-1))
            call("nmg_weight_create", self.gt, self.in_features, self.out_features, ctypes.c_void_p(buf.ctypes.data), 0,
                 self.device, ctypes.byref(h))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.lib().nmg_weight_destroy(h)
            except Exception:
                pass
            self._h = None

    @property
    def handle(self):
        return self._h

    def type(self) -> int:
        t = ctypes.c_int()
        call("nmg_weight_info", self._h, ctypes.byref(t), None, None)
        return t.value

    def row_bytes(self) -> int:
        return type_size_bytes(self.gt, self.in_features)

    def _act(self) -> int:
        return 1 if self.fp32_act else 0

    def matvec(self, x: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
        """y[out] = W x for a device fp32 x[in] (src/quant_i8.hpp:351-428)."""
        x = _dev(x).float().contiguous()
        if x.numel() != self.in_features:
            raise ValueError(f"matvec: {x.numel()} values for In={self.in_features}")
        if out is None:
            out = torch.empty(self.out_features, dtype=torch.float32, device=x.device)
        call("nmg_weight_matvec", self._h, _ptr(x), _ptr(out), self._act(), _stream(x.device))
        return out

    def matmul(self, x: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
        """Y[rows][out] for device fp32 X[rows][in] (src/quant_i8.hpp:430-514)."""
        x = _dev(x).float().contiguous()
        if x.dim() != 2 or x.shape[1] != self.in_features:
            raise ValueError(f"matmul: activations {tuple(x.shape)} for In={self.in_features}")
        if out is None:
            out = torch.empty(x.shape[0], self.out_features, dtype=torch.float32, device=x.device)
        call("nmg_weight_matmul", self._h, int(x.shape[0]), _ptr(x), _ptr(out), self._act(), _stream(x.device))
        return out

    def gather_rows(self, rows) -> torch.Tensor:
        """Rows dequantised to fp32 [len(rows)][in] (src/quant.hpp:469-475)."""
        ids = np.ascontiguousarray(np.asarray(rows, dtype=np.int32).reshape(-1))
        out = torch.empty(len(ids), self.in_features, dtype=torch.float32, device=f"cuda:{self.device}")
        call("nmg_weight_gather_rows", self._h, ctypes.c_void_p(ids.ctypes.data), len(ids), _ptr(out),
             _stream(self.device))
        return out

    def dequant_row(self, o: int) -> torch.Tensor:
        return self.gather_rows([o])[0]


def quantize_activations(x: torch.Tensor, act_type: int) -> torch.Tensor:
    """quantize_row_q8_0 / quantize_row_q8_K of each row of device fp32 x
    [rows][n]: the reference's packed blocks as a uint8 tensor [rows][bytes]."""
    x = _dev(x).float().contiguous()
    x2 = x.view(-1, x.shape[-1])
    rb = type_size_bytes(act_type, x2.shape[1])
    out = torch.empty(x2.shape[0], rb, dtype=torch.uint8, device=x.device)
    call("nmg_quantize_activations", int(act_type), int(x2.shape[0]), int(x2.shape[1]), _ptr(x2), _ptr(out),
         _stream(x.device))
    return out


# ---- multi-GPU: output rows assembled by the attention epilogue -------------

class SharedRows:
    """A [rows, width] device buffer other processes of the node can map.

    ``handle`` (64 bytes) goes to the other ranks, which pass it to
    :func:`open_peer`; every rank then hands all ranks' pointers to
    :func:`attend_fanout`, whose epilogue writes its heads into each of them."""

    def __init__(self, rows: int, width: int, dtype=torch.bfloat16, device: int = 0):
        self.rows, self.width, self.dtype, self.device = int(rows), int(width), dtype, int(device)
        nbytes = self.rows * self.width * torch.tensor([], dtype=dtype).element_size()
        self._ptr = ctypes.c_void_p()
        h = (ctypes.c_char * 64)()
        call("nmg_shared_alloc", nbytes, self.device, ctypes.byref(self._ptr), h)
        self.handle = bytes(h)

    @property
    def ptr(self) -> int:
        return self._ptr.value

    def tensor(self) -> torch.Tensor:
        return _from_ptr(self.ptr, self.rows * self.width, self.device, self.dtype).view(self.rows, self.width)

    def close(self):
        if self._ptr.value:
            call("nmg_shared_free", self._ptr)
            self._ptr = ctypes.c_void_p()


def open_peer(handle: bytes, device: int) -> int:
    """Map another process's SharedRows into this one; returns the device pointer."""
    h = (ctypes.c_char * 64).from_buffer_copy(handle)
    p = ctypes.c_void_p()
    call("nmg_ipc_open", h, int(device), ctypes.byref(p))
    return p.value


def close_peer(ptr: int) -> None:
    call("nmg_ipc_close", ctypes.c_void_p(ptr))


def attend_fanout(cache: _Cache, q: torch.Tensor, at: int, scale: float | None, outs, row_elems: int, col0: int,
                  out_dtype=torch.bfloat16) -> None:
    """attend() with each output row written to every pointer in ``outs`` at
    column ``col0`` of rows ``row_elems`` elements long."""
    q = _dev(q)
    hq = q.shape[-1] // cache.head_dim
    arr = (ctypes.c_void_p * len(outs))(*[int(p) for p in outs])
    call("nmg_attend_fanout", cache.handle, hq, _ptr(q), _DT[q.dtype], q.shape[0], int(at),
         ctypes.c_float(scale if scale is not None else 1.0), 0 if scale is None else 1, arr, len(outs),
         int(row_elems), int(col0), _DT[out_dtype], _stream(q.device))
