"""nmg_attend_noalloc, the decode entry point for callers that cannot allocate device memory.

Some callers may not call cudaMalloc: engines whose device memory belongs to
their own arena allocator, or serving loops that cannot afford the device-wide
synchronisation an allocation can cause.  This entry point keeps its scratch in
a fixed device array instead.  Here it must agree with the allocating entry
point (nmg_attend) within the suite's tolerance, on two calls in a row (the
second call finds the first call's leftovers in the shared array).

The file sorts last so that a failure here never hides the rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from helpers import MAX_ABS, REL_L2, assert_close
from hero_b200 import _lib, nm

pytestmark = pytest.mark.gpu


def _call(fn, cache, q, first_query, scale, out, use_scale=1):
    L = _lib.lib()
    hq = q.shape[1] // cache.head_dim
    stream = ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)
    code = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}
    _lib.check(getattr(L, fn)(cache.handle, hq, ctypes.c_void_p(q.data_ptr()), code[q.dtype], q.shape[0],
                              first_query, ctypes.c_float(scale), use_scale, ctypes.c_void_p(out.data_ptr()),
                              code[out.dtype], stream))


@pytest.mark.parametrize("dtype,hq,hkv,dh,rows", [("f32", 16, 8, 128, 1024), ("bf16", 8, 4, 256, 20000),
                                                   ("f16", 64, 8, 128, 9000)])
def test_noalloc_matches_nmg_attend_twice(dev, dtype, hq, hkv, dh, rows):
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    g = torch.Generator(device=dev)
    g.manual_seed(rows)
    cache = nm.FullAttentionCache(hkv, dh, capacity=rows, dtype=dtype)
    cache.append(0, torch.randn(rows, hkv * dh, device=dev, generator=g).to(tdt),
                 torch.randn(rows, hkv * dh, device=dev, generator=g).to(tdt))
    scale = 1.0 / np.sqrt(dh)
    for call in range(2):
        q = torch.randn(1, hq * dh, device=dev, generator=g).to(tdt)
        want = torch.empty(1, hq * dh, device=dev)
        got = torch.full((1, hq * dh), float("nan"), device=dev)
        _call("nmg_attend", cache, q, rows - 1, scale, want)
        _call("nmg_attend_noalloc", cache, q, rows - 1, scale, got)
        torch.cuda.synchronize(dev)
        assert_close(got.cpu().numpy(), want.cpu().numpy(), MAX_ABS, REL_L2, what=f"{dtype} call {call}")


def test_noalloc_against_the_oracle(dev):
    hq, hkv, dh, rows = 4, 2, 64, 3000
    k = oracle.normal(21, 1, rows * hkv * dh).reshape(rows, -1)
    v = oracle.normal(21, 2, rows * hkv * dh).reshape(rows, -1)
    q = oracle.normal(21, 3, hq * dh).reshape(1, -1)
    cache = nm.FullAttentionCache(hkv, dh, capacity=rows)
    cache.append(0, torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev))
    out = torch.empty(1, hq * dh, device=dev)
    for _ in range(2):
        _call("nmg_attend_noalloc", cache, torch.from_numpy(q).to(dev), rows - 1, 0.125, out)
        want = oracle.attend(k, v, 0, 0, hkv, dh, q, hq, rows - 1, scale=np.float32(0.125))
        assert_close(out.cpu().numpy(), want, what="noalloc vs oracle")


def test_noalloc_rejects_work_beyond_its_fixed_scratch(dev):
    # thousands of query rows need far more than the fixed array holds
    hkv, dh, rows = 8, 128, 4096
    cache = nm.FullAttentionCache(hkv, dh, capacity=rows)
    cache.append(0, torch.zeros(rows, hkv * dh, device=dev), torch.zeros(rows, hkv * dh, device=dev))
    q = torch.zeros(rows, 64 * dh, device=dev)
    out = torch.empty_like(q)
    with pytest.raises(_lib.LengthError, match="scratch"):
        _call("nmg_attend_noalloc", cache, q, 0, 1.0, out)


def test_noalloc_wrapped_window_and_several_rows(dev):
    # A sliding-window cache whose ring has wrapped (positions far beyond the
    # physical slots), with 8 query rows whose windows start at different
    # positions: the window floor and the per-row split arithmetic.
    hq, hkv, dh, W, cap = 8, 4, 128, 1024, 1536
    g = torch.Generator(device=dev)
    g.manual_seed(12)
    cache = nm.LocalAttentionCache(hkv, dh, W, capacity=cap, dtype="f16")
    total = 5000
    kf = torch.randn(total, hkv * dh, device=dev, generator=g).half()
    vf = torch.randn(total, hkv * dh, device=dev, generator=g).half()
    for s0 in range(0, total, 500):
        cache.append(s0, kf[s0:s0 + 500], vf[s0:s0 + 500])
    rows = 8
    q = torch.randn(rows, hq * dh, device=dev, generator=g).half()
    first = total - rows
    want = torch.empty(rows, hq * dh, device=dev)
    _call("nmg_attend", cache, q, first, dh ** -0.5, want)
    oldest = cache.position(0)
    kk = kf[oldest:].float().cpu().numpy()
    vv = vf[oldest:].float().cpu().numpy()
    ref = oracle.attend(kk, vv, oldest, W, hkv, dh, q.float().cpu().numpy(), hq, first, scale=np.float32(dh ** -0.5))
    for call in range(2):
        got = torch.full((rows, hq * dh), float("nan"), device=dev)
        _call("nmg_attend_noalloc", cache, q, first, dh ** -0.5, got)
        torch.cuda.synchronize(dev)
        assert_close(got.cpu().numpy(), want.cpu().numpy(), what=f"noalloc vs nmg_attend, call {call}")
        assert_close(got.cpu().numpy(), ref, what=f"noalloc vs oracle, call {call}")


def test_noalloc_wide_heads_long_cache(dev):
    # Gemma 4 12B's full-attention layers: head_dim 512, 16 query heads over
    # one K/V head, bf16 cache, one decode row over 40000 keys.  The fixed
    # array holds this row's partials only with longer splits than
    # nmg_attend would pick.
    hq, hkv, dh, rows = 16, 1, 512, 40000
    g = torch.Generator(device=dev)
    g.manual_seed(13)
    cache = nm.FullAttentionCache(hkv, dh, capacity=rows, dtype="bf16")
    k = torch.randn(rows, hkv * dh, device=dev, generator=g).bfloat16()
    v = torch.randn(rows, hkv * dh, device=dev, generator=g).bfloat16()
    cache.append(0, k, v)
    q = (torch.randn(1, hq * dh, device=dev, generator=g) * 0.05).bfloat16()
    want = torch.empty(1, hq * dh, device=dev)
    _call("nmg_attend", cache, q, rows - 1, 1.0, want, use_scale=0)
    ref = oracle.attend(k.float().cpu().numpy(), v.float().cpu().numpy(), 0, 0, hkv, dh,
                        q.float().cpu().numpy(), hq, rows - 1, use_scale=False)
    for call in range(2):
        got = torch.full((1, hq * dh), float("nan"), device=dev)
        _call("nmg_attend_noalloc", cache, q, rows - 1, 1.0, got, use_scale=0)
        torch.cuda.synchronize(dev)
        assert_close(got.cpu().numpy(), want.cpu().numpy(), what=f"dh512 noalloc vs nmg_attend, call {call}")
        assert_close(got.cpu().numpy(), ref, what=f"dh512 noalloc vs oracle, call {call}")


def test_noalloc_wait_timeout_survives_the_next_call(dev):
    # A wait that gave up in this path raises the path's own error word, which
    # the next call must not erase: nmg_device_status reports it afterwards.
    hq, hkv, dh, rows = 4, 2, 64, 512
    cache = nm.FullAttentionCache(hkv, dh, capacity=rows)
    cache.append(0, torch.randn(rows, hkv * dh, device=dev), torch.randn(rows, hkv * dh, device=dev))
    q = torch.randn(1, hq * dh, device=dev)
    out = torch.empty(1, hq * dh, device=dev)
    nm.device_status(0)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.call("nmg_selftest_wait_timeout", 0, 1, stream)
    _call("nmg_attend_noalloc", cache, q, rows - 1, 0.125, out)
    with pytest.raises(_lib.DeviceTimeout):
        nm.device_status(0)
    _call("nmg_attend_noalloc", cache, q, rows - 1, 0.125, out)
    nm.device_status(0)
