"""Q8_0 K/V cache storage: the quantiser bit for bit, exact read-back, attention parity.

A Q8_0 cache keeps K and V as blocks of 32 int8 quants with an fp16 scale,
quantised on append exactly as the reference's quantize_row_q8_0
(src/quant_i8.hpp:69-81; the oracle's restatement is pinned to that function in
tests/test_oracle.py).  Attention over it must equal the reference reduction
(qwen35.hpp:360-382) over the dequantised rows (scale * quant, the values the
cache's key()/value() return) within max abs 2e-3 / rel L2 1e-3.
"""
import math

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close
from hero_b200 import _lib, nm

pytestmark = pytest.mark.gpu


def _rows(seed, n, width, scale=1.0):
    return (oracle.normal(seed, 1, n * width).reshape(n, width) * np.float32(scale)).astype(np.float32)


def _deq(x, hkv, dh):
    """The values a Q8_0 cache holds for rows x [n, hkv*dh] (the oracle quantiser)."""
    q, d = oracle.quantize_q8_0(x.reshape(-1, hkv, dh))
    return oracle.dequantize_q8_0(q, d).reshape(x.shape)


@pytest.mark.parametrize("src", [torch.float32, torch.float16, torch.bfloat16])
def test_append_quantises_like_the_reference(dev, src):
    hkv, dh, n = 2, 128, 300
    x = _rows(3, n, hkv * dh, 2.5)
    x[7, :32] = 0.0  # an all-zero block: d = 0, quants 0
    tie = np.float32(1.7) / np.float32(127)
    x[9, 32:64] = (np.arange(32, dtype=np.float32) - np.float32(15.5)) * tie  # values on half steps
    x[9, 32] = np.float32(1.7)
    xt = torch.from_numpy(x).to(dev).to(src)
    x_in = xt.float().cpu().numpy()  # the fp32 values the quantiser sees
    cache = nm.FullAttentionCache(hkv, dh, capacity=n, dtype="q8_0")
    cache.append(0, xt, xt * 0.5)
    torch.cuda.synchronize(dev)
    for h in range(hkv):
        kq, ks, vq, vs = cache.q8_blocks(h)
        wq, wd = oracle.quantize_q8_0(x_in.reshape(n, hkv, dh)[:, h])
        assert np.array_equal(kq[:n], wq) and np.array_equal(ks[:n], wd), f"K head {h}"
        wq, wd = oracle.quantize_q8_0((x_in * np.float32(0.5)).reshape(n, hkv, dh)[:, h]) if src == torch.float32 \
            else oracle.quantize_q8_0((xt * 0.5).float().cpu().numpy().reshape(n, hkv, dh)[:, h])
        assert np.array_equal(vq[:n], wq) and np.array_equal(vs[:n], wd), f"V head {h}"
    # key()/value() return scale * quant exactly
    deq = _deq(x_in, hkv, dh).reshape(n, hkv, dh)
    for row in (0, 7, 9, n - 1):
        assert np.array_equal(cache.key(row, 1).numpy(), deq[row, 1])


def test_ring_append_and_read_back(dev):
    # A sliding-window Q8_0 cache that wraps: chronological rows read back exactly.
    hkv, dh, W, cap = 1, 64, 100, 128
    x = _rows(5, 700, hkv * dh)
    cache = nm.LocalAttentionCache(hkv, dh, W, capacity=cap, dtype="q8_0")
    for s0 in range(0, 700, 70):
        cache.append(s0, torch.from_numpy(x[s0:s0 + 70]).to(dev), torch.from_numpy(x[s0:s0 + 70]).to(dev))
    deq = _deq(x, hkv, dh)
    first = cache.position(0)
    for row in (0, cache.size() // 2, cache.size() - 1):
        assert np.array_equal(cache.value(row, 0).numpy(), deq[first + row])


@pytest.mark.parametrize("q_dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_batched_decode_config5_shape(dev, q_dtype):
    # Config 5's heads (64 query heads over 8 K/V heads, head_dim 128) over
    # ragged Q8_0 caches, one query per sequence.
    hq, hkv, dh = 64, 8, 128
    lens = [4100, 777, 6000]
    caches, kv = [], []
    for i, L in enumerate(lens):
        k, v = _rows(20 + i, L, hkv * dh), _rows(40 + i, L, hkv * dh)
        c = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="q8_0")
        c.append(0, torch.from_numpy(k).to(dev).half(), torch.from_numpy(v).to(dev).half())
        caches.append(c)
        kv.append((_deq(oracle.round_fp16(k), hkv, dh), _deq(oracle.round_fp16(v), hkv, dh)))
    q = torch.from_numpy(_rows(60, len(lens), hq * dh)).to(dev).to(q_dtype)
    scale = 1.0 / math.sqrt(dh)
    out = nm.attend_batch(caches, q, scale, out_dtype=torch.float32).cpu().numpy()
    qh = q.float().cpu().numpy()
    for b, L in enumerate(lens):
        want = oracle.attend(kv[b][0], kv[b][1], 0, 0, hkv, dh, qh[b:b + 1], hq, L - 1, scale=np.float32(scale))
        assert_close(out[b:b + 1], want, what=f"sequence {b} ({L} rows)")


def test_batched_decode_gemma_global_shape(dev):
    # Config 4's heads (8 query heads over 4 K/V heads, head_dim 256, scale 1)
    # over ragged Q8_0 caches filled from bf16 rows: the fragments built from
    # the quants in registers at head_dim 256, with key splits merged.
    hq, hkv, dh = 8, 4, 256
    lens = [9000, 130, 4097]
    caches, kv = [], []
    for i, L in enumerate(lens):
        k, v = oracle.round_bf16(_rows(80 + i, L, hkv * dh)), oracle.round_bf16(_rows(90 + i, L, hkv * dh))
        c = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="q8_0")
        c.append(0, torch.from_numpy(k).to(dev).bfloat16(), torch.from_numpy(v).to(dev).bfloat16())
        caches.append(c)
        kv.append((_deq(k, hkv, dh), _deq(v, hkv, dh)))
    q = torch.from_numpy(_rows(99, len(lens), hq * dh, 0.1)).to(dev).bfloat16()
    out = nm.attend_batch(caches, q, None, out_dtype=torch.float32).cpu().numpy()
    qh = q.float().cpu().numpy()
    for b, L in enumerate(lens):
        want = oracle.attend(kv[b][0], kv[b][1], 0, 0, hkv, dh, qh[b:b + 1], hq, L - 1, use_scale=False)
        assert_close(out[b:b + 1], want, what=f"sequence {b} ({L} rows)")


@pytest.mark.parametrize("dh,hq,hkv", [(64, 4, 2), (128, 8, 2), (128, 32, 2), (256, 8, 4)])
def test_rows_and_window_decode(dev, dh, hq, hkv):
    # Several query rows over a wrapped sliding-window Q8_0 cache (scale 1, the
    # Gemma form), at head dims 64, 128 (groups of 4, fragments built from the
    # quants in registers, and of 16, converted through shared memory) and 256.
    W, cap, total = 300, 512, 1400
    k, v = _rows(71, total, hkv * dh), _rows(72, total, hkv * dh)
    q = _rows(73, 5, hq * dh, 0.1)
    cache = nm.LocalAttentionCache(hkv, dh, W, capacity=cap, dtype="q8_0")
    for s0 in range(0, total, 200):
        cache.append(s0, torch.from_numpy(k[s0:s0 + 200]).to(dev), torch.from_numpy(v[s0:s0 + 200]).to(dev))
    oldest = cache.position(0)
    out = nm.attend(cache, torch.from_numpy(q).to(dev), total - 5, None).cpu().numpy()
    kd, vd = _deq(k, hkv, dh)[oldest:], _deq(v, hkv, dh)[oldest:]
    want = oracle.attend(kd, vd, oldest, W, hkv, dh, q, hq, total - 5, use_scale=False)
    assert_close(out, want, what=f"window decode dh={dh}")


def test_prologue_appends_quantised_rows(dev):
    # The attention prologue into a Q8_0 cache: RoPE'd K quantised on append.
    hq, hkv, dh, T = 4, 2, 128, 40
    qg, k, v = _rows(81, T, 2 * hq * dh), _rows(82, T, hkv * dh), _rows(83, T, hkv * dh)
    gam = np.ones(dh, np.float32)
    cache = nm.FullAttentionCache(hkv, dh, capacity=64, dtype="q8_0")
    t = lambda a: torch.from_numpy(a).to(dev)
    nm.attn_prologue(cache, 0, t(qg), t(k), t(v), t(gam), t(gam), 1e-6, 1e7, 1, 4, q_dtype=torch.float32)
    _, ko, vo = oracle.attn_prologue(qg, k, v, gam, gam, hq, hkv, dh, 0, 1e-6, 1e7, 1, 4)
    kd = _deq(ko, hkv, dh).reshape(T, hkv, dh)
    vd = _deq(vo, hkv, dh).reshape(T, hkv, dh)
    for row in (0, T - 1):
        for h in range(hkv):
            assert np.abs(cache.key(row, h).numpy() - kd[row, h]).max() <= 1e-6 + 0.01 * np.abs(kd[row, h]).max()
            assert np.array_equal(cache.value(row, h).numpy(), vd[row, h])


def test_unsupported_uses_are_refused(dev):
    cache = nm.FullAttentionCache(1, 64, capacity=64, dtype="q8_0")
    x = torch.randn(8, 64, device=dev)
    cache.append(0, x, x)
    import ctypes

    out = torch.empty(1, 64, device=dev)
    q = torch.randn(1, 64, device=dev)
    st = _lib.lib().nmg_attend_noalloc(cache.handle, 1, ctypes.c_void_p(q.data_ptr()), _lib.F32, 1, 7,
                                       ctypes.c_float(1.0), 1, ctypes.c_void_p(out.data_ptr()), _lib.F32,
                                       ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert st == _lib.UNSUPPORTED
    with pytest.raises(_lib.Unsupported):
        nm.FullAttentionCache(1, 48, capacity=64, dtype="q8_0")
