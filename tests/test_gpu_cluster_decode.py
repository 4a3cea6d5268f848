"""The fp32 decode kernel (cluster merge and ticket merge) against the oracle.

fp32 caches at head_dim 128 / 256 decode on 8-warp CTAs whose key splits meet
in distributed shared memory (short decodes) or through global partials and a
ticket (long decodes over few heads).  Checked here across GQA groups 1-8 (and
an odd group), split counts from one to eight (short caches leave splits
empty), query rows that each see a different window of a wrapped ring, ragged
batches, fp16 / bf16 queries and outputs, and repeat calls, all against the
reference reduction (qwen35.hpp:360-382, gemma4.hpp:593-615) within max abs
2e-3 / rel L2 1e-3.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close
from hero_b200 import nm

pytestmark = pytest.mark.gpu


def _rows(seed, stream, n, width, scale=1.0):
    return (oracle.normal(seed, stream, n * width).reshape(n, width) * np.float32(scale)).astype(np.float32)


def _t(a, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dtype)


@pytest.mark.parametrize("hq,hkv,dh,L", [(16, 8, 128, 1024), (16, 8, 128, 1), (16, 8, 128, 65), (8, 8, 128, 1000),
                                         (24, 8, 128, 777), (32, 4, 128, 3000), (64, 8, 128, 2048),
                                         (8, 4, 256, 1024), (4, 4, 256, 300), (32, 4, 256, 1500)])
def test_decode_groups_and_lengths(dev, hq, hkv, dh, L):
    seed = hq + 7 * hkv + L
    k, v = _rows(seed, 1, L, hkv * dh), _rows(seed, 2, L, hkv * dh)
    q = _rows(seed, 3, 1, hq * dh)
    cache = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="f32")
    cache.append(0, _t(k, dev), _t(v, dev))
    scale = float(np.float32(1 / np.sqrt(np.float32(dh))))
    out = nm.attend(cache, _t(q, dev), L - 1, scale, out_dtype=torch.float32).cpu().numpy()
    want = oracle.attend(k, v, 0, 0, hkv, dh, q, hq, L - 1, scale=np.float32(scale))
    assert_close(out, want, what=f"hq={hq} hkv={hkv} dh={dh} L={L}")


@pytest.mark.parametrize("dh", [128, 256])
def test_rows_over_a_wrapped_window(dev, dh):
    # Five query rows over a sliding-window cache whose ring has wrapped: each
    # row sees its own window, and key tiles straddle the ring's end.
    hq, hkv, W, cap, total = 8, 2, 700, 768, 2000
    k, v = _rows(31, 1, total, hkv * dh), _rows(31, 2, total, hkv * dh)
    q = _rows(31, 3, 5, hq * dh, 0.2)
    cache = nm.LocalAttentionCache(hkv, dh, W, capacity=cap, dtype="f32")
    for s0 in range(0, total, 250):
        cache.append(s0, _t(k[s0:s0 + 250], dev), _t(v[s0:s0 + 250], dev))
    oldest = cache.position(0)
    out = nm.attend(cache, _t(q, dev), total - 5, None, out_dtype=torch.float32).cpu().numpy()
    want = oracle.attend(k[oldest:], v[oldest:], oldest, W, hkv, dh, q, hq, total - 5, use_scale=False)
    assert_close(out, want, what=f"window rows dh={dh}")


@pytest.mark.parametrize("q_dtype,out_dtype", [(torch.float16, torch.float32), (torch.bfloat16, torch.bfloat16),
                                               (torch.float32, torch.float16)])
def test_ragged_batch_and_dtypes(dev, q_dtype, out_dtype):
    hq, hkv, dh = 16, 4, 128
    lens = [1, 40, 513, 1024, 2900, 130]
    caches, kv = [], []
    for i, L in enumerate(lens):
        k, v = _rows(50 + i, 1, L, hkv * dh), _rows(50 + i, 2, L, hkv * dh)
        c = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="f32")
        c.append(0, _t(k, dev), _t(v, dev))
        caches.append(c)
        kv.append((k, v))
    q = _t(_rows(70, 3, len(lens), hq * dh), dev, q_dtype)
    scale = 0.0883883
    out = nm.attend_batch(caches, q, scale, out_dtype=out_dtype).float().cpu().numpy()
    qh = q.float().cpu().numpy()
    for b, L in enumerate(lens):
        want = oracle.attend(kv[b][0], kv[b][1], 0, 0, hkv, dh, qh[b:b + 1], hq, L - 1, scale=np.float32(scale))
        if out_dtype == torch.float32:
            assert_close(out[b:b + 1], want, what=f"sequence {b} ({L} rows)")
        else:
            # the fp32 result rounded once to the output type
            rounded = oracle.round_bf16(want) if out_dtype == torch.bfloat16 else oracle.round_fp16(want)
            step = 2.0 ** -7 if out_dtype == torch.bfloat16 else 2.0 ** -10
            bound = 2e-3 + step * np.abs(want).max()
            assert np.abs(out[b:b + 1] - rounded.reshape(want.shape)).max() <= bound, f"sequence {b}, {out_dtype}"


def test_repeat_calls_agree_bit_for_bit(dev):
    # No tickets or scratch carry state from one call to the next.
    hq, hkv, dh, L = 16, 8, 128, 1024
    k, v = _rows(90, 1, L, hkv * dh), _rows(90, 2, L, hkv * dh)
    cache = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="f32")
    cache.append(0, _t(k, dev), _t(v, dev))
    q = _t(_rows(90, 3, 1, hq * dh), dev)
    first = nm.attend(cache, q, L - 1, 0.1)
    for _ in range(3):
        assert torch.equal(nm.attend(cache, q, L - 1, 0.1), first)


def test_long_fp32_decode_ticket_merge(dev):
    # One row over 20,000 fp32 keys (82 MB): too few (row, head) units for
    # clusters to fill the GPU, so the splits merge through global partials
    # and a ticket; the tickets return to zero, so repeat calls agree exactly.
    hq, hkv, dh, L = 16, 8, 128, 20000
    k, v = _rows(95, 1, L, hkv * dh), _rows(95, 2, L, hkv * dh)
    q = _rows(95, 3, 1, hq * dh)
    cache = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="f32")
    cache.append(0, _t(k, dev), _t(v, dev))
    qd = _t(q, dev)
    out = nm.attend(cache, qd, L - 1, 0.0883883, out_dtype=torch.float32)
    want = oracle.attend(k, v, 0, 0, hkv, dh, q, hq, L - 1, scale=np.float32(0.0883883))
    assert_close(out.cpu().numpy(), want, what="20000 fp32 keys")
    for _ in range(2):
        assert torch.equal(nm.attend(cache, qd, L - 1, 0.0883883, out_dtype=torch.float32), out)


def test_ragged_pair_ticket_merge(dev):
    # Two sequences (9000 and 300 rows) at head_dim 256: the short one leaves
    # most of its splits empty.
    hq, hkv, dh = 8, 4, 256
    lens = [9000, 300]
    caches, kv = [], []
    for i, L in enumerate(lens):
        k, v = _rows(97 + i, 1, L, hkv * dh), _rows(97 + i, 2, L, hkv * dh)
        c = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="f32")
        c.append(0, _t(k, dev), _t(v, dev))
        caches.append(c)
        kv.append((k, v))
    q = _rows(99, 3, 2, hq * dh, 0.1)
    out = nm.attend_batch(caches, _t(q, dev), None, out_dtype=torch.float32).cpu().numpy()
    for b, L in enumerate(lens):
        want = oracle.attend(kv[b][0], kv[b][1], 0, 0, hkv, dh, q[b:b + 1], hq, L - 1, use_scale=False)
        assert_close(out[b:b + 1], want, what=f"sequence {b} ({L} rows)")
