"""Head dim 512: the full-attention layers of Gemma 4 (FULL_HEAD_DIM = 512 in
nm/src/gemma4.hpp:26 and :505; one K/V head in the 12B, two in E4B) through the
split-KV kernel, prefill rows, decode and batched decode, against the oracle.

Tolerance as everywhere: max abs <= 2e-3 and rel L2 <= 1e-3 versus the fp32
reference path on identical pre-rounded inputs.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close
from hero_b200 import nm
from hero_b200._lib import Unsupported

pytestmark = pytest.mark.gpu
DH = 512
DT = {"bf16": torch.bfloat16, "f16": torch.float16}


def normed(code, seed, stream, rows, heads):
    """N(0,1) rows with a per-head RMS norm (unit gain, eps 1e-6), rounded to the cache dtype."""
    x = oracle.normal(seed, stream, rows * heads * DH).reshape(-1, DH).astype(np.float64)
    x = (x / np.sqrt((x * x).mean(axis=1, keepdims=True) + 1e-6)).astype(np.float32)
    r = oracle.round_bf16 if code == "bf16" else oracle.round_fp16
    return r(x).reshape(rows, heads * DH)


def plain(code, seed, stream, rows, heads):
    x = oracle.normal(seed, stream, rows * heads * DH)
    r = oracle.round_bf16 if code == "bf16" else oracle.round_fp16
    return r(x).reshape(rows, heads * DH)


def dev_t(a, dev, code):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(DT[code])


@pytest.mark.parametrize("code,hq,hkv,S,scaled", [("bf16", 16, 1, 300, False), ("f16", 8, 2, 2100, True)])
def test_full_layer_prefill_then_decode(dev, code, hq, hkv, S, scaled):
    # 12B full layer (Gemma scale 1, 16 query heads on one K/V head) and an
    # E4B-shaped one with an explicit score scale and enough keys for splits.
    scale = float(np.float32(1 / np.sqrt(DH))) if scaled else None
    k, q = normed(code, 21, 1, S, hkv), normed(code, 21, 3, S, hq)
    v = plain(code, 21, 2, S, hkv)
    cache = nm.FullAttentionCache(hkv, DH, capacity=S + 1, dtype=code)
    out = nm.append_attend(cache, 0, dev_t(k, dev, code), dev_t(v, dev, code), dev_t(q, dev, code), scale,
                           out_dtype=torch.float32).cpu().numpy()
    kw = dict(scale=np.float32(scale)) if scaled else dict(use_scale=False)
    rows = sorted({0, 1, 31, 32, 33, S // 2, S - 1} | set(np.random.default_rng(2).integers(0, S, 8).tolist()))
    for r in rows:
        want = oracle.attend(k[:r + 1], v[:r + 1], 0, 0, hkv, DH, q[r:r + 1], hq, r, **kw)
        assert_close(out[r:r + 1], want, what=f"{code} head_dim 512 row {r}")
    # one decode step appended at position S
    qd, kd, vd = normed(code, 21, 5, 1, hq), normed(code, 21, 6, 1, hkv), plain(code, 21, 7, 1, hkv)
    outd = nm.append_attend(cache, S, dev_t(kd, dev, code), dev_t(vd, dev, code), dev_t(qd, dev, code), scale,
                            out_dtype=torch.float32).cpu().numpy()
    want = oracle.attend(np.concatenate([k, kd]), np.concatenate([v, vd]), 0, 0, hkv, DH, qd, hq, S, **kw)
    assert_close(outd, want, what=f"{code} head_dim 512 decode")


def test_batched_decode_over_ragged_caches(dev):
    hq, hkv, code = 16, 1, "bf16"
    lens = [7, 640, 3000]
    caches, ks, vs = [], [], []
    for b, L in enumerate(lens):
        k, v = normed(code, 22, 10 + 2 * b, L, hkv), plain(code, 22, 11 + 2 * b, L, hkv)
        c = nm.FullAttentionCache(hkv, DH, capacity=L, dtype=code)
        c.append(0, dev_t(k, dev, code), dev_t(v, dev, code))
        caches.append(c)
        ks.append(k)
        vs.append(v)
    q = normed(code, 22, 1, len(lens), hq)
    out = nm.attend_batch(caches, dev_t(q, dev, code), None, out_dtype=torch.float32).cpu().numpy()
    for b, L in enumerate(lens):
        want = oracle.attend(ks[b], vs[b], 0, 0, hkv, DH, q[b:b + 1], hq, L - 1, use_scale=False)
        assert_close(out[b:b + 1], want, what=f"batched head_dim 512 sequence {b}")


def test_fp32_cache_at_head_dim_512_is_refused(dev):
    # Two 32-key fp32 tiles of 2 KB rows do not fit the kernel's shared memory:
    # the call is refused before any launch.
    cache = nm.FullAttentionCache(1, DH, capacity=4)
    x = torch.randn(4, DH, device=dev)
    cache.append(0, x, x)
    with pytest.raises(Unsupported):
        nm.attend(cache, torch.randn(1, DH, device=dev), 3, 1.0)


def test_gemma_full_layer_prologue_then_attend(dev):
    # A Gemma 4 E4B full-attention layer on a bf16 cache: per-head RMS norm and
    # partial RoPE (1/4 of 512 planes, base 1e6, gemma4.hpp:397) written into the
    # cache by the prologue, then the reduction at head_dim 512 with scale 1.
    hq, hkv, Tt = 8, 2, 24
    x = oracle.normal(23, 1, Tt * hq * DH).reshape(Tt, hq * DH) * np.float32(2)
    k = oracle.normal(23, 2, Tt * hkv * DH).reshape(Tt, hkv * DH) * np.float32(3)
    v = oracle.normal(23, 3, Tt * hkv * DH).reshape(Tt, hkv * DH)
    qg = oracle.normal(23, 4, DH) * np.float32(0.5) + np.float32(1)
    kg = oracle.normal(23, 5, DH) * np.float32(0.5) + np.float32(1)
    f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)
    cache = nm.FullAttentionCache(hkv, DH, capacity=32, dtype="bf16")
    Q = nm.attn_prologue(cache, 0, f32(x), f32(k), f32(v), f32(qg), f32(kg), 1e-6, 1000000, 1, 4, gated=False,
                         v_norm=True)
    assert Q.dtype == torch.bfloat16 and cache.size() == Tt
    # the prepared values are the oracle's, rounded to the cache's bf16
    wq, wk, wv = oracle.attn_prologue(x, k, v, qg, kg, hq, hkv, DH, 0, 1e-6, 1000000, 1, 4, gated=False, v_norm=True)
    keys = np.stack([np.concatenate([cache.key(r, h).numpy() for h in range(hkv)]) for r in range(Tt)])
    vals = np.stack([np.concatenate([cache.value(r, h).numpy() for h in range(hkv)]) for r in range(Tt)])
    qv = Q.float().cpu().numpy()
    for got, want in ((qv, wq), (keys, wk), (vals, wv)):
        assert np.all(np.abs(got - want) <= 2.0 ** -7 * np.maximum(np.abs(want), 2.0 ** -14) + 1e-5)
    # and the reduction over exactly what the device holds matches the oracle's
    out = nm.attend(cache, Q, 0, None, out_dtype=torch.float32).cpu().numpy()
    assert_close(out, oracle.attend(keys, vals, 0, 0, hkv, DH, qv, hq, 0, use_scale=False),
                 what="Gemma full layer at head_dim 512")
