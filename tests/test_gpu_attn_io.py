"""The attention prologue (per-head RMSNorm + RoPE of Q and K, optional
scale-free V norm, append to the cache) and the output gate on the device,
against the oracle (oracle/nm_oracle.c, pinned to the reference in
tests/test_oracle_attn_io.py)."""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close
from hero_b200 import nm
from hero_b200._lib import InvalidArgument, Unsupported

pytestmark = pytest.mark.gpu

QWEN = dict(base=10000000, num=1, den=4)  # Qwen 3.5: head_dim 256, partial rotary 1/4
GEMMA_FULL = dict(base=1000000, num=1, den=4)  # Gemma 4 global layers: head_dim 512
GEMMA_LOCAL = dict(base=10000, num=1, den=1)  # Gemma 4 sliding layers: head_dim 256


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


def _inputs(seed, T_, hq, hkv, dh, gated):
    q = oracle.normal(seed, 1, T_ * (2 if gated else 1) * hq * dh).reshape(T_, -1) * np.float32(2)
    k = oracle.normal(seed, 2, T_ * hkv * dh).reshape(T_, -1) * np.float32(3)
    v = oracle.normal(seed, 3, T_ * hkv * dh).reshape(T_, -1)
    qgam = oracle.normal(seed, 4, dh) * np.float32(0.5) + np.float32(1)
    kgam = oracle.normal(seed, 5, dh) * np.float32(0.5) + np.float32(1)
    return q, k, v, qgam, kgam


def _cached(cache, rows, hkv):
    keys = np.stack([np.concatenate([cache.key(r, h).numpy() for h in range(hkv)]) for r in range(rows)])
    vals = np.stack([np.concatenate([cache.value(r, h).numpy() for h in range(hkv)]) for r in range(rows)])
    return keys, vals


@pytest.mark.parametrize("hq,hkv,dh,rope,gated,v_norm,pos", [
    (16, 4, 256, QWEN, True, False, 0),
    (8, 2, 512, GEMMA_FULL, False, True, 70000),  # large angles: the sincos slow path
    (4, 1, 256, GEMMA_LOCAL, False, True, 5),
    (3, 3, 64, dict(base=10000, num=1, den=1), True, False, 1000),
])
def test_prologue_matches_oracle(dev, hq, hkv, dh, rope, gated, v_norm, pos):
    T_ = 37
    q, k, v, qgam, kgam = _inputs(81, T_, hq, hkv, dh, gated)
    wq, wk, wv = oracle.attn_prologue(q, k, v, qgam, kgam, hq, hkv, dh, pos, 1e-6, rope["base"], rope["num"],
                                      rope["den"], gated=gated, v_norm=v_norm)
    cache = nm.FullAttentionCache(hkv, dh, capacity=64)  # the first append sets the cache's first position
    got = nm.attn_prologue(cache, pos, T(q, dev), T(k, dev), T(v, dev), T(qgam, dev), T(kgam, dev), 1e-6, rope["base"],
                           rope["num"], rope["den"], gated=gated, v_norm=v_norm)
    assert got.dtype == torch.float32 and cache.size() == T_ and cache.position(0) == pos
    # sin/cos of angles up to 7e4 rad: the device's and glibc's agree to a few ulp of the angle's own rounding
    tol = 2e-5 if pos < 10000 else 2e-4
    assert_close(got.cpu().numpy(), wq, max_abs=tol, rel=1e-5, what="Q")
    keys, vals = _cached(cache, T_, hkv)
    assert_close(keys, wk, max_abs=tol, rel=1e-5, what="K")
    assert_close(vals, wv, max_abs=2e-6 if v_norm else 0, rel=1e-6 if v_norm else 0, what="V")


def test_prologue_non_rotary_planes_are_only_normalised(dev):
    # Partial rotary: planes at and beyond num*dh/den/2 carry gamma * x * inverse_rms unchanged.
    hq, hkv, dh = 2, 2, 256
    q, k, v, qgam, kgam = _inputs(82, 9, hq, hkv, dh, True)
    cache = nm.FullAttentionCache(hkv, dh, capacity=16)
    got = nm.attn_prologue(cache, 3, T(q, dev), T(k, dev), T(v, dev), T(qgam, dev), T(kgam, dev), 1e-6, 1e7, 1,
                           4).cpu().numpy().reshape(9, hq, dh)
    normed = oracle.rmsnorm(q.reshape(9, hq, 2, dh)[:, :, 0, :], qgam, 1e-6)
    planes = np.r_[32:128, 160:256]
    assert_close(got[..., planes], normed[..., planes], max_abs=2e-6, rel=1e-6, what="non-rotary planes")


def test_prologue_across_calls_equals_one_call(dev):
    hq, hkv, dh = 4, 2, 128
    q, k, v, qgam, kgam = _inputs(83, 12, hq, hkv, dh, True)
    wq, wk, _ = oracle.attn_prologue(q, k, v, qgam, kgam, hq, hkv, dh, 0, 1e-6, 10000, 1, 2)
    cache = nm.FullAttentionCache(hkv, dh, capacity=16)
    parts = [nm.attn_prologue(cache, t0, T(q[t0:t1], dev), T(k[t0:t1], dev), T(v[t0:t1], dev), T(qgam, dev),
                              T(kgam, dev), 1e-6, 10000, 1, 2).cpu().numpy() for t0, t1 in ((0, 1), (1, 5), (5, 12))]
    assert_close(np.concatenate(parts), wq, max_abs=2e-5, rel=1e-5, what="Q")
    assert_close(_cached(cache, 12, hkv)[0], wk, max_abs=2e-5, rel=1e-5, what="K")


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_prologue_rounds_q_like_the_reference(dev, dtype):
    # Q in a 16-bit cache dtype is the fp32 result rounded to nearest even (core.hpp:61-100):
    # equal to the rounded oracle except where the fp32 values straddle a rounding boundary.
    hq, hkv, dh = 8, 2, 256
    q, k, v, qgam, kgam = _inputs(84, 50, hq, hkv, dh, True)
    wq, _, _ = oracle.attn_prologue(q, k, v, qgam, kgam, hq, hkv, dh, 17, 1e-6, 1e7, 1, 4)
    cache = nm.FullAttentionCache(hkv, dh, capacity=128, dtype=dtype)
    got = nm.attn_prologue(cache, 17, T(q, dev), T(k, dev), T(v, dev), T(qgam, dev), T(kgam, dev), 1e-6, 1e7, 1, 4)
    assert got.dtype == {"bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    want = (oracle.round_bf16 if dtype == "bf16" else oracle.round_fp16)(wq.copy()).reshape(wq.shape)
    g = got.float().cpu().numpy()
    assert np.mean(g == want) > 0.999
    ulp = np.float32(2.0 ** (-7 if dtype == "bf16" else -10))  # one ulp, relative, at worst
    assert np.all(np.abs(g - want) <= ulp * np.maximum(np.abs(want), np.float32(2.0 ** -14)))


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("hq,dh", [(16, 256), (3, 6)])
def test_gate_matches_oracle(dev, dtype, hq, dh):
    T_ = 33
    qg = oracle.normal(85, 1, T_ * 2 * hq * dh).reshape(T_, -1) * np.float32(4)
    a = oracle.normal(85, 2, T_ * hq * dh).reshape(T_, -1)
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    if dtype != "f32":
        a = (oracle.round_bf16 if dtype == "bf16" else oracle.round_fp16)(a.copy()).reshape(a.shape)
    ad = T(a, dev).to(tdt)
    out = nm.attn_gate(T(qg, dev), ad, dh)
    assert out.data_ptr() == ad.data_ptr()
    want = oracle.attn_gate(qg, a, dh)
    if dtype == "f32":
        assert_close(out.cpu().numpy(), want, max_abs=1e-6, rel=1e-6, what="gate")
    else:
        want = (oracle.round_bf16 if dtype == "bf16" else oracle.round_fp16)(want.copy()).reshape(want.shape)
        ulp = np.float32(2.0 ** (-7 if dtype == "bf16" else -10))  # one ulp, relative, at worst
        diff = np.abs(out.float().cpu().numpy() - want)
        assert np.all(diff <= ulp * np.maximum(np.abs(want), np.float32(2.0 ** -14)))


@pytest.mark.parametrize("cache_dtype", ["f32", "bf16"])
def test_gated_attention_chain_matches_oracle(dev, cache_dtype):
    # A Qwen 3.5 attention layer between its projections, in two prefill calls
    # and a decode step: prologue -> attend (scale 1/sqrt(dh)) -> gate.
    hq, hkv, dh = 16, 4, 256
    Tt = 161
    q, k, v, qgam, kgam = _inputs(86, Tt, hq, hkv, dh, True)
    wq, wk, wv = oracle.attn_prologue(q, k, v, qgam, kgam, hq, hkv, dh, 0, 1e-6, 1e7, 1, 4)
    if cache_dtype == "bf16":  # what a bf16 cache holds: bf16 Q, K and V values (V stored exactly as fp16)
        wq, wk = oracle.round_bf16(wq.copy()).reshape(wq.shape), oracle.round_bf16(wk.copy()).reshape(wk.shape)
        wv = oracle.round_bf16(wv.copy()).reshape(wv.shape)
    scale = float(np.float32(1) / np.sqrt(np.float32(dh)))
    want = oracle.attn_gate(q, oracle.attend(wk, wv, 0, 0, hkv, dh, wq, hq, 0, scale), dh)
    cache = nm.FullAttentionCache(hkv, dh, capacity=256, dtype=cache_dtype)
    outs = []
    for t0, t1 in ((0, 100), (100, 160), (160, 161)):
        qq = T(q[t0:t1], dev)
        Q = nm.attn_prologue(cache, t0, qq, T(k[t0:t1], dev), T(v[t0:t1], dev), T(qgam, dev), T(kgam, dev), 1e-6,
                             1e7, 1, 4)
        A = nm.attend(cache, Q, t0, scale, out_dtype="f32")
        outs.append(nm.attn_gate(qq, A, dh).cpu().numpy())
    assert_close(np.concatenate(outs), want, what=f"gated attention, {cache_dtype} cache")


def test_prepare_then_append_attend_on_a_sliding_window(dev):
    # A Gemma 4 sliding layer whose batch evicts: the cacheless prepare, then
    # append_attend's token-by-token windows (gemma4.hpp:237-253), no score scale.
    hq, hkv, dh, W, Tt = 8, 4, 256, 64, 300
    q, k, v, qgam, kgam = _inputs(87, Tt, hq, hkv, dh, False)
    wq, wk, wv = oracle.attn_prologue(q, k, v, qgam, kgam, hq, hkv, dh, 0, 1e-6, 10000, gated=False, v_norm=True)
    Q, K, V = nm.attn_prepare(hkv, dh, 0, T(q, dev), T(k, dev), T(v, dev), T(qgam, dev), T(kgam, dev), 1e-6, 10000,
                              gated=False, v_norm=True)
    assert_close(Q.cpu().numpy(), wq, max_abs=2e-5, rel=1e-5, what="Q")
    assert_close(K.cpu().numpy(), wk, max_abs=2e-5, rel=1e-5, what="K")
    assert_close(V.cpu().numpy(), wv, max_abs=2e-6, rel=1e-6, what="V")
    cache = nm.LocalAttentionCache(hkv, dh, W)
    out = nm.append_attend(cache, 0, K, V, Q, None).cpu().numpy()
    want = oracle.attend(wk, wv, 0, W, hkv, dh, wq, hq, 0, use_scale=False)
    assert_close(out, want, what="sliding-window layer")


def test_prologue_rejects_bad_arguments(dev):
    cache = nm.FullAttentionCache(2, 128, capacity=8)
    z = lambda *s: torch.zeros(*s, device=dev)
    with pytest.raises(InvalidArgument):  # Hq not a multiple of Hkv
        nm.attn_prologue(cache, 0, z(1, 3 * 128), z(1, 256), z(1, 256), z(128), z(128), 1e-6, 1e4, gated=False)
    with pytest.raises(InvalidArgument):  # rotary fraction above one
        nm.attn_prologue(cache, 0, z(1, 4 * 128), z(1, 256), z(1, 256), z(128), z(128), 1e-6, 1e4, 5, 4)
    with pytest.raises(InvalidArgument):  # positions must continue the cache
        nm.attn_prologue(cache, 0, z(1, 4 * 128), z(1, 256), z(1, 256), z(128), z(128), 1e-6, 1e4)
        nm.attn_prologue(cache, 3, z(1, 4 * 128), z(1, 256), z(1, 256), z(128), z(128), 1e-6, 1e4)
    odd = nm.FullAttentionCache(1, 96, capacity=8)
    with pytest.raises(Unsupported):
        nm.attn_prologue(odd, 0, z(1, 2 * 96), z(1, 96), z(1, 96), z(96), z(96), 1e-6, 1e4)
