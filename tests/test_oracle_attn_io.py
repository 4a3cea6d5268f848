"""Pins the oracle's restatement of the steps either side of the attention
reduction (oracle/nm_oracle.c: nmo_rope_freqs, nmo_rope, nmo_rmsnorm,
nmo_attn_prologue, nmo_attn_gate) before the device path is checked against it.

1. The reference's own property tests: partial RoPE leaves the non-rotary
   planes exactly unchanged and rotates the prefix (tests/gemma4_tests.cpp:110-120);
   the half-split RoPE score depends only on the offset
   (tests/property_tests.cpp:136-151); RMSNorm and the scale-free RMSNorm are
   scale invariant (property_tests.cpp:152-165, gemma4_tests.cpp:96-108).
2. Against the reference engine's own types (oracle/_ref): RotaryEmbedding's
   Matrix overload, PerHeadNorm<RMSNorm>, PerHeadNorm<RMSNormNoScale> and
   sigmoid, on seeded inputs at the Qwen 3.5 and Gemma 4 shapes.
"""
import ctypes

import numpy as np
import pytest

import oracle

ref = oracle.ref()
needs_ref = pytest.mark.skipif(ref is None, reason="reference library not built")
_fp = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def test_partial_rope_keeps_non_rotary_planes():
    # gemma4_tests.cpp:110-120: RotaryEmbedding<8, 10000, 1, 2> at position 7.
    x = np.arange(1, 9, dtype=np.float32).reshape(1, 1, 8)
    y = oracle.rope(x, 7, 10000, 1, 2)
    assert y[0, 0, [2, 3, 6, 7]].tolist() == [3.0, 4.0, 7.0, 8.0]
    assert y[0, 0, 0] != 1.0 and y[0, 0, 4] != 5.0
    assert oracle.rope_freqs(8, 10000, 1, 2).tolist()[2:] == [0.0, 0.0]


def test_rope_score_depends_only_on_offset():
    # property_tests.cpp:136-151: (R(p) q) . (R(m) k) is a function of m - p.
    q0 = np.arange(1, 9, dtype=np.float32).reshape(1, 1, 8)

    def score(p, m):
        return float(np.dot(oracle.rope(q0, p, 10000)[0, 0], oracle.rope(q0, m, 10000)[0, 0]))

    a, b, c = score(3, 1), score(10, 8), score(60, 58)
    assert abs(a - b) < 1e-4 and abs(b - c) < 1e-4


def test_rmsnorm_scale_invariance():
    # property_tests.cpp:152-165 (unit gamma) and gemma4_tests.cpp:96-108 (no scale).
    a = np.array([2, 4, 6, 8], np.float32)
    for gamma in (np.ones(4, np.float32), None):
        na, nb = oracle.rmsnorm(a, gamma, 1e-6), oracle.rmsnorm(a * np.float32(7.5), gamma, 1e-6)
        assert np.abs(na - nb).max() < 1e-5


def test_rope_at_position_zero_is_identity():
    x = oracle.normal(71, 1, 3 * 64).reshape(1, 3, 64)
    assert np.array_equal(oracle.rope(x, 0, 10000), x)


@needs_ref
@pytest.mark.parametrize("dh,base,num,den,heads", [(8, 10000, 1, 2, 1), (8, 10000, 1, 1, 1), (256, 10000000, 1, 4, 2),
                                                   (256, 10000, 1, 1, 2), (512, 1000000, 1, 4, 1), (64, 10000, 1, 1, 3)])
def test_rope_matches_reference(dh, base, num, den, heads):
    rows, first = 9, 70000  # large angles: cos/sin far from their first period
    x = oracle.normal(72, dh, rows * heads * dh).reshape(rows, heads, dh)
    want = np.array(x, order="C")
    assert ref.nmref_rope(dh, base, num, den, heads, rows, first, _fp(want)) == 0
    got = oracle.rope(x, first, base, num, den)
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=2e-6)
    rotary = num * dh // den // 2
    planes = np.r_[rotary:dh // 2, dh // 2 + rotary:dh]
    assert np.array_equal(got[..., planes], x[..., planes])  # untouched planes are bit-exact


@needs_ref
@pytest.mark.parametrize("n,heads", [(256, 2), (512, 1), (64, 3), (4, 1)])
@pytest.mark.parametrize("scaled", [True, False])
def test_head_norm_matches_reference(n, heads, scaled):
    rows = 11
    x = oracle.normal(73, n, rows * heads * n).reshape(rows, heads * n) * np.float32(3)
    gamma = oracle.normal(73, 1000 + n, n) if scaled else None
    want = np.empty_like(x)
    assert ref.nmref_head_norm(n, heads, rows, None if gamma is None else _fp(gamma), 1e-6, _fp(x), _fp(want)) == 0
    got = oracle.rmsnorm(x.reshape(rows, heads, n), gamma, 1e-6).reshape(rows, heads * n)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)


@needs_ref
def test_sigmoid_matches_reference():
    x = np.concatenate([oracle.normal(74, 1, 4096) * np.float32(8), np.array([-100, -88, 0, 88, 100], np.float32)])
    want = np.empty_like(x)
    ref.nmref_sigmoid_n(x.size, _fp(x), _fp(want))
    qg = np.stack([np.zeros_like(x), x], 0).reshape(1, 2 * x.size)  # one head: [q | gate]
    got = oracle.attn_gate(qg, np.ones((1, x.size), np.float32), x.size)
    assert np.array_equal(got[0], want)


@needs_ref
@pytest.mark.parametrize("gated,v_norm", [(True, False), (False, True)])
def test_attn_prologue_is_the_reference_composition(gated, v_norm):
    # Qwen 3.5 (gated, plain V) and Gemma 4 (ungated, scale-free V norm) at
    # head_dim 256, 2 heads of each, partial rotary 1/4 with base 1e7.
    T, hq, hkv, dh, pos = 6, 2, 2, 256, 123
    q = oracle.normal(75, 1, T * (2 if gated else 1) * hq * dh).reshape(T, -1)
    k = oracle.normal(75, 2, T * hkv * dh).reshape(T, -1)
    v = oracle.normal(75, 3, T * hkv * dh).reshape(T, -1)
    qgam, kgam = oracle.normal(75, 4, dh), oracle.normal(75, 5, dh)
    Q, K, V = oracle.attn_prologue(q, k, v, qgam, kgam, hq, hkv, dh, pos, 1e-6, 10000000, 1, 4, gated=gated,
                                   v_norm=v_norm)
    qs = np.ascontiguousarray(q.reshape(T, hq, -1)[:, :, :dh].reshape(T, hq * dh))  # split_head_pairs' .first
    wq, wk = np.empty_like(qs), np.empty_like(k)
    assert ref.nmref_head_norm(dh, hq, T, _fp(qgam), 1e-6, _fp(qs), _fp(wq)) == 0
    assert ref.nmref_head_norm(dh, hkv, T, _fp(kgam), 1e-6, _fp(k), _fp(wk)) == 0
    assert ref.nmref_rope(dh, 10000000, 1, 4, hq, T, pos, _fp(wq)) == 0
    assert ref.nmref_rope(dh, 10000000, 1, 4, hkv, T, pos, _fp(wk)) == 0
    np.testing.assert_allclose(Q, wq, rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(K, wk, rtol=2e-6, atol=2e-6)
    if v_norm:
        wv = np.empty_like(v)
        assert ref.nmref_head_norm(dh, hkv, T, None, 1e-6, _fp(v), _fp(wv)) == 0
        np.testing.assert_allclose(V, wv, rtol=1e-6, atol=1e-6)
    else:
        assert np.array_equal(V, v)


def test_attn_gate_uses_the_second_half_of_each_pair():
    T, hq, dh = 3, 4, 8
    qg = oracle.normal(76, 1, T * 2 * hq * dh).reshape(T, hq, 2, dh)
    a = oracle.normal(76, 2, T * hq * dh).reshape(T, hq * dh)
    got = oracle.attn_gate(qg.reshape(T, -1), a, dh)
    want = a * (1 / (1 + np.exp(-qg[:, :, 1, :].astype(np.float64)))).reshape(T, -1)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-7)
