"""Pins the oracle's restatement of the steps either side of the delta rule
(oracle/nm_oracle.c: nmo_conv_run, nmo_silu, nmo_delta_prologue,
nmo_delta_epilogue) before the device path is checked against it.

1. The reference's own known-answer tests (tests/qwen35_tests.cpp:132-155 for
   the causal conv1d, :188-197 for softplus and the L2 norm).
2. Against the reference engine's own types (oracle/_ref): CausalConv1dState,
   Silu, RMSNorm, l2_normalize, sigmoid, softplus on seeded inputs.
"""
import ctypes

import numpy as np
import pytest

import oracle

ref = oracle.ref()
needs_ref = pytest.mark.skipif(ref is None, reason="reference library not built")
_fp = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def test_conv1d_known_answers():
    # qwen35_tests.cpp:132-155: taps [1, 10, 100] on two channels.
    w = np.array([[1, 10, 100], [1, 10, 100]], np.float32)
    x = np.array([[1, 0], [2, 0], [3, 0]], np.float32)
    y, hist = oracle.conv_run(w, x)
    assert y[:, 0].tolist() == [100.0, 210.0, 321.0]
    again, _ = oracle.conv_run(w, x[:1])
    assert again[0, 0] == y[0, 0]  # a fresh state reproduces the first token
    assert hist.tolist() == [[2.0, 0.0], [3.0, 0.0]]  # the last W - 1 inputs, oldest first


def test_conv1d_history_carries_across_calls():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((24, 4)).astype(np.float32)
    x = rng.standard_normal((37, 24)).astype(np.float32)
    whole, hw = oracle.conv_run(w, x)
    a, h = oracle.conv_run(w, x[:2])
    b, h = oracle.conv_run(w, x[2:17], h)
    c, h = oracle.conv_run(w, x[17:], h)
    np.testing.assert_array_equal(np.concatenate([a, b, c]), whole)
    np.testing.assert_array_equal(h, hw)


@needs_ref
@pytest.mark.parametrize("channels,width,T", [(2, 3, 5), (24, 4, 37), (1024, 4, 19)])
def test_conv1d_equals_reference(channels, width, T):
    w = oracle.normal(21, 1, channels * width).reshape(channels, width)
    x = oracle.normal(21, 2, T * channels).reshape(T, channels)
    want = np.empty_like(x)
    assert ref.nmref_conv_run(channels, width, _fp(w), _fp(x), T, _fp(want)) == 0
    got, _ = oracle.conv_run(w, x)
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=2e-6)


@needs_ref
def test_silu_equals_reference():
    x = np.concatenate([oracle.normal(22, 1, 500) * np.float32(8), np.array([0, -90, 90, 1e-30], np.float32)])
    want = np.empty_like(x)
    ref.nmref_silu(x.size, _fp(x), _fp(want))
    np.testing.assert_array_equal(oracle.silu(x), want)


@needs_ref
def test_prologue_equals_reference_pieces():
    hk, hv, dk, dv, W, T = 2, 4, 128, 128, 4, 9
    C = 2 * hk * dk + hv * dv
    w = oracle.normal(23, 1, C * W).reshape(C, W)
    qkv = oracle.normal(23, 2, T * C).reshape(T, C)
    br, ar = oracle.normal(23, 3, T * hv).reshape(T, hv), oracle.normal(23, 4, T * hv).reshape(T, hv)
    dt, ds = oracle.normal(23, 5, hv), -np.exp(oracle.normal(23, 6, hv))
    q, k, v, beta, gate, _ = oracle.delta_prologue(w, qkv, br, ar, dt, ds, hk, hv, dk, dv)
    # the same steps through the reference's own functions (qwen35.hpp:436-446)
    conv = np.empty_like(qkv)
    assert ref.nmref_conv_run(C, W, _fp(w), _fp(qkv), T, _fp(conv)) == 0
    stream = np.empty_like(conv)
    ref.nmref_silu(conv.size, _fp(conv), _fp(stream))
    for t in range(T):
        for h in range(hk):
            qn, kn = np.empty(dk, np.float32), np.empty(dk, np.float32)
            assert ref.nmref_l2_normalize(dk, _fp(np.ascontiguousarray(stream[t, h * dk:(h + 1) * dk])), _fp(qn)) == 0
            assert ref.nmref_l2_normalize(dk, _fp(np.ascontiguousarray(stream[t, hk * dk + h * dk:hk * dk + (h + 1) * dk])),
                                          _fp(kn)) == 0
            np.testing.assert_allclose(q[t, h], qn * np.float32(1 / np.sqrt(dk)), rtol=2e-6, atol=2e-7)
            np.testing.assert_allclose(k[t, h], kn, rtol=2e-6, atol=2e-7)
        np.testing.assert_allclose(v[t].ravel(), stream[t, 2 * hk * dk:], rtol=2e-6, atol=2e-7)
        for h in range(hv):
            assert beta[t, h] == np.float32(ref.nmref_sigmoid(float(br[t, h])))
            assert gate[t, h] == np.float32(np.float32(ds[h]) * np.float32(ref.nmref_softplus(float(np.float32(ar[t, h] + dt[h])))))


@needs_ref
def test_epilogue_equals_reference_pieces():
    rows, dv, eps = 7, 128, 1e-6
    o = oracle.normal(24, 1, rows * dv).reshape(rows, dv)
    z = oracle.normal(24, 2, rows * dv).reshape(rows, dv)
    gamma = oracle.normal(24, 3, dv)
    got = oracle.delta_epilogue(o, z, gamma, eps)
    normed = np.empty_like(o)
    assert ref.nmref_rmsnorm(dv, rows, _fp(gamma), eps, _fp(o), _fp(normed)) == 0
    gate = np.empty_like(z)
    ref.nmref_silu(z.size, _fp(z), _fp(gate))
    np.testing.assert_allclose(got, normed * gate, rtol=2e-6, atol=2e-7)
