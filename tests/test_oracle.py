"""Pins the CPU oracle (oracle/nm_oracle.c) before anything is checked against it.

1. The reference's own known-answer tests, restated:
   tests/property_tests.cpp:187-223, :301-316, :318-338;
   tests/gemma4_tests.cpp:122-173; tests/qwen35_tests.cpp:157-197.
2. The oracle against the reference engine itself (oracle/_ref, the reference
   headers compiled by oracle/Makefile) on seeded random inputs: equal up to
   fp32 rounding (|diff| <= 2e-6 + 2e-6*|x|; the compiler may contract a*b+c
   into an FMA differently in the two builds; most cases are bit-identical).
3. The committed golden fixtures (tests/golden, written by the reference).
"""
import ctypes
import glob
import os

import numpy as np
import pytest

import oracle
from helpers import delta_inputs, load_attn_fixture

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


def test_causal_attention_equation():
    # property_tests.cpp:187-215: one KV head, keys e0/e1, values 10 / 30,
    # queries e0 at position 0 and e1 at position 1, scale 1/sqrt(2).
    keys = np.array([[1, 0], [0, 1]], np.float32)
    values = np.array([[10, 0], [30, 0]], np.float32)
    q = np.array([[1, 0], [0, 1]], np.float32)
    scale = np.float32(1 / np.sqrt(np.float32(2)))
    out = oracle.attend(keys, values, 0, 0, 1, 2, q, 1, 0, scale=scale)
    w1 = np.exp(scale) / (1 + np.exp(scale))
    assert out[0, 0] == 10.0
    assert abs(out[1, 0] - ((1 - w1) * 10 + w1 * 30)) < 1e-5


def test_local_window_of_one():
    # property_tests.cpp:217-222: a window of one keeps only the current position.
    keys = np.array([[1, 0], [0, 1]], np.float32)
    values = np.array([[10, 0], [30, 0]], np.float32)
    q = np.array([[0, 1]], np.float32)
    out = oracle.attend(keys, values, 0, 1, 1, 2, q, 1, 1, scale=np.float32(1 / np.sqrt(2)))
    assert out[0, 0] == 30.0


def test_gqa_heads_share_kv_with_scale_one():
    # gemma4_tests.cpp:122-145.
    keys = np.array([[1, 0], [0, 1]], np.float32)
    values = np.array([[10, 20], [30, 40]], np.float32)
    q = np.array([[1, 0, 1, 0]], np.float32)
    out = oracle.attend(keys, values, 0, 0, 1, 2, q, 2, 1, use_scale=False)
    p0 = np.exp(np.float32(1)) / (np.exp(np.float32(1)) + 1)
    assert abs(out[0, 0] - (p0 * 10 + (1 - p0) * 30)) < 1e-5
    assert out[0, 0] == out[0, 2]
    # gemma4_tests.cpp:147-151: the local window excludes position 0.
    local = oracle.attend(keys[1:], values[1:], 1, 1, 1, 2, q, 2, 1, use_scale=False)
    assert local[0, 0] == 30 and local[0, 1] == 40


def test_no_visible_key_is_an_error():
    # property_tests.cpp:301-316: window 2, key at 0, query at 9.
    with pytest.raises(oracle.NoVisibleKeys):
        oracle.attend(np.ones((1, 2), np.float32), np.ones((1, 2), np.float32), 0, 2, 1, 2,
                      np.ones((1, 2), np.float32), 1, 9)
    m = oracle.CacheModel(2, local=True)
    m.append(0)
    with pytest.raises(oracle.NoVisibleKeys):
        m.visible_rows(9)


def test_visible_rows_is_contains_in_closed_form():
    # property_tests.cpp:318-338, the exhaustive box.
    for width in range(5):
        for anchor in range(4):
            for rows in range(6):
                for query in range(10):
                    f, e = oracle.visible_rows(width, query, anchor, rows)
                    for row in range(rows):
                        assert (f <= row < e) == oracle.contains(width, anchor + row, query)


def test_ring_order_and_batch_retention():
    # gemma4_tests.cpp:153-172.
    m = oracle.CacheModel(2, local=True)
    for p in range(3):
        m.append(p)
    assert m.size == 2 and m.position(0) == 1 and m.position(1) == 2
    m.begin_batch_retention(2)
    m.append(3)
    m.append(4)
    assert m.size == 4 and m.position(0) == 1 and m.position(3) == 4
    m.end_batch_retention()
    assert m.size == 2 and m.position(0) == 3 and m.position(1) == 4


def test_delta_rule_known_answers():
    # qwen35_tests.cpp:157-186.
    k = np.array([[[1, 0]]], np.float32)
    v = np.array([[[3, -5]]], np.float32)
    out, s = oracle.delta_run(np.zeros((1, 2, 2), np.float32), k, k, v, np.zeros((1, 1), np.float32),
                              np.ones((1, 1), np.float32), 1)
    assert abs(out[0, 0, 0] - 3) < 1e-6 and abs(out[0, 0, 1] + 5) < 1e-6
    orth = np.array([[[0, 1]]], np.float32)
    miss, _ = oracle.delta_run(s, orth, orth, np.zeros((1, 1, 2), np.float32), np.zeros((1, 1), np.float32),
                               np.zeros((1, 1), np.float32), 1)
    assert abs(miss).max() < 1e-6
    faded, _ = oracle.delta_run(s, k, k, np.zeros((1, 1, 2), np.float32), np.full((1, 1), -4, np.float32),
                                np.zeros((1, 1), np.float32), 1)
    assert abs(faded[0, 0, 0] - 3 * np.exp(np.float32(-4))) < 1e-5


def test_softplus_and_l2():
    # qwen35_tests.cpp:188-197.
    assert abs(oracle.softplus(0.0) - np.log(2)) < 1e-6
    assert oracle.softplus(60.0) == 60.0
    u = oracle.l2_normalize(np.array([3, 4], np.float32))
    assert abs(u[0] - 0.6) < 1e-6 and abs(u[1] - 0.8) < 1e-6


def test_rounding_matches_core_hpp():
    # The vectorised numpy rounding equals the C restatement of core.hpp:61-100,
    # and (where built) the reference's own conversions.
    x = oracle.normal(3, 1, 4000) * np.float32(7)
    x[:6] = [0.0, -0.0, 65519.0, 1e-7, 3e38, -6.1e-5]
    L, R = oracle.lib(), oracle.ref()
    bb, hb = oracle.bf16_bits(x), oracle.fp16_bits(x)
    for i, v in enumerate(x):
        assert bb[i] == L.nmo_fp32_to_bf16(float(v))
        assert hb[i] == L.nmo_fp32_to_fp16(float(v))
        if R is not None and i % 7 == 0:
            assert bb[i] == R.nmref_fp32_to_bf16(float(v)) and hb[i] == R.nmref_fp32_to_fp16(float(v))


# ---- the oracle against the reference's own code -----------------------------

ref = oracle.ref()
needs_ref = pytest.mark.skipif(ref is None, reason="oracle/_ref (reference build) not present")
_fp = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _same(got, want):
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=2e-6)


@needs_ref
@pytest.mark.parametrize("hq,hkv,dh,rows,qrows,scale", [(16, 8, 128, 300, 4, True), (8, 4, 256, 200, 3, False),
                                                        (2, 1, 2, 5, 2, True), (64, 8, 128, 129, 1, True),
                                                        # Gemma 4 full-attention layers (head_dim 512): 12B, E4B
                                                        (16, 1, 512, 150, 3, False), (8, 2, 512, 90, 2, False)])
def test_oracle_equals_reference_full(hq, hkv, dh, rows, qrows, scale):
    k = oracle.normal(11, 1, rows * hkv * dh).reshape(rows, -1)
    v = oracle.normal(11, 2, rows * hkv * dh).reshape(rows, -1)
    q = oracle.normal(11, 3, qrows * hq * dh).reshape(qrows, -1)
    s = np.float32(1 / np.sqrt(dh))
    want = np.zeros_like(q)
    assert ref.nmref_attend_full(hkv, dh, _fp(k), _fp(v), rows, 5, _fp(q), qrows, hq, 5 + rows - qrows, s,
                                 int(scale), _fp(want)) == 0
    got = oracle.attend(k, v, 5, 0, hkv, dh, q, hq, 5 + rows - qrows, scale=s, use_scale=scale)
    _same(got, want)


@needs_ref
@pytest.mark.parametrize("window,rows,qrows", [(64, 300, 200), (64, 100, 30), (1, 10, 10), (128, 128, 128)])
def test_oracle_equals_reference_local(window, rows, qrows):
    hq, hkv, dh = 4, 2, 64
    k = oracle.normal(12, 1, rows * hkv * dh).reshape(rows, -1)
    v = oracle.normal(12, 2, rows * hkv * dh).reshape(rows, -1)
    q = oracle.normal(12, 3, qrows * hq * dh).reshape(qrows, -1)
    want = np.zeros_like(q)
    assert ref.nmref_attend_local(hkv, dh, window, _fp(k), _fp(v), rows, 3, _fp(q), qrows, hq, 1.0, 0, _fp(want)) == 0
    got = oracle.attend(k, v, 3, window, hkv, dh, q, hq, 3 + rows - qrows, use_scale=False)
    _same(got, want)


@needs_ref
def test_oracle_equals_reference_delta():
    q, k, v, g, b = delta_inputs(13, 24, 16, 32, 128)
    s0 = oracle.normal(13, 9, 32 * 128 * 128).reshape(32, 128, 128) * np.float32(0.1)
    got, gs = oracle.delta_run(s0, q, k, v, g, b, 16)
    want = np.zeros_like(got)
    ws = s0.copy()
    assert ref.nmref_delta_run(32, 128, 128, _fp(ws), 24, 16, _fp(q), _fp(k), _fp(v), _fp(g), _fp(b), _fp(want)) == 0
    _same(got, want)
    _same(gs, ws)


@needs_ref
def test_cache_model_equals_reference_scripts():
    rng = np.random.default_rng(5)
    for trial in range(200):
        window = int(rng.integers(1, 6))
        ops, pos, model = [], 0, oracle.CacheModel(window, local=True)
        expect_fail = None
        for _ in range(int(rng.integers(1, 14))):
            r = rng.random()
            if r < 0.7:
                ops.append((0, pos))
                try:
                    model.append(pos)
                except Exception as e:
                    expect_fail = (len(ops) - 1, type(e))
                    break
                pos += 1
            elif r < 0.85:
                n = int(rng.integers(0, 4))
                ops.append((1, n))
                try:
                    model.begin_batch_retention(n)
                except Exception as e:
                    expect_fail = (len(ops) - 1, type(e))
                    break
            else:
                ops.append((2, 0))
                try:
                    model.end_batch_retention()
                except Exception as e:
                    expect_fail = (len(ops) - 1, type(e))
                    break
        arr = np.array(ops, np.int64).reshape(-1)
        size, failed = ctypes.c_int64(), ctypes.c_int64()
        positions = np.zeros(64, np.int64)
        st = ref.nmref_local_script(window, arr.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), len(ops),
                                    ctypes.byref(size), positions.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), 64,
                                    ctypes.byref(failed))
        if expect_fail is None:
            assert st == 0, (ops, st)
            assert size.value == model.size
            assert list(positions[:size.value]) == [model.position(r) for r in range(model.size)]
        else:
            assert st != 0 and failed.value == expect_fail[0], (ops, st, failed.value)


# ---- committed golden fixtures (written by the reference, tests/golden/make_golden.py) ----

@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "attn_*.npz"))))
def test_oracle_matches_golden_attention(path):
    z = load_attn_fixture(path)
    got = oracle.attend(z["k"], z["v"], int(z["oldest"]), int(z["window"]), int(z["hkv"]), int(z["dh"]), z["q"],
                        int(z["hq"]), int(z["first_query"]), scale=np.float32(z["scale"]),
                        use_scale=bool(z["use_scale"]))
    _same(got, z["out"])


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "delta_*.npz"))))
def test_oracle_matches_golden_delta(path):
    z = np.load(path)
    out, state = oracle.delta_run(z["state0"], z["q"], z["k"], z["v"], z["g"], z["beta"], int(z["hk"]))
    _same(out, z["out"])
    _same(state, z["state1"])


def test_golden_fixtures_exist():
    assert len(glob.glob(os.path.join(GOLDEN, "*.npz"))) >= 6


@needs_ref
def test_golden_fixtures_reproduce_from_the_reference(tmp_path, capsys):
    # The committed fixtures are what tests/golden/make_golden.py and
    # make_quant_golden.py write from the reference build today: rerun them
    # into a scratch directory and compare.
    scratch = tmp_path / "golden"
    scratch.mkdir()
    for script in ("make_golden.py", "make_quant_golden.py"):
        src = open(os.path.join(GOLDEN, script)).read()
        exec(compile(src, script, "exec"), {"__file__": str(scratch / script), "__name__": "__main__"})
    committed = sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))
    assert sorted(p.name for p in scratch.glob("*.npz")) == [os.path.basename(p) for p in committed]
    for p in committed:
        a, b = np.load(p), np.load(scratch / os.path.basename(p))
        assert set(a.files) == set(b.files), p
        for key in a.files:
            assert np.array_equal(a[key], b[key]), (p, key)


@pytest.mark.skipif(oracle.ref() is None, reason="reference library not built")
@pytest.mark.parametrize("heads,tq,tk,scale", [(12, 40, 360, 1.0), (4, 37, 300, 0.125)])
def test_dense_attention_is_the_reference_sdpa(heads, tq, tk, scale):
    # scaled_dot_product_attention<Heads, 64, 64> (attention.hpp:124-139), the
    # vision ViT's call at 12 heads and scale 1 (gemma4_vision.hpp:167): the
    # oracle's reduction with every key visible (all queries at the newest row).
    d = 64
    q = oracle.normal(91, 1, tq * heads * d).reshape(tq, heads * d)
    k = oracle.normal(91, 2, tk * heads * d).reshape(tk, heads * d)
    v = oracle.normal(91, 3, tk * heads * d).reshape(tk, heads * d)
    want = np.empty_like(q)
    fp = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    assert oracle.ref().nmref_sdpa(heads, d, tq, tk, fp(q), fp(k), fp(v), scale, fp(want)) == 0
    got = oracle.attend(k, v, 0, 0, heads, d, q, heads, tk - 1, scale=np.float32(scale))
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=2e-6)


def _q8_cases():
    rng = np.random.default_rng(8)
    rows = [rng.standard_normal(4096).astype(np.float32),
            (rng.standard_normal(4096) * 1e-3).astype(np.float32),
            (rng.standard_normal(4096) * 3e4).astype(np.float32),
            np.zeros(64, np.float32)]
    # values on exact half-steps of the block scale: x = (k + 0.5) * amax / 127
    amax = np.float32(1.7)
    ties = (np.arange(-127, 127, dtype=np.float32)[:224] + np.float32(0.5)) * (amax / np.float32(127))
    ties[0] = -amax
    rows.append(ties.astype(np.float32))
    return rows


@pytest.mark.skipif(oracle.ref() is None, reason="reference build (oracle/_ref) not present")
def test_q8_0_quantiser_matches_the_reference_bit_for_bit():
    # quantize_row_q8_0 (quant_i8.hpp:69-81): the C restatement against the
    # reference's own function, every quant and every fp16 scale.
    for x in _q8_cases():
        q0, d0 = oracle.quantize_q8_0(x)
        q1, d1 = oracle.quantize_q8_0(x, use_ref=True)
        assert np.array_equal(q0, q1) and np.array_equal(d0, d1)


def test_q8_0_round_trip_error_is_half_a_step():
    x = _q8_cases()[0].reshape(-1, 32)
    q, d = oracle.quantize_q8_0(x)
    back = oracle.dequantize_q8_0(q, d)
    # quants are taken against the fp32 scale amax / 127, the block keeps its
    # fp16 rounding: half a step plus 127 times that rounding
    d32 = (np.abs(x).max(axis=1) / np.float32(127)).astype(np.float32)[:, None]
    d16 = oracle.from_fp16_bits(d)[:, None]
    assert np.all(np.abs(back - x) <= 0.5 * d32 + 127 * np.abs(d16 - d32) + 1e-7)
