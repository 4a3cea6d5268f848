"""The quantised-weight oracle (oracle/nm_quant_oracle.c) pinned to the reference.

Against tests/golden/quant_i8.npz, written by the reference's own
Weight<In,Out>::matvec / matmul, dequant_to_f32 and activation quantisers
(tests/golden/make_quant_golden.py), and, where oracle/_ref is built, against
the reference code directly on further seeds.  Integer and byte results
(activation blocks, dequantised weights) must be identical; the float sums
agree up to the compiler's fused multiply-add choices (a few ulp).
"""
import os

import numpy as np
import pytest

import oracle
from helpers import assert_close
from oracle import quant as Q

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "quant_i8.npz")
TYPES = (Q.Q8_0, Q.Q4_0, Q.Q4_K, Q.Q5_K, Q.Q6_K)


def ulp_close(got, want, what=""):
    """Equal up to a few ulp of the largest output (fused multiply-add choices)."""
    scale = max(1.0, float(np.abs(want).max()))
    assert_close(got, want, max_abs=2e-6 * scale, rel=1e-6, what=what)


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(GOLD))


def test_block_sizes_match_ggml():
    assert [Q.BLOCK[t][1] for t in TYPES] == [34, 18, 144, 176, 210]
    assert Q.row_bytes(Q.Q4_K, 4096) == 16 * 144
    assert Q.row_bytes(Q.Q8_K, 512) == 2 * 292


def test_activation_blocks_are_the_references(gold):
    x = gold["x"]
    assert np.array_equal(Q.quantize_act(x, Q.Q8_0), gold["act_q8_0"])
    assert np.array_equal(Q.quantize_act(x, Q.Q8_K), gold["act_q8_k"])


def test_q8_k_rounds_the_exact_product_on_ties(gold):
    """Inputs whose fp32 products sit on .5: the reference build rounds the
    exact product (fused multiply-add), which the oracle follows."""
    got = Q.quantize_act(gold["tie_x"], Q.Q8_K)
    assert np.array_equal(got, gold["tie_q8_k"])
    x = gold["tie_x"]
    mx = x[np.arange(len(x)), np.argmax(np.abs(x), axis=1)]
    iscale = (np.float32(-127) / mx).astype(np.float32)
    rounded_product = np.minimum(np.rint((iscale[:, None] * x).astype(np.float32)), 127).astype(np.int8)
    qs = got[:, 4:260].view(np.int8)
    assert (qs != rounded_product).sum() > 100, "the fixture no longer exercises the tie cases"


@pytest.mark.parametrize("t", TYPES)
def test_dequant_is_bit_exact(gold, t):
    name = Q.NAMES[t]
    got = Q.dequant(t, gold["w_" + name], int(gold["n"]))
    assert np.array_equal(got.view(np.uint32), gold["deq_" + name].view(np.uint32))


@pytest.mark.parametrize("t", TYPES)
def test_products_match_the_reference(gold, t):
    name, x, w = Q.NAMES[t], gold["x"], gold["w_" + Q.NAMES[t]]
    ulp_close(Q.matmul(t, w, x[0]), gold["mv_" + name], what=f"{name} matvec")
    ulp_close(Q.matmul(t, w, x), gold["mm_" + name], what=f"{name} matmul")
    ulp_close(Q.matmul(t, w, x, fp32_act=True), gold["f32_" + name], what=f"{name} fp32 activations")


def test_reference_quantised_weights(gold):
    x = gold["x"]
    ulp_close(Q.matmul(Q.Q8_0, gold["wq8_0"], x[0]), gold["mvq8_0"], what="quantize_q8_0 weights")
    ulp_close(Q.matmul(Q.Q4_0, gold["wq4_0"], x[0]), gold["mvq4_0"], what="quantize_q4_0 weights")


@pytest.mark.parametrize("t", (Q.Q8_0, Q.Q4_0, Q.Q4_K, Q.Q6_K))
def test_integer_path_differs_from_fp32_path(gold, t):
    """Activation quantisation moves the products well past the parity
    tolerance, so a device path must follow the integer path to match."""
    name, x = Q.NAMES[t], gold["x"]
    a, b = gold["mm_" + name], gold["f32_" + name]
    assert np.linalg.norm(a - b) / np.linalg.norm(b) > 2e-3


def test_q5_k_high_plane_adds_sixteen():
    """quant_tests.cpp:134-150: the fifth bit moves the value by 16 quanta."""
    blk = np.zeros(176, np.uint8)
    one = int(oracle.fp16_bits(np.float32([1.0]))[0])
    blk[0], blk[1] = one & 0xFF, one >> 8
    blk[4] = 1  # sub-block 0 scale 1, min 0
    blk[48] = 3  # low nibble of element 0
    low = Q.dequant(Q.Q5_K, blk, 256)[0]
    blk[16] = 1  # element 0's fifth bit
    high = Q.dequant(Q.Q5_K, blk, 256)[0]
    assert low[0] == 3.0 and high[0] == 19.0


@pytest.mark.skipif(oracle.ref() is None, reason="reference not built here")
@pytest.mark.parametrize("t", TYPES)
def test_oracle_against_reference_code(t):
    n, out = 1024, 16
    w = Q.random_weight(t, out, n, seed=40 + t)
    x = oracle.normal(41 + t, 1, 3 * n).reshape(3, n)
    assert np.array_equal(Q.dequant(t, w, n), Q.dequant(t, w, n, use_ref=True))
    if t in Q.I8_TYPES:
        at = Q.act_type(t)
        a = Q.quantize_act(x, at)
        assert np.array_equal(a, Q.quantize_act(x, at, use_ref=True))
        for o in range(out):
            assert abs(Q.vec_dot_i8(t, n, w[o], a[1]) - Q.vec_dot_i8(t, n, w[o], a[1], use_ref=True)) <= 1e-6
    for o in range(out):
        assert Q.dot_fp32(t, n, w[o], x[2]) == Q.dot_fp32(t, n, w[o], x[2], use_ref=True)
    ulp_close(Q.matmul(t, w, x), Q.ref_product(t, w, x))
