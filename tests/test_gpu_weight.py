"""The device quantised projections (nmg_weight_*) against the oracle.

Weight<In,Out>::matvec / matmul / gather_rows (src/quant.hpp:439-487,
src/quant_i8.hpp:351-514) for Q8_0, Q4_0, Q4_K, Q5_K, Q6_K and F32 weights:

* the activation quantisers bit for bit (quantize_row_q8_0 / _q8_K, including
  the tie cases the reference build rounds through a fused multiply-add);
* gather_rows bit for bit (dequant_to_f32);
* products within the north-star tolerance (max abs 2e-3, rel L2 1e-3) of
  the oracle's integer-activation path (the reference default) and of its
  fp32-activation path (NM_FP32_ACT), and of the reference's own outputs in
  tests/golden/quant_i8.npz; at Qwen3.5-9B projection shapes too;
* the errors the reference raises.
"""
import os

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close
from hero_b200 import _lib, nm
from oracle import quant as Q

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "quant_i8.npz")
TYPES = (Q.Q8_0, Q.Q4_0, Q.Q4_K, Q.Q5_K, Q.Q6_K, Q.F32)


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(GOLD))


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


@pytest.mark.parametrize("atype", (Q.Q8_0, Q.Q8_K))
def test_activation_quantisers_are_bit_exact(dev, gold, atype):
    x = np.concatenate([gold["x"], oracle.normal(21, 1, 5 * 512).reshape(5, 512) * np.float32(7.0)])
    x[3, 40:72] = 0.0  # an all-zero Q8_0 block
    got = nm.quantize_activations(_t(x, dev), atype).cpu().numpy()
    assert np.array_equal(got, Q.quantize_act(x, atype))
    key = "act_q8_k" if atype == Q.Q8_K else "act_q8_0"
    assert np.array_equal(got[:3], gold[key])


def test_q8_k_ties_round_the_exact_product(dev, gold):
    got = nm.quantize_activations(_t(gold["tie_x"], dev), Q.Q8_K).cpu().numpy()
    assert np.array_equal(got, gold["tie_q8_k"])


def test_q8_k_zero_block_and_first_maximum(dev):
    x = np.zeros((2, 256), np.float32)
    x[1, 10], x[1, 200] = -3.0, 3.0  # equal magnitudes: the first one sets the sign
    got = nm.quantize_activations(_t(x, dev), Q.Q8_K).cpu().numpy()
    assert np.array_equal(got, Q.quantize_act(x, Q.Q8_K))
    assert not got[0].any()


@pytest.mark.parametrize("t", TYPES)
def test_gather_rows_bit_exact(dev, t):
    n, out = 1024, 40
    w = Q.random_weight(t, out, n, seed=30 + t)
    W = nm.Weight(t, n, out, w)
    rows = [0, 39, 7, 7, 22]
    got = W.gather_rows(rows).cpu().numpy()
    want = Q.dequant(t, w[rows], n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("rows", (1, 3, 8, 13))
def test_products_match_the_oracle(dev, t, rows):
    n, out = 2048, 200
    w = Q.random_weight(t, out, n, seed=50 + t)
    x = oracle.normal(51 + t, rows, rows * n).reshape(rows, n)
    W = nm.Weight(t, n, out, w)
    xt = _t(x, dev)
    got = (W.matvec(xt[0])[None] if rows == 1 else W.matmul(xt)).cpu().numpy()
    assert_close(got, Q.matmul(t, w, x, threads=8), what=f"{Q.NAMES.get(t)} rows {rows}")
    W32 = nm.Weight(t, n, out, w, fp32_act=True)
    got32 = W32.matmul(xt).cpu().numpy()
    assert_close(got32, Q.matmul(t, w, x, fp32_act=True, threads=8), what=f"{Q.NAMES.get(t)} fp32 act rows {rows}")


@pytest.mark.parametrize("t", (Q.Q8_0, Q.Q4_0, Q.Q4_K, Q.Q6_K))
@pytest.mark.parametrize("rows,n,out", [(200, 2048, 300), (129, 2080, 136), (512, 4096, 1024)])
def test_tensor_core_batches_match_the_oracle(dev, t, rows, n, out):
    """Batches past 8 rows take the int8 tensor-core tiles: partial row and
    output tiles, and (Q8_0/Q4_0) rows that end inside a 256-value superblock."""
    if n % Q.BLOCK[t][0]:
        pytest.skip("row is not whole blocks of this type")
    w = Q.random_weight(t, out, n, seed=90 + t)
    x = oracle.normal(91 + t, 1, rows * n).reshape(rows, n)
    got = nm.Weight(t, n, out, w).matmul(_t(x, dev)).cpu().numpy()
    assert_close(got, Q.matmul(t, w, x, threads=16), what=f"{Q.NAMES[t]} {rows}x{n}->{out}")


@pytest.mark.parametrize("t", (Q.Q8_0, Q.Q4_0, Q.Q4_K, Q.Q5_K, Q.Q6_K))
def test_products_match_the_reference_fixture(dev, gold, t):
    name = Q.NAMES[t]
    n, out = int(gold["n"]), int(gold["out"])
    W = nm.Weight(t, n, out, gold["w_" + name])
    x = _t(gold["x"], dev)
    assert_close(W.matvec(x[0]).cpu().numpy(), gold["mv_" + name], what=name + " matvec")
    assert_close(W.matmul(x).cpu().numpy(), gold["mm_" + name], what=name + " matmul")
    W32 = nm.Weight(t, n, out, gold["w_" + name], fp32_act=True)
    assert_close(W32.matmul(x).cpu().numpy(), gold["f32_" + name], what=name + " fp32 activations")


def test_reference_quantised_weights(dev, gold):
    x = _t(gold["x"], dev)
    n, out = int(gold["n"]), int(gold["out"])
    for t, key in ((Q.Q8_0, "q8_0"), (Q.Q4_0, "q4_0")):
        W = nm.Weight(t, n, out, gold["wq" + key[1:]])
        assert_close(W.matvec(x[0]).cpu().numpy(), gold["mvq" + key[1:]], what=key)


@pytest.mark.parametrize("t,n,out", [(Q.Q4_K, 4096, 12288), (Q.Q6_K, 12288, 4096), (Q.Q8_0, 4096, 8192),
                                     (Q.Q4_0, 4096, 4096), (Q.Q5_K, 4096, 4096)])
def test_qwen35_9b_projection_shapes(dev, t, n, out):
    """Qwen3.5-9B (qwen35.hpp:62-83, D = 4096, FF = 12288) projection shapes:
    gate/up, down, the delta layer's qkv, out, and a Q5_K tensor."""
    w = Q.random_weight(t, out, n, seed=60 + t)
    x = oracle.normal(61, 1, 2 * n).reshape(2, n)
    W = nm.Weight(t, n, out, w)
    got = W.matmul(_t(x, dev)).cpu().numpy()
    assert_close(got, Q.matmul(t, w, x, threads=16), what=f"{Q.NAMES[t]} {n}->{out}")


@pytest.mark.parametrize("src", ("f16", "bf16"))
def test_sixteen_bit_rows_are_widened(dev, src):
    n, out = 512, 24
    v = oracle.normal(70, 1, out * n).reshape(out, n) * np.float32(0.05)
    bits = oracle.fp16_bits(v) if src == "f16" else oracle.bf16_bits(v)
    vals = oracle.from_fp16_bits(bits) if src == "f16" else oracle.from_bf16_bits(bits)
    W = nm.Weight(nm.GT.F16 if src == "f16" else nm.GT.BF16, n, out, bits.astype(np.uint16))
    assert W.type() == nm.GT.F32
    x = oracle.normal(71, 1, n)
    got = W.matvec(_t(x, dev)).cpu().numpy()
    assert_close(got, Q.matmul(Q.F32, vals.astype(np.float32).view(np.uint8), x))
    assert np.array_equal(W.gather_rows([3]).cpu().numpy()[0], vals.astype(np.float32)[3])


def test_device_resident_bytes_and_empty_batch(dev):
    n, out = 512, 16
    w = Q.random_weight(Q.Q4_K, out, n, seed=80)
    W = nm.Weight(Q.Q4_K, n, out, torch.from_numpy(w).to(dev))
    x = oracle.normal(81, 1, n)
    assert_close(W.matvec(_t(x, dev)).cpu().numpy(), Q.matmul(Q.Q4_K, w, x))
    assert W.matmul(torch.empty(0, n, device=dev)).shape == (0, out)


def test_errors(dev):
    with pytest.raises(_lib.InvalidArgument):
        nm.Weight(7, 512, 4, np.zeros(4 * 512, np.uint8))  # not a weight type
    with pytest.raises(_lib.InvalidArgument):
        nm.Weight(Q.Q4_K, 300, 4, np.zeros(4 * 1024, np.uint8))  # ragged row
    with pytest.raises(_lib.Unsupported):
        nm.Weight(Q.F32, 6, 4, np.zeros(4 * 6 * 4, np.uint8))
    W = nm.Weight(Q.Q8_0, 64, 4, Q.random_weight(Q.Q8_0, 4, 64))
    with pytest.raises(_lib.OutOfRange):
        W.gather_rows([4])
    with pytest.raises(_lib.InvalidArgument):
        nm.quantize_activations(torch.zeros(2, 100, device=dev), Q.Q8_0)
