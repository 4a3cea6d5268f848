"""Writes tests/golden/quant_i8.npz from the reference engine's own quantised
weight code (Weight<In,Out>::matvec / matmul, dequant_to_f32, the activation
quantisers), instantiated by oracle/ref_shim.cpp.

Run where the reference sources are present and oracle/_ref is built
(``make -C oracle``): ``python tests/golden/make_quant_golden.py``.

Per weight type (Q8_0, Q4_0, Q4_K, Q5_K, Q6_K) at In = 512, Out = 24:
  w_<T>      GGUF bytes [24][row bytes]: random quant bytes with fp16 scales
             set for O(1) products (oracle.quant.random_weight, seed 11)
  x          fp32 activations [3][512] (oracle.normal(12, 1, ...))
  mv_<T>     the reference's Weight::matvec(x[0]) (its default integer path
             for Q8_0/Q4_0/Q4_K/Q6_K, the fp32 path for Q5_K)
  mm_<T>     the reference's Weight::matmul(x) [3][24]
  f32_<T>    the fp32-activation path (dot_block_* per row) [3][24]
  deq_<T>    dequant_to_f32 of the rows [24][512]
  act_q8_0, act_q8_k   quantize_row_q8_0 / quantize_row_q8_K of x (packed blocks)
  tie_x, tie_q8_k      Q8_K inputs whose products land on .5 after fp32
                       rounding: the reference build rounds the exact product
                       (its nearest_int contracts to a fused multiply-add)
  wq8_0, wq4_0, mvq8_0, mvq4_0   weights made by the reference's own quantize_q8_0 /
                       quantize_q4_0 from U(-2, 2) values (as
                       tests/quant_tests.cpp:197-203 builds them) and their matvec.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402
from oracle import quant as Q  # noqa: E402

if oracle.ref() is None:
    sys.exit("oracle/_ref/libnmref.so is not built (needs the reference sources)")


def tie_inputs(rows=8, n=256, seed=13):
    rng = np.random.default_rng(seed)
    x = np.zeros((rows, n), np.float32)
    for r in range(rows):
        mx = np.float32(rng.uniform(0.5, 3.0)) * (1 if r % 2 else -1)
        x[r, 0] = mx
        iscale = np.float32(-127.0) / mx
        k = rng.integers(-126, 126, size=n - 1)
        x[r, 1:] = ((k + 0.5) / np.float64(iscale)).astype(np.float32)
        step = rng.integers(-2, 3, size=n - 1)
        for j in range(1, n):
            for _ in range(abs(step[j - 1])):
                x[r, j] = np.nextafter(x[r, j], np.float32(np.inf) if step[j - 1] > 0 else np.float32(-np.inf))
    return x


def main():
    n, out, rows = 512, 24, 3
    x = oracle.normal(12, 1, rows * n).reshape(rows, n)
    z = {"x": x, "n": n, "out": out}
    for t in (Q.Q8_0, Q.Q4_0, Q.Q4_K, Q.Q5_K, Q.Q6_K):
        name = Q.NAMES[t]
        w = Q.random_weight(t, out, n, seed=11)
        z["w_" + name] = w
        z["mv_" + name] = Q.ref_product(t, w, x[0])
        z["mm_" + name] = Q.ref_product(t, w, x)
        z["f32_" + name] = np.float32([[Q.dot_fp32(t, n, w[o], x[r], use_ref=True) for o in range(out)]
                                       for r in range(rows)])
        z["deq_" + name] = Q.dequant(t, w, n, use_ref=True)
    z["act_q8_0"] = Q.quantize_act(x, Q.Q8_0, use_ref=True)
    z["act_q8_k"] = Q.quantize_act(x, Q.Q8_K, use_ref=True)
    tx = tie_inputs()
    z["tie_x"] = tx
    z["tie_q8_k"] = Q.quantize_act(tx, Q.Q8_K, use_ref=True)
    rng = np.random.default_rng(14)
    wf = rng.uniform(-2, 2, size=(out, n)).astype(np.float32)
    R = oracle.ref()
    for t, fn, bb in ((Q.Q8_0, R.nmref_quantize_q8_0_weights, 34), (Q.Q4_0, R.nmref_quantize_q4_0_weights, 18)):
        wq = np.empty((out, n // 32 * bb), np.uint8)
        for o in range(out):
            fn(wf[o].ctypes.data, n, wq[o].ctypes.data)
        key = Q.NAMES[t].lower()
        z["wq" + key[1:]] = wq
        z["mvq" + key[1:]] = Q.ref_product(t, wq, x[0])
    np.savez_compressed(os.path.join(HERE, "quant_i8.npz"), **z)


if __name__ == "__main__":
    main()
