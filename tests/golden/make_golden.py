"""Writes tests/golden/*.npz from the reference engine's own code.

Run where the reference sources are present and oracle/_ref is built
(``make -C oracle``): ``python tests/golden/make_golden.py``.  Inputs come from
the seeded generator in oracle/ and are stored as bf16/fp16 bit patterns (the
values the reference then computes on in fp32); outputs are the reference's
fp32 results.  Shapes are BASELINE-config shapes cut down to fixture size.
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))  # tests/, for helpers
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402

R = oracle.ref()
if R is None:
    sys.exit("oracle/_ref/libnmref.so is not built (needs the reference sources)")
fp = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def bf16(seed, stream, shape):
    return oracle.round_bf16(oracle.normal(seed, stream, int(np.prod(shape)))).reshape(shape)


def f16(seed, stream, shape):
    return oracle.round_fp16(oracle.normal(seed, stream, int(np.prod(shape)))).reshape(shape)


def attn_full(name, seed, hq, hkv, dh, rows, qrows, first, use_scale, rnd=bf16):
    k = rnd(seed, 1, (rows, hkv * dh))
    v = rnd(seed, 2, (rows, hkv * dh))
    q = rnd(seed, 3, (qrows, hq * dh))
    scale = np.float32(1 / np.sqrt(np.float32(dh)))
    out = np.zeros_like(q)
    fq = first + rows - qrows
    st = R.nmref_attend_full(hkv, dh, fp(k), fp(v), rows, first, fp(q), qrows, hq, fq, scale, int(use_scale), fp(out))
    assert st == 0, st
    save(name, k, v, q, out, hq, hkv, dh, first, 0, fq, scale, use_scale, rnd)


def attn_local(name, seed, hq, hkv, dh, window, rows, qrows, first, rnd=bf16):
    k = rnd(seed, 1, (rows, hkv * dh))
    v = rnd(seed, 2, (rows, hkv * dh))
    q = rnd(seed, 3, (qrows, hq * dh))
    out = np.zeros_like(q)
    st = R.nmref_attend_local(hkv, dh, window, fp(k), fp(v), rows, first, fp(q), qrows, hq, 1.0, 0, fp(out))
    assert st == 0, st
    save(name, k, v, q, out, hq, hkv, dh, first, window, first + rows - qrows, np.float32(1), False, rnd)


def save(name, k, v, q, out, hq, hkv, dh, oldest, window, first_query, scale, use_scale, rnd):
    bits = oracle.bf16_bits if rnd is bf16 else oracle.fp16_bits
    np.savez_compressed(os.path.join(HERE, name + ".npz"), k_bits=bits(k), v_bits=bits(v), q_bits=bits(q), out=out, hq=hq, hkv=hkv, dh=dh, oldest=oldest, window=window,
                        first_query=first_query, scale=scale, use_scale=use_scale,
                        dtype="bf16" if rnd is bf16 else "f16")


def delta(name, seed, hv, hk, d, T):
    sys.path.insert(0, os.path.dirname(HERE))
    from helpers import delta_inputs

    q, k, v, g, b = delta_inputs(seed, T, hk, hv, d)
    s0 = np.zeros((hv, d, d), np.float32)
    s1 = s0.copy()
    out = np.zeros((T, hv, d), np.float32)
    st = R.nmref_delta_run(hv, d, d, fp(s1), T, hk, fp(q), fp(k), fp(v), fp(g), fp(b), fp(out))
    assert st == 0, st
    np.savez_compressed(os.path.join(HERE, name + ".npz"), q=q, k=k, v=v, g=g, beta=b, hk=hk, state0=s0,
                        state1=s1, out=out)


if __name__ == "__main__":
    # config 1 (decode, 16q/8kv, d128), cut to 96 cached rows
    attn_full("attn_c1_decode", 101, 16, 8, 128, 96, 1, 0, True)
    # config 2 (causal GQA prefill, group 4, d128), one KV head, 130 rows
    attn_full("attn_c2_prefill", 102, 4, 1, 128, 130, 130, 0, True)
    # config 4 (Gemma, d256, scale 1, window): local ring, token-by-token path
    attn_local("attn_c4_local", 104, 2, 1, 256, 64, 150, 100, 0)
    # config 5 (group 8, fp16 cache), 200 rows from position 7
    attn_full("attn_c5_f16", 105, 8, 1, 128, 200, 1, 7, True, rnd=f16)
    # toy shapes of the reference unit tests
    attn_full("attn_toy", 106, 2, 1, 2, 6, 3, 0, False)
    # config 3 (delta rule, tiled key heads), 4 value heads over 2 key heads, 12 tokens
    delta("delta_c3", 103, 4, 2, 128, 12)
    delta("delta_toy", 107, 2, 1, 2, 9)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))
