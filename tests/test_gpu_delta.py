"""Gated delta-rule state, step and prefill parity against the oracle and fixtures."""
import glob
import os

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close, delta_inputs
from hero_b200 import nm
from hero_b200._lib import OutOfRange

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


def test_delta_rule_known_answers(dev):
    # qwen35_tests.cpp:157-186, one head of DeltaNetState<1,2,2>
    st = nm.DeltaNetState(1, 2, 2)
    k, v = T([1, 0], dev), T([3, -5], dev)
    out = nm.gated_delta_step(st.head(0), k, k, v, 0.0, 1.0).cpu().numpy()
    assert abs(out[0] - 3) < 1e-6 and abs(out[1] + 5) < 1e-6
    orth = T([0, 1], dev)
    miss = nm.gated_delta_step(st.head(0), orth, orth, T([0, 0], dev), 0.0, 0.0).cpu().numpy()
    assert abs(miss).max() < 1e-6
    decaying = nm.DeltaNetState(1, 2, 2)
    nm.gated_delta_step(decaying.head(0), k, k, v, 0.0, 1.0)
    faded = nm.gated_delta_step(decaying.head(0), k, k, T([0, 0], dev), -4.0, 0.0).cpu().numpy()
    assert abs(faded[0] - 3 * np.exp(np.float32(-4))) < 1e-5
    with pytest.raises(OutOfRange):  # recurrent.hpp:128
        st.head(1)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(HERE, "golden", "delta_*.npz"))))
@pytest.mark.parametrize("chunk", [0, 64])
def test_golden_fixtures(dev, path, chunk):
    z = np.load(path)
    hv, d = z["state0"].shape[0], z["state0"].shape[1]
    st = nm.DeltaNetState(hv, d, d)
    out = nm.delta_prefill(st, T(z["q"], dev), T(z["k"], dev), T(z["v"], dev), T(z["g"], dev), T(z["beta"], dev),
                           int(z["hk"]), chunk=chunk)
    assert_close(out.cpu().numpy(), z["out"], what="out")
    assert_close(st.tensor().cpu().numpy(), z["state1"], what="state")


def test_config3_sequential_prefill_then_decode(dev):
    # 32 value heads over 16 tiled key heads, Dk = Dv = 128 (config 3), cut to
    # 192 prefill tokens + 16 decode steps so the sequential oracle is quick.
    hv, hk, d, Tp, Td = 32, 16, 128, 192, 16
    q, k, v, g, b = delta_inputs(3, Tp + Td, hk, hv, d)
    st = nm.DeltaNetState(hv, d, d)
    out = nm.delta_prefill(st, T(q[:Tp], dev), T(k[:Tp], dev), T(v[:Tp], dev), T(g[:Tp], dev), T(b[:Tp], dev), hk,
                           chunk=0).cpu().numpy()
    want, ws = oracle.delta_run(np.zeros((hv, d, d), np.float32), q[:Tp], k[:Tp], v[:Tp], g[:Tp], b[:Tp], hk)
    assert_close(out, want, what="prefill out")
    assert_close(st.tensor().cpu().numpy(), ws, what="prefill state")
    for t in range(Tp, Tp + Td):
        o = nm.delta_step(st, T(q[t], dev), T(k[t], dev), T(v[t], dev), T(g[t], dev), T(b[t], dev), hk).cpu().numpy()
        wo, ws = oracle.delta_run(ws, q[t:t + 1], k[t:t + 1], v[t:t + 1], g[t:t + 1], b[t:t + 1], hk)
        assert_close(o, wo[0], what=f"decode step {t}")
    assert_close(st.tensor().cpu().numpy(), ws, what="final state")


def test_step_equals_prefill(dev):
    # qwen35_tests.cpp:224-255's property at the kernel level: token-by-token
    # decode equals one-shot prefill (tolerance 1e-4 as there).
    hv, hk, d, n = 8, 4, 64, 40
    q, k, v, g, b = delta_inputs(9, n, hk, hv, d)
    a, c = nm.DeltaNetState(hv, d, d), nm.DeltaNetState(hv, d, d)
    whole = nm.delta_prefill(a, T(q, dev), T(k, dev), T(v, dev), T(g, dev), T(b, dev), hk, chunk=0).cpu().numpy()
    steps = np.stack([nm.delta_step(c, T(q[t], dev), T(k[t], dev), T(v[t], dev), T(g[t], dev), T(b[t], dev), hk)
                      .cpu().numpy() for t in range(n)])
    assert np.abs(whole - steps).max() < 1e-4
    assert np.abs(a.tensor().cpu().numpy() - c.tensor().cpu().numpy()).max() < 1e-4


def _random_state(seed, hv, d):
    return (oracle.normal(seed, 7, hv * d * d).reshape(hv, d, d) * np.float32(0.05)).astype(np.float32)


@pytest.mark.parametrize("n", [1, 12, 63, 64, 65, 130, 700, 2100, 4100])
def test_chunked_prefill_matches_oracle(dev, n):
    # Chunk 64, tcgen05 tf32 path: ragged last chunk, single partial chunk,
    # exact multiples; a non-zero starting state; value heads over tiled key heads;
    # 2100 and 4100 tokens (33 and 65 chunks) for longer state chains.
    hv, hk, d = 4, 2, 128
    q, k, v, g, b = delta_inputs(11 + n, n, hk, hv, d)
    s0 = _random_state(n, hv, d)
    st = nm.DeltaNetState(hv, d, d)
    st.tensor().copy_(T(s0, dev))
    out = nm.delta_prefill(st, T(q, dev), T(k, dev), T(v, dev), T(g, dev), T(b, dev), hk, chunk=64).cpu().numpy()
    want, ws = oracle.delta_run(s0, q, k, v, g, b, hk)
    assert_close(out, want, what=f"chunked out T={n}")
    assert_close(st.tensor().cpu().numpy(), ws, what=f"chunked state T={n}")


@pytest.mark.parametrize("hv,hk,dv", [(3, 2, 64), (2, 1, 96)])
def test_chunked_prefill_other_head_layouts(dev, hv, hk, dv):
    # value heads not a multiple of key heads; Dv of 2 and 3 column slices
    d, n = 128, 150
    q, k, _, g, b = delta_inputs(5, n, hk, hv, d)
    v = oracle.normal(5, 9, n * hv * dv).reshape(n, hv, dv)
    st = nm.DeltaNetState(hv, d, dv)
    out = nm.delta_prefill(st, T(q, dev), T(k, dev), T(v, dev), T(g, dev), T(b, dev), hk, chunk=64).cpu().numpy()
    want, ws = oracle.delta_run(np.zeros((hv, d, dv), np.float32), q, k, v, g, b, hk)
    assert_close(out, want, what="out")
    assert_close(st.tensor().cpu().numpy(), ws, what="state")


def test_chunked_config3_heads_then_decode(dev):
    # Config 3's head layout (32 value heads, 16 key heads, 128 x 128 states)
    # over 1024 prefill tokens in 16 chunks, then decode steps continue from
    # the chunked kernel's final state.
    hv, hk, d, Tp, Td = 32, 16, 128, 1024, 8
    q, k, v, g, b = delta_inputs(3, Tp + Td, hk, hv, d)
    st = nm.DeltaNetState(hv, d, d)
    out = nm.delta_prefill(st, T(q[:Tp], dev), T(k[:Tp], dev), T(v[:Tp], dev), T(g[:Tp], dev), T(b[:Tp], dev), hk,
                           chunk=64).cpu().numpy()
    want, ws = oracle.delta_run(np.zeros((hv, d, d), np.float32), q[:Tp], k[:Tp], v[:Tp], g[:Tp], b[:Tp], hk)
    assert_close(out, want, what="prefill out")
    assert_close(st.tensor().cpu().numpy(), ws, what="prefill state")
    for t in range(Tp, Tp + Td):
        o = nm.delta_step(st, T(q[t], dev), T(k[t], dev), T(v[t], dev), T(g[t], dev), T(b[t], dev), hk).cpu().numpy()
        wo, ws = oracle.delta_run(ws, q[t:t + 1], k[t:t + 1], v[t:t + 1], g[t:t + 1], b[t:t + 1], hk)
        assert_close(o, wo[0], what=f"decode step {t}")


def test_chunked_equals_sequential_at_full_length(dev):
    # Config 3 at its full 8192 tokens: the chunked kernel against the
    # token-sequential kernel (both on the device; the oracle would take
    # minutes here), outputs and final state.
    hv, hk, d, n = 32, 16, 128, 8192
    gen = torch.Generator(device="cpu").manual_seed(0)
    q = torch.nn.functional.normalize(torch.randn(n, hk, d, generator=gen), dim=-1) / d ** 0.5
    k = torch.nn.functional.normalize(torch.randn(n, hk, d, generator=gen), dim=-1)
    v = torch.randn(n, hv, d, generator=gen)
    g = -torch.nn.functional.softplus(torch.randn(n, hv, generator=gen))
    b = torch.sigmoid(torch.randn(n, hv, generator=gen))
    q, k, v, g, b = (x.to(dev) for x in (q, k, v, g, b))
    a, s = nm.DeltaNetState(hv, d, d), nm.DeltaNetState(hv, d, d)
    oc = nm.delta_prefill(a, q, k, v, g, b, hk, chunk=64).cpu().numpy()
    os_ = nm.delta_prefill(s, q, k, v, g, b, hk, chunk=0).cpu().numpy()
    assert_close(oc, os_, what="chunked vs sequential out")
    assert_close(a.tensor().cpu().numpy(), s.tensor().cpu().numpy(), what="chunked vs sequential state")


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_decode_attention_after_chunked_prefill(dev, dtype):
    # The chunked prefill leaves its tiles in the library's device scratch; the
    # split-KV decode kernels that run next (CUDA-core f32, tensor-core f16)
    # keep their merge tickets elsewhere and must be unaffected.
    hv, hk, d, n = 4, 2, 128, 300
    q, k, v, g, b = delta_inputs(17, n, hk, hv, d)
    st = nm.DeltaNetState(hv, d, d)
    nm.delta_prefill(st, T(q, dev), T(k, dev), T(v, dev), T(g, dev), T(b, dev), hk, chunk=64)
    hq, hkv, dh, rows = 8, 4, 128, 5000
    rnd = oracle.round_fp16 if dtype == "f16" else (lambda x: x)
    tdt = torch.float16 if dtype == "f16" else torch.float32
    kk = rnd(oracle.normal(23, 1, rows * hkv * dh).reshape(rows, -1))
    vv = rnd(oracle.normal(23, 2, rows * hkv * dh).reshape(rows, -1))
    qq = rnd(oracle.normal(23, 3, hq * dh).reshape(1, -1))
    cache = nm.FullAttentionCache(hkv, dh, capacity=rows, dtype=dtype)
    cache.append(0, T(kk, dev).to(tdt), T(vv, dev).to(tdt))
    want = oracle.attend(kk, vv, 0, 0, hkv, dh, qq, hq, rows - 1, scale=np.float32(dh ** -0.5))
    for _ in range(2):
        got = nm.attend(cache, T(qq, dev).to(tdt), rows - 1, dh ** -0.5, out_dtype=torch.float32).cpu().numpy()
        assert_close(got, want, what=f"{dtype} decode after chunked prefill")


@pytest.mark.parametrize("batch,steps", [(5, 3), (130, 1)])
def test_step_batch_matches_oracle_per_sequence(dev, batch, steps):
    # Decode steps for a batch of sequences, each with its own (non-zero)
    # state: the batched kernel against the reference recurrence, sequence by
    # sequence; 130 sequences take two launches.
    hv, hk, d = 32, 16, 128
    states, host = [], []
    for b in range(batch):
        s0 = _random_state(1000 + b, hv, d)
        st = nm.DeltaNetState(hv, d, d)
        st.tensor().copy_(T(s0, dev))
        states.append(st)
        host.append(s0)
    for t in range(steps):
        q, k, v, g, bt = delta_inputs(500 + t, batch, hk, hv, d)  # token axis used as the batch axis
        out = nm.delta_step_batch(states, T(q, dev), T(k, dev), T(v, dev), T(g, dev), T(bt, dev), hk).cpu().numpy()
        for b in range(batch):
            wo, host[b] = oracle.delta_run(host[b], q[b:b + 1], k[b:b + 1], v[b:b + 1], g[b:b + 1], bt[b:b + 1], hk)
            assert_close(out[b], wo[0], what=f"step {t} sequence {b}")
    for b in (0, batch // 2, batch - 1):
        assert_close(states[b].tensor().cpu().numpy(), host[b], what=f"state of sequence {b}")


def test_step_batch_other_shapes_run_per_sequence(dev):
    # Dv = 96 is not built for the batched kernel: the same result through the
    # one-sequence step, launched per sequence.
    hv, hk, dk, dv, batch = 4, 2, 64, 96, 3
    states = [nm.DeltaNetState(hv, dk, dv) for _ in range(batch)]
    q, k, _, g, bt = delta_inputs(77, batch, hk, hv, dk)
    v = oracle.normal(77, 9, batch * hv * dv).reshape(batch, hv, dv)
    out = nm.delta_step_batch(states, T(q, dev), T(k, dev), T(v, dev), T(g, dev), T(bt, dev), hk).cpu().numpy()
    for b in range(batch):
        wo, ws = oracle.delta_run(np.zeros((hv, dk, dv), np.float32), q[b:b + 1], k[b:b + 1], v[b:b + 1],
                                  g[b:b + 1], bt[b:b + 1], hk)
        assert_close(out[b], wo[0], what=f"sequence {b}")
        assert_close(states[b].tensor().cpu().numpy(), ws, what=f"state {b}")
