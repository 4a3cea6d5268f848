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
@pytest.mark.parametrize("chunk", [0])
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
