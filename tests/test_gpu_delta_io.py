"""The delta-net prologue and epilogue on the device against the oracle
(oracle/nm_oracle.c, pinned to the reference in tests/test_oracle_delta_io.py)."""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close
from hero_b200 import nm
from hero_b200._lib import InvalidArgument

pytestmark = pytest.mark.gpu


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


def test_conv1d_known_answers(dev):
    # qwen35_tests.cpp:132-155: taps [1, 10, 100], the causal zero pad, the window.
    conv = nm.ConvState(2, 3)
    w = T([[1, 10, 100], [1, 10, 100]], dev)
    ys = [conv.step(w, T([[x, 0]], dev))[0, 0].item() for x in (1, 2, 3)]
    assert ys == [100.0, 210.0, 321.0]
    assert conv.history().cpu().numpy().tolist() == [[2.0, 0.0], [3.0, 0.0]]
    conv.clear()
    assert conv.step(w, T([[1, 0]], dev))[0, 0].item() == 100.0  # a cleared state starts again
    whole = nm.ConvState(2, 3).step(w, T([[1, 0], [2, 0], [3, 0]], dev))  # one call over three tokens
    assert whole[:, 0].cpu().numpy().tolist() == [100.0, 210.0, 321.0]


@pytest.mark.parametrize("channels,width,splits", [(24, 4, (2, 15, 20)), (300, 1, (7,)), (1000, 8, (40, 1, 33))])
def test_conv1d_matches_oracle_across_calls(dev, channels, width, splits):
    w = oracle.normal(31, 1, channels * width).reshape(channels, width)
    x = oracle.normal(31, 2, sum(splits) * channels).reshape(-1, channels)
    want, hist = oracle.conv_run(w, x)
    conv = nm.ConvState(channels, width)
    got, t = [], 0
    for n in splits:
        got.append(conv.step(T(w, dev), T(x[t:t + n], dev), silu=False).cpu().numpy())
        t += n
    assert_close(np.concatenate(got), want, max_abs=1e-5, rel=1e-6, what="conv")
    if width > 1:
        assert_close(conv.history().cpu().numpy(), hist, max_abs=0, rel=0, what="history")
    y = nm.ConvState(channels, width).step(T(w, dev), T(x, dev), silu=True).cpu().numpy()
    assert_close(y, oracle.silu(want), max_abs=1e-5, rel=1e-6, what="conv + silu")


def _prologue_inputs(seed, T_, hk, hv, dk, dv, W):
    C = 2 * hk * dk + hv * dv
    w = oracle.normal(seed, 1, C * W).reshape(C, W) * np.float32(0.5)
    qkv = oracle.normal(seed, 2, T_ * C).reshape(T_, C)
    br = oracle.normal(seed, 3, T_ * hv).reshape(T_, hv)
    ar = oracle.normal(seed, 4, T_ * hv).reshape(T_, hv) * np.float32(4)  # both softplus branches
    dt = oracle.normal(seed, 5, hv)
    ds = -np.exp(oracle.normal(seed, 6, hv)).astype(np.float32)
    return w, qkv, br, ar, dt, ds


@pytest.mark.parametrize("hk,hv,dk,dv,splits", [(2, 4, 128, 128, (37, 63)), (1, 3, 64, 96, (5,)), (16, 32, 128, 128, (300,))])
def test_prologue_matches_oracle(dev, hk, hv, dk, dv, splits):
    W = 4
    w, qkv, br, ar, dt, ds = _prologue_inputs(41, sum(splits), hk, hv, dk, dv, W)
    want = oracle.delta_prologue(w, qkv, br, ar, dt, ds, hk, hv, dk, dv)
    conv = nm.ConvState(2 * hk * dk + hv * dv, W)
    parts, t = [], 0
    for n in splits:
        parts.append([a.cpu().numpy() for a in nm.delta_prologue(conv, T(w, dev), T(qkv[t:t + n], dev), T(br[t:t + n], dev),
                                                                  T(ar[t:t + n], dev), T(dt, dev), T(ds, dev), hk, hv, dk, dv)])
        t += n
    for i, name in enumerate(("q", "k", "v", "beta", "gate")):
        got = np.concatenate([p[i] for p in parts])
        assert_close(got, want[i], max_abs=2e-5, rel=2e-6, what=name)
    assert_close(conv.history().cpu().numpy(), want[5], max_abs=0, rel=0, what="conv history")


def test_prologue_rejects_mismatched_state(dev):
    conv = nm.ConvState(100, 4)
    x = torch.zeros(2, 100, device=dev)
    with pytest.raises(InvalidArgument):
        nm.delta_prologue(conv, torch.zeros(100, 4, device=dev), x, torch.zeros(2, 1, device=dev),
                          torch.zeros(2, 1, device=dev), torch.zeros(1, device=dev), torch.zeros(1, device=dev),
                          1, 1, 32, 32)


@pytest.mark.parametrize("hv,dv,T_,eps", [(32, 128, 300, 1e-6), (3, 96, 17, 1e-5)])
def test_epilogue_matches_oracle(dev, hv, dv, T_, eps):
    o = oracle.normal(51, 1, T_ * hv * dv).reshape(T_, hv, dv)
    z = oracle.normal(51, 2, T_ * hv * dv).reshape(T_, hv, dv) * np.float32(3)
    gamma = oracle.normal(51, 3, dv)
    got = nm.delta_epilogue(T(o, dev), T(z, dev), T(gamma, dev), eps).cpu().numpy()
    assert_close(got, oracle.delta_epilogue(o, z, gamma, eps), max_abs=2e-5, rel=2e-6, what="epilogue")


@pytest.mark.parametrize("chunk", [0, 64])
def test_recurrent_layer_core_matches_oracle(dev, chunk):
    # prologue -> delta rule -> epilogue, the on-device core of a Qwen 3.5
    # recurrent layer between its projections, in two prefill calls.  The
    # RMS norm rescales each head to unit RMS, so the chunked (tf32) path's
    # relative error reappears at the output's scale: its absolute bound is
    # the contract's 2e-3 relative to the largest output.
    hk, hv, dk, dv, W = 2, 4, 128, 128, 4
    Tt = 200
    w, qkv, br, ar, dt, ds = _prologue_inputs(61, Tt, hk, hv, dk, dv, W)
    z = oracle.normal(61, 7, Tt * hv * dv).reshape(Tt, hv, dv)
    gamma = oracle.normal(61, 8, dv)
    q, k, v, beta, gate, _ = oracle.delta_prologue(w, qkv, br, ar, dt, ds, hk, hv, dk, dv)
    o, _ = oracle.delta_run(np.zeros((hv, dk, dv), np.float32), q, k, v, gate, beta, hk)
    want = oracle.delta_epilogue(o, z, gamma, 1e-6)
    conv, st = nm.ConvState(2 * hk * dk + hv * dv, W), nm.DeltaNetState(hv, dk, dv)
    outs = []
    for t0, t1 in ((0, 77), (77, Tt)):
        dq, dk_, dvv, db, dg = nm.delta_prologue(conv, T(w, dev), T(qkv[t0:t1], dev), T(br[t0:t1], dev),
                                                 T(ar[t0:t1], dev), T(dt, dev), T(ds, dev), hk, hv, dk, dv)
        do = nm.delta_prefill(st, dq, dk_, dvv, dg, db, hk, chunk=chunk)
        outs.append(nm.delta_epilogue(do, T(z[t0:t1], dev), T(gamma, dev), 1e-6).cpu().numpy())
    scale = 1.0 if chunk == 0 else max(1.0, float(np.abs(want).max()))
    assert_close(np.concatenate(outs), want, max_abs=2e-3 * scale, what=f"layer core, chunk {chunk}")
