"""The fused single-token layer core (nmg_delta_decode_token) against the oracle.

One launch does the prologue (conv + SiLU + per-key-head L2 norms + gates),
the recurrent step and the gated output norm (qwen35.hpp:396-461 at T = 1).
Checked token by token against the oracle's chain of delta_prologue (pinned
to the reference's conv, SiLU, norms and gates), delta_run (the reference
recurrence) and delta_epilogue, within max abs 2e-3 / rel L2 1e-3; against
the library's own three launches within 1e-4; the conv history exactly and
the state after the tokens; and for the shapes it refuses.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close
from hero_b200 import _lib, nm

pytestmark = pytest.mark.gpu


def _layer(seed, hk, hv, dk, dv, W, ntok):
    C = 2 * hk * dk + hv * dv
    n = lambda s, shape, sc=1.0: (oracle.normal(seed, s, int(np.prod(shape))).reshape(shape) * np.float32(sc)).astype(np.float32)
    return {
        "w": n(1, (C, W), 0.5), "qkv": n(2, (ntok, C)), "br": n(3, (ntok, hv)), "ar": n(4, (ntok, hv)),
        "dtb": n(5, (hv,)), "dsc": -np.abs(n(6, (hv,))), "z": n(7, (ntok, hv, dv)), "gamma": n(8, (dv,)),
    }


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


@pytest.mark.parametrize("hk,hv,dk,dv", [(16, 32, 128, 128), (4, 4, 128, 256), (2, 8, 128, 64)])
def test_tokens_match_the_oracle_chain(dev, hk, hv, dk, dv):
    W, ntok, eps = 4, 12, 1e-6
    L = _layer(11 + hk + dv, hk, hv, dk, dv, W, ntok)
    st = nm.DeltaNetState(hv, dk, dv)
    conv = nm.ConvState(2 * hk * dk + hv * dv, W)
    w, dtb, dsc, gamma = (_t(L[x], dev) for x in ("w", "dtb", "dsc", "gamma"))
    state = np.zeros((hv, dk, dv), np.float32)
    hist = None
    for t in range(ntok):
        out = nm.delta_decode_token(st, conv, w, _t(L["qkv"][t], dev), _t(L["br"][t], dev), _t(L["ar"][t], dev), dtb,
                                    dsc, hk, _t(L["z"][t], dev), gamma, eps).cpu().numpy()
        q, k, v, beta, gate, hist = oracle.delta_prologue(L["w"], L["qkv"][t:t + 1], L["br"][t:t + 1], L["ar"][t:t + 1],
                                                          L["dtb"], L["dsc"], hk, hv, dk, dv, history=hist)
        o, state = oracle.delta_run(state, q, k, v, gate, beta, hk)
        want = oracle.delta_epilogue(o, L["z"][t:t + 1], L["gamma"], eps)[0]
        assert_close(out, want, what=f"token {t}")
    assert np.array_equal(conv.history().cpu().numpy(), hist), "conv history"
    assert_close(st.tensor().cpu().numpy(), state, what="state after the tokens")


def test_agrees_with_the_three_launches(dev):
    hk, hv, dk, dv, W, ntok, eps = 16, 32, 128, 128, 4, 6, 1e-6
    L = _layer(5, hk, hv, dk, dv, W, ntok)
    C = 2 * hk * dk + hv * dv
    st1, st2 = nm.DeltaNetState(hv, dk, dv), nm.DeltaNetState(hv, dk, dv)
    cv1, cv2 = nm.ConvState(C, W), nm.ConvState(C, W)
    w, dtb, dsc, gamma = (_t(L[x], dev) for x in ("w", "dtb", "dsc", "gamma"))
    for t in range(ntok):
        qkv, br, ar, z = (_t(L[x][t], dev) for x in ("qkv", "br", "ar", "z"))
        fused = nm.delta_decode_token(st1, cv1, w, qkv, br, ar, dtb, dsc, hk, z, gamma, eps)
        q, k, v, beta, gate = nm.delta_prologue(cv2, w, qkv[None], br[None], ar[None], dtb, dsc, hk, hv, dk, dv)
        o = nm.delta_step(st2, q[0], k[0], v[0], gate[0], beta[0], hk)
        three = nm.delta_epilogue(o[None], z[None], gamma, eps)[0]
        assert (fused - three).abs().max().item() <= 1e-4, f"token {t}"
    assert torch.equal(cv1.history(), cv2.history())
    assert (st1.tensor() - st2.tensor()).abs().max().item() <= 1e-5


@pytest.mark.parametrize("hk,hv,dk,dv", [(2, 8, 128, 128), (4, 4, 64, 64)])
def test_unbuilt_shapes_are_refused(dev, hk, hv, dk, dv):
    W = 4
    st = nm.DeltaNetState(hv, dk, dv)
    conv = nm.ConvState(2 * hk * dk + hv * dv, W)
    L = _layer(3, hk, hv, dk, dv, W, 1)
    with pytest.raises(_lib.Unsupported):
        nm.delta_decode_token(st, conv, _t(L["w"], dev), _t(L["qkv"][0], dev), _t(L["br"][0], dev),
                              _t(L["ar"][0], dev), _t(L["dtb"], dev), _t(L["dsc"], dev), hk, _t(L["z"][0], dev),
                              _t(L["gamma"], dev), 1e-6)
