"""Parity against the CPU oracle at the benchmark configurations' full sizes.

Configs 3, 4 (decode) and 5 are compared with the oracle (a C restatement of
the reference's arithmetic, pinned to the reference build) on the sizes the
benchmark times, not on cut-down shapes:

* config 3: 8192 prefill tokens at chunk 64, then 256 decode steps from the
  final state (qwen35.hpp:436-456), outputs of every token and the final state;
* config 4: decode of batch 16 with 32768 cached rows per sequence, query at
  position 32767, through a global layer and a sliding-window (1024) layer
  (gemma4.hpp:593-615, :687-709), every sequence;
* config 5: the seed-1 ragged lengths in [4096, 131072] over all 64 sequences
  in one batched call, a deterministic subset checked that includes the
  shortest and the longest sequence (qwen35.hpp:360-382).
"""
import math

import numpy as np
import pytest
import torch

import oracle
from bench import ragged_lengths
from helpers import assert_close, delta_inputs
from hero_b200 import nm

pytestmark = pytest.mark.gpu


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


def test_config3_full_prefill_then_256_decode_steps(dev):
    hv, hk, d, Tp, Td = 32, 16, 128, 8192, 256
    q, k, v, g, b = delta_inputs(3, Tp + Td, hk, hv, d)
    st = nm.DeltaNetState(hv, d, d)
    out = nm.delta_prefill(st, _t(q[:Tp], dev), _t(k[:Tp], dev), _t(v[:Tp], dev), _t(g[:Tp], dev), _t(b[:Tp], dev),
                           hk, chunk=64).cpu().numpy()
    want, ws = oracle.delta_run(np.zeros((hv, d, d), np.float32), q[:Tp], k[:Tp], v[:Tp], g[:Tp], b[:Tp], hk)
    assert_close(out, want, what="prefill out (8192 tokens)")
    assert_close(st.tensor().cpu().numpy(), ws, what="prefill state")
    qd, kd, vd, gd, bd = (_t(x[Tp:], dev) for x in (q, k, v, g, b))
    od = torch.empty(Td, hv, d, device=dev)
    for t in range(Td):
        nm.delta_step(st, qd[t], kd[t], vd[t], gd[t], bd[t], hk, out=od[t])
    wd, ws = oracle.delta_run(ws, q[Tp:], k[Tp:], v[Tp:], g[Tp:], b[Tp:], hk)
    assert_close(od.cpu().numpy(), wd, what="256 decode steps")
    assert_close(st.tensor().cpu().numpy(), ws, what="state after 256 decode steps")


def _rms(x):
    return x / x.pow(2).mean(dim=-1, keepdim=True).add(1e-6).sqrt()


def test_config4_decode_batch16_32768_rows(dev):
    hq, hkv, dh, W, B, L = 8, 4, 256, 1024, 16, 32768
    g = torch.Generator(device=dev)
    g.manual_seed(44)
    gcaches, lcaches, host = [], [], []
    for _ in range(B):
        kk = _rms(torch.randn(L, hkv, dh, device=dev, generator=g)).reshape(L, hkv * dh).bfloat16()
        vv = torch.randn(L, hkv * dh, device=dev, generator=g).bfloat16()
        c = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="bf16")
        c.append(0, kk, vv)
        gcaches.append(c)
        lc = nm.LocalAttentionCache(hkv, dh, W, capacity=2 * W, dtype="bf16")
        lc.append(L - W, kk[L - W:], vv[L - W:])
        lcaches.append(lc)
        host.append((kk, vv))
    q = _rms(torch.randn(B, hq, dh, device=dev, generator=g)).reshape(B, hq * dh).bfloat16()
    og = nm.attend_batch(gcaches, q, None, out_dtype=torch.float32).cpu().numpy()
    ol = nm.attend_batch(lcaches, q, None, out_dtype=torch.float32).cpu().numpy()
    qh = q.float().cpu().numpy()
    for bi, (kk, vv) in enumerate(host):
        kf, vf = kk.float().cpu().numpy(), vv.float().cpu().numpy()
        wg = oracle.attend(kf, vf, 0, 0, hkv, dh, qh[bi:bi + 1], hq, L - 1, use_scale=False)
        wl = oracle.attend(kf[L - W:], vf[L - W:], L - W, W, hkv, dh, qh[bi:bi + 1], hq, L - 1, use_scale=False)
        assert_close(og[bi:bi + 1], wg, what=f"global layer, sequence {bi}")
        assert_close(ol[bi:bi + 1], wl, what=f"sliding-window layer, sequence {bi}")


def test_config5_ragged_batch64(dev):
    B, hq, hkv, dh = 64, 64, 8, 128
    lens = ragged_lengths(1, B, 4096, 131072)
    scale = 1.0 / math.sqrt(dh)

    def rows(b, L):
        g = torch.Generator(device=dev)
        g.manual_seed(5000 + b)
        return (torch.randn(L, hkv * dh, device=dev, generator=g).half(),
                torch.randn(L, hkv * dh, device=dev, generator=g).half())

    caches = []
    for b, L in enumerate(lens):
        k, v = rows(b, L)
        c = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="f16")
        c.append(0, k, v)
        caches.append(c)
        del k, v
    gq = torch.Generator(device=dev)
    gq.manual_seed(55)
    q = torch.randn(B, hq * dh, device=dev, generator=gq).half()
    out = nm.attend_batch(caches, q, scale, out_dtype=torch.float32).cpu().numpy()
    qh = q.float().cpu().numpy()
    order = sorted(range(B), key=lambda i: lens[i])
    check = sorted({order[0], order[-1], order[B // 2], 0, 1, B - 1})
    assert lens[order[-1]] > 100000 and lens[order[0]] < 10000
    for b in check:
        k, v = rows(b, lens[b])
        want = oracle.attend(k.float().cpu().numpy(), v.float().cpu().numpy(), 0, 0, hkv, dh, qh[b:b + 1], hq,
                             lens[b] - 1, scale=np.float32(scale))
        assert_close(out[b:b + 1], want, what=f"sequence {b} ({lens[b]} rows)")
