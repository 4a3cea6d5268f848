"""The two prefill kernels against the oracle across the shapes that pick them.

head_dim 128 with an even GQA group runs the two-head kernel (two query heads
of one group per unit, sharing every K/V block) when its units fill the GPU
(query tiles x head pairs >= 148); an odd group, or fewer units (a sharded
launch's few heads), runs the one-head kernel.  Both are checked here on
ragged tiles, sliding windows, chunked prefill into a cache that already
holds rows and many units per persistent CTA, all against the reference reduction
(qwen35.hpp:360-382, gemma4.hpp:593-615) within max abs 2e-3 / rel L2 1e-3.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close
from hero_b200 import nm

pytestmark = pytest.mark.gpu


def _rnd(code, seed, stream, shape):
    x = oracle.normal(seed, stream, int(np.prod(shape))).reshape(shape)
    return oracle.round_bf16(x).reshape(shape) if code == "bf16" else oracle.round_fp16(x).reshape(shape)


def _dev(a, dev, code):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(torch.bfloat16 if code == "bf16" else torch.float16)


@pytest.mark.parametrize("hq,hkv,S,code", [(32, 8, 1200, "bf16"), (32, 4, 1150, "f16"),
                                            (8, 4, 1000, "bf16"), (16, 2, 777, "f16"), (6, 2, 600, "bf16"),
                                           (4, 4, 300, "bf16"), (64, 8, 1280, "bf16")])
def test_prefill_groups_match_oracle(dev, hq, hkv, S, code):
    dh = 128
    seed = 100 + hq + S
    k, v, q = _rnd(code, seed, 1, (S, hkv * dh)), _rnd(code, seed, 2, (S, hkv * dh)), _rnd(code, seed, 3, (S, hq * dh))
    cache = nm.FullAttentionCache(hkv, dh, capacity=(S + 127) // 128 * 128, dtype=code)
    cache.append(0, _dev(k, dev, code), _dev(v, dev, code))
    scale = dh ** -0.5
    out = nm.attend(cache, _dev(q, dev, code), 0, scale, out_dtype=torch.float32).cpu().numpy()
    want = oracle.attend(k, v, 0, 0, hkv, dh, q, hq, 0, scale=np.float32(scale))
    assert_close(out, want, what=f"hq={hq} hkv={hkv} S={S} {code}")


def test_prefill_pair_chunked_into_a_filled_cache(dev):
    # Rows 500.. of a sequence whose first 500 rows are cached already: query
    # tiles start mid key block, and the first tile sees 4+ blocks.
    hq, hkv, dh, S0, S1 = 32, 8, 128, 500, 1200  # 10 tiles x 16 head pairs: the two-head kernel
    S = S0 + S1
    k, v, q = _rnd("bf16", 7, 1, (S, hkv * dh)), _rnd("bf16", 7, 2, (S, hkv * dh)), _rnd("bf16", 7, 3, (S1, hq * dh))
    cache = nm.FullAttentionCache(hkv, dh, capacity=1792, dtype="bf16")
    cache.append(0, _dev(k[:S0], dev, "bf16"), _dev(v[:S0], dev, "bf16"))
    out = nm.append_attend(cache, S0, _dev(k[S0:], dev, "bf16"), _dev(v[S0:], dev, "bf16"), _dev(q, dev, "bf16"),
                           0.09, out_dtype=torch.float32).cpu().numpy()
    want = oracle.attend(k, v, 0, 0, hkv, dh, q, hq, S0, scale=np.float32(0.09))
    assert_close(out, want, what="chunked prefill")


@pytest.mark.parametrize("W", [300, 1024])
def test_prefill_pair_sliding_window(dev, W):
    # A Gemma-style local layer (scale 1) through the two-head kernel: the
    # window's lower edge masks inside blocks and whole blocks drop out.
    hq, hkv, dh, S = 32, 16, 128, 2500  # 20 tiles x 16 head pairs: the two-head kernel
    k, v, q = _rnd("bf16", 9, 1, (S, hkv * dh)), _rnd("bf16", 9, 2, (S, hkv * dh)), _rnd("bf16", 9, 3, (S, hq * dh))
    q = q * np.float32(0.05)
    q = oracle.round_bf16(q).reshape(q.shape)
    cap = ((S + W + 127) // 128) * 128
    cache = nm.LocalAttentionCache(hkv, dh, W, capacity=cap, dtype="bf16")
    out = nm.append_attend(cache, 0, _dev(k, dev, "bf16"), _dev(v, dev, "bf16"), _dev(q, dev, "bf16"), None,
                           out_dtype=torch.float32).cpu().numpy()
    for r0, r1 in ((0, 256), (1100, 1400), (S - 300, S)):
        want = oracle.attend(k[:r1], v[:r1], 0, W, hkv, dh, q[r0:r1], hq, r0, use_scale=False)
        assert_close(out[r0:r1], want, what=f"W={W} rows {r0}:{r1}")


def test_prefill_pair_key_splits_repeat_exactly(dev):
    # Two query heads over 3000 causal rows: one head pair, too few units for
    # the two-head kernel, so the heads run as units of their own; repeated
    # calls agree bit for bit.
    hq, hkv, dh, S = 2, 1, 128, 3000
    k, v, q = _rnd("bf16", 11, 1, (S, hkv * dh)), _rnd("bf16", 11, 2, (S, hkv * dh)), _rnd("bf16", 11, 3, (S, hq * dh))
    cache = nm.FullAttentionCache(hkv, dh, capacity=3072, dtype="bf16")
    cache.append(0, _dev(k, dev, "bf16"), _dev(v, dev, "bf16"))
    qd = _dev(q, dev, "bf16")
    out = nm.attend(cache, qd, 0, dh ** -0.5, out_dtype=torch.float32)
    want = oracle.attend(k, v, 0, 0, hkv, dh, q, hq, 0, scale=np.float32(dh ** -0.5))
    assert_close(out.cpu().numpy(), want, what="split pair")
    for _ in range(2):
        assert torch.equal(nm.attend(cache, qd, 0, dh ** -0.5, out_dtype=torch.float32), out)
