"""Device KV cache + attention parity against the oracle (and the reference's fixtures).

Tolerance (north star): max abs <= 2e-3 and rel L2 <= 1e-3 versus the fp32
reference path on identical pre-rounded inputs; positions, visible rows and
window membership exact.
"""
import glob
import os

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close, load_attn_fixture
from hero_b200 import nm
from hero_b200._lib import InvalidArgument, LengthError, LogicError, NoVisibleKeys, OutOfRange

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def T(a, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dtype)


def TD(a, dev, code):
    return T(a, dev, {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[code])


def rnd(code, seed, stream, shape):
    x = oracle.normal(seed, stream, int(np.prod(shape))).reshape(shape)
    if code == "bf16":
        return oracle.round_bf16(x).reshape(shape)
    if code == "f16":
        return oracle.round_fp16(x).reshape(shape)
    return x


# ---- the reference's known-answer tests through the device path ---------------

def test_causal_attention_equation(dev):
    # property_tests.cpp:187-215
    cache = nm.FullAttentionCache(1, 2, capacity=8)
    keys = T([[1, 0], [0, 1]], dev)
    values = T([[10, 0], [30, 0]], dev)
    cache.append(0, keys, values)
    q = T([[1, 0], [0, 1]], dev)
    scale = float(np.float32(1 / np.sqrt(np.float32(2))))
    out = nm.attend(cache, q, 0, scale).cpu().numpy()
    w1 = np.exp(np.float32(scale)) / (1 + np.exp(np.float32(scale)))
    assert out[0, 0] == 10.0
    assert abs(out[1, 0] - ((1 - w1) * 10 + w1 * 30)) < 1e-5
    # the local cache owns its width-1 visibility (property_tests.cpp:217-222)
    local = nm.LocalAttentionCache(1, 2, 1)
    local.append(0, keys[0], values[0])
    local.append(1, keys[1], values[1])
    assert nm.attend(local, q[1:], 1, scale).cpu().numpy()[0, 0] == 30.0


def test_gemma_gqa_window_and_ring(dev):
    # gemma4_tests.cpp:122-172
    k0, v0, k1, v1 = T([1, 0], dev), T([10, 20], dev), T([0, 1], dev), T([30, 40], dev)
    full = nm.FullAttentionCache(1, 2, capacity=4)
    full.append(0, k0, v0)
    full.append(1, k1, v1)
    q = T([[1, 0, 1, 0]], dev)
    r = nm.attend(full, q, 1).cpu().numpy()
    p0 = np.exp(np.float32(1)) / (np.exp(np.float32(1)) + 1)
    assert abs(r[0, 0] - (p0 * 10 + (1 - p0) * 30)) < 1e-5 and r[0, 0] == r[0, 2]
    local = nm.LocalAttentionCache(1, 2, 1)
    local.append(0, k0, v0)
    local.append(1, k1, v1)
    r = nm.attend(local, q, 1).cpu().numpy()
    assert r[0, 0] == 30 and r[0, 1] == 40
    ring = nm.LocalAttentionCache(1, 2, 2)
    k2, v2 = T([2, 2], dev), T([50, 60], dev)
    ring.append(0, k0, v0)
    ring.append(1, k1, v1)
    ring.append(2, k2, v2)
    assert ring.size() == 2 and ring.position(0) == 1 and ring.position(1) == 2
    assert torch.equal(ring.key(0, 0), torch.tensor([0.0, 1.0])) and torch.equal(ring.value(1, 0), torch.tensor([50.0, 60.0]))
    ring.begin_batch_retention(2)
    ring.append(3, k0, v0)
    ring.append(4, k1, v1)
    assert ring.size() == 4 and ring.position(0) == 1 and ring.position(3) == 4
    # during retention the rows are all readable, in chronological order
    assert torch.equal(ring.value(0, 0), torch.tensor([30.0, 40.0])) and torch.equal(ring.value(3, 0), torch.tensor([30.0, 40.0]))
    ring.end_batch_retention()
    assert ring.size() == 2 and ring.position(0) == 3 and ring.position(1) == 4


def test_errors_match_the_reference(dev):
    cache = nm.LocalAttentionCache(1, 2, 2)
    cache.append(0, T([1, 0], dev), T([5, 0], dev))
    with pytest.raises(NoVisibleKeys):  # property_tests.cpp:301-316
        cache.visible_rows(9)
    with pytest.raises(NoVisibleKeys):
        nm.attend(cache, T([[1, 0]], dev), 9)
    with pytest.raises(InvalidArgument):  # attention.hpp:322
        cache.append(5, T([1, 0], dev), T([5, 0], dev))
    with pytest.raises(OutOfRange):  # attention.hpp:380-385
        cache.key(3, 0)
    with pytest.raises(OutOfRange):
        cache.key(0, 1)
    with pytest.raises(LogicError):  # attention.hpp:295
        cache.begin_batch_retention(3)
        cache.end_batch_retention()
    empty = nm.FullAttentionCache(1, 2, capacity=2)
    with pytest.raises(NoVisibleKeys):
        empty.visible_rows(0)
    full = nm.FullAttentionCache(1, 2, capacity=2)
    full.append(0, T([[1, 0], [0, 1]], dev), T([[1, 0], [0, 1]], dev))
    with pytest.raises(LengthError):  # device capacity
        full.append(2, T([1, 0], dev), T([1, 0], dev))
    with pytest.raises(InvalidArgument):  # Hq not a multiple of Hkv
        nm.attend(nm.FullAttentionCache(2, 2, capacity=2), T([[1, 0]], dev), 0)


def test_empty_inputs_do_nothing(dev):
    # Zero rows append nothing and reduce nothing; zero tokens leave the delta state as it was.
    cache = nm.FullAttentionCache(2, 128, capacity=4, dtype="bf16")
    z = torch.empty(0, 2 * 128, device=dev, dtype=torch.bfloat16)
    cache.append(0, z, z)
    assert cache.size() == 0
    q0 = torch.empty(0, 4 * 128, device=dev, dtype=torch.bfloat16)
    assert nm.append_attend(cache, 0, z, z, q0, 0.1).shape == (0, 4 * 128)
    assert cache.size() == 0
    st = nm.DeltaNetState(2, 128, 128)
    before = st.tensor().clone()
    e = lambda *shape: torch.empty(*shape, device=dev)
    out = nm.delta_prefill(st, e(0, 1, 128), e(0, 1, 128), e(0, 2, 128), e(0, 2), e(0, 2), 1, chunk=64)
    assert out.shape == (0, 2, 128) and torch.equal(st.tensor(), before)


def test_visible_rows_exhaustive_box(dev):
    # property_tests.cpp:318-338 through the device cache's bookkeeping
    for width in range(1, 5):
        for anchor in range(4):
            for rows in range(1, 6):
                c = nm.LocalAttentionCache(1, 2, width, capacity=8)
                m = oracle.CacheModel(width, local=True)
                for r in range(rows):
                    c.append(anchor + r, T([0, 0], dev), T([0, 0], dev))
                    m.append(anchor + r)
                assert c.size() == m.size
                for query in range(10):
                    try:
                        want = m.visible_rows(query)
                    except oracle.NoVisibleKeys:
                        with pytest.raises(NoVisibleKeys):
                            c.visible_rows(query)
                        continue
                    got = c.visible_rows(query)
                    assert (got.first, got.end) == want


# ---- golden fixtures written by the reference ---------------------------------

@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(HERE, "golden", "attn_*.npz"))))
def test_golden_fixtures(dev, path):
    z = load_attn_fixture(path)
    hq, hkv, dh = int(z["hq"]), int(z["hkv"]), int(z["dh"])
    window, first_query, oldest = int(z["window"]), int(z["first_query"]), int(z["oldest"])
    code = str(z["dtype"]) if dh >= 64 else "f32"
    rows, qrows = z["k"].shape[0], z["q"].shape[0]
    scale = float(z["scale"]) if bool(z["use_scale"]) else None
    if window:
        cache = nm.LocalAttentionCache(hkv, dh, window, capacity=((rows + window + 127) // 128) * 128, dtype=code)
        hist = rows - qrows
        if hist:
            cache.append(oldest, TD(z["k"][:hist], dev, code), TD(z["v"][:hist], dev, code))
        out = nm.append_attend(cache, oldest + hist, TD(z["k"][hist:], dev, code), TD(z["v"][hist:], dev, code),
                               TD(z["q"], dev, code), scale, out_dtype=torch.float32)
    else:
        cache = nm.FullAttentionCache(hkv, dh, capacity=((rows + 127) // 128) * 128, dtype=code)
        cache.append(oldest, TD(z["k"], dev, code), TD(z["v"], dev, code))
        out = nm.attend(cache, TD(z["q"], dev, code), first_query, scale, out_dtype=torch.float32)
    assert_close(out.cpu().numpy(), z["out"], what=os.path.basename(path))


# ---- seeded random parity at BASELINE shapes -----------------------------------

def test_config1_decode_fp32(dev):
    hq, hkv, dh, rows = 16, 8, 128, 1024
    k, v = rnd("f32", 0, 1, (rows, hkv * dh)), rnd("f32", 0, 2, (rows, hkv * dh))
    q = rnd("f32", 0, 3, (1, hq * dh))
    cache = nm.FullAttentionCache(hkv, dh, capacity=rows)
    cache.append(0, T(k, dev), T(v, dev))
    s = float(np.float32(1 / np.sqrt(np.float32(dh))))
    out = nm.attend(cache, T(q, dev), rows - 1, s).cpu().numpy()
    want = oracle.attend(k, v, 0, 0, hkv, dh, q, hq, rows - 1, scale=np.float32(s))
    assert_close(out, want, what="config 1")


@pytest.mark.parametrize("S", [128, 200, 640])
def test_config2_prefill_bf16(dev, S):
    hq, hkv, dh = 32, 8, 128
    k, v = rnd("bf16", 0, 1, (S, hkv * dh)), rnd("bf16", 0, 2, (S, hkv * dh))
    q = rnd("bf16", 0, 3, (S, hq * dh))
    cache = nm.FullAttentionCache(hkv, dh, capacity=((S + 127) // 128) * 128, dtype="bf16")
    s = float(np.float32(1 / np.sqrt(np.float32(dh))))
    out = nm.append_attend(cache, 0, TD(k, dev, "bf16"), TD(v, dev, "bf16"), TD(q, dev, "bf16"), s,
                           out_dtype=torch.float32).cpu().numpy()
    want = oracle.attend(k, v, 0, 0, hkv, dh, q, hq, 0, scale=np.float32(s))
    assert_close(out, want, what=f"config 2 S={S}")


def test_config2_full_size_rows_subset(dev):
    # S = 4096 through the kernel; the oracle checks a spread of rows (first,
    # last, tile edges, random) so it finishes in seconds.
    S, hq, hkv, dh = 4096, 32, 8, 128
    k, v = rnd("bf16", 0, 1, (S, hkv * dh)), rnd("bf16", 0, 2, (S, hkv * dh))
    q = rnd("bf16", 0, 3, (S, hq * dh))
    cache = nm.FullAttentionCache(hkv, dh, capacity=S, dtype="bf16")
    s = float(np.float32(1 / np.sqrt(np.float32(dh))))
    out = nm.append_attend(cache, 0, TD(k, dev, "bf16"), TD(v, dev, "bf16"), TD(q, dev, "bf16"), s,
                           out_dtype=torch.float32).cpu().numpy()
    rows = sorted({0, 1, 127, 128, 129, 1023, 2048, 4095} | set(np.random.default_rng(0).integers(0, S, 24).tolist()))
    for r in rows:
        want = oracle.attend(k, v, 0, 0, hkv, dh, q[r:r + 1], hq, r, scale=np.float32(s))
        assert_close(out[r:r + 1], want, what=f"config 2 row {r}")
    # bf16 output (the bench's dtype) stays within bf16 rounding of the fp32 result
    out16 = nm.attend(cache, TD(q, dev, "bf16"), 0, s).float().cpu().numpy()
    assert np.abs(out16 - out).max() <= 2.0 ** -8 * max(1.0, np.abs(out).max())


@pytest.mark.parametrize("S,window", [(2048, 1024), (1500, 256), (700, 1024)])
def test_config4_gemma_prefill_window(dev, S, window):
    # Gemma local layers: scale 1.0, RMS-normed q/k, window 1024, batch larger
    # than the window -> the reference's token-by-token path.
    hq, hkv, dh = 8, 4, 256

    def normed(seed, stream, shape):
        x = oracle.normal(seed, stream, int(np.prod(shape))).reshape(-1, dh).astype(np.float64)
        x = x / np.sqrt((x * x).mean(axis=1, keepdims=True) + 1e-6)
        return oracle.round_bf16(x.astype(np.float32)).reshape(shape)

    k, q = normed(4, 1, (S, hkv * dh)), normed(4, 3, (S, hq * dh))
    v = rnd("bf16", 4, 2, (S, hkv * dh))
    cache = nm.LocalAttentionCache(hkv, dh, window, capacity=((S + window + 127) // 128) * 128, dtype="bf16")
    out = nm.append_attend(cache, 0, TD(k, dev, "bf16"), TD(v, dev, "bf16"), TD(q, dev, "bf16"), None,
                           out_dtype=torch.float32).cpu().numpy()
    rows = sorted({0, 1, window - 1, window, window + 1, S - 1} & set(range(S)) |
                  set(np.random.default_rng(1).integers(0, S, 12).tolist()))
    for r in rows:
        want = oracle.attend(k[:r + 1], v[:r + 1], 0, window, hkv, dh, q[r:r + 1], hq, r, use_scale=False)
        assert_close(out[r:r + 1], want, what=f"config 4 row {r}")
    # the ring now holds the reference's logical window
    assert cache.size() == min(S, window) and cache.position(0) == S - min(S, window)
    # and decode continues from it: the global/local decode step of config 4
    qd = normed(4, 5, (1, hq * dh))
    kd, vd = normed(4, 6, (1, hkv * dh)), rnd("bf16", 4, 7, (1, hkv * dh))
    outd = nm.append_attend(cache, S, TD(kd, dev, "bf16"), TD(vd, dev, "bf16"), TD(qd, dev, "bf16"), None,
                            out_dtype=torch.float32).cpu().numpy()
    kk, vv = np.concatenate([k, kd]), np.concatenate([v, vd])
    want = oracle.attend(kk, vv, 0, window, hkv, dh, qd, hq, S, use_scale=False)
    assert_close(outd, want, what="config 4 decode")


def test_config5_ragged_batch_f16_group8(dev):
    hq, hkv, dh, B = 64, 8, 128, 6
    lens = [17, 130, 1000, 4096, 5000, 257]
    caches, ks, vs = [], [], []
    for b, L in enumerate(lens):
        k, v = rnd("f16", 5, 10 + 2 * b, (L, hkv * dh)), rnd("f16", 5, 11 + 2 * b, (L, hkv * dh))
        c = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="f16")
        c.append(0, TD(k, dev, "f16"), TD(v, dev, "f16"))
        caches.append(c)
        ks.append(k)
        vs.append(v)
    q = rnd("f16", 5, 1, (B, hq * dh))
    s = float(np.float32(1 / np.sqrt(np.float32(dh))))
    out = nm.attend_batch(caches, TD(q, dev, "f16"), s, out_dtype=torch.float32).cpu().numpy()
    for b, L in enumerate(lens):
        want = oracle.attend(ks[b], vs[b], 0, 0, hkv, dh, q[b:b + 1], hq, L - 1, scale=np.float32(s))
        assert_close(out[b:b + 1], want, what=f"config 5 seq {b} len {L}")


def test_ring_wraps_across_many_batches(dev):
    # A local cache whose physical ring wraps many times, attended after every
    # batch (decode-style and short-batch-style) against the oracle's window.
    hq, hkv, dh, W = 4, 2, 64, 96
    cache = nm.LocalAttentionCache(hkv, dh, W, capacity=128, dtype="f32")
    total = 700
    k, v = rnd("f32", 6, 1, (total, hkv * dh)), rnd("f32", 6, 2, (total, hkv * dh))
    q = rnd("f32", 6, 3, (total, hq * dh))
    pos, sizes = 0, [1, 5, 33, 1, 64, 7, 1, 100, 1, 200, 31, 1, 2]
    for n in sizes:
        out = nm.append_attend(cache, pos, T(k[pos:pos + n], dev), T(v[pos:pos + n], dev), T(q[pos:pos + n], dev),
                               0.125).cpu().numpy()
        for r in range(n):
            p = pos + r
            lo = max(0, p - W + 1)
            want = oracle.attend(k[lo:p + 1], v[lo:p + 1], lo, W, hkv, dh, q[p:p + 1], hq, p, scale=np.float32(0.125))
            assert_close(out[r:r + 1], want, what=f"ring pos {p}")
        pos += n
    assert cache.size() == W and cache.position(0) == pos - W


def test_dense_sdpa(dev):
    # scaled_dot_product_attention<Heads,D,D> (attention.hpp:124-139): no mask.
    heads, dh, tq, tk = 4, 64, 37, 300
    q, k, v = rnd("f32", 8, 1, (tq, heads * dh)), rnd("f32", 8, 2, (tk, heads * dh)), rnd("f32", 8, 3, (tk, heads * dh))
    out = nm.scaled_dot_product_attention(T(q, dev), T(k, dev), T(v, dev), heads, 0.125).cpu().numpy()
    want = oracle.attend(k, v, 0, 0, heads, dh, q, heads, tk - 1, scale=np.float32(0.125))
    assert_close(out, want, what="sdpa")
    # bf16 through the tensor-core kernel
    qb, kb, vb = (rnd("bf16", 8, i, s) for i, s in ((4, (256, heads * 128)), (5, (256, heads * 128)), (6, (256, heads * 128))))
    out = nm.scaled_dot_product_attention(TD(qb, dev, "bf16"), TD(kb, dev, "bf16"), TD(vb, dev, "bf16"), heads, 0.1,
                                          out_dtype=torch.float32).cpu().numpy()
    want = oracle.attend(kb, vb, 0, 0, heads, 128, qb, heads, 255, scale=np.float32(0.1))
    assert_close(out, want, what="sdpa bf16")


def test_first_launch_in_a_fresh_process(dev):
    # The first tensor-core prefill launch of a process runs against cold
    # caches (and leftover shared/tensor memory); a synchronisation slip shows
    # up there and nowhere else, so check it in a new interpreter each time.
    import subprocess
    import sys

    code = r"""
import sys, math, torch
sys.path.insert(0, %r)
from hero_b200 import nm
dev = torch.device('cuda:0')
torch.manual_seed(int(sys.argv[1]))
hq, hkv, T, dh, scale = 4, 4, 256, 128, 0.1
q = torch.randn(T, hq*dh, device=dev).bfloat16(); k = torch.randn(T, hkv*dh, device=dev).bfloat16()
v = torch.randn(T, hkv*dh, device=dev).bfloat16()
qf, kf, vf = q.float().view(T, hq, dh), k.float().view(T, hkv, dh), v.half().float().view(T, hkv, dh)
ref = torch.einsum('hts,shd->thd', torch.softmax(torch.einsum('thd,shd->hts', qf, kf) * scale, -1), vf)
c = nm.FullAttentionCache(hkv, dh, capacity=T, dtype='bf16'); c.append(0, k, v)
out = torch.full((T, hq*dh), float('nan'), device=dev)
nm.attend(c, q, T - 1, scale, out=out)
nm.device_status(0)
print(float((out.view(T, hq, dh) - ref).abs().max()))
""" % (os.path.dirname(HERE),)
    for seed in range(3):
        r = subprocess.run([sys.executable, "-c", code, str(seed)], capture_output=True, text=True, timeout=120)
        assert r.returncode == 0, r.stderr[-2000:]
        assert float(r.stdout.strip().splitlines()[-1]) < 2e-3


@pytest.mark.parametrize("rows", [256, 3])
def test_attend_fanout_writes_every_output(dev, rows):
    # The multi-GPU gather rides on this: each output row lands in every
    # buffer at the given column offset (tcgen05 epilogue for 256 rows, the
    # staged copy for a decode-sized call), bit-identical to nmg_attend.
    hq, hkv, dh, S = 8, 2, 128, 512
    g = torch.Generator(device=dev)
    g.manual_seed(rows)
    cache = nm.FullAttentionCache(hkv, dh, capacity=S, dtype="bf16")
    cache.append(0, torch.randn(S, hkv * dh, device=dev, generator=g).bfloat16(),
                 torch.randn(S, hkv * dh, device=dev, generator=g).bfloat16())
    q = torch.randn(rows, hq * dh, device=dev, generator=g).bfloat16()
    at = S - rows
    want = nm.attend(cache, q, at, dh ** -0.5, out_dtype=torch.bfloat16)
    width, col0 = 3 * hq * dh, hq * dh
    outs = [torch.full((rows, width), float("nan"), device=dev, dtype=torch.bfloat16) for _ in range(2)]
    nm.attend_fanout(cache, q, at, dh ** -0.5, [o.data_ptr() for o in outs], width, col0, torch.bfloat16)
    torch.cuda.synchronize(dev)
    for o in outs:
        assert torch.equal(o[:, col0:col0 + hq * dh], want)
        assert torch.isnan(o[:, :col0].float()).all() and torch.isnan(o[:, col0 + hq * dh:].float()).all()


def test_attend_fanout_rejects_columns_that_do_not_fit(dev):
    cache = nm.FullAttentionCache(2, 128, capacity=128, dtype="bf16")
    cache.append(0, torch.zeros(128, 256, device=dev).bfloat16(), torch.zeros(128, 256, device=dev).bfloat16())
    q = torch.zeros(128, 8 * 128, device=dev).bfloat16()
    o = torch.empty(128, 8 * 128, device=dev, dtype=torch.bfloat16)
    with pytest.raises(InvalidArgument):
        nm.attend_fanout(cache, q, 0, 1.0, [o.data_ptr()], 8 * 128, 128, torch.bfloat16)


def test_prefill_key_splits_match_oracle(dev):
    # 4 query heads over 4096 causal rows is little work for the GPU, so the
    # heavy query tiles are split over several CTAs (8 key blocks each) whose
    # partials the last CTA merges; the heaviest and lightest tiles against
    # the reference reduction.
    hq, hkv, dh, S = 4, 2, 128, 4096
    k, v, q = rnd("bf16", 31, 1, (S, hkv * dh)), rnd("bf16", 31, 2, (S, hkv * dh)), rnd("bf16", 31, 3, (S, hq * dh))
    cache = nm.FullAttentionCache(hkv, dh, capacity=S, dtype="bf16")
    cache.append(0, TD(k, dev, "bf16"), TD(v, dev, "bf16"))
    scale = dh ** -0.5
    out = nm.attend(cache, TD(q, dev, "bf16"), 0, scale, out_dtype=torch.float32).cpu().numpy()
    for r0, r1 in ((S - 256, S), (0, 128)):
        want = oracle.attend(k, v, 0, 0, hkv, dh, q[r0:r1], hq, r0, scale=np.float32(scale))
        assert_close(out[r0:r1], want, what=f"rows {r0}:{r1}")
    for _ in range(2):  # tickets return to zero: the same result again
        again = nm.attend(cache, TD(q, dev, "bf16"), 0, scale, out_dtype=torch.float32).cpu().numpy()
        assert np.array_equal(again, out)


def test_prefill_key_splits_with_fanout(dev):
    hq, hkv, dh, S = 4, 2, 128, 4096
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    cache = nm.FullAttentionCache(hkv, dh, capacity=S, dtype="bf16")
    cache.append(0, torch.randn(S, hkv * dh, device=dev, generator=g).bfloat16(),
                 torch.randn(S, hkv * dh, device=dev, generator=g).bfloat16())
    q = torch.randn(S, hq * dh, device=dev, generator=g).bfloat16()
    want = nm.attend(cache, q, 0, dh ** -0.5, out_dtype=torch.bfloat16)
    width, col0 = 2 * hq * dh, hq * dh
    outs = [torch.zeros(S, width, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    nm.attend_fanout(cache, q, 0, dh ** -0.5, [o.data_ptr() for o in outs], width, col0, torch.bfloat16)
    torch.cuda.synchronize(dev)
    for o in outs:
        assert torch.equal(o[:, col0:], want)
        assert not o[:, :col0].any()


def test_prefill_many_units_per_cta_match_oracle(dev):
    # 10 query tiles x 32 heads = 320 units on at most 148 persistent CTAs:
    # each CTA takes two or three units in snake order, alternating its two
    # O accumulators, so unit boundaries, the overlapped epilogue and the
    # next unit's first S all run; every row against the reference.
    hq, hkv, dh, S = 32, 8, 128, 1280
    k, v, q = rnd("bf16", 41, 1, (S, hkv * dh)), rnd("bf16", 41, 2, (S, hkv * dh)), rnd("bf16", 41, 3, (S, hq * dh))
    cache = nm.FullAttentionCache(hkv, dh, capacity=S, dtype="bf16")
    cache.append(0, TD(k, dev, "bf16"), TD(v, dev, "bf16"))
    scale = dh ** -0.5
    out = nm.attend(cache, TD(q, dev, "bf16"), 0, scale, out_dtype=torch.float32).cpu().numpy()
    want = oracle.attend(k, v, 0, 0, hkv, dh, q, hq, 0, scale=np.float32(scale))
    assert_close(out, want, what="all rows")
    bf = nm.attend(cache, TD(q, dev, "bf16"), 0, scale, out_dtype=torch.bfloat16)
    assert torch.equal(bf, torch.from_numpy(out).to(dev).to(torch.bfloat16))  # the epilogue rounds like a cast


def test_prefill_head_dim_256_window_many_units(dev):
    # head_dim 256 (one O accumulator: each unit's epilogue is waited for
    # before the next unit's first P.V) with a sliding window, 304 units.
    hq, hkv, dh, S, W = 8, 4, 256, 4864, 1024
    k, v, q = rnd("bf16", 43, 1, (S, hkv * dh)), rnd("bf16", 43, 2, (S, hkv * dh)), rnd("bf16", 43, 3, (S, hq * dh))
    cache = nm.LocalAttentionCache(hkv, dh, W, capacity=((S + W + 127) // 128) * 128, dtype="bf16")
    out = nm.append_attend(cache, 0, TD(k, dev, "bf16"), TD(v, dev, "bf16"), TD(q, dev, "bf16"), None,
                           out_dtype=torch.float32).cpu().numpy()
    for r0, r1 in ((0, 256), (2304, 2560), (S - 256, S)):
        want = oracle.attend(k[:r1], v[:r1], 0, W, hkv, dh, q[r0:r1], hq, r0, use_scale=False)
        assert_close(out[r0:r1], want, what=f"rows {r0}:{r1}")


@pytest.mark.parametrize("dtype,slots,window", [("bf16", 1856, 256), ("f16", 1856, 0), ("f16", 1920, 700)])
def test_prefill_head_dim_256_block_sizes(dev, dtype, slots, window):
    # head_dim 256 runs 128-key blocks (K in four 64-dimension pieces, V in two
    # 64-key pieces) when the cache's slots are a multiple of 128, and 64-key
    # blocks otherwise (1856 = 29 x 64); both against the oracle.
    hq, hkv, dh, S = 8, 4, 256, 1500
    k, v, q = rnd(dtype, 44, 1, (S, hkv * dh)), rnd(dtype, 44, 2, (S, hkv * dh)), rnd(dtype, 44, 3, (S, hq * dh))
    cache = (nm.LocalAttentionCache(hkv, dh, window, capacity=slots, dtype=dtype) if window
             else nm.FullAttentionCache(hkv, dh, capacity=slots, dtype=dtype))
    out = nm.append_attend(cache, 0, TD(k, dev, dtype), TD(v, dev, dtype), TD(q, dev, dtype), None,
                           out_dtype=torch.float32).cpu().numpy()
    for r0, r1 in ((0, 192), (640, 800), (S - 200, S)):
        want = oracle.attend(k[:r1], v[:r1], 0, window, hkv, dh, q[r0:r1], hq, r0, use_scale=False)
        assert_close(out[r0:r1], want, what=f"{dtype} slots {slots} rows {r0}:{r1}")


@pytest.mark.parametrize("dtype,window", [("bf16", 0), ("f16", 0), ("bf16", 200)])
def test_prefill_head_dim_64_matches_oracle(dev, dtype, window):
    # head_dim 64 through the tensor-core kernel (128-key blocks, P.V with N = 64).
    hq, hkv, dh, S = 6, 2, 64, 700
    k, v, q = rnd(dtype, 44, 1, (S, hkv * dh)), rnd(dtype, 44, 2, (S, hkv * dh)), rnd(dtype, 44, 3, (S, hq * dh))
    if window:
        cache = nm.LocalAttentionCache(hkv, dh, window, capacity=((S + window + 127) // 128) * 128, dtype=dtype)
    else:
        cache = nm.FullAttentionCache(hkv, dh, capacity=768, dtype=dtype)
    out = nm.append_attend(cache, 0, TD(k, dev, dtype), TD(v, dev, dtype), TD(q, dev, dtype), 0.125,
                           out_dtype=torch.float32).cpu().numpy()
    want = oracle.attend(k, v, 0, window, hkv, dh, q, hq, 0, scale=np.float32(0.125))
    assert_close(out, want, what=f"head_dim 64 {dtype} window {window}")


def test_sdpa_vision_shape(dev):
    # scaled_dot_product_attention<12, 64, 64> with scale 1 (gemma4_vision.hpp:167)
    # at the ViT's largest image, 2520 patch tokens, in bf16 on the tensor cores.
    heads, dh, n = 12, 64, 2520
    q, k, v = (rnd("bf16", 45, i, (n, heads * dh)) for i in (1, 2, 3))
    q = oracle.round_bf16(q * np.float32(0.125)).reshape(q.shape)  # normed Q/K keep scale-1 scores moderate
    out = nm.scaled_dot_product_attention(TD(q, dev, "bf16"), TD(k, dev, "bf16"), TD(v, dev, "bf16"), heads, 1.0,
                                          out_dtype=torch.float32).cpu().numpy()
    want = oracle.attend(k, v, 0, 0, heads, dh, q, heads, n - 1, scale=np.float32(1.0))
    assert_close(out, want, what="vision sdpa")
