"""The multi-GPU split on the CPU: two gloo ranks each reduce their KV-head
shard with the oracle, gather the shards, and lay them back into rows; the
result must equal the unsharded reduction exactly (heads are independent).
Also the handle exchange the GPU path uses to map peer buffers."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

from hero_b200.shard import decode_shard, delta_shard, heads_to_rows, kv_shard, take_heads

HQ, HKV, DH, S = 8, 4, 16, 40


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests"))
    import torch
    import torch.distributed as dist

    import oracle
    from hero_b200.shard import exchange, kv_shard, take_heads

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        k = oracle.normal(5, 1, S * HKV * DH).reshape(S, HKV * DH)
        v = oracle.normal(5, 2, S * HKV * DH).reshape(S, HKV * DH)
        q = oracle.normal(5, 3, S * HQ * DH).reshape(S, HQ * DH)
        sh = kv_shard(rank, world, HKV, HQ)
        part = oracle.attend(take_heads(k, HKV, DH, sh.kv0, sh.kv1), take_heads(v, HKV, DH, sh.kv0, sh.kv1), 0, 0,
                             sh.kv1 - sh.kv0, DH, take_heads(q, HQ, DH, sh.q0, sh.q1), sh.q1 - sh.q0, 0,
                             scale=np.float32(0.25), threads=1)
        parts = [torch.empty(S, part.shape[1]) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part))
        # rank r's block is the column range [q0_r * DH, q1_r * DH) of every row
        rows = np.zeros((S, HQ * DH), np.float32)
        for r, p in enumerate(parts):
            sr = kv_shard(r, world, HKV, HQ)
            rows[:, sr.out_col0(DH):sr.q1 * DH] = p.numpy()
        want = oracle.attend(k, v, 0, 0, HKV, DH, q, HQ, 0, scale=np.float32(0.25), threads=1)
        handles = exchange(dist, bytes([rank]) * 64)
        results[rank] = (bool(np.array_equal(rows, want)), handles == [bytes([r]) * 64 for r in range(world)])
    finally:
        dist.destroy_process_group()


def test_kv_head_shards_gathered_equal_the_whole_reduction():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: (True, True), 1: (True, True)}


def test_shard_plan():
    shards = [kv_shard(r, 4, 8, 32) for r in range(4)]
    assert [(s.kv0, s.kv1, s.q0, s.q1) for s in shards] == [(0, 2, 0, 8), (2, 4, 8, 16), (4, 6, 16, 24), (6, 8, 24, 32)]
    assert shards[2].out_col0(128) == 16 * 128
    with pytest.raises(ValueError):
        kv_shard(0, 3, 8, 32)  # 3 ranks do not divide 8 KV heads
    x = np.arange(2 * 4 * 3).reshape(2, 12)
    assert (take_heads(x, 4, 3, 1, 3) == x[:, 3:9]).all()
    assert (heads_to_rows(np.arange(2 * 3 * 4).reshape(2, 3, 4), 2, 3, 4)
            == np.concatenate([np.arange(12).reshape(3, 4), np.arange(12, 24).reshape(3, 4)], axis=1)).all()


def test_plans_for_more_ranks_than_kv_heads():
    # prefill: the 2 ranks of a KV head split its query heads; blocks still tile each row in rank order
    shards = [kv_shard(r, 8, 4, 8) for r in range(8)]
    assert [(s.kv0, s.q0, s.q1) for s in shards] == [(r // 2, r, r + 1) for r in range(8)]
    with pytest.raises(ValueError):
        kv_shard(0, 8, 4, 4)  # a group of one query head cannot be split in two
    # decode: KV heads across 4 ranks, the batch of 16 in two parts
    d = [decode_shard(r, 8, 4, 8, 16) for r in range(8)]
    assert [(x.heads.kv0, x.heads.q0, x.b0, x.b1) for x in d] == \
        [(r % 4, 2 * (r % 4), 8 * (r // 4), 8 * (r // 4) + 8) for r in range(8)]
    assert all(x.kv_world == 4 and x.parts == 2 for x in d)
    assert decode_shard(3, 4, 8, 64, 64).parts == 1
    with pytest.raises(ValueError):
        decode_shard(0, 8, 4, 8, 3)  # 2 parts do not divide 3 sequences
    # delta rule: key-head groups with the tiled value heads (h reads key head h % 16)
    for world in (1, 2, 4, 8, 16):
        owned = []
        for r in range(world):
            s = delta_shard(r, world, 16, 32)
            assert s.hk == 16 // world and s.hv == 32 // world
            for i, h in enumerate(s.v_heads):
                assert h % 16 == s.k0 + i % s.hk  # local head i reads local key head i % hk
            owned += s.v_heads
        assert sorted(owned) == list(range(32))
    with pytest.raises(ValueError):
        delta_shard(0, 3, 16, 32)


def _rank_more(rank, world, port, results):
    """Each rank runs its shard of three splits through the oracle; the
    gathered, reassembled result must equal the unsharded one bit for bit."""
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch
    import torch.distributed as dist

    import oracle
    from hero_b200.shard import decode_shard, delta_shard, heads_to_rows, kv_shard, take_heads

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))

    def gather(a):
        a = np.ascontiguousarray(a, dtype=np.float32)
        parts = [torch.empty(a.shape) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(a))
        return np.stack([p.numpy() for p in parts])

    try:
        ok = []
        # (1) gated delta rule by key-head group: hk = 4, hv = 8, T = 12
        hk, hv, d, T = 4, 8, 8, 12
        q = oracle.l2_normalize(oracle.normal(9, 1, T * hk * d).reshape(T, hk, d)) * np.float32(d ** -0.5)
        k = oracle.l2_normalize(oracle.normal(9, 2, T * hk * d).reshape(T, hk, d))
        v = oracle.normal(9, 3, T * hv * d).reshape(T, hv, d)
        g = -np.log1p(np.exp(oracle.normal(9, 4, T * hv))).astype(np.float32).reshape(T, hv)
        b = (1 / (1 + np.exp(-oracle.normal(9, 5, T * hv)))).astype(np.float32).reshape(T, hv)
        s = delta_shard(rank, world, hk, hv)
        hs = list(s.v_heads)
        out, st = oracle.delta_run(np.zeros((s.hv, d, d), np.float32), q[:, s.k0:s.k1], k[:, s.k0:s.k1], v[:, hs],
                                   g[:, hs], b[:, hs], s.hk)
        R = hv // hk
        rows = heads_to_rows(gather(out.reshape(T * R, s.hk * d)), world, T * R, s.hk * d).reshape(T, hv, d)
        want, want_st = oracle.delta_run(np.zeros((hv, d, d), np.float32), q, k, v, g, b, hk)
        ok.append(bool(np.array_equal(rows, want)) and bool(np.array_equal(st, want_st[hs])))
        # (2) batched decode with more ranks than KV heads: hkv = 1, batch parts
        hq, hkv, dh, B = 2, 1, 8, 4
        lens = [5, 9, 3, 7]
        ks = [oracle.normal(11, 10 + i, n * hkv * dh).reshape(n, hkv * dh) for i, n in enumerate(lens)]
        vs = [oracle.normal(11, 20 + i, n * hkv * dh).reshape(n, hkv * dh) for i, n in enumerate(lens)]
        qd = oracle.normal(11, 30, B * hq * dh).reshape(B, hq * dh)
        ds = decode_shard(rank, world, hkv, hq, B)
        sh = ds.heads
        mine = np.concatenate([
            oracle.attend(take_heads(ks[i], hkv, dh, sh.kv0, sh.kv1), take_heads(vs[i], hkv, dh, sh.kv0, sh.kv1), 0, 0,
                          sh.kv1 - sh.kv0, dh, take_heads(qd[i:i + 1], hq, dh, sh.q0, sh.q1), sh.q1 - sh.q0,
                          lens[i] - 1, scale=np.float32(0.5), threads=1)
            for i in range(ds.b0, ds.b1)])
        gd = gather(mine)
        cols = (sh.q1 - sh.q0) * dh
        per = ds.b1 - ds.b0
        got = np.concatenate([heads_to_rows(gd[p * ds.kv_world:(p + 1) * ds.kv_world], ds.kv_world, per, cols)
                              for p in range(ds.parts)])
        want = np.concatenate([oracle.attend(ks[i], vs[i], 0, 0, hkv, dh, qd[i:i + 1], hq, lens[i] - 1,
                                             scale=np.float32(0.5), threads=1) for i in range(B)])
        ok.append(bool(np.array_equal(got, want)))
        # (3) causal prefill with more ranks than KV heads: the query heads of one group split
        S = 10
        kp = oracle.normal(12, 1, S * hkv * dh).reshape(S, hkv * dh)
        vp = oracle.normal(12, 2, S * hkv * dh).reshape(S, hkv * dh)
        qp = oracle.normal(12, 3, S * hq * dh).reshape(S, hq * dh)
        sp = kv_shard(rank, world, hkv, hq)
        part = oracle.attend(take_heads(kp, hkv, dh, sp.kv0, sp.kv1), take_heads(vp, hkv, dh, sp.kv0, sp.kv1), 0, 0,
                             sp.kv1 - sp.kv0, dh, take_heads(qp, hq, dh, sp.q0, sp.q1), sp.q1 - sp.q0, 0,
                             scale=np.float32(0.5), threads=1)
        got = heads_to_rows(gather(part), world, S, (sp.q1 - sp.q0) * dh)
        want = oracle.attend(kp, vp, 0, 0, hkv, dh, qp, hq, 0, scale=np.float32(0.5), threads=1)
        ok.append(bool(np.array_equal(got, want)))
        results[rank] = tuple(ok)
    finally:
        dist.destroy_process_group()


def test_delta_and_decode_shards_gathered_equal_the_whole():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_more, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: (True, True, True), 1: (True, True, True)}
