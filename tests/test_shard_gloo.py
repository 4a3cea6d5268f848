"""The multi-GPU split on the CPU: two gloo ranks each reduce their KV-head
shard with the oracle, gather the shards, and lay them back into rows; the
result must equal the unsharded reduction exactly (heads are independent).
Also the handle exchange the GPU path uses to map peer buffers."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

from hero_b200.shard import kv_shard, take_heads

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
