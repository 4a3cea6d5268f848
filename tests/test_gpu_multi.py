"""Two-process multi-GPU head sharding (one rank per GPU, NCCL): the attention
epilogue's stores into every rank's mapped rows, and the NCCL all-gather path,
against one GPU's unsharded reduction.  Needs two GPUs; skipped otherwise."""
import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu

HQ, HKV, DH, S = 8, 4, 128, 384


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    import ctypes
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    from hero_b200 import _lib, nm

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        g = torch.Generator(device=dev)
        g.manual_seed(7)  # every rank draws the same full problem
        k = torch.randn(S, HKV * DH, device=dev, generator=g).bfloat16()
        v = torch.randn(S, HKV * DH, device=dev, generator=g).bfloat16()
        q = torch.randn(S, HQ * DH, device=dev, generator=g).bfloat16()
        full_cache = nm.FullAttentionCache(HKV, DH, capacity=S, dtype="bf16", device=rank)
        full_cache.append(0, k, v)
        want = nm.attend(full_cache, q, 0, DH ** -0.5, out_dtype=torch.bfloat16)

        hkv_l, hq_l = HKV // world, HQ // world
        ks = k.view(S, HKV, DH)[:, rank * hkv_l:(rank + 1) * hkv_l].reshape(S, -1).contiguous()
        vs = v.view(S, HKV, DH)[:, rank * hkv_l:(rank + 1) * hkv_l].reshape(S, -1).contiguous()
        qs = q.view(S, HQ, DH)[:, rank * hq_l:(rank + 1) * hq_l].reshape(S, -1).contiguous()
        cache = nm.FullAttentionCache(hkv_l, DH, capacity=S, dtype="bf16", device=rank)
        cache.append(0, ks, vs)

        # fused: every rank writes its heads into all ranks' rows
        rows = nm.SharedRows(S, HQ * DH, torch.bfloat16, rank)
        handles = [None] * world
        dist.all_gather_object(handles, rows.handle)
        ptrs = [rows.ptr if r == rank else nm.open_peer(handles[r], rank) for r in range(world)]
        uid = (ctypes.c_char * 128)()
        if rank == 0:
            _lib.call("nmg_comm_unique_id", uid)
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=0)
        uid = (ctypes.c_char * 128).from_buffer_copy(obj[0])
        comm = ctypes.c_void_p()
        _lib.call("nmg_comm_init", uid, rank, world, rank, ctypes.byref(comm))
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        nm.attend_fanout(cache, qs, 0, DH ** -0.5, ptrs, HQ * DH, rank * hq_l * DH, torch.bfloat16)
        _lib.call("nmg_comm_barrier", comm, stream)
        torch.cuda.synchronize(dev)
        fused_ok = torch.equal(rows.tensor(), want)

        # unfused: local heads, NCCL all-gather, head-to-row permutation
        o = nm.attend(cache, qs, 0, DH ** -0.5, out_dtype=torch.bfloat16)
        gathered = torch.empty(world, S, hq_l * DH, device=dev, dtype=torch.bfloat16)
        full = torch.empty(S, HQ * DH, device=dev, dtype=torch.bfloat16)
        _lib.call("nmg_allgather", comm, ctypes.c_void_p(o.data_ptr()), ctypes.c_void_p(gathered.data_ptr()),
                  o.numel() * 2, stream)
        _lib.call("nmg_gather_heads_to_rows", ctypes.c_void_p(gathered.data_ptr()), ctypes.c_void_p(full.data_ptr()),
                  world, S, hq_l * DH * 2, stream)
        torch.cuda.synchronize(dev)
        nccl_ok = torch.equal(full, want)

        dist.barrier()
        for r, p in enumerate(ptrs):
            if r != rank:
                nm.close_peer(p)
        dist.barrier()
        rows.close()
        _lib.lib().nmg_comm_destroy(comm)
        results[rank] = (fused_ok, nccl_ok)
    finally:
        dist.destroy_process_group()


def test_head_sharded_prefill_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: (True, True), 1: (True, True)}
