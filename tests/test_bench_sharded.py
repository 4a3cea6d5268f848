"""The multi-GPU bench extras' host logic on the CPU.

bench.py's sharded_config1/3/4/5 run on every rank of a torchrun job; here
each runs its small variant as one rank of 2, 4 and 8, with the device calls
replaced by fakes that check every shape, dtype and position the real calls
would be given, and the all-gather / head-to-row permutation replaced by
checks of the byte counts the C ABI would receive.  No GPU is touched."""
import sys
import types

import pytest
import torch

import bench


class _Cache:
    def __init__(self, hkv, head_dim, window, capacity, dtype):
        assert capacity and capacity > 0 and (window == 0 or capacity >= window)
        self.hkv, self.head_dim, self.window, self.cap, self.dtype = hkv, head_dim, window, capacity, dtype
        self.n, self.first = 0, None

    def append(self, pos, k, v):
        assert k.shape == v.shape and k.dim() == 2 and k.shape[1] == self.hkv * self.head_dim
        assert k.dtype == {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[self.dtype]
        if self.first is None:
            self.first = pos
        assert pos == self.first + self.n, "appends must be consecutive"
        self.n += k.shape[0]
        assert self.window or self.n <= self.cap, "a full cache cannot outgrow its capacity"

    def reset(self):
        self.n, self.first = 0, None


class FakeNm(types.SimpleNamespace):
    def __init__(self):
        def full(hkv, head_dim, *, capacity, dtype="f32", device=0):
            return _Cache(hkv, head_dim, 0, capacity, dtype)

        def local(hkv, head_dim, window, *, capacity=None, dtype="f32", device=0):
            return _Cache(hkv, head_dim, window, capacity, dtype)

        super().__init__(FullAttentionCache=full, LocalAttentionCache=local)

    @staticmethod
    def attend(cache, q, at, scale=None, *, out=None, out_dtype=None):
        assert q.dim() == 2 and q.shape[1] % cache.head_dim == 0
        assert (q.shape[1] // cache.head_dim) % cache.hkv == 0
        assert cache.first is not None and at + q.shape[0] - 1 <= cache.first + cache.n - 1
        assert out.shape == q.shape

    @classmethod
    def append_attend(cls, cache, pos, k, v, q, scale=None, *, out=None, out_dtype=None):
        cache.append(pos, k, v)
        assert q.shape[0] == k.shape[0]
        cls.attend(cache, q, pos, scale, out=out)

    @staticmethod
    def attend_batch(caches, q, scale=None, *, queries_at=None, out=None, out_dtype=None):
        assert q.shape[0] == len(caches) and q.is_contiguous() and out.shape == q.shape
        assert all(c.hkv == caches[0].hkv and c.n > 0 for c in caches)
        assert (q.shape[1] // caches[0].head_dim) % caches[0].hkv == 0

    class DeltaNetState:
        def __init__(self, heads, dk, dv, device=0):
            self.heads, self.dk, self.dv = heads, dk, dv

        def clear(self):
            pass

    @staticmethod
    def delta_prefill(st, q, k, v, gate, beta, hk, *, chunk=64, out=None):
        T = v.shape[0]
        assert q.shape == (T, hk, st.dk) == k.shape and q.is_contiguous() and k.is_contiguous()
        assert v.shape == (T, st.heads, st.dv) and v.is_contiguous() and st.heads % hk == 0
        assert gate.shape == beta.shape == (T, st.heads) and gate.is_contiguous() and beta.is_contiguous()
        assert out.shape == (T, st.heads, st.dv)

    @staticmethod
    def delta_step(st, q, k, v, gate, beta, hk, *, out=None):
        assert q.shape == k.shape == (hk, st.dk) and q.is_contiguous() and k.is_contiguous()
        assert v.shape == (st.heads, st.dv) and gate.shape == beta.shape == (st.heads,)
        assert out.shape == (st.heads, st.dv) and out.is_contiguous()


class FakeRanks(bench.Ranks):
    """One rank of `world`: collectives become checks of what the C ABI would get."""

    def __init__(self, rank, world):
        self.torch, self.dev, self.rank, self.world = torch, torch.device("cpu"), rank, world
        self.gathers = 0

    def barrier(self):
        pass

    def max_over(self, *vals):
        return list(vals)

    def all_ok(self, ok):
        return ok

    def gather(self, send, gathered):
        assert send.is_contiguous() and gathered.is_contiguous() and send.dtype == gathered.dtype
        assert gathered.numel() == self.world * send.numel()
        self.gathers += 1

    def to_rows(self, gathered, out, world, rows, row_bytes):
        assert gathered.is_contiguous() and out.is_contiguous()
        assert gathered.numel() * gathered.element_size() == world * rows * row_bytes
        assert out.numel() * out.element_size() == world * rows * row_bytes
        assert row_bytes % 16 == 0  # the vectorised permutation

    def graph_ms(self, fn, reps, inner):
        fn()
        return 1.0

    def event_ms(self, fn, reps):
        fn()
        return 1.0

    def release(self):
        pass

    def close(self):
        pass


@pytest.fixture
def fake_nm(monkeypatch):
    import hero_b200

    nm = FakeNm()
    monkeypatch.setattr(hero_b200, "nm", nm, raising=False)
    monkeypatch.setitem(sys.modules, "hero_b200.nm", nm)
    return nm


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("name", ["sharded_config1", "sharded_config3", "sharded_config4", "sharded_config5"])
def test_sharded_extra_host_logic(fake_nm, name, world):
    for rank in (0, world - 1):
        rk = FakeRanks(rank, world)
        res = getattr(bench, name)(rk, small=True)
        assert rk.gathers > 0, "every extra gathers its head outputs"
        assert "workload" in res and "error" not in res


_REAL_ALL_OK = bench.Ranks.all_ok


class GlooRanks(FakeRanks):
    """FakeRanks whose agreement steps are real collectives (two gloo ranks)."""

    def __init__(self, rank, world, dist):
        super().__init__(rank, world)
        self.dist = dist

    def all_ok(self, ok):
        return _REAL_ALL_OK(self, ok)


def _rank_protocol(rank, world, port, results):
    import os
    from datetime import timedelta

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch.distributed as dist

    import hero_b200

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        nm = FakeNm()
        hero_b200.nm = nm
        sys.modules["hero_b200.nm"] = nm
        if rank == 1:  # fails alone while setting up config 3 (before its first checkpoint)
            def broken_state(*a, **k):
                raise MemoryError("injected")
            nm.DeltaNetState = broken_state
        if rank == 0:  # fails alone between config 4's prefill and decode phases (its 6th ring)
            made, local = [0], nm.LocalAttentionCache

            def sixth_ring_fails(*a, **k):
                made[0] += 1
                if made[0] == 6:
                    raise ValueError("injected")
                return local(*a, **k)
            nm.LocalAttentionCache = sixth_ring_fails
        real = {n: getattr(bench, n) for n in ("sharded_config1", "sharded_config3", "sharded_config4",
                                                "sharded_config5")}
        for n, fn in real.items():  # the small variants
            setattr(bench, n, lambda rk, fn=fn: fn(rk, small=True))
        rk = GlooRanks(rank, world, dist)
        bench.Ranks = lambda *a: rk
        extra = bench.sharded_extras(None, dist, None, rank, world)
        results[rank] = {k: ("error" in v) for k, v in extra.items()}
    finally:
        dist.destroy_process_group()


def test_one_rank_failing_stops_that_extra_on_every_rank():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    procs = [ctx.Process(target=_rank_protocol, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    want = {"config1": False, "config3": True, "config4": True, "config5": False}
    assert dict(results) == {0: want, 1: want}
