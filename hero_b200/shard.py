"""Host side of the multi-GPU split: which heads a rank owns and how its
output columns sit in the reference's [rows][H*D] layout.

One process per GPU; KV heads are split evenly across ranks and each KV head
takes its Hq/Hkv query heads with it (the grouped mapping of the reference,
query head h reads KV head h // (Hq/Hkv)), so every rank's attention is
independent and its output is the contiguous column block
[q0 * head_dim, q1 * head_dim) of every row.
"""
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    kv0: int  # KV heads [kv0, kv1)
    kv1: int
    q0: int  # query heads [q0, q1)
    q1: int

    def out_col0(self, head_dim: int) -> int:
        """First output column (elements) of this rank's heads in a [rows][Hq*D] row."""
        return self.q0 * head_dim


def kv_shard(rank: int, world: int, hkv: int, hq: int) -> Shard:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if hq % hkv:
        raise ValueError(f"{hq} query heads is not a multiple of {hkv} KV heads")
    if hkv % world:
        raise ValueError(f"{world} ranks do not divide {hkv} KV heads")
    per = hkv // world
    g = hq // hkv
    return Shard(rank, world, rank * per, (rank + 1) * per, rank * per * g, (rank + 1) * per * g)


def take_heads(x, heads: int, head_dim: int, h0: int, h1: int):
    """Rows [T][heads*head_dim] -> the contiguous rows [T][(h1-h0)*head_dim] of heads [h0, h1)
    (torch tensors or numpy arrays)."""
    rows = x.shape[0]
    part = x.reshape(rows, heads, head_dim)[:, h0:h1].reshape(rows, (h1 - h0) * head_dim)
    return part.contiguous() if hasattr(part, "contiguous") else part.copy()


def exchange(dist, obj):
    """Every rank's `obj` (for example a 64-byte IPC handle), in rank order."""
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out
