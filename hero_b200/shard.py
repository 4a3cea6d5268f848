"""Host side of the multi-GPU split: which heads a rank owns and how its
output columns sit in the reference's [rows][H*D] layout.

One process per GPU; KV heads are split evenly across ranks and each KV head
takes its Hq/Hkv query heads with it (the grouped mapping of the reference,
query head h reads KV head h // (Hq/Hkv)), so every rank's attention is
independent and its output is the contiguous column block
[q0 * head_dim, q1 * head_dim) of every row.  With more ranks than KV heads
the ranks that share a KV head split its query heads (prefill: each keeps a
copy of that head's K/V) or the batch (decode: `decode_shard`).

The gated delta rule splits by key-head group (`delta_shard`): value head h
reads key head h % Hk (src/qwen35.hpp:172), so a rank that owns a range of
key heads owns every value head that reads one of them, and no state or
activation crosses ranks until the outputs are gathered.

After an all-gather of equal per-rank blocks, [world][rows][cols] ->
[rows][world * cols] is the head-to-row permutation `heads_to_rows` restates
(on the device: nmg_gather_heads_to_rows).
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
    """KV heads [kv0, kv1) and their query heads for `rank`.  When there are
    more ranks than KV heads (world = hkv * s), the s ranks of one KV head take
    consecutive 1/s slices of its query heads; either way rank r's query heads
    are [r * hq / world, (r + 1) * hq / world), so the output blocks tile every
    row in rank order."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if hq % hkv:
        raise ValueError(f"{hq} query heads is not a multiple of {hkv} KV heads")
    g = hq // hkv
    if world > hkv:
        if world % hkv or g % (world // hkv):
            raise ValueError(f"{world} ranks split neither {hkv} KV heads nor their groups of {g} query heads")
        per_q = hq // world
        kv = rank // (world // hkv)
        return Shard(rank, world, kv, kv + 1, rank * per_q, (rank + 1) * per_q)
    if hkv % world:
        raise ValueError(f"{world} ranks do not divide {hkv} KV heads")
    per = hkv // world
    return Shard(rank, world, rank * per, (rank + 1) * per, rank * per * g, (rank + 1) * per * g)


@dataclass(frozen=True)
class DecodeShard:
    heads: Shard  # the KV-head shard among the `kv_world` ranks of this batch part
    kv_world: int
    part: int  # batch part: sequences [b0, b1)
    parts: int
    b0: int
    b1: int


def decode_shard(rank: int, world: int, hkv: int, hq: int, batch: int) -> DecodeShard:
    """Batched decode: KV heads across min(world, hkv) ranks; with more ranks
    than KV heads the batch is cut into world / hkv parts as well, so no two
    ranks read the same cache rows.  Ranks of one part are consecutive
    (rank = part * kv_world + kv_rank): after an all-gather, the blocks of part
    p are gathered[p * kv_world:(p + 1) * kv_world] and fill rows [b0, b1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    kv_world = min(world, hkv)
    if world % kv_world:
        raise ValueError(f"{world} ranks are not a whole number of {kv_world}-rank KV-head groups")
    parts = world // kv_world
    if batch % parts:
        raise ValueError(f"{parts} batch parts do not divide a batch of {batch}")
    part, kv_rank = divmod(rank, kv_world)
    per = batch // parts
    return DecodeShard(kv_shard(kv_rank, kv_world, hkv, hq), kv_world, part, parts, part * per, (part + 1) * per)


@dataclass(frozen=True)
class DeltaShard:
    rank: int
    world: int
    k0: int  # key heads [k0, k1)
    k1: int
    v_heads: tuple  # the global value heads of this rank, in local order

    @property
    def hk(self) -> int:
        return self.k1 - self.k0

    @property
    def hv(self) -> int:
        return len(self.v_heads)


def delta_shard(rank: int, world: int, hk: int, hv: int) -> DeltaShard:
    """Key heads [k0, k1) = the rank's 1/world of the hk key heads, and the
    value heads h with h % hk in that range (src/qwen35.hpp:172).  Local order
    is repeat-major: local value head m * (k1 - k0) + j is global value head
    m * hk + k0 + j, so local value head i reads local key head i % (k1 - k0)
    -- the shard is a smaller instance of the same tiled map and runs through
    the same kernels.  In a gathered output row block [m][k1 - k0][dv] per
    rank, row t of rank r splits into hv / hk runs; viewing every row as
    hv / hk rows of (k1 - k0) * dv values turns the assembly into one
    `heads_to_rows` over T * hv / hk rows."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if hv % hk:
        raise ValueError(f"{hv} value heads is not a multiple of {hk} key heads")
    if hk % world:
        raise ValueError(f"{world} ranks do not divide {hk} key heads")
    per = hk // world
    k0, k1 = rank * per, (rank + 1) * per
    heads = tuple(m * hk + k0 + j for m in range(hv // hk) for j in range(per))
    return DeltaShard(rank, world, k0, k1, heads)


def heads_to_rows(gathered, world: int, rows: int, cols: int):
    """[world][rows][cols] -> [rows][world * cols] (numpy), the permutation
    nmg_gather_heads_to_rows performs on the device."""
    return gathered.reshape(world, rows, cols).transpose(1, 0, 2).reshape(rows, world * cols)


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
