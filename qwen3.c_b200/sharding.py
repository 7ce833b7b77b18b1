"""Host-side work partitioning across GPUs (one process per GPU).

Decode shards by request: rank r of N owns a contiguous block of the global
batch, with its own KV cache and GDN state; no collective touches the data
path. Prefill shards by head: rank r computes a contiguous block of query
heads (GQA) / value heads (GDN) and the per-rank outputs are all-gathered.
The reference engine is single-sequence and single-device (c/qwen.c:131-137),
so none of this has a reference counterpart.
"""


def request_shard(batch, world, rank):
    """[begin, end) of the global requests owned by `rank` (balanced blocks)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(batch, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def head_shard(n_heads, world, rank):
    """[begin, end) of the heads computed by `rank`; heads must split evenly."""
    if n_heads % world:
        raise ValueError(f"{n_heads} heads do not split over {world} ranks")
    per = n_heads // world
    return rank * per, (rank + 1) * per


def kv_heads_for(q_begin, q_end, group):
    """KV heads a block of query heads reads (query head h uses KV head h // group)."""
    return q_begin // group, (q_end - 1) // group + 1


def max_over_ranks(value, group=None):
    """Max of a host float over the process group (gloo or nccl)."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
