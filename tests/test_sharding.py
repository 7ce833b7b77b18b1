"""Host logic of the multi-GPU paths, on CPU with the gloo backend (world size 2)."""
import os

import pytest
import torch.multiprocessing as mp

from conftest import load_pkg


def test_request_shards_cover_batch():
    sh = load_pkg().sharding
    for B in (1, 7, 64, 256):
        for N in (1, 2, 4, 8):
            blocks = [sh.request_shard(B, N, r) for r in range(N)]
            assert blocks[0][0] == 0 and blocks[-1][1] == B
            assert all(blocks[i][1] == blocks[i + 1][0] for i in range(N - 1))
            assert max(e - b for b, e in blocks) - min(e - b for b, e in blocks) <= 1


def test_head_shards_and_kv_mapping():
    sh = load_pkg().sharding
    # GQA: 16 query heads over 8 ranks, KV head = h // 8
    assert [sh.kv_heads_for(*sh.head_shard(16, 8, r), 8) for r in range(8)] == [(0, 1)] * 4 + [(1, 2)] * 4
    # GDN: 32 V heads / 16 K heads: V head h uses K head h // 2
    assert sh.kv_heads_for(*sh.head_shard(32, 4, 1), 2) == (4, 8)
    with pytest.raises(ValueError):
        sh.head_shard(16, 3, 0)


def _worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sh = load_pkg().sharding
    out[rank] = (sh.max_over_ranks(1.5 + rank), sh.request_shard(64, world, rank))
    dist.destroy_process_group()


def test_max_over_ranks_gloo():
    import random
    port = random.randint(20000, 40000)
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
        res = dict(out)
    assert res[0][0] == res[1][0] == 2.5
    assert res[0][1] == (0, 32) and res[1][1] == (32, 64)
