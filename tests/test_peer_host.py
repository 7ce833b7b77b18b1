"""Host logic of the fused-gather plumbing (peer.PeerBuffer / PeerBarrier) on
CPU with gloo, world size 2, against a fake backend: handle exchange, the
peer pointer table, barrier epochs and the unmap / free order."""
import os
import random

import torch.multiprocessing as mp

from conftest import load_pkg


class FakeBackend:
    def __init__(self, rank):
        self.rank, self.log, self.next = rank, [], 1000 * (rank + 1)

    def ipc_alloc(self, nbytes):
        self.next += 1
        self.log.append(("alloc", nbytes))
        return self.next, f"h{self.rank}:{self.next}".encode()

    def ipc_open(self, handle):
        self.log.append(("open", handle))
        return "mapped:" + handle.decode()

    def ipc_close(self, ptr):
        self.log.append(("close", ptr))

    def ipc_free(self, ptr, nbytes):
        self.log.append(("free", ptr, nbytes))

    def peer_barrier(self, flags, rank, epoch):
        self.log.append(("barrier", tuple(flags), rank, epoch))

    def sync(self):
        pass


def _worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    peer = load_pkg().peer
    be = FakeBackend(rank)
    buf = peer.PeerBuffer(be, 4096, world, rank)
    bar = peer.PeerBarrier(be, world, rank)
    bar()
    bar()
    ptrs = list(buf.ptrs)
    buf.close()
    bar.close()
    out[rank] = (ptrs, be.log)
    dist.destroy_process_group()


def test_peer_buffers_gloo():
    port = random.randint(20000, 40000)
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
        res = dict(out)
    for rank in (0, 1):
        ptrs, log = res[rank]
        other = 1 - rank
        assert ptrs[rank] == 1000 * (rank + 1) + 1                      # own allocation, unmapped
        assert ptrs[other] == f"mapped:h{other}:{1000 * (other + 1) + 1}"  # the peer's, from its handle
        barriers = [e for e in log if e[0] == "barrier"]
        assert [b[3] for b in barriers] == [1, 2] and all(b[2] == rank for b in barriers)
        # the peer mapping is closed before the local buffer is freed
        kinds = [e[0] for e in log]
        assert kinds.index("close") < kinds.index("free")
