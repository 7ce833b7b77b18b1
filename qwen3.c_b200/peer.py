"""Peer-mapped device buffers for head-sharded prefill with the all-gather
fused into the output kernels (one process per GPU, torch.distributed for the
handle exchange only).

Each rank cudaMalloc's its gathered buffer through the backend
(coli_cuda_ipc_alloc), the 64-byte CUDA IPC handles are exchanged with
all_gather_object, and every rank maps the others' buffers
(coli_cuda_ipc_open). The prefill kernels then store their output block into
all ranks' buffers directly (coli_cuda_*_prefill_heads_gather_dev), and
PeerBarrier ends a layer: a device-side barrier over IPC-mapped flag words,
ordered on the compute stream like any kernel.
"""
import torch.distributed as dist


class PeerBuffer:
    """One device buffer per rank, every rank's buffer mapped in every rank.
    ptrs[r] is rank r's buffer as seen from this process."""

    def __init__(self, be, nbytes, world, rank, group=None):
        self.be, self.nbytes, self.world, self.rank, self.group = be, nbytes, world, rank, group
        self.local, handle = be.ipc_alloc(nbytes)
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs = [self.local if r == rank else be.ipc_open(h) for r, h in enumerate(handles)]

    def close(self):
        """Unmap the peers' buffers, then (after every peer has unmapped this
        one) free the local buffer."""
        self.be.sync()
        dist.barrier(group=self.group)
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self.be.ipc_close(p)
        dist.barrier(group=self.group)
        self.be.ipc_free(self.local, self.nbytes)
        self.ptrs = []


class PeerBarrier:
    """Cross-rank barrier on the device: call it on every rank, in the same
    order; epochs count the calls."""

    def __init__(self, be, world, rank, group=None):
        self.be, self.rank = be, rank
        self.flags = PeerBuffer(be, 4 * world, world, rank, group)
        self.epoch = 0

    def __call__(self):
        self.epoch += 1
        self.be.peer_barrier(self.flags.ptrs, self.rank, self.epoch)

    def close(self):
        self.flags.close()
