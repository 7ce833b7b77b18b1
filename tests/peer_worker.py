"""Worker of test_gpu_peer (run under torchrun, one process per GPU, NCCL):
head-sharded prefill of a short mixer stack (6 GatedDeltaNet + 2 GQA layers)
with the layer outputs gathered by NCCL and by the fused peer stores of the
output kernels; the gathered outputs of the last layer of each kind must be
bit-identical. Prints "PEER OK <rank>" on success."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from conftest import load_pkg  # noqa: E402


def copy_out(ptr, like):
    """Device buffer at ptr (this process's own allocation) -> a torch tensor."""
    from cuda.bindings import runtime as rt
    out = torch.empty_like(like)
    err, = rt.cudaMemcpy(out.data_ptr(), ptr, out.numel() * out.element_size(),
                         rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
    assert int(err) == 0, err
    return out


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    pkg = load_pkg()
    pkg.build()
    be = pkg.Backend(local)
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    be.set_stream(st.cuda_stream)
    S = int(os.environ.get("PEER_S", "320"))

    ref = pkg.stack.MixerStack(be, n_layers=8, seed=3)
    ref.setup_prefill(S, world, rank, fused=False)
    be.gdn_reset()
    ref.prefill()
    torch.cuda.synchronize()
    want_ctx, want_y = ref.ctx_all.clone(), ref.y_all.clone()

    fus = pkg.stack.MixerStack(be, n_layers=8, seed=3)   # same seed: same inputs and weights
    fus.setup_prefill(S, world, rank, fused=True)
    be.gdn_reset()
    fus.prefill()
    be.sync()
    torch.cuda.synchronize()
    n_gqa = sum(k == "gqa" for k in fus.kinds)
    n_gdn = len(fus.kinds) - n_gqa
    got_ctx = copy_out(fus.gq_bufs[(n_gqa - 1) % 2].ptrs[rank], want_ctx)
    got_y = copy_out(fus.gd_bufs[(n_gdn - 1) % 2].ptrs[rank], want_y)
    assert torch.equal(got_ctx, want_ctx), "GQA gathered output differs from the NCCL all-gather"
    assert torch.equal(got_y, want_y), "GDN gathered output differs from the NCCL all-gather"
    assert float(want_y.float().abs().sum()) > 0 and float(want_ctx.float().abs().sum()) > 0
    fus.close_prefill()
    be.shutdown()
    dist.destroy_process_group()
    print(f"PEER OK {rank}", flush=True)


if __name__ == "__main__":
    main()
