"""coli_cuda_gqa_decode_noalloc: the decode entry point for callers that cannot
allocate device memory while serving.

It must give the same results as coli_cuda_gqa_decode_dev (within the parity
tolerance used everywhere in these tests) on consecutive calls that share its
fixed scratch array, and refuse a batch that does not fit that array. The
file is named to be collected last; it also passes on its own in a fresh
process.
"""
import numpy as np
import pytest

from conftest import load_pkg
from helpers import H, HD, KH, assert_close

pytestmark = pytest.mark.gpu

LAYER = 7


@pytest.fixture(scope="module")
def be():
    pkg = load_pkg()
    pkg.build()
    b = pkg.Backend(0)
    yield b
    b.shutdown()


def _setup(be, torch, B, T, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    be.kv_ensure(LAYER, B, KH, T)
    be.gqa_norm_weight(LAYER, (torch.randn(HD, generator=g, device="cuda") * 0.1).cpu().numpy(),
                       (torch.randn(HD, generator=g, device="cuda") * 0.1).cpu().numpy())
    rows_k = torch.randn(KH * T, HD, generator=g, device="cuda").bfloat16()
    rows_v = torch.randn(KH * T, HD, generator=g, device="cuda").bfloat16()
    torch.cuda.synchronize()
    for r in range(B):
        be.kv_rows_dev(LAYER, r, 0, KH * T, rows_k.data_ptr(), rows_v.data_ptr(), 1)
    be.sync()
    return g


def _inputs(torch, g, B, T):
    qg = torch.randn(B, H, 2 * HD, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, KH, HD, generator=g, device="cuda").bfloat16()
    v = torch.randn(B, KH, HD, generator=g, device="cuda").bfloat16()
    pos = torch.randint(0, T, (B,), generator=g, device="cuda", dtype=torch.int32)
    pos[0] = T - 1
    return qg, k, v, pos


def test_noalloc_matches_allocating_entry_on_two_calls(be):
    import torch
    B, T = 16, 3000
    g = _setup(be, torch, B, T, seed=11)
    for call in range(2):
        qg, k, v, pos = _inputs(torch, g, B, T)
        want = torch.zeros(B, H, HD, dtype=torch.bfloat16, device="cuda")
        got = torch.full((B, H, HD), float("nan"), dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
        be.gqa_decode_dev(LAYER, B, qg.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(),
                          want.data_ptr())
        # the same new K/V rows are written again at the same positions, so
        # both calls see identical caches
        be.gqa_decode_noalloc(LAYER, B, qg.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(),
                              got.data_ptr())
        be.sync()
        assert_close(got.float().cpu().numpy(), want.float().cpu().numpy(),
                     what=f"noalloc call {call}")


def test_noalloc_cuts_splits_to_fit_and_allocates_nothing(be):
    """64 requests at T = 8192: the default plan (8 KV splits) needs ~16 MB of
    partial sums, more than the fixed 8 MiB array, so the call runs with fewer
    splits; its results equal the allocating entry's. The allocation-failure
    hook is armed around the call (any device allocation would be refused and
    the call would fail), and the backend's allocation total is unchanged."""
    import torch
    B, T = 64, 8192
    g = _setup(be, torch, B, T, seed=5)
    qg, k, v, pos = _inputs(torch, g, B, T)
    want = torch.zeros(B, H, HD, dtype=torch.bfloat16, device="cuda")
    got = torch.full((B, H, HD), float("nan"), dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    be.gqa_decode_dev(LAYER, B, qg.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), want.data_ptr())
    be.sync()
    before = be.mem_info()
    be.lib.coli_cuda_debug_fail_alloc(0)
    try:
        be.gqa_decode_noalloc(LAYER, B, qg.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(),
                              got.data_ptr())
        be.sync()
    finally:
        be.lib.coli_cuda_debug_fail_alloc(-1)
    assert be.mem_info() == before
    assert_close(got.float().cpu().numpy(), want.float().cpu().numpy(), what="noalloc with fewer splits")


def test_noalloc_rejects_batch_beyond_fixed_scratch(be):
    import torch
    BackendError = load_pkg().BackendError
    B, T = 400, 64
    be.kv_ensure(LAYER, B, KH, T)
    be.gqa_norm_weight(LAYER, np.zeros(HD, np.float32), np.zeros(HD, np.float32))
    qg = torch.zeros(B, H, 2 * HD, dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros(B, KH, HD, dtype=torch.bfloat16, device="cuda")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    ctx = torch.zeros(B, H, HD, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(BackendError, match="fixed"):
        be.gqa_decode_noalloc(LAYER, B, qg.data_ptr(), kv.data_ptr(), kv.data_ptr(), pos.data_ptr(),
                              ctx.data_ptr())
    be.sync()
