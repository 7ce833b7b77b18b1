"""Head-sharded prefill (the multi-GPU prefill mode) emulated on one GPU:
every rank's head block is computed through the sharded entry points in turn,
the blocks are gathered the way the all-gather lays them out, and the result
must match the unsharded prefill of the same inputs."""
import numpy as np
import pytest

from conftest import load_pkg
from helpers import CD, H, HD, KH, VD, VH_G, assert_close, gdn_params

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    pkg = load_pkg()
    pkg.build()
    b = pkg.Backend(0)
    yield b
    b.shutdown()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gqa_head_sharded_prefill(be, world):
    import torch
    sh = load_pkg().sharding
    S = 300
    g = torch.Generator(device="cuda").manual_seed(world)
    qn = (0.1 * torch.randn(HD, generator=g, device="cuda")).cpu().numpy()
    kn = (0.1 * torch.randn(HD, generator=g, device="cuda")).cpu().numpy()
    qg = torch.randn(S, H, 2 * HD, generator=g, device="cuda").bfloat16()
    k = torch.randn(S, KH, HD, generator=g, device="cuda").bfloat16()
    v = torch.randn(S, KH, HD, generator=g, device="cuda").bfloat16()
    full = torch.zeros(S, H, HD, dtype=torch.bfloat16, device="cuda")
    be.kv_ensure(20, 1, KH, S)
    be.gqa_norm_weight(20, qn, kn)
    torch.cuda.synchronize()
    be.gqa_step_dev(20, 0, S, 0, qg.data_ptr(), k.data_ptr(), v.data_ptr(), full.data_ptr())
    be.sync()
    parts = []
    for r in range(world):
        h0, h1 = sh.head_shard(H, world, r)
        k0, k1 = sh.kv_heads_for(h0, h1, 8)
        layer = 21 + r
        be.kv_ensure(layer, 1, k1 - k0, S)
        be.gqa_norm_weight(layer, qn, kn)
        ctx = torch.zeros(S, h1 - h0, HD, dtype=torch.bfloat16, device="cuda")
        be.gqa_prefill_heads_dev(layer, 0, S, 0, qg.data_ptr(), k.data_ptr(), v.data_ptr(),
                                 ctx.data_ptr(), h0, h1 - h0)
        be.sync()
        parts.append(ctx)
    got = torch.cat(parts, dim=1)
    assert_close(got.float().cpu().numpy(), full.float().cpu().numpy(), max_abs=1e-2, min_cos=0.99999,
                 what=f"gqa sharded x{world}")


@pytest.mark.parametrize("world", [2, 8])
def test_gdn_head_sharded_prefill(be, world):
    import torch
    sh = load_pkg().sharding
    S = 200
    prm = gdn_params(f"gdn_shard_{world}")
    g = torch.Generator(device="cuda").manual_seed(100 + world)
    qkv = torch.randn(S, CD, generator=g, device="cuda").bfloat16()
    z = torch.randn(S, VH_G * VD, generator=g, device="cuda").bfloat16()
    a = torch.randn(S, VH_G, generator=g, device="cuda").bfloat16()
    b = torch.randn(S, VH_G, generator=g, device="cuda").bfloat16()
    full = torch.zeros(S, VH_G * VD, dtype=torch.bfloat16, device="cuda")
    be.gdn_setup(20, 1, prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["gnorm"])
    be.gdn_reset()
    torch.cuda.synchronize()
    be.gdn_prefill_dev(20, 0, S, qkv.data_ptr(), z.data_ptr(), a.data_ptr(), b.data_ptr(), full.data_ptr())
    be.sync()
    state_full = be.gdn_state_get(20, 0)
    parts, states = [], []
    lib = be.lib
    be.gdn_reset()  # every shard starts from zero state and history, as the full run did
    for r in range(world):
        k0, k1 = sh.head_shard(16, world, r)
        layer = 21 + r
        nv = 2 * (k1 - k0)
        assert lib.coli_cuda_gdn_state_ensure(layer, 1, nv, 128, 128) == 1
        assert lib.coli_cuda_gdn_conv_ensure(layer, 1, 4, CD) == 1
        cw = np.ascontiguousarray(prm["conv_w"], np.float32)
        import ctypes
        fp = ctypes.POINTER(ctypes.c_float)
        assert lib.coli_cuda_gdn_conv_weight(layer, cw.ctypes.data_as(fp), 4, CD) == 1
        arrs = [np.ascontiguousarray(prm[n], np.float32) for n in ("A_log", "dt_bias", "gnorm")]
        assert lib.coli_cuda_gdn_params(layer, *[x.ctypes.data_as(fp) for x in arrs], VH_G, VD) == 1
        y = torch.zeros(S, nv * VD, dtype=torch.bfloat16, device="cuda")
        be.gdn_prefill_heads_dev(layer, 0, S, qkv.data_ptr(), z.data_ptr(), a.data_ptr(), b.data_ptr(),
                                 y.data_ptr(), k0, k1 - k0)
        be.sync()
        parts.append(y)
        s = np.zeros((nv, 128, 128), np.float32)
        assert lib.coli_cuda_gdn_state_get(layer, 0, s.ctypes.data_as(fp)) == 1
        states.append(s)
    got = torch.cat(parts, dim=1)
    assert_close(got.float().cpu().numpy(), full.float().cpu().numpy(), max_abs=1e-2, min_cos=0.99999,
                 what=f"gdn sharded x{world}")
    np.testing.assert_allclose(np.concatenate(states), state_full, rtol=1e-4, atol=1e-5)
