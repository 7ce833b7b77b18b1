"""GatedDeltaNet decode on the GPU vs the CPU oracle (and the reference's own
golden outputs), through the C ABI."""
import numpy as np
import pytest

from conftest import golden, load_pkg
from helpers import (CD, CONVK, KD, KH_G, STATE_REL_L2, VD, VH_G, assert_close, gdn_inputs,
                     gdn_params, gdn_state0, record, rel_l2)
import make_golden_shim as mg
from oracle import Oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    pkg = load_pkg()
    pkg.build()
    b = pkg.Backend(0)
    yield b
    b.shutdown()


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def _setup(be, layer, batch, prm, states):
    be.gdn_setup(layer, batch, prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["gnorm"])
    for r, (s, ring) in enumerate(states):
        be.gdn_state_set(layer, r, s)
        be.gdn_conv_set(layer, r, ring)


def test_golden_reference_sequence(be):
    """The reference's own gdn_step outputs (tests/golden/gdn_seq.npz)."""
    g = golden("gdn_seq.npz")
    state, ring = mg.gdn_init_state("golden_gdn_seq")
    prm = dict(conv_w=g["conv"], A_log=g["A_log"], dt_bias=g["dt_bias"], gnorm=g["gnorm"])
    _setup(be, 0, 1, prm, [(state, ring)])
    for s in range(g["qkv"].shape[0]):
        y = be.gdn_decode(0, g["qkv"][s:s + 1], g["z"][s:s + 1], g["a"][s:s + 1], g["b"][s:s + 1])
        assert_close(y[0], g["y"][s], what=f"step {s}")
    got_ring = be.gdn_conv_get(0, 0)
    np.testing.assert_array_equal(got_ring[1:], g["ring_final"])
    sfin = be.gdn_state_get(0, 0).reshape(-1)
    assert rel_l2(sfin[::97], g["state_sample"]) < 1e-5


@pytest.mark.parametrize("B", [1, 5, 64])
def test_batched_decode_vs_oracle(be, orc, B):
    cfg = f"gdn_batch{B}"
    prm = gdn_params(cfg)
    st = [gdn_state0(cfg, r) for r in range(B)]
    _setup(be, 1, B, prm, st)
    steps = 3
    ins = [gdn_inputs(cfg, steps, r) for r in range(B)]
    want = []
    for r in range(B):
        s0, r0 = st[r][0].copy(), st[r][1].copy()
        y = orc.gdn_seq(ins[r]["qkv"], ins[r]["z"], ins[r]["a"], ins[r]["b"], prm["conv_w"],
                        prm["A_log"], prm["dt_bias"], prm["gnorm"], r0, s0, KH=KH_G, KD=KD)
        want.append((y, s0, r0))
    for t in range(steps):
        y = be.gdn_decode(1, *[np.stack([ins[r][k][t] for r in range(B)]) for k in ("qkv", "z", "a", "b")])
        for r in range(B):
            assert_close(y[r], want[r][0][t], what=f"req {r} step {t}")
    for r in range(B):
        assert rel_l2(be.gdn_state_get(1, r), want[r][1]) < 1e-5
        np.testing.assert_allclose(be.gdn_conv_get(1, r)[1:], want[r][2][1:], rtol=0, atol=0)


def test_prenormalised_mirror(be, orc):
    """coli_cuda_gdn: the reference's coli_vk_gdn contract (post-norm inputs)."""
    cfg = "gdn_prenorm"
    prm = gdn_params(cfg)
    state, ring = gdn_state0(cfg)
    _setup(be, 2, 1, prm, [(state, ring)])
    import synth
    qn = synth.normal(synth.seed_of(cfg, "qn"), (KH_G * KD,), std=0.05)
    kn = synth.normal(synth.seed_of(cfg, "kn"), (KH_G * KD,), std=0.09)
    v = synth.normal(synth.seed_of(cfg, "v"), (VH_G * VD,))
    z = synth.normal(synth.seed_of(cfg, "z"), (VH_G * VD,))
    decay = synth.uniform(synth.seed_of(cfg, "decay"), (VH_G,), 0.5, 1.0)
    beta = synth.uniform(synth.seed_of(cfg, "beta"), (VH_G,), 0.0, 1.0)
    s_ref = state.copy()
    want = orc.gdn_recur(qn, kn, v, z, decay, beta, prm["gnorm"], s_ref, KH=KH_G)
    got = be.gdn(2, qn, kn, v, z, decay, beta, prm["gnorm"])
    assert_close(got, want, what="prenorm y")
    assert rel_l2(be.gdn_state_get(2, 0), s_ref) < 1e-5


def test_state_after_4096_steps(be, orc):
    """North-star state parity: rel-L2 <= 1e-3 after 4096 sequential decode steps."""
    cfg = "gdn_4096"
    S = 4096
    prm = gdn_params(cfg)
    state, ring = gdn_state0(cfg)
    _setup(be, 3, 1, prm, [(state, ring)])
    ins = gdn_inputs(cfg, S)
    s_ref, r_ref = state.copy(), ring.copy()
    y_ref = orc.gdn_seq(ins["qkv"], ins["z"], ins["a"], ins["b"], prm["conv_w"], prm["A_log"],
                        prm["dt_bias"], prm["gnorm"], r_ref, s_ref, KH=KH_G, KD=KD)
    y = np.concatenate([be.gdn_decode(3, ins["qkv"][t:t + 1], ins["z"][t:t + 1], ins["a"][t:t + 1],
                                      ins["b"][t:t + 1]) for t in range(S)])
    err = rel_l2(be.gdn_state_get(3, 0), s_ref)
    record("decode 4096 steps state rel-L2", err)
    assert err <= STATE_REL_L2, err
    assert_close(y[-64:], y_ref[-64:], what="last outputs")


@pytest.mark.parametrize("S", [64, 100, 1000, 4096])
def test_chunked_prefill_vs_sequential_oracle(be, orc, S):
    """S >= 64 tokens run the chunk-parallel kernels; the oracle is the
    reference's token-by-token recurrence from the same carried state."""
    cfg = f"gdn_chunked_{S}"
    prm = gdn_params(cfg)
    state, ring = gdn_state0(cfg)
    _setup(be, 5, 1, prm, [(state, ring)])
    ins = gdn_inputs(cfg, S)
    s_ref, r_ref = state.copy(), ring.copy()
    y_ref = orc.gdn_seq(ins["qkv"], ins["z"], ins["a"], ins["b"], prm["conv_w"], prm["A_log"],
                        prm["dt_bias"], prm["gnorm"], r_ref, s_ref, KH=KH_G, KD=KD)
    y = be.gdn_prefill(5, 0, ins["qkv"], ins["z"], ins["a"], ins["b"])
    assert_close(y, y_ref, what=f"chunked prefill S={S}")
    err = rel_l2(be.gdn_state_get(5, 0), s_ref)
    record(f"chunked prefill S={S} state rel-L2", err)
    assert err <= STATE_REL_L2, err
    np.testing.assert_array_equal(be.gdn_conv_get(5, 0)[1:], r_ref[1:])


def test_bf16_device_path(be, orc):
    """The *_dev entry with bf16 activations (the benchmark path)."""
    import torch
    cfg = "gdn_bf16"
    B = 8
    prm = gdn_params(cfg)
    st = [gdn_state0(cfg, r) for r in range(B)]
    _setup(be, 4, B, prm, st)
    ins = [gdn_inputs(cfg, 1, r, bf16=True) for r in range(B)]
    dev = {k: torch.tensor(np.concatenate([ins[r][k] for r in range(B)]), device="cuda").bfloat16()
           for k in ("qkv", "z", "a", "b")}
    y = torch.zeros(B, VH_G * VD, dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    be.gdn_decode_dev(4, B, dev["qkv"].data_ptr(), dev["z"].data_ptr(), dev["a"].data_ptr(),
                      dev["b"].data_ptr(), y.data_ptr())
    be.sync()
    for r in range(B):
        s0, r0 = st[r][0].copy(), st[r][1].copy()
        want = orc.gdn_seq(ins[r]["qkv"], ins[r]["z"], ins[r]["a"], ins[r]["b"], prm["conv_w"],
                           prm["A_log"], prm["dt_bias"], prm["gnorm"], r0, s0, KH=KH_G, KD=KD)
        assert_close(y[r].float().cpu().numpy(), want[0], what=f"bf16 req {r}")


@pytest.mark.parametrize("kh0,nkh", [(0, 2), (6, 2), (8, 4), (4, 8)])
def test_head_sharded_segmented_prefill_vs_oracle(be, orc, kh0, nkh):
    """A head shard of 2-8 K heads at S = 4096 walks its 64 chunks as several
    segments in parallel (segment maps, fp32 chaining, replay); outputs and
    final state of the owned heads against the token-by-token oracle from a
    nonzero carried state."""
    import ctypes
    import torch
    S = 4096
    cfg = "gdn_segmented"
    prm = gdn_params(cfg)
    state, ring = gdn_state0(cfg)
    ins = gdn_inputs(cfg, S)
    s_ref, r_ref = state.copy(), ring.copy()
    y_ref = orc.gdn_seq(ins["qkv"], ins["z"], ins["a"], ins["b"], prm["conv_w"], prm["A_log"],
                        prm["dt_bias"], prm["gnorm"], r_ref, s_ref, KH=KH_G, KD=KD)
    layer, nv, v0 = 30, 2 * nkh, 2 * kh0
    lib = be.lib
    fp = ctypes.POINTER(ctypes.c_float)
    assert lib.coli_cuda_gdn_state_ensure(layer, 1, nv, KD, VD) == 1
    assert lib.coli_cuda_gdn_conv_ensure(layer, 1, CONVK, CD) == 1
    cw = np.ascontiguousarray(prm["conv_w"], np.float32)
    assert lib.coli_cuda_gdn_conv_weight(layer, cw.ctypes.data_as(fp), CONVK, CD) == 1
    arrs = [np.ascontiguousarray(prm[n], np.float32) for n in ("A_log", "dt_bias", "gnorm")]
    assert lib.coli_cuda_gdn_params(layer, *[x.ctypes.data_as(fp) for x in arrs], VH_G, VD) == 1
    be.gdn_state_set(layer, 0, np.ascontiguousarray(state[v0:v0 + nv]))
    be.gdn_conv_set(layer, 0, ring)
    dev = {k: torch.from_numpy(np.ascontiguousarray(ins[k], np.float32)).cuda() for k in ("qkv", "z", "a", "b")}
    y = torch.zeros(S, nv * VD, dtype=torch.float32, device="cuda")
    be.gdn_prefill_heads_dev(layer, 0, S, dev["qkv"].data_ptr(), dev["z"].data_ptr(), dev["a"].data_ptr(),
                             dev["b"].data_ptr(), y.data_ptr(), kh0, nkh, dtype=0)
    be.sync()
    assert_close(y.cpu().numpy(), y_ref.reshape(S, VH_G * VD)[:, v0 * VD:(v0 + nv) * VD],
                 what=f"segmented prefill heads {kh0}+{nkh}")
    err = rel_l2(be.gdn_state_get(layer, 0, VH=nv), s_ref[v0:v0 + nv])
    record(f"segmented prefill heads {kh0}+{nkh} state rel-L2", err)
    assert err <= STATE_REL_L2, err
