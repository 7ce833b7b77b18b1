"""Parity at the configurations bench.py measures, through
the C ABI, against the fp32 CPU oracle.

The inputs of these sizes are drawn on the device (seeded torch generator,
bf16, the benchmark's distributions) and the pieces the oracle needs are
copied back, so the oracle and the kernels read bit-identical values and the
host never holds a whole 32k-token activation in fp32:

* GQA prefill S = 8192 / 32768 (config 4a): the whole bf16 KV cache the
  prologue wrote is compared with the oracle's normed + roped rows, and the
  attention output is checked on sampled query rows (the first and last 64,
  one row per 4096), where the oracle's cost is O(rows x S).
* GDN prefill S = 8192 / 32768 (config 4b): every output row and the final
  state against the token-by-token oracle, walked in blocks of 2048 tokens.
* GQA decode, 64 requests at context 32768 (config 2, the headline): ragged
  positions, 8 requests checked.
* GDN decode, batch 256 (config 3): every request, outputs and states.

bf16 outputs are compared with max-abs 2e-2 plus half a bf16 ulp of the
expected value (the rounding of the output itself: bf16 keeps 8 significant
bits, so half an ulp of x is 2^(floor(log2|x|) - 8)), cosine >= 0.9999.
"""
import numpy as np
import pytest

from conftest import load_pkg
from helpers import (CD, CONVK, H, HD, KD, KH, KH_G, MAX_ABS, MIN_COS, STATE_REL_L2, VD, VH_G, cosine,
                     gdn_params, record, rel_l2)
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


def half_ulp_bf16(x):
    x = np.abs(np.asarray(x, np.float64))
    return np.where(x > 0, np.exp2(np.floor(np.log2(np.maximum(x, 1e-300))) - 8), 0.0)


def assert_close_bf16(got, want, what):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    excess = np.abs(got - want) - half_ulp_bf16(want)
    err = float(np.max(excess))
    cos = cosine(got, want)
    record(what, {"max_abs_beyond_bf16": err, "cos": cos})
    assert err <= MAX_ABS and cos >= MIN_COS, f"{what}: max-abs {err:.3e} cosine {cos:.8f}"


def _randn(shape, seed, std=1.0):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda", dtype=torch.float32) * std).bfloat16()


def _host(t):
    return np.ascontiguousarray(t.float().cpu().numpy())


@pytest.mark.parametrize("S", [8192, 32768])
def test_gqa_prefill_at_bench_size(be, orc, S):
    import torch
    layer = 40 if S == 8192 else 44
    rng = np.random.default_rng(S)
    qnw = (rng.standard_normal(HD) * 0.1).astype(np.float32)
    knw = (rng.standard_normal(HD) * 0.1).astype(np.float32)
    be.kv_ensure(layer, 1, KH, S)
    be.gqa_norm_weight(layer, qnw, knw)
    qg = _randn((S, H, 2 * HD), 11 + S)
    k = _randn((S, KH, HD), 12 + S)
    v = _randn((S, KH, HD), 13 + S)
    ctx = torch.zeros(S, H, HD, dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    be.gqa_step_dev(layer, 0, S, 0, qg.data_ptr(), k.data_ptr(), v.data_ptr(), ctx.data_ptr())
    be.sync()
    # the oracle's cache: normed + roped k, raw v, block by block
    Kc = np.zeros((KH, S, HD), np.float32)
    Vc = np.zeros_like(Kc)
    blk = 2048
    for s0 in range(0, S, blk):
        qz = np.zeros((blk, H, 2 * HD), np.float32)
        orc.gqa_prologue(qz, _host(k[s0:s0 + blk]), _host(v[s0:s0 + blk]), qnw, knw, s0, Kc, Vc)
    for kh in range(KH):
        kd, vd = be.kv_read(layer, 0, kh * S, S)
        assert_close_bf16(kd, Kc[kh], f"gqa prefill S={S} k cache head {kh}")
        np.testing.assert_array_equal(vd, _host(v[:, kh]))
    Kb = np.ascontiguousarray(_host(torch.from_numpy(Kc).bfloat16()))
    Vb = np.ascontiguousarray(Vc)   # already bf16 values
    rows = [(0, 64), (S - 64, 64)] + [(r, 1) for r in range(4095, S - 64, 4096)]
    for r0, n in rows:
        q1 = _host(qg[r0:r0 + n])
        k1 = _host(k[r0:r0 + n])
        Kd, Vd = np.zeros((KH, S, HD), np.float32), np.zeros((KH, S, HD), np.float32)
        orc.gqa_prologue(q1, k1, _host(v[r0:r0 + n]), qnw, knw, r0, Kd, Vd)
        want = orc.gqa_attend(q1, Kb, Vb, r0)
        assert_close_bf16(_host(ctx[r0:r0 + n]), want, f"gqa prefill S={S} rows {r0}+{n}")


@pytest.mark.parametrize("S", [8192, 32768])
def test_gdn_prefill_at_bench_size(be, orc, S):
    import torch
    layer = 41 if S == 8192 else 45
    cfg = f"gdn_bench_{S}"
    prm = gdn_params(cfg)
    be.gdn_setup(layer, 1, prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["gnorm"])
    # the benchmark's start: zero state and conv history
    state = np.zeros((VH_G, KD, VD), np.float32)
    ring = np.zeros((CONVK, CD), np.float32)
    be.gdn_state_set(layer, 0, state)
    be.gdn_conv_set(layer, 0, ring)
    qkv = _randn((S, CD), 21 + S)
    z = _randn((S, VH_G * VD), 22 + S)
    a = _randn((S, VH_G), 23 + S)
    b = _randn((S, VH_G), 24 + S)
    y = torch.zeros(S, VH_G * VD, dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    be.gdn_prefill_dev(layer, 0, S, qkv.data_ptr(), z.data_ptr(), a.data_ptr(), b.data_ptr(), y.data_ptr())
    be.sync()
    blk = 2048
    worst = (-1.0, 1.0)
    for s0 in range(0, S, blk):
        sl = slice(s0, s0 + blk)
        want = orc.gdn_seq(_host(qkv[sl]), _host(z[sl]), _host(a[sl]), _host(b[sl]), prm["conv_w"],
                           prm["A_log"], prm["dt_bias"], prm["gnorm"], ring, state, KH=KH_G, KD=KD)
        got = _host(y[sl])
        excess = np.abs(got.astype(np.float64) - want) - half_ulp_bf16(want)
        worst = (max(worst[0], float(excess.max())), min(worst[1], cosine(got, want)))
    record(f"gdn prefill S={S} y", {"max_abs_beyond_bf16": worst[0], "min_block_cos": worst[1]})
    assert worst[0] <= MAX_ABS and worst[1] >= MIN_COS, worst
    err = rel_l2(be.gdn_state_get(layer, 0), state)
    record(f"gdn prefill S={S} state rel-L2", err)
    assert err <= STATE_REL_L2, err
    np.testing.assert_array_equal(be.gdn_conv_get(layer, 0)[1:], ring[1:])


def test_gqa_decode_headline_config(be, orc):
    """64 requests, context 32768, ragged positions; 8 requests checked."""
    import torch
    layer, B, T = 42, 64, 32768
    rng = np.random.default_rng(64)
    pos = np.array([T - 1] + list(rng.integers(1, T, size=B - 1)), np.int32)
    qnw = (rng.standard_normal(HD) * 0.1).astype(np.float32)
    knw = (rng.standard_normal(HD) * 0.1).astype(np.float32)
    be.kv_ensure(layer, B, KH, T)
    be.gqa_norm_weight(layer, qnw, knw)

    def cache(r):
        return _randn((2, KH, T, HD), 1000 + r)

    for r in range(B):
        c = cache(r)
        torch.cuda.synchronize()   # c is drawn on torch's stream, the copies run on the backend's
        for kh in range(KH):
            be.kv_rows_dev(layer, r, kh * T, int(pos[r]), c[0, kh].data_ptr(), c[1, kh].data_ptr(), dtype=1)
        be.sync()   # the copies run on the backend's stream: finish them before c is freed
        del c
    qg = _randn((B, H, 2 * HD), 31)
    k = _randn((B, KH, HD), 32)
    v = _randn((B, KH, HD), 33, std=1.0 / 16)
    pd = torch.tensor(pos, device="cuda")
    ctx = torch.zeros(B, H, HD, dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    be.gqa_decode_dev(layer, B, qg.data_ptr(), k.data_ptr(), v.data_ptr(), pd.data_ptr(), ctx.data_ptr())
    be.sync()
    for r in [0, 1, 7, 20, 33, 47, 58, 63]:
        c = cache(r)
        Kc, Vc = _host(c[0]), _host(c[1])
        q1, k1 = _host(qg[r:r + 1]), _host(k[r:r + 1])
        orc.gqa_prologue(q1, k1, _host(v[r:r + 1]), qnw, knw, int(pos[r]), Kc, Vc)
        Kc[:, int(pos[r])] = _host(torch.from_numpy(Kc[:, int(pos[r])]).bfloat16())
        want = orc.gqa_attend(q1, Kc, Vc, int(pos[r]))
        assert_close_bf16(_host(ctx[r]), want[0], f"gqa decode B=64 T=32k req {r} pos {pos[r]}")


def test_gdn_decode_batch_256(be, orc):
    """Every request of a 256-request decode step: outputs and states."""
    layer, B = 43, 256
    cfg = "gdn_decode_256"
    prm = gdn_params(cfg)
    be.gdn_setup(layer, B, prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["gnorm"])
    rng = np.random.default_rng(256)
    states = [(rng.standard_normal((VH_G, KD, VD)) * 0.1).astype(np.float32) for _ in range(B)]
    rings = [rng.standard_normal((CONVK, CD)).astype(np.float32) for _ in range(B)]
    for r in range(B):
        rings[r][0] = 0.0
        be.gdn_state_set(layer, r, states[r])
        be.gdn_conv_set(layer, r, rings[r])
    for step in range(2):
        qkv = rng.standard_normal((B, CD)).astype(np.float32)
        z = rng.standard_normal((B, VH_G * VD)).astype(np.float32)
        a = rng.standard_normal((B, VH_G)).astype(np.float32)
        b = rng.standard_normal((B, VH_G)).astype(np.float32)
        y = be.gdn_decode(layer, qkv, z, a, b)
        want = np.stack([orc.gdn_seq(qkv[r:r + 1], z[r:r + 1], a[r:r + 1], b[r:r + 1], prm["conv_w"],
                                     prm["A_log"], prm["dt_bias"], prm["gnorm"], rings[r], states[r],
                                     KH=KH_G, KD=KD)[0] for r in range(B)])
        err = float(np.max(np.abs(y - want)))
        cos = cosine(y, want)
        record(f"gdn decode B=256 step {step}", {"max_abs": err, "cos": cos})
        assert err <= MAX_ABS and cos >= MIN_COS, (err, cos)
    worst = max(rel_l2(be.gdn_state_get(layer, r), states[r]) for r in range(B))
    record("gdn decode B=256 worst state rel-L2", worst)
    assert worst <= 1e-4, worst
