"""Gated GQA attention on the GPU vs the CPU oracle and the reference's own
golden outputs, through the C ABI."""
import numpy as np
import pytest

import synth
from conftest import golden, load_pkg
from helpers import H, HD, KH, assert_close
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


def _cache(cfg, T, req=0):
    """bf16-representable cache rows (treated as already roped)."""
    Kc = synth.bf16_round(synth.normal(synth.seed_of(cfg, "K", req), (KH, T, HD)))
    Vc = synth.bf16_round(synth.normal(synth.seed_of(cfg, "V", req), (KH, T, HD)))
    return Kc, Vc


def _upload(be, layer, req, Kc, Vc, n):
    max_t = Kc.shape[1]
    for kh in range(KH):
        be.kv_rows(layer, req, kh * max_t, Kc[kh, :n], Vc[kh, :n])


def _norm_w(cfg):
    return (synth.normal(synth.seed_of(cfg, "qn"), (HD,), std=0.1),
            synth.normal(synth.seed_of(cfg, "kn"), (HD,), std=0.1))


def test_golden_reference_prefill_then_decode(be):
    """tests/golden/gqa_seq.npz: the reference's attention() outputs."""
    g = golden("gqa_seq.npz")
    max_t = int(g["max_t"])
    be.kv_ensure(0, 1, KH, max_t)
    be.gqa_norm_weight(0, g["qn"], g["kn"])
    row = 0
    for pos, S in g["calls"]:
        ctx = be.gqa_step(0, 0, int(pos), g["qg"][row:row + S], g["k"][row:row + S], g["v"][row:row + S])
        assert_close(ctx, g["ctx"][row:row + S], what=f"call at pos {pos}")
        row += S
    k, v = be.kv_read(0, 0, 0, KH * max_t)
    n = row
    kc = k.reshape(KH, max_t, HD)[:, :n]
    vc = v.reshape(KH, max_t, HD)[:, :n]
    np.testing.assert_allclose(kc, g["Kc_final"][:, :n], atol=2e-2, rtol=1e-2)
    np.testing.assert_allclose(vc, g["Vc_final"][:, :n], atol=2e-2, rtol=1e-2)


def test_golden_reference_long_context(be):
    g = golden("gqa_long.npz")
    T = int(g["T"])
    Kc, Vc = mg.gqa_long_cache("golden_gqa_long", T)
    be.kv_ensure(1, 1, KH, T)
    be.gqa_norm_weight(1, g["qn"], g["kn"])
    _upload(be, 1, 0, Kc, Vc, T - 1)
    ctx = be.gqa_step(1, 0, T - 1, g["qg"], g["k"], g["v"])
    assert_close(ctx, g["ctx"], what="decode at T=4096")


# (1, 4096): a grid far below one wave (one tile per warp); (1, 32768): 74
# KV splits merged by the combine's warps four at a time
@pytest.mark.parametrize("B,tmax", [(1, 1), (3, 17), (16, 5000), (4, 32768), (1, 4096), (1, 32768)])
def test_batched_decode_vs_oracle(be, orc, B, tmax):
    cfg = f"gqa_b{B}_t{tmax}"
    rng = np.random.default_rng(B * 7919 + tmax)
    pos = np.array([tmax - 1] + list(rng.integers(0, tmax, size=B - 1)), np.int32)
    max_t = tmax
    be.kv_ensure(2, B, KH, max_t)
    qnw, knw = _norm_w(cfg)
    be.gqa_norm_weight(2, qnw, knw)
    caches = []
    for r in range(B):
        Kc, Vc = _cache(cfg, max_t, r)
        _upload(be, 2, r, Kc, Vc, int(pos[r]))
        caches.append((Kc, Vc))
    qg = synth.normal(synth.seed_of(cfg, "qg"), (B, H, 2 * HD))
    k = synth.normal(synth.seed_of(cfg, "k"), (B, KH, HD))
    v = synth.normal(synth.seed_of(cfg, "v"), (B, KH, HD), std=1.0 / 16)
    ctx = be.gqa_decode(2, qg, k, v, pos)
    for r in range(B):
        Kc, Vc = caches[r][0].copy(), caches[r][1].copy()
        q1, k1, v1 = qg[r:r + 1].copy(), k[r:r + 1].copy(), v[r:r + 1].copy()
        orc.gqa_prologue(q1, k1, v1, qnw, knw, int(pos[r]), Kc, Vc)
        want = orc.gqa_attend(q1, Kc, Vc, int(pos[r]))
        assert_close(ctx[r], want[0], what=f"req {r} pos {pos[r]}")


def test_core_mirror_roped_q(be, orc):
    """coli_cuda_gqa: S causal rows over a pre-filled cache (coli_vk_gqa contract)."""
    cfg = "gqa_core"
    T, S = 300, 7
    be.kv_ensure(3, 1, KH, T)
    Kc, Vc = _cache(cfg, T)
    _upload(be, 3, 0, Kc, Vc, T)
    q = synth.normal(synth.seed_of(cfg, "q"), (S, H, 2 * HD))
    ctx = be.gqa(3, q, T, T)
    want = orc.gqa_attend(q, Kc, Vc, T - S)
    assert_close(ctx, want, what="core")


def test_prefill_rows_vs_oracle(be, orc):
    cfg = "gqa_prefill_small"
    S = 300
    be.kv_ensure(4, 1, KH, 512)
    qnw, knw = _norm_w(cfg)
    be.gqa_norm_weight(4, qnw, knw)
    qg = synth.normal(synth.seed_of(cfg, "qg"), (S, H, 2 * HD))
    k = synth.normal(synth.seed_of(cfg, "k"), (S, KH, HD))
    v = synth.normal(synth.seed_of(cfg, "v"), (S, KH, HD))
    ctx = be.gqa_step(4, 0, 0, qg, k, v)
    Kc = np.zeros((KH, 512, HD), np.float32)
    Vc = np.zeros_like(Kc)
    q1, k1 = qg.copy(), k.copy()
    orc.gqa_prologue(q1, k1, v.copy(), qnw, knw, 0, Kc, Vc)
    # the device cache holds bf16 K/V: give the oracle the same rounded rows
    want = orc.gqa_attend(q1, synth.bf16_round(Kc), synth.bf16_round(Vc), 0)
    assert_close(ctx, want, what="prefill")


@pytest.mark.parametrize("rot", [2, 36, 64, 256])
def test_prologue_rotary_widths(be, orc, rot):
    """q/k norm + partial RoPE for rotary widths whose half is / is not a
    multiple of 8 (lane-shuffle vs shared-memory partner exchange), at a row
    count that takes the four-rows-per-CTA launch, then attention."""
    cfg = f"gqa_rot{rot}"
    S = 2050
    be.kv_ensure(4, 1, KH, 2304)
    qnw, knw = _norm_w(cfg)
    be.gqa_norm_weight(4, qnw, knw)
    qg = synth.normal(synth.seed_of(cfg, "qg"), (S, H, 2 * HD))
    k = synth.normal(synth.seed_of(cfg, "k"), (S, KH, HD))
    v = synth.normal(synth.seed_of(cfg, "v"), (S, KH, HD))
    ctx = be.gqa_step(4, 0, 0, qg, k, v, rot=rot)
    Kc = np.zeros((KH, 2304, HD), np.float32)
    Vc = np.zeros_like(Kc)
    q1, k1 = qg.copy(), k.copy()
    orc.gqa_prologue(q1, k1, v.copy(), qnw, knw, 0, Kc, Vc, rot=rot)
    # the cache rows carry the normed + roped k
    for kh in range(KH):
        kd, vd = be.kv_read(4, 0, kh * 2304, S)
        assert_close(kd, Kc[kh, :S], what=f"rot {rot} k cache")
        np.testing.assert_array_equal(vd, synth.bf16_round(v[:, kh]))
    # the roped q, through attention: the first and the last 64 rows
    Kb, Vb = synth.bf16_round(Kc), synth.bf16_round(Vc)
    assert_close(ctx[:64], orc.gqa_attend(q1[:64], Kb, Vb, 0), what=f"rot {rot} head rows")
    assert_close(ctx[S - 64:], orc.gqa_attend(q1[S - 64:], Kb, Vb, S - 64), what=f"rot {rot} tail rows")


@pytest.mark.parametrize("rot", [36, 256])
def test_small_batch_decode_rotary_widths(be, orc, rot):
    """Decode batches of up to 8 rows run the prologue inside the split
    kernel; rotary widths whose half is not a multiple of 8 (36) take its
    shared-memory RoPE exchange, the full width (256) ropes every dim."""
    cfg = f"gqa_fused_rot{rot}"
    B, max_t = 3, 700
    pos = np.array([699, 130, 64], np.int32)
    be.kv_ensure(6, B, KH, max_t)
    qnw, knw = _norm_w(cfg)
    be.gqa_norm_weight(6, qnw, knw)
    caches = []
    for r in range(B):
        Kc, Vc = _cache(cfg, max_t, r)
        _upload(be, 6, r, Kc, Vc, int(pos[r]))
        caches.append((Kc, Vc))
    qg = synth.normal(synth.seed_of(cfg, "qg"), (B, H, 2 * HD))
    k = synth.normal(synth.seed_of(cfg, "k"), (B, KH, HD))
    v = synth.normal(synth.seed_of(cfg, "v"), (B, KH, HD), std=1.0 / 16)
    ctx = be.gqa_decode(6, qg, k, v, pos, rot=rot)
    for r in range(B):
        Kc, Vc = caches[r][0].copy(), caches[r][1].copy()
        q1, k1, v1 = qg[r:r + 1].copy(), k[r:r + 1].copy(), v[r:r + 1].copy()
        orc.gqa_prologue(q1, k1, v1, qnw, knw, int(pos[r]), Kc, Vc, rot=rot)
        for kh in range(KH):   # the appended row: normed + roped k, v as given
            kd, vd = be.kv_read(6, r, kh * max_t + int(pos[r]), 1)
            assert_close(kd[0], Kc[kh, pos[r]], what=f"rot {rot} req {r} appended k")
            np.testing.assert_array_equal(vd[0], synth.bf16_round(v[r, kh]))
        want = orc.gqa_attend(q1, Kc, Vc, int(pos[r]))
        assert_close(ctx[r], want[0], what=f"rot {rot} req {r} pos {pos[r]}")


def test_bf16_device_path(be, orc):
    import torch
    cfg = "gqa_dev"
    B, T = 8, 2000
    be.kv_ensure(5, B, KH, T)
    qnw, knw = _norm_w(cfg)
    be.gqa_norm_weight(5, qnw, knw)
    caches = [_cache(cfg, T, r) for r in range(B)]
    for r in range(B):
        _upload(be, 5, r, caches[r][0], caches[r][1], T - 1)
    qg = synth.bf16_round(synth.normal(synth.seed_of(cfg, "qg"), (B, H, 2 * HD)))
    k = synth.bf16_round(synth.normal(synth.seed_of(cfg, "k"), (B, KH, HD)))
    v = synth.bf16_round(synth.normal(synth.seed_of(cfg, "v"), (B, KH, HD)))
    pos = np.full(B, T - 1, np.int32)
    d = {n: torch.tensor(a, device="cuda").bfloat16() for n, a in (("qg", qg), ("k", k), ("v", v))}
    pd = torch.tensor(pos, device="cuda")
    ctx = torch.zeros(B, H, HD, dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    be.gqa_decode_dev(5, B, d["qg"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(), pd.data_ptr(),
                      ctx.data_ptr())
    be.sync()
    for r in range(B):
        Kc, Vc = caches[r][0].copy(), caches[r][1].copy()
        q1, k1 = qg[r:r + 1].copy(), k[r:r + 1].copy()
        orc.gqa_prologue(q1, k1, v[r:r + 1].copy(), qnw, knw, T - 1, Kc, Vc)
        want = orc.gqa_attend(q1, Kc, Vc, T - 1)
        assert_close(ctx[r].float().cpu().numpy(), want[0], what=f"bf16 req {r}")


@pytest.mark.parametrize("S,pos_base", [(64, 0), (1000, 0), (200, 77), (130, 4000)])
def test_tensor_core_prefill_vs_oracle(be, orc, S, pos_base):
    """S >= 64 rows of one request run the tcgen05 prefill kernel."""
    cfg = f"gqa_tc_prefill_{S}_{pos_base}"
    max_t = pos_base + S + 5
    be.kv_ensure(6, 1, KH, max_t)
    qnw, knw = _norm_w(cfg)
    be.gqa_norm_weight(6, qnw, knw)
    Kc, Vc = _cache(cfg, max_t)
    Kc[:, pos_base:] = 0
    Vc[:, pos_base:] = 0
    if pos_base:
        _upload(be, 6, 0, Kc, Vc, pos_base)
    qg = synth.normal(synth.seed_of(cfg, "qg"), (S, H, 2 * HD))
    k = synth.normal(synth.seed_of(cfg, "k"), (S, KH, HD))
    v = synth.normal(synth.seed_of(cfg, "v"), (S, KH, HD))
    ctx = be.gqa_step(6, 0, pos_base, qg, k, v)
    q1, k1 = qg.copy(), k.copy()
    orc.gqa_prologue(q1, k1, v.copy(), qnw, knw, pos_base, Kc, Vc)
    want = orc.gqa_attend(q1, synth.bf16_round(Kc), synth.bf16_round(Vc), pos_base)
    assert_close(ctx, want, what=f"tc prefill S={S} pos_base={pos_base}")
