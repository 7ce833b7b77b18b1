"""Block-level entry points (projections + mixer + out-projection) on the GPU
against the fp32 CPU path: numpy fp32 projections (the reference's matmul(),
c/qwen.c:178-189) around the C oracle, and where the reference harness was
built, the reference's own attention() / gdn_step() with the same weights."""
import numpy as np
import pytest

from conftest import load_pkg
from helpers import (CD, CONVK, KD, KH, KH_G, H, HD, VD, VH_G, assert_close, gdn_params, gdn_state0,
                     record, rel_l2)
from oracle import Oracle, Reference
import synth

pytestmark = pytest.mark.gpu
D = 2048          # hidden size of the benchmark container


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


def _w(cfg, name, O, I, std=0.02):
    return synth.normal(synth.seed_of(cfg, name), (O, I), std=std)


def _dense(be, w, **kw):
    return load_pkg().coli_cuda.DenseTensor(be, w, **kw)


@pytest.mark.parametrize("S", [1, 7, 64, 300])
def test_linear_vs_bf16_product(be, S):
    """y = x W^T for O not a multiple of the 128-row tile, decode (split-K)
    and prefill shapes; the reference product uses the same bf16 operands."""
    W = _w("lin", "W", 1000, D)
    x = synth.normal(synth.seed_of("lin", "x", S), (S, D))
    t = _dense(be, W)
    y = be.matmul(t, x)
    ref = synth.bf16_round(x).astype(np.float64) @ synth.bf16_round(W).astype(np.float64).T
    err = np.max(np.abs(y - ref))
    assert err <= 1e-4 * np.max(np.abs(ref)) + 1e-6, err
    t.free()


@pytest.mark.parametrize("S", [1, 5, 16, 20])
def test_linear_multi_launch_vs_bf16_product(be, S):
    """coli_cuda_matmul_multi_dev: four projections of one x (output widths
    1000, 512, 32, 32: not multiples of the tile, two of them smaller than
    one tile) in one launch for S <= 16 (shared grid, split-K across a
    cluster), one by one above; against the bf16-operand product."""
    import torch
    Os = (1000, 512, 32, 32)
    Ws = [_w("linm", f"W{i}", O, D) for i, O in enumerate(Os)]
    x = synth.normal(synth.seed_of("linm", "x", S), (S, D))
    ts = [_dense(be, W) for W in Ws]
    xd = torch.from_numpy(synth.bf16_round(x)).cuda().bfloat16()
    ys = [torch.full((S, O), float("nan"), device="cuda") for O in Os]
    torch.cuda.synchronize()
    be.matmul_multi_dev(ts, xd.data_ptr(), S, [y.data_ptr() for y in ys], 0)
    be.sync()
    for W, y, O in zip(Ws, ys, Os):
        ref = synth.bf16_round(x).astype(np.float64) @ synth.bf16_round(W).astype(np.float64).T
        err = np.max(np.abs(y.cpu().numpy() - ref))
        assert err <= 1e-4 * np.max(np.abs(ref)) + 1e-6, (O, err)
    for t in ts:
        t.free()


def test_linear_int8_rows(be):
    rng = np.random.default_rng(5)
    q = rng.integers(-127, 128, size=(384, D), dtype=np.int8)
    s = (rng.random(384).astype(np.float32) + 0.5) * 1e-3
    x = synth.normal(synth.seed_of("lin8", "x"), (3, D))
    t = _dense(be, q, scales=s, fmt=1)
    y = be.matmul(t, x)
    Wd = synth.bf16_round(q.astype(np.float32) * s[:, None])
    ref = synth.bf16_round(x).astype(np.float64) @ Wd.astype(np.float64).T
    assert np.max(np.abs(y - ref)) <= 1e-4 * np.max(np.abs(ref)) + 1e-6
    assert t.nbytes == 384 * D * 2
    t.free()


def test_gqa_block_prefill_then_decode(be, orc):
    """Prefill 130 rows (tcgen05 path), one decode row, then 5 rows through the
    split-KV path, all continuing one cache; against fp32 projections around
    the oracle with an fp32 cache."""
    cfg = "gqa_block"
    Wq, Wk, Wv = _w(cfg, "q", H * 2 * HD, D), _w(cfg, "k", KH * HD, D), _w(cfg, "v", KH * HD, D)
    Wo = _w(cfg, "o", D, H * HD)
    qnw = synth.normal(synth.seed_of(cfg, "qn"), (HD,), std=0.1)
    knw = synth.normal(synth.seed_of(cfg, "kn"), (HD,), std=0.1)
    T = 256
    layer = 8
    be.kv_ensure(layer, 1, KH, T)
    be.gqa_norm_weight(layer, qnw, knw)
    tq, tk, tv, to = (_dense(be, w) for w in (Wq, Wk, Wv, Wo))
    Kc = np.zeros((KH, T, HD), np.float32)
    Vc = np.zeros_like(Kc)
    ref = Reference(path=None) if Reference.available() else None
    Kr, Vr = np.zeros_like(Kc), np.zeros_like(Kc)
    pos = 0
    for S in (130, 1, 5):
        x = synth.normal(synth.seed_of(cfg, "x", pos), (S, D))
        got = be.gqa_full(layer, x, tq, tk, tv, to, pos, max_t=T)
        qg = (x @ Wq.T).reshape(S, H, 2 * HD)
        k = (x @ Wk.T).reshape(S, KH, HD)
        v = (x @ Wv.T).reshape(S, KH, HD)
        orc.gqa_prologue(qg, k, v, qnw, knw, pos, Kc, Vc)
        ctx = orc.gqa_attend(qg, Kc, Vc, pos)
        want = ctx.reshape(S, H * HD) @ Wo.T
        assert_close(got, want, what=f"gqa block S={S} pos={pos}")
        if ref is not None:   # the reference's own attention() on the same weights
            rout = ref.attention(x, pos, H, KH, HD, Wq, Wk, Wv, Wo, qnw, knw, Kr, Vr)
            assert_close(got, rout, what=f"gqa block vs reference S={S}")
        pos += S
    for t in (tq, tk, tv, to):
        t.free()


@pytest.mark.parametrize("S", [1, 20, 100])
def test_gdn_block_vs_oracle(be, orc, S):
    """in_proj_qkv / in_proj_z -> conv + delta rule + gated norm -> out_proj
    with the engine's params packing (decay | beta | gnorm), from a nonzero
    carried state; S = 1 is coli_cuda_gdn_full, 20 the token-stepped sequence,
    100 the chunk-parallel prefill."""
    cfg = f"gdn_block_{S}"
    prm = gdn_params(cfg)
    state, ring = gdn_state0(cfg)
    Wqkv, Wz = _w(cfg, "qkv", CD, D), _w(cfg, "z", VH_G * VD, D)
    Wa, Wb, Wo = _w(cfg, "a", VH_G, D), _w(cfg, "b", VH_G, D), _w(cfg, "o", D, VH_G * VD)
    x = synth.normal(synth.seed_of(cfg, "x"), (S, D))
    a, b = x @ Wa.T, x @ Wb.T
    sp = np.where(a + prm["dt_bias"] > 20, a + prm["dt_bias"], np.log1p(np.exp(a + prm["dt_bias"])))
    decay = np.exp(-np.exp(prm["A_log"]) * sp).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-b))).astype(np.float32)
    params = np.concatenate([decay, beta, np.broadcast_to(prm["gnorm"], (S, VD))], axis=1)
    layer = 12 + S % 7
    be.gdn_setup(layer, 1, prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["gnorm"])
    be.gdn_state_set(layer, 0, state)
    be.gdn_conv_set(layer, 0, ring)
    tqkv, tz, to = _dense(be, Wqkv), _dense(be, Wz), _dense(be, Wo)
    got = be.gdn_full_seq(layer, x, params, tqkv, tz, to)
    s_ref, r_ref = state.copy(), ring.copy()
    y = orc.gdn_seq(x @ Wqkv.T, x @ Wz.T, a, b, prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["gnorm"],
                    r_ref, s_ref, KH=KH_G, KD=KD)
    want = y.reshape(S, VH_G * VD) @ Wo.T
    assert_close(got, want, what=f"gdn block S={S}")
    # The block's projections run on bf16 weights and activations while the
    # oracle here is fed fp32 projections, so the state difference includes the
    # projections' bf16 rounding; the recurrence's own bound (rel-L2 1e-3) is
    # asserted with identical inputs in test_gpu_gdn.py / test_gpu_bench_configs.py.
    err = rel_l2(be.gdn_state_get(layer, 0), s_ref)
    record(f"gdn block S={S} state rel-L2 (bf16 projections)", err)
    assert err <= 1e-2, err
    for t in (tqkv, tz, to):
        t.free()


@pytest.mark.parametrize("S", [1, 20, 100])
def test_gdn_block_device_ab_vs_oracle(be, orc, S):
    """coli_cuda_gdn_full_ab: the a / b projections on the device too, in the
    same launch as in_proj_qkv / in_proj_z (c/qwen.c:709-711), the gates from
    the layer's A_log / dt_bias (c/qwen.c:722-727) inside the mixer kernels.
    The checker's projections take the same bf16-rounded operands (x and W)
    with fp32 accumulation and feed the oracle's gdn_step loop, so the state
    is held to the recurrence's own bound (rel-L2 1e-3)."""
    cfg = f"gdn_block_ab_{S}"
    prm = gdn_params(cfg)
    state, ring = gdn_state0(cfg)
    Ws = {n: synth.bf16_round(_w(cfg, n, O, D)) for n, O in
          (("qkv", CD), ("z", VH_G * VD), ("a", VH_G), ("b", VH_G))}
    Wo = synth.bf16_round(_w(cfg, "o", D, VH_G * VD))
    x = synth.normal(synth.seed_of(cfg, "x"), (S, D))
    xb = synth.bf16_round(x)
    layer = 20 + S % 7
    be.gdn_setup(layer, 1, prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["gnorm"])
    be.gdn_state_set(layer, 0, state)
    be.gdn_conv_set(layer, 0, ring)
    ts = {n: _dense(be, w) for n, w in Ws.items()}
    to = _dense(be, Wo)
    got = be.gdn_full_ab(layer, x, ts["qkv"], ts["z"], ts["a"], ts["b"], to)
    s_ref, r_ref = state.copy(), ring.copy()
    p = {n: xb @ w.T for n, w in Ws.items()}
    y = orc.gdn_seq(p["qkv"], p["z"], p["a"], p["b"], prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["gnorm"],
                    r_ref, s_ref, KH=KH_G, KD=KD)
    want = synth.bf16_round(y.reshape(S, VH_G * VD)) @ Wo.T
    assert_close(got, want, what=f"gdn block (device a/b) S={S}")
    err = rel_l2(be.gdn_state_get(layer, 0), s_ref)
    record(f"gdn block S={S} state rel-L2 (device a/b)", err)
    assert err <= 1e-3, err
    for t in list(ts.values()) + [to]:
        t.free()


def _rmsnorm_zc(x, w, eps=1e-6):
    """c/qwen.c:326-330 (double accumulation of the mean square)."""
    x = np.asarray(x, np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    r = (1.0 / np.sqrt((ms + eps).astype(np.float32))).astype(np.float32)
    return (x * r * (1.0 + w)).astype(np.float32)


def test_gqa_route_tail(be, orc):
    """in_ln on the device, the GQA block, then resid + delta, post_ln and the
    router logits (coli_cuda_gqa_full_route) for 3 prompt rows."""
    cfg = "gqa_route"
    E, S, T, layer, ln_layer = 8, 3, 64, 9, 3
    Wq, Wk, Wv = _w(cfg, "q", H * 2 * HD, D), _w(cfg, "k", KH * HD, D), _w(cfg, "v", KH * HD, D)
    Wo, Wr = _w(cfg, "o", D, H * HD), _w(cfg, "r", E, D)
    qnw = synth.normal(synth.seed_of(cfg, "qn"), (HD,), std=0.1)
    knw = synth.normal(synth.seed_of(cfg, "kn"), (HD,), std=0.1)
    in_ln = synth.normal(synth.seed_of(cfg, "in"), (D,), std=0.1)
    post_ln = synth.normal(synth.seed_of(cfg, "post"), (D,), std=0.1)
    resid = synth.normal(synth.seed_of(cfg, "resid"), (S, D))
    be.kv_ensure(layer, 1, KH, T)
    be.gqa_norm_weight(layer, qnw, knw)
    be.layer_norm_weight(ln_layer, in_ln, post_ln)
    ts = [_dense(be, w) for w in (Wq, Wk, Wv, Wo, Wr)]
    ro, nr, pr = be.gqa_full_route(layer, resid, *ts[:4], ts[4], ln_layer, 0, max_t=T)
    x = _rmsnorm_zc(resid, in_ln)
    qg = (x @ Wq.T).reshape(S, H, 2 * HD)
    k = (x @ Wk.T).reshape(S, KH, HD)
    v = (x @ Wv.T).reshape(S, KH, HD)
    Kc = np.zeros((KH, T, HD), np.float32)
    Vc = np.zeros_like(Kc)
    orc.gqa_prologue(qg, k, v, qnw, knw, 0, Kc, Vc)
    delta = orc.gqa_attend(qg, Kc, Vc, 0).reshape(S, H * HD) @ Wo.T
    want_ro = resid + delta
    want_nr = _rmsnorm_zc(want_ro, post_ln)
    assert_close(ro, want_ro, what="resid_out")
    assert_close(nr, want_nr, what="nrm_out")
    assert_close(pr, want_nr @ Wr.T, what="router logits")
    for t in ts:
        t.free()


def test_gdn_route_tail(be, orc):
    """One GDN token with the route tail (coli_cuda_gdn_full_route); x_in is
    the host-normed input the caller also derives b/a from."""
    cfg = "gdn_route"
    E, layer, ln_layer = 8, 20, 4
    prm = gdn_params(cfg)
    state, ring = gdn_state0(cfg)
    Wqkv, Wz = _w(cfg, "qkv", CD, D), _w(cfg, "z", VH_G * VD, D)
    Wa, Wb, Wo, Wr = _w(cfg, "a", VH_G, D), _w(cfg, "b", VH_G, D), _w(cfg, "o", D, VH_G * VD), _w(cfg, "r", E, D)
    in_ln = synth.normal(synth.seed_of(cfg, "in"), (D,), std=0.1)
    post_ln = synth.normal(synth.seed_of(cfg, "post"), (D,), std=0.1)
    resid = synth.normal(synth.seed_of(cfg, "resid"), (1, D))
    x = _rmsnorm_zc(resid, in_ln)
    a, b = x @ Wa.T, x @ Wb.T
    sp = np.where(a + prm["dt_bias"] > 20, a + prm["dt_bias"], np.log1p(np.exp(a + prm["dt_bias"])))
    decay = np.exp(-np.exp(prm["A_log"]) * sp).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-b))).astype(np.float32)
    params = np.concatenate([decay, beta, prm["gnorm"][None, :]], axis=1)
    be.gdn_setup(layer, 1, prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["gnorm"])
    be.gdn_state_set(layer, 0, state)
    be.gdn_conv_set(layer, 0, ring)
    be.layer_norm_weight(ln_layer, in_ln, post_ln)
    ts = [_dense(be, w) for w in (Wqkv, Wz, Wo, Wr)]
    ro, nr, pr = be.gdn_full_route(layer, x[0], resid[0], params[0], ts[0], ts[1], ts[2], ts[3], ln_layer)
    s_ref, r_ref = state.copy(), ring.copy()
    y = orc.gdn_seq(x @ Wqkv.T, x @ Wz.T, a, b, prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["gnorm"],
                    r_ref, s_ref, KH=KH_G, KD=KD)
    want_ro = resid[0] + (y.reshape(1, VH_G * VD) @ Wo.T)[0]
    want_nr = _rmsnorm_zc(want_ro, post_ln)
    assert_close(ro, want_ro, what="resid_out")
    assert_close(nr, want_nr, what="nrm_out")
    assert_close(pr, want_nr @ Wr.T, what="router logits")
    for t in ts:
        t.free()


def test_snapshot_layers_end_to_end(be, orc, tmp_path):
    """A two-layer container (layer 0 GatedDeltaNet, layer 1 gated GQA, the
    benchmark shapes, bf16 weights N(0, 0.02)) written as safetensors, loaded
    through coli_cuda_st_* into resident tensors, then one prompt of 5 rows
    through both blocks against fp32 references built from the same stored
    values."""
    import json
    import st_writer
    snapmod = load_pkg().snapshot
    cfg = {"hidden_size": D, "num_hidden_layers": 2, "layer_types": ["linear_attention", "full_attention"],
           "num_attention_heads": H, "num_key_value_heads": KH, "head_dim": HD, "partial_rotary_factor": 0.25,
           "rope_theta": 1e7, "rms_norm_eps": 1e-6, "linear_num_key_heads": KH_G, "linear_key_head_dim": KD,
           "linear_num_value_heads": VH_G, "linear_value_head_dim": VD, "linear_conv_kernel_dim": CONVK}
    c = "snap"
    prm = gdn_params(c)
    t = {}
    for i in (0, 1):
        t[f"model.layers.{i}.input_layernorm.weight"] = ("F32", synth.normal(synth.seed_of(c, "in", i), (D,), std=0.1))
        t[f"model.layers.{i}.post_attention_layernorm.weight"] = ("F32", synth.normal(synth.seed_of(c, "po", i), (D,), std=0.1))
    p0, p1 = "model.layers.0.linear_attn.", "model.layers.1.self_attn."
    t.update({p0 + "in_proj_qkv.weight": ("BF16", _w(c, "qkv", CD, D)), p0 + "in_proj_z.weight": ("BF16", _w(c, "z", VH_G * VD, D)),
              p0 + "in_proj_a.weight": ("BF16", _w(c, "a", VH_G, D)), p0 + "in_proj_b.weight": ("BF16", _w(c, "b", VH_G, D)),
              p0 + "out_proj.weight": ("BF16", _w(c, "o", D, VH_G * VD)),
              p0 + "conv1d.weight": ("BF16", prm["conv_w"].reshape(CD, 1, CONVK)),
              p0 + "A_log": ("F32", prm["A_log"]), p0 + "dt_bias": ("F32", prm["dt_bias"]), p0 + "norm.weight": ("F32", prm["gnorm"]),
              p1 + "q_proj.weight": ("BF16", _w(c, "q", H * 2 * HD, D)), p1 + "k_proj.weight": ("BF16", _w(c, "k", KH * HD, D)),
              p1 + "v_proj.weight": ("BF16", _w(c, "v", KH * HD, D)), p1 + "o_proj.weight": ("BF16", _w(c, "oo", D, H * HD)),
              p1 + "q_norm.weight": ("F32", synth.normal(synth.seed_of(c, "qn"), (HD,), std=0.1)),
              p1 + "k_norm.weight": ("F32", synth.normal(synth.seed_of(c, "kn"), (HD,), std=0.1))})
    st_writer.write(str(tmp_path / "model-00001-of-00001.safetensors"), t)
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    snap = snapmod.Snapshot(be.lib, str(tmp_path))
    gdn = snapmod.load_mixer_layer(be, snap, 0, slot=24)
    gqa = snapmod.load_mixer_layer(be, snap, 1, slot=10, max_t=64)
    S = 5
    x = synth.normal(synth.seed_of(c, "x"), (S, D))
    # GDN layer 0 from zero state and history
    be.gdn_state_set(24, 0, np.zeros((VH_G, KD, VD), np.float32))
    be.gdn_conv_set(24, 0, np.zeros((CONVK, CD), np.float32))
    got = be.gdn_full_seq(24, x, snapmod.gdn_params(gdn, x), gdn["qkv"], gdn["z"], gdn["out"])
    rd = lambda n: snap.read(n)
    a, b = x @ rd(p0 + "in_proj_a.weight").T, x @ rd(p0 + "in_proj_b.weight").T
    s_ref, r_ref = np.zeros((VH_G, KD, VD), np.float32), np.zeros((CONVK, CD), np.float32)
    y = orc.gdn_seq(x @ rd(p0 + "in_proj_qkv.weight").T, x @ rd(p0 + "in_proj_z.weight").T, a, b,
                    rd(p0 + "conv1d.weight").reshape(CD, CONVK), prm["A_log"], prm["dt_bias"], prm["gnorm"],
                    r_ref, s_ref, KH=KH_G, KD=KD)
    assert_close(got, y.reshape(S, VH_G * VD) @ rd(p0 + "out_proj.weight").T, what="snapshot GDN layer")
    # GQA layer 1
    got = be.gqa_full(10, x, gqa["q"], gqa["k"], gqa["v"], gqa["o"], 0, max_t=64)
    qg = (x @ rd(p1 + "q_proj.weight").T).reshape(S, H, 2 * HD)
    k = (x @ rd(p1 + "k_proj.weight").T).reshape(S, KH, HD)
    v = (x @ rd(p1 + "v_proj.weight").T).reshape(S, KH, HD)
    Kc = np.zeros((KH, 64, HD), np.float32)
    Vc = np.zeros_like(Kc)
    orc.gqa_prologue(qg, k, v, rd(p1 + "q_norm.weight"), rd(p1 + "k_norm.weight"), 0, Kc, Vc)
    want = orc.gqa_attend(qg, Kc, Vc, 0).reshape(S, H * HD) @ rd(p1 + "o_proj.weight").T
    assert_close(got, want, what="snapshot GQA layer")
    for lt in (gdn, gqa):
        for v_ in lt.values():
            if hasattr(v_, "free"):
                v_.free()
    snap.close()
