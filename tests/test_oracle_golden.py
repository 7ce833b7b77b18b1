"""Pin the CPU oracle (oracle/oracle.c) to the reference's own outputs.

The fixtures under tests/golden/ were produced by the reference's unmodified
attention() / gdn_step() (c/qwen.c:581-666, :669-776) via
tests/golden/make_golden.py. The oracle restates those functions' arithmetic
in the same operation order, so agreement is expected to the last bit; the
test allows 1e-6 relative.
"""
import numpy as np
import pytest

from conftest import golden
import synth
from oracle import Oracle, Reference

RTOL = 1e-6


def _close(a, b, rtol=RTOL):
    err = np.max(np.abs(a - b)) / max(1e-30, np.max(np.abs(b)))
    assert err <= rtol, err


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def test_gqa_seq_prefill_then_decode(orc):
    g = golden("gqa_seq.npz")
    max_t = int(g["max_t"])
    KH, HD = g["k"].shape[1], g["k"].shape[2]
    Kc = np.zeros((KH, max_t, HD), np.float32)
    Vc = np.zeros_like(Kc)
    row = 0
    for pos, S in g["calls"]:
        qg = g["qg"][row:row + S].copy()
        k = g["k"][row:row + S].copy()
        v = g["v"][row:row + S].copy()
        orc.gqa_prologue(qg, k, v, g["qn"], g["kn"], int(pos), Kc, Vc)
        ctx = orc.gqa_attend(qg, Kc, Vc, int(pos))
        _close(ctx, g["ctx"][row:row + S])
        row += S
    _close(Kc, g["Kc_final"])
    _close(Vc, g["Vc_final"])


def test_gqa_long_context_decode(orc):
    import make_golden_shim as mg
    g = golden("gqa_long.npz")
    T = int(g["T"])
    Kc, Vc = mg.gqa_long_cache("golden_gqa_long", T)
    qg, k, v = g["qg"].copy(), g["k"].copy(), g["v"].copy()
    orc.gqa_prologue(qg, k, v, g["qn"], g["kn"], T - 1, Kc, Vc)
    _close(Kc[:, T - 1], g["k_row"]) if np.any(g["k_row"]) else None
    ctx = orc.gqa_attend(qg, Kc, Vc, T - 1)
    _close(ctx, g["ctx"])


def test_gdn_seq(orc):
    import make_golden_shim as mg
    g = golden("gdn_seq.npz")
    state, ring = mg.gdn_init_state("golden_gdn_seq")
    y = orc.gdn_seq(g["qkv"], g["z"], g["a"], g["b"], g["conv"], g["A_log"], g["dt_bias"],
                    g["gnorm"], ring, state, KH=16, KD=128)
    _close(y, g["y"])
    _close(ring[1:], g["ring_final"])
    flat = state.reshape(-1).astype(np.float64)
    assert abs(flat.sum() - g["state_sum"]) <= 1e-6 * abs(g["state_sumsq"]) ** 0.5 * 100
    assert abs((flat * flat).sum() - g["state_sumsq"]) <= 1e-6 * g["state_sumsq"]
    _close(state.reshape(-1)[::97], g["state_sample"])


@pytest.mark.skipif(not Reference.available(), reason="reference harness not built")
def test_oracle_matches_reference_block_directly(orc):
    """Where oracle/_ref exists, run the reference and the oracle side by side
    on fresh seeded inputs (a GDN block at the real head shapes)."""
    import make_golden_shim as mg
    ref = Reference()
    D, CD = 4096, 8192
    cfg = "live_gdn"
    Wqkv = synth.normal(synth.seed_of(cfg, "Wqkv"), (CD, D), std=0.02)
    Wz = synth.normal(synth.seed_of(cfg, "Wz"), (D, D), std=0.02)
    Wa = synth.normal(synth.seed_of(cfg, "Wa"), (32, D), std=0.02)
    Wb = synth.normal(synth.seed_of(cfg, "Wb"), (32, D), std=0.02)
    conv = synth.normal(synth.seed_of(cfg, "conv"), (CD, 4), std=0.3)
    A_log = synth.uniform(synth.seed_of(cfg, "A_log"), (32,), 0.0, float(np.log(16.0)))
    dt_bias = synth.normal(synth.seed_of(cfg, "dt_bias"), (32,))
    gnorm = synth.normal(synth.seed_of(cfg, "gnorm"), (128,), std=0.1, mean=1.0)
    x = synth.normal(synth.seed_of(cfg, "x"), (3, D))
    s_ref, r_ref = mg.gdn_init_state(cfg)
    s_orc, r_orc = s_ref.copy(), r_ref.copy()
    out = ref.gdn_steps(x, 16, 128, 32, 128, 4, Wqkv, Wz, Wa, Wb, conv, A_log, dt_bias, gnorm,
                        np.eye(D, dtype=np.float32), s_ref, r_ref)
    y = orc.gdn_seq(ref.matmul(x, Wqkv), ref.matmul(x, Wz), ref.matmul(x, Wa), ref.matmul(x, Wb),
                    conv, A_log, dt_bias, gnorm, r_orc, s_orc, KH=16, KD=128)
    _close(y, out)
    _close(s_orc, s_ref)
