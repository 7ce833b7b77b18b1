"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference's OWN functions — attention() and gdn_step() from
c/qwen.c, compiled unmodified into oracle/_ref/libqwenref.so by
oracle/Makefile — on seeded inputs at the Qwen3.5-35B-A3B token-mixer shapes
and stores their inputs (post-projection, i.e. what the token-mixer core
consumes) and outputs as .npz files next to this script.

The out-projection weight is the identity (hidden = H*hd for GQA and
VH*VD for GDN), so the block output the reference returns IS the mixer core
output (ctx for GQA, the gated-RMSNorm y for GDN), exactly. The projected
inputs (q|gate, k, v; qkv, z, a, b) are recomputed with the reference's own
matmul() on the same x and weights, so they are bit-identical to what the
reference computed inside the block.

Usage (in the build container, where the reference sources exist):
    make -C oracle && python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "qwen3.c_b200"))

import synth  # noqa: E402
from oracle import Reference  # noqa: E402

H, KH, HD = 16, 2, 256
KD, VD, GKH, GVH, CONVK = 128, 128, 16, 32, 4


def gqa_weights(cfg):
    D = H * HD
    W = {
        "Wq": synth.normal(synth.seed_of(cfg, "Wq"), (H * 2 * HD, D), std=0.02),
        "Wk": synth.normal(synth.seed_of(cfg, "Wk"), (KH * HD, D), std=0.02),
        "Wv": synth.normal(synth.seed_of(cfg, "Wv"), (KH * HD, D), std=0.02),
        "Wo": np.eye(D, dtype=np.float32),
        "qn": synth.normal(synth.seed_of(cfg, "qn"), (HD,), std=0.1),
        "kn": synth.normal(synth.seed_of(cfg, "kn"), (HD,), std=0.1),
    }
    return D, W


def make_gqa_seq(ref):
    """Prefill of 12 tokens at pos 0, then 3 single-token decode steps."""
    cfg = "golden_gqa_seq"
    D, W = gqa_weights(cfg)
    max_t = 16
    Kc = np.zeros((KH, max_t, HD), np.float32)
    Vc = np.zeros((KH, max_t, HD), np.float32)
    calls = [(0, 12), (12, 1), (13, 1), (14, 1)]
    qg_all, k_all, v_all, ctx_all, pos_all = [], [], [], [], []
    for ci, (pos, S) in enumerate(calls):
        x = synth.normal(synth.seed_of(cfg, "x", ci), (S, D))
        qg_all.append(ref.matmul(x, W["Wq"]))
        k_all.append(ref.matmul(x, W["Wk"]))
        v_all.append(ref.matmul(x, W["Wv"]))
        out = ref.attention(x, pos, H, KH, HD, W["Wq"], W["Wk"], W["Wv"], W["Wo"], W["qn"],
                            W["kn"], Kc, Vc)
        ctx_all.append(out)
        pos_all.append(np.full(S, pos, np.int32) + np.arange(S, dtype=np.int32))
    np.savez_compressed(
        os.path.join(HERE, "gqa_seq.npz"),
        qg=np.concatenate(qg_all).reshape(-1, H, 2 * HD),
        k=np.concatenate(k_all).reshape(-1, KH, HD),
        v=np.concatenate(v_all).reshape(-1, KH, HD),
        ctx=np.concatenate(ctx_all).reshape(-1, H, HD),
        calls=np.array(calls, np.int32), qn=W["qn"], kn=W["kn"], max_t=np.int32(max_t),
        Kc_final=Kc, Vc_final=Vc)


def gqa_long_cache(cfg, T):
    """Seeded, bf16-representable cache rows [0, T-1) (treated as roped)."""
    Kc = synth.bf16_round(synth.normal(synth.seed_of(cfg, "Kc"), (KH, T, HD), std=1.0))
    Vc = synth.bf16_round(synth.normal(synth.seed_of(cfg, "Vc"), (KH, T, HD), std=1.0))
    Kc[:, T - 1] = 0
    Vc[:, T - 1] = 0
    return Kc, Vc


def make_gqa_long(ref, T=4096):
    """One decode step at position T-1 over a seeded T-1 row cache."""
    cfg = "golden_gqa_long"
    D, W = gqa_weights(cfg)
    Kc, Vc = gqa_long_cache(cfg, T)
    x = synth.normal(synth.seed_of(cfg, "x"), (1, D))
    qg, k, v = ref.matmul(x, W["Wq"]), ref.matmul(x, W["Wk"]), ref.matmul(x, W["Wv"])
    out = ref.attention(x, T - 1, H, KH, HD, W["Wq"], W["Wk"], W["Wv"], W["Wo"], W["qn"], W["kn"],
                        Kc, Vc)
    np.savez_compressed(os.path.join(HERE, "gqa_long.npz"), qg=qg.reshape(1, H, 2 * HD),
                        k=k.reshape(1, KH, HD), v=v.reshape(1, KH, HD),
                        ctx=out.reshape(1, H, HD), qn=W["qn"], kn=W["kn"], T=np.int32(T),
                        k_row=Kc[:, T - 1].copy(), v_row=Vc[:, T - 1].copy())


def gdn_init_state(cfg):
    state = synth.normal(synth.seed_of(cfg, "state0"), (GVH, KD, VD), std=0.1)
    CD = 2 * GKH * KD + GVH * VD
    ring = synth.normal(synth.seed_of(cfg, "ring0"), (CONVK, CD), std=1.0)
    return state, ring


def make_gdn_seq(ref, S=6):
    cfg = "golden_gdn_seq"
    D = GVH * VD
    CD = 2 * GKH * KD + GVH * VD
    Wqkv = synth.normal(synth.seed_of(cfg, "Wqkv"), (CD, D), std=0.02)
    Wz = synth.normal(synth.seed_of(cfg, "Wz"), (GVH * VD, D), std=0.02)
    Wa = synth.normal(synth.seed_of(cfg, "Wa"), (GVH, D), std=0.02)
    Wb = synth.normal(synth.seed_of(cfg, "Wb"), (GVH, D), std=0.02)
    conv = synth.normal(synth.seed_of(cfg, "conv"), (CD, CONVK), std=0.3)
    A_log = synth.uniform(synth.seed_of(cfg, "A_log"), (GVH,), 0.0, float(np.log(16.0)))
    dt_bias = synth.normal(synth.seed_of(cfg, "dt_bias"), (GVH,))
    gnorm = synth.normal(synth.seed_of(cfg, "gnorm"), (VD,), std=0.1, mean=1.0)
    Wout = np.eye(D, dtype=np.float32)
    x = synth.normal(synth.seed_of(cfg, "x"), (S, D))
    state, ring = gdn_init_state(cfg)
    out = ref.gdn_steps(x, GKH, KD, GVH, VD, CONVK, Wqkv, Wz, Wa, Wb, conv, A_log, dt_bias, gnorm,
                        Wout, state, ring)
    qkv, z = ref.matmul(x, Wqkv), ref.matmul(x, Wz)
    a, b = ref.matmul(x, Wa), ref.matmul(x, Wb)
    flat = state.reshape(-1).astype(np.float64)
    np.savez_compressed(
        os.path.join(HERE, "gdn_seq.npz"), qkv=qkv, z=z, a=a, b=b, conv=conv, A_log=A_log,
        dt_bias=dt_bias, gnorm=gnorm, y=out, ring_final=ring[1:].copy(),
        state_sum=np.float64(flat.sum()), state_sumsq=np.float64((flat * flat).sum()),
        state_sample=state.reshape(-1)[::97].copy())


def main():
    ref = Reference()
    make_gqa_seq(ref)
    make_gqa_long(ref)
    make_gdn_seq(ref)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
