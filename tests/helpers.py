"""Shared helpers for the GPU parity tests (tolerances from the north star:
layer outputs max-abs <= 2e-2 and cosine >= 0.9999 against the fp32 CPU
oracle; GDN state after 4096 steps relative-L2 <= 1e-3)."""
import numpy as np

import synth

MAX_ABS = 2e-2
MIN_COS = 0.9999
STATE_REL_L2 = 1e-3

KH_G, KD, VH_G, VD, CONVK = 16, 128, 32, 128, 4
CD = 2 * KH_G * KD + VH_G * VD
H, KH, HD = 16, 2, 256


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-300))


def assert_close(got, want, max_abs=MAX_ABS, min_cos=MIN_COS, what=""):
    err = float(np.max(np.abs(np.asarray(got, np.float64) - np.asarray(want, np.float64))))
    cos = cosine(got, want)
    assert err <= max_abs and cos >= min_cos, f"{what}: max-abs {err:.3e} cosine {cos:.8f}"
    return err, cos


def gdn_params(cfg):
    """Per-layer GDN parameters with the benchmark distributions."""
    return dict(
        conv_w=synth.normal(synth.seed_of(cfg, "conv"), (CD, CONVK), std=0.3),
        A_log=synth.uniform(synth.seed_of(cfg, "A_log"), (VH_G,), 0.0, float(np.log(16.0))),
        dt_bias=synth.normal(synth.seed_of(cfg, "dt_bias"), (VH_G,)),
        gnorm=synth.normal(synth.seed_of(cfg, "gnorm"), (VD,), std=0.1, mean=1.0),
    )


def gdn_inputs(cfg, S, req=0, bf16=False):
    """Post-projection GDN inputs for S tokens: qkv/z ~ N(0,1), a/b ~ N(0,1)."""
    f = synth.bf16_round if bf16 else (lambda x: x)
    return dict(
        qkv=f(synth.normal(synth.seed_of(cfg, "qkv", req), (S, CD))),
        z=f(synth.normal(synth.seed_of(cfg, "z", req), (S, VH_G * VD))),
        a=f(synth.normal(synth.seed_of(cfg, "a", req), (S, VH_G))),
        b=f(synth.normal(synth.seed_of(cfg, "b", req), (S, VH_G))),
    )


def gdn_state0(cfg, req=0):
    state = synth.normal(synth.seed_of(cfg, "state0", req), (VH_G, KD, VD), std=0.1)
    ring = synth.normal(synth.seed_of(cfg, "ring0", req), (CONVK, CD))
    ring[0] = 0.0  # dead slot: overwritten before any use
    return state, ring


def record(what, value):
    """Append a measured error to the file named by COLI_PARITY_LOG (if set),
    one JSON object per line, so a GPU run leaves the actual margins behind."""
    import json
    import os
    path = os.environ.get("COLI_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({what: value}) + "\n")

