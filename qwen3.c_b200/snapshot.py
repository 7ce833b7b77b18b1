"""Snapshot (safetensors container) loading for the token-mixer layers,
through the C ABI's reader (coli_cuda_st_*): the mixer part of the
reference's model_init (c/qwen.c:433-485) and load_cfg (c/qwen.c:344-400).

A loaded layer leaves its weights resident on the device: dense projections
as bf16 tensors, q/k norm weights, conv taps, A_log / dt_bias / gnorm and the
in/post layer norms in the backend's per-layer slots. The tiny GDN a/b
projections stay on the host, where the engine computes them (c/qwen.c:677-686).
"""
import ctypes
import json
import os

import numpy as np

from . import coli_cuda


class Snapshot:
    def __init__(self, lib, snap_dir):
        self.lib = lib
        self.dir = snap_dir
        self.h = lib.coli_cuda_st_open(snap_dir.encode())
        if self.h < 0:
            raise coli_cuda.BackendError(lib.coli_cuda_last_error().decode())
        with open(os.path.join(snap_dir, "config.json")) as f:
            self.cfg = json.load(f)

    # ---- config (load_cfg)
    def layer_is_full(self, i):
        lt = self.cfg.get("layer_types")
        if lt is not None:
            return lt[i] == "full_attention"
        return (i + 1) % 4 == 0

    # ---- tensors
    def info(self, name):
        shape = (ctypes.c_longlong * 8)()
        nd, dt = ctypes.c_int(), ctypes.c_int()
        if not self.lib.coli_cuda_st_info(self.h, name.encode(), shape, ctypes.byref(nd), ctypes.byref(dt)):
            return None
        return tuple(shape[i] for i in range(nd.value)), dt.value

    def read(self, name):
        inf = self.info(name)
        if inf is None:
            raise KeyError(name)
        shape = inf[0]
        out = np.zeros(int(np.prod(shape)) if shape else 1, np.float32)
        n = self.lib.coli_cuda_st_read_f32(self.h, name.encode(), out.ctypes.data_as(coli_cuda._fp), out.size)
        if n < 0:
            raise coli_cuda.BackendError(self.lib.coli_cuda_last_error().decode())
        return out.reshape(shape)

    def dense(self, be, name):
        t = coli_cuda.DenseTensor.__new__(coli_cuda.DenseTensor)
        t.be = be
        t.h = ctypes.c_void_p()
        be._ok(self.lib.coli_cuda_st_dense(self.h, name.encode(), ctypes.byref(t.h)), "st_dense " + name)
        t.O, t.I = self.info(name)[0]
        return t

    def close(self):
        if self.h >= 0:
            self.lib.coli_cuda_st_close(self.h)
            self.h = -1


def load_mixer_layer(be, snap, i, slot, batch=1, max_t=4096):
    """Model layer i's mixer onto the device. slot is the KV layer (full
    attention) or GDN layer index of the backend; the in/post layer norms go
    to norm slot i. Returns the dense tensors (and, for GDN, the host a/b
    projections and the gate parameters the caller packs per token)."""
    c = snap.cfg
    p = f"model.layers.{i}."
    be.layer_norm_weight(i, snap.read(p + "input_layernorm.weight"), snap.read(p + "post_attention_layernorm.weight"))
    if snap.layer_is_full(i):
        be.kv_ensure(slot, batch, c["num_key_value_heads"], max_t, c["head_dim"])
        be.gqa_norm_weight(slot, snap.read(p + "self_attn.q_norm.weight"), snap.read(p + "self_attn.k_norm.weight"))
        return {"kind": "gqa", **{k: snap.dense(be, p + f"self_attn.{k}_proj.weight") for k in "qkvo"}}
    kh, kd = c["linear_num_key_heads"], c["linear_key_head_dim"]
    vh, vd, ck = c["linear_num_value_heads"], c["linear_value_head_dim"], c["linear_conv_kernel_dim"]
    cd = 2 * kh * kd + vh * vd
    conv = snap.read(p + "linear_attn.conv1d.weight").reshape(cd, ck)
    A_log, dt_bias = snap.read(p + "linear_attn.A_log"), snap.read(p + "linear_attn.dt_bias")
    gnorm = snap.read(p + "linear_attn.norm.weight")
    be.gdn_setup(slot, batch, conv, A_log, dt_bias, gnorm, KH=kh, KD=kd, VH=vh, VD=vd, conv_k=ck)
    return {"kind": "gdn",
            "qkv": snap.dense(be, p + "linear_attn.in_proj_qkv.weight"),
            "z": snap.dense(be, p + "linear_attn.in_proj_z.weight"),
            "out": snap.dense(be, p + "linear_attn.out_proj.weight"),
            "Wa": snap.read(p + "linear_attn.in_proj_a.weight"), "Wb": snap.read(p + "linear_attn.in_proj_b.weight"),
            "A_log": A_log, "dt_bias": dt_bias, "gnorm": gnorm}


def gdn_params(layer, x_in):
    """[decay | beta | gnorm] per token from the host a/b projections, as the
    engine packs them (c/qwen.c:677-686)."""
    x_in = np.atleast_2d(np.asarray(x_in, np.float32))
    a, b = x_in @ layer["Wa"].T, x_in @ layer["Wb"].T
    z = a + layer["dt_bias"]
    sp = np.where(z > 20, z, np.log1p(np.exp(np.minimum(z, 20))))
    decay = np.exp(-np.exp(layer["A_log"]) * sp).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-b))).astype(np.float32)
    return np.concatenate([decay, beta, np.broadcast_to(layer["gnorm"], (x_in.shape[0], layer["gnorm"].size))],
                          axis=1).astype(np.float32)
