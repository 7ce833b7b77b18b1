"""Writes BASELINE config 1's random container for the engine-level tests: a
4-layer Qwen3.5-MoE-shaped snapshot (layers 0-2 GatedDeltaNet, layer 3 gated
GQA; hidden 2048, vocab 248320, 8 routed experts top-2 of width 512 plus a
shared expert, RMSNorm eps 1e-6) in the layout the reference engine loads
(config.json keys of c/qwen.c:344-401, tensor names of c/qwen.c:433-475,
int8 experts with per-row ".qs" scales as c/qwen.c:509-536 reads them), and
the oracle-mode ref.json (prompt_ids / full_ids, c/qwen.c:2093-2137).

Weight matrices are N(0, 0.02) fp32. The small per-layer vectors take the
values a freshly initialised model has, so the mixers are not degenerate:
zero-centred RMSNorm weights 0 (scale 1 + w), GDN gated-norm weight 1,
A_log = log U(1, 16), dt_bias 1, conv taps N(0, 0.3). Seeded; no public data.

With int8_dense=True every matrix the engine quantises for a device
(vk_dense_init, c/qwen.c:1829-1850: the mixer projections, the shared expert,
router, GDN a/b and the tied lm_head) is stored already round-tripped through
the engine's per-row int8 (quant_rows fmt 1, c/qwen.c:266-275). The engine's
own quantisation then reproduces the same int8 rows, so its CPU run and its
device run compute with the same weights.
"""
import json
import os
import struct

import numpy as np

CFG = dict(hidden_size=2048, num_hidden_layers=4, vocab_size=248320, num_attention_heads=16,
           num_key_value_heads=2, head_dim=256, partial_rotary_factor=0.25, rope_theta=1e7,
           rms_norm_eps=1e-6, linear_num_key_heads=16, linear_key_head_dim=128,
           linear_num_value_heads=32, linear_value_head_dim=128, linear_conv_kernel_dim=4,
           num_experts=8, num_experts_per_tok=2, moe_intermediate_size=512,
           shared_expert_intermediate_size=512, expert_bits=8,
           layer_types=["linear_attention"] * 3 + ["full_attention"])


def _tensors(c):
    """(name, dtype, shape, kind) in file order; kind picks the generator."""
    D, V = c["hidden_size"], c["vocab_size"]
    H, KH, hd = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
    gkh, gkd, gvh, gvd = (c["linear_num_key_heads"], c["linear_key_head_dim"],
                          c["linear_num_value_heads"], c["linear_value_head_dim"])
    CD = 2 * gkh * gkd + gvh * gvd
    E, I, SI = c["num_experts"], c["moe_intermediate_size"], c["shared_expert_intermediate_size"]
    out = [("model.embed_tokens.weight", "F32", (V, D), "w"), ("model.norm.weight", "F32", (D,), "zero")]
    for i, lt in enumerate(c["layer_types"]):
        p = f"model.layers.{i}."
        out += [(p + "input_layernorm.weight", "F32", (D,), "zero"),
                (p + "post_attention_layernorm.weight", "F32", (D,), "zero")]
        if lt == "full_attention":
            out += [(p + "self_attn.q_proj.weight", "F32", (H * 2 * hd, D), "w"),
                    (p + "self_attn.k_proj.weight", "F32", (KH * hd, D), "w"),
                    (p + "self_attn.v_proj.weight", "F32", (KH * hd, D), "w"),
                    (p + "self_attn.o_proj.weight", "F32", (D, H * hd), "w"),
                    (p + "self_attn.q_norm.weight", "F32", (hd,), "zero"),
                    (p + "self_attn.k_norm.weight", "F32", (hd,), "zero")]
        else:
            out += [(p + "linear_attn.in_proj_qkv.weight", "F32", (CD, D), "w"),
                    (p + "linear_attn.in_proj_z.weight", "F32", (gvh * gvd, D), "w"),
                    (p + "linear_attn.in_proj_b.weight", "F32", (gvh, D), "w"),
                    (p + "linear_attn.in_proj_a.weight", "F32", (gvh, D), "w"),
                    (p + "linear_attn.conv1d.weight", "F32", (CD, c["linear_conv_kernel_dim"]), "conv"),
                    (p + "linear_attn.dt_bias", "F32", (gvh,), "one"),
                    (p + "linear_attn.A_log", "F32", (gvh,), "alog"),
                    (p + "linear_attn.norm.weight", "F32", (gvd,), "one"),
                    (p + "linear_attn.out_proj.weight", "F32", (D, gvh * gvd), "w")]
        out += [(p + "mlp.gate.weight", "F32", (E, D), "w"),
                (p + "mlp.shared_expert.gate_proj.weight", "F32", (SI, D), "w"),
                (p + "mlp.shared_expert.up_proj.weight", "F32", (SI, D), "w"),
                (p + "mlp.shared_expert.down_proj.weight", "F32", (D, SI), "w"),
                (p + "mlp.shared_expert_gate.weight", "F32", (1, D), "w")]
        for e in range(E):
            for pj, shp in (("gate_proj", (I, D)), ("up_proj", (I, D)), ("down_proj", (D, I))):
                n = f"{p}mlp.experts.{e}.{pj}.weight"
                out += [(n, "I8", shp, "q8"), (n + ".qs", "F32", (shp[0],), "q8s")]
    return out


def _q8_roundtrip(w):
    amax = np.abs(w).max(axis=1, keepdims=True)
    sc = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(w / sc), -127, 127)
    return (q * sc).astype(np.float32)


def _gen(rng, kind, shape, cache):
    if kind in ("w", "wq"):
        w = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
        return _q8_roundtrip(w) if kind == "wq" else w
    if kind == "zero":
        return np.zeros(shape, np.float32)
    if kind == "one":
        return np.ones(shape, np.float32)
    if kind == "conv":
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.3))
    if kind == "alog":
        return np.log(rng.uniform(1.0, 16.0, shape)).astype(np.float32)
    if kind == "q8":   # per-row symmetric int8 of an N(0, 0.02) matrix; the scales follow
        w = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
        s = np.maximum(np.abs(w).max(axis=1), 1e-12) / 127.0
        cache["qs"] = s.astype(np.float32)
        return np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    if kind == "q8s":
        return cache.pop("qs")
    raise ValueError(kind)


def write(snap_dir, seed=1, n_prompt=128, n_new=32, int8_dense=False):
    """Write config.json, model.safetensors and ref.json into snap_dir."""
    os.makedirs(snap_dir, exist_ok=True)
    with open(os.path.join(snap_dir, "config.json"), "w") as f:
        json.dump(CFG, f)
    items = _tensors(CFG)
    if int8_dense:
        items = [(n, dt, shp, "wq" if k == "w" and not n.endswith("shared_expert_gate.weight") else k)
                 for n, dt, shp, k in items]
    esize = {"F32": 4, "I8": 1}
    header, off = {}, 0
    for name, dt, shape, _ in items:
        nb = int(np.prod(shape)) * esize[dt]
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + nb]}
        off += nb
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    rng = np.random.default_rng(seed)
    cache = {}
    with open(os.path.join(snap_dir, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for name, dt, shape, kind in items:
            if kind in ("w", "wq") and shape[0] > 4096:   # the embedding: in row blocks
                for r0 in range(0, shape[0], 16384):
                    rows = min(16384, shape[0] - r0)
                    f.write(_gen(rng, kind, (rows,) + tuple(shape[1:]), cache).tobytes())
            else:
                f.write(np.ascontiguousarray(_gen(rng, kind, shape, cache)).tobytes())
    prompt = rng.integers(0, CFG["vocab_size"], size=n_prompt).tolist()
    with open(os.path.join(snap_dir, "ref.json"), "w") as f:
        # full_ids only sets how many tokens the engine generates (its own
        # continuation is what the tests compare)
        json.dump({"prompt_ids": prompt, "full_ids": prompt + [0] * n_new}, f)
    return os.path.join(snap_dir, "ref.json")


def read_dump(path):
    """Records of the adapter's COLI_VK_DUMP file, in call order."""
    buf = open(path, "rb").read()
    i, out = 0, []

    def ints(n):
        nonlocal i
        v = struct.unpack_from(f"<{n}i", buf, i)
        i += 4 * n
        return v

    def flt(n):
        nonlocal i
        a = np.frombuffer(buf, np.float32, n, i).copy()
        i += 4 * n
        return a
    while i < len(buf):
        kind = ints(1)[0]
        if kind == 1:
            layer, row, hd = ints(3)
            out.append(("kv", layer, row, flt(hd), flt(hd)))
        elif kind == 2:
            layer, S, H, KH, hd, max_t, T = ints(7)
            scale = flt(1)[0]
            q = flt(S * H * 2 * hd).reshape(S, H, 2 * hd)
            ctx = flt(S * H * hd).reshape(S, H, hd)
            out.append(("gqa", layer, dict(S=S, H=H, KH=KH, hd=hd, max_t=max_t, T=T, scale=scale, q=q, ctx=ctx)))
        elif kind == 3:
            layer, KH, KD, VH, VD = ints(5)
            eps = flt(1)[0]
            rec = dict(KH=KH, KD=KD, VH=VH, VD=VD, eps=eps, qn=flt(KH * KD), kn=flt(KH * KD),
                       v=flt(VH * VD), z=flt(VH * VD), decay=flt(VH), beta=flt(VH), gnorm=flt(VD),
                       y=flt(VH * VD))
            out.append(("gdn", layer, rec))
        elif kind == 4:
            layer, S, D, H, KH, hd, rot, pos_base, max_t, Dout = ints(10)
            eps, theta = flt(2)
            out.append(("gqa_full", layer, dict(S=S, D=D, H=H, KH=KH, hd=hd, rot=rot, pos_base=pos_base,
                                                max_t=max_t, eps=eps, theta=theta, x=flt(S * D).reshape(S, D),
                                                out=flt(S * Dout).reshape(S, Dout))))
        elif kind == 5:
            layer, S, D, H, KH, hd, rot, pos_base, max_t, ln_layer, E = ints(11)
            eps, theta = flt(2)
            out.append(("gqa_full_route", layer, dict(
                S=S, D=D, H=H, KH=KH, hd=hd, rot=rot, pos_base=pos_base, max_t=max_t, ln_layer=ln_layer, E=E,
                eps=eps, theta=theta, resid=flt(S * D).reshape(S, D), resid_out=flt(S * D).reshape(S, D),
                nrm_out=flt(S * D).reshape(S, D), pr_out=flt(S * E).reshape(S, E))))
        elif kind == 6:
            layer, S, D, VH, VD, Dout = ints(6)
            eps = flt(1)[0]
            out.append(("gdn_full", layer, dict(S=S, D=D, VH=VH, VD=VD, eps=eps, x=flt(S * D).reshape(S, D),
                                                params=flt(S * (2 * VH + VD)).reshape(S, 2 * VH + VD),
                                                out=flt(S * Dout).reshape(S, Dout))))
        elif kind == 7:
            layer, D, VH, VD, ln_layer, E = ints(6)
            eps = flt(1)[0]
            out.append(("gdn_full_route", layer, dict(
                D=D, VH=VH, VD=VD, ln_layer=ln_layer, E=E, eps=eps, x=flt(D)[None], params=flt(2 * VH + VD)[None],
                resid=flt(D)[None], resid_out=flt(D)[None], nrm_out=flt(D)[None], pr_out=flt(E)[None])))
        else:
            raise ValueError(f"bad dump record {kind} at {i}")
    return out


def open_tensors(snap_dir):
    """name -> numpy view (memory-mapped) of model.safetensors."""
    path = os.path.join(snap_dir, "model.safetensors")
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    dt = {"F32": np.float32, "I8": np.int8}
    out = {}
    for name, t in header.items():
        if name == "__metadata__":
            continue
        a, b = t["data_offsets"]
        out[name] = mm[8 + n + a:8 + n + b].view(dt[t["dtype"]]).reshape(t["shape"])
    return out
