"""The reference engine itself on the B200 backend.

The unmodified c/qwen.c is built twice (oracle/Makefile, qwen3.c_b200/engine/
Makefile): once as it ships, whose CPU path (`--no-vulkan`) is the oracle, and
once with -DCOLI_VULKAN linked against libcoli_vk_cuda.so, the engine's Vulkan
ABI served by this backend. Both run the random 4-layer container on the same
128-token prompt and greedily generate 32 tokens (oracle mode, c/qwen.c:
2093-2137), dumping every step's logits.

* Staged mode (`--no-dense`): the projections stay on the engine's fp32 CPU
  path and only the token mixers run on the GPU (coli_vk_kv_row + coli_vk_gqa
  at c/qwen.c:611-634, coli_vk_gdn at c/qwen.c:732-746). The adapter dumps
  every mixer call with its inputs and outputs, and each call is replayed
  through the CPU oracle along the engine's own layer loop (c/qwen.c:
  1297-1387): GQA ctx against the attention core over the fp32 rows the engine
  mirrored, GDN y against the recurrence with the oracle's own state chained
  over all 160 steps of each layer. Tolerance: max-abs 2e-2, cosine 0.9999.
  The generated ids must equal the CPU engine's, and the logits agree at
  every step.
* Block mode (the engine's default with a device: dense projections
  quantised to int8 rows by the engine, c/qwen.c:1810-1872, and uploaded as
  bf16; whole-block calls coli_vk_gqa_full(_route) / coli_vk_gdn_full_seq /
  coli_vk_gdn_full_route, projections on the tcgen05 linear kernel). It runs
  a second container whose matrices are stored already int8-round-tripped,
  so the CPU run computes with the very weights the device holds; the
  device keeps activations between the steps in bf16. Every block call is
  dumped and replayed through the oracle mixers with the oracle's own KV
  cache / GDN state chained over the run, between projections that take the
  device's bf16-rounded operands with fp32 accumulation (the a / b gate
  projections stay fp32 on the host, as the engine computes them), and must
  agree within max-abs 2e-2 / cosine 0.9999,
  residual / post-norm / router outputs of the route tail included. The
  generated ids are recorded, not asserted: the top-2 expert choice and the
  greedy argmax are discontinuous, so a bf16-level difference in a block
  output can move a near-tied routing decision and the continuation.
"""
import os
import re
import subprocess

import numpy as np
import pytest

import engine_container as ec
from helpers import MAX_ABS, MIN_COS, cosine, record
import synth
from oracle import Oracle

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CPU_ENGINE = os.path.join(ROOT, "oracle", "_ref", "qwen")
GPU_ENGINE = os.path.join(ROOT, "qwen3.c_b200", "engine", "_build", "qwen_vk_cuda")
VOCAB = ec.CFG["vocab_size"]


def _run(exe, snap, args, logits, env_extra=None):
    env = dict(os.environ)
    env.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 8))
    env.update(env_extra or {})
    cmd = [exe, "--snap", snap, "--experts", "0", "--logits", logits] + args + [os.path.join(snap, "ref.json")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    m = re.search(r"C engine : ([0-9 ]+)", r.stdout)
    assert m, r.stdout[-2000:]
    ids = [int(t) for t in m.group(1).split()]
    lg = np.fromfile(logits, np.float32).reshape(-1, VOCAB)
    rate = re.search(r"Prefill: ([0-9.]+)s .*decode: \d+ tok in [0-9.]+s \(([0-9.]+) tok/s\)", r.stdout)
    if rate:
        record(f"engine {os.path.basename(exe)} {' '.join(args) or 'default'}",
               {"prefill_s_128": float(rate.group(1)), "decode_tok_s": float(rate.group(2))})
    return ids, lg, r.stdout


@pytest.fixture(scope="module")
def container(tmp_path_factory):
    if not (os.path.exists(CPU_ENGINE) and os.path.exists(GPU_ENGINE)):
        pytest.fail("engine binaries missing: build() with the reference sources present builds "
                    "oracle/_ref/qwen and qwen3.c_b200/engine/_build/qwen_vk_cuda")
    d = str(tmp_path_factory.mktemp("config1"))
    ec.write(d)
    ids, lg, _ = _run(CPU_ENGINE, d, ["--no-vulkan"], os.path.join(d, "cpu_logits.bin"))
    return d, ids, lg


def test_engine_staged_mixers_on_gpu(container):
    snap, cpu_ids, cpu_lg = container
    dump = os.path.join(snap, "mixers.bin")
    ids, lg, out = _run(GPU_ENGINE, snap, ["--no-dense"], os.path.join(snap, "gpu_logits.bin"),
                        {"COLI_VK_DUMP": dump})
    assert "GatedDeltaNet recurrence ENABLED" in out and "device KV mirror" in out, out[-3000:]
    # per-call parity along the engine's own loop
    orc = Oracle()
    recs = ec.read_dump(dump)
    caches, states = {}, {}
    n_gqa = n_gdn = 0
    worst = {"gqa": (0.0, 1.0), "gdn": (0.0, 1.0)}
    for r in recs:
        if r[0] == "kv":
            _, layer, row, k, v = r
            caches.setdefault(layer, {})[row] = (k, v)
        elif r[0] == "gqa":
            _, layer, c = r
            KH, max_t, hd = c["KH"], c["max_t"], c["hd"]
            Kc = np.zeros((KH, max_t, hd), np.float32)
            Vc = np.zeros_like(Kc)
            for row, (k, v) in caches.get(layer, {}).items():
                Kc[row // max_t, row % max_t] = k
                Vc[row // max_t, row % max_t] = v
            want = orc.gqa_attend(c["q"], Kc, Vc, c["T"] - c["S"], scale=c["scale"])
            err = float(np.max(np.abs(c["ctx"] - want)))
            cos = cosine(c["ctx"], want)
            worst["gqa"] = (max(worst["gqa"][0], err), min(worst["gqa"][1], cos))
            assert err <= MAX_ABS and cos >= MIN_COS, (layer, c["S"], c["T"], err, cos)
            n_gqa += 1
        else:
            _, layer, c = r
            st = states.setdefault(layer, np.zeros((c["VH"], c["KD"], c["VD"]), np.float32))
            want = orc.gdn_recur(c["qn"], c["kn"], c["v"], c["z"], c["decay"], c["beta"], c["gnorm"], st,
                                 KH=c["KH"], eps=float(c["eps"]))
            err = float(np.max(np.abs(c["y"] - want)))
            cos = cosine(c["y"], want)
            worst["gdn"] = (max(worst["gdn"][0], err), min(worst["gdn"][1], cos))
            assert err <= MAX_ABS and cos >= MIN_COS, (layer, n_gdn, err, cos)
            n_gdn += 1
    # 1 GQA layer: one 128-row prefill call + 31 decode calls; 3 GDN layers x 159 tokens
    assert n_gqa == 32 and n_gdn == 3 * 159, (n_gqa, n_gdn)
    match = sum(a == b for a, b in zip(ids, cpu_ids))
    lcos = [cosine(lg[i], cpu_lg[i]) for i in range(min(len(lg), len(cpu_lg)))]
    lerr = float(np.max(np.abs(lg[0] - cpu_lg[0])))
    record("engine staged", {"gqa_worst": worst["gqa"], "gdn_worst": worst["gdn"], "ids_matching": match,
                             "prefill_logits_max_abs": lerr, "min_step_logit_cos": min(lcos)})
    assert ids == cpu_ids, (match, ids, cpu_ids)
    assert lerr <= MAX_ABS and min(lcos) >= MIN_COS, (lerr, min(lcos))


def _rms_zc(x, w, eps):
    """rmsnorm_zc (c/qwen.c:326-330): mean square in double, scale 1 + w."""
    x = np.asarray(x, np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    return (x * (1.0 / np.sqrt((ms + eps).astype(np.float32))) * (1.0 + w)).astype(np.float32)


def bf(a):
    return synth.bf16_round(np.ascontiguousarray(a, np.float32))


def _check(what, got, want, worst):
    err = float(np.max(np.abs(np.asarray(got, np.float64) - want)))
    cos = cosine(got, want)
    w = worst.get(what, (0.0, 1.0))
    worst[what] = (max(w[0], err), min(w[1], cos))
    assert err <= MAX_ABS and cos >= MIN_COS, (what, err, cos)


def test_engine_whole_blocks_on_gpu(tmp_path_factory):
    if not (os.path.exists(CPU_ENGINE) and os.path.exists(GPU_ENGINE)):
        pytest.fail("engine binaries missing")
    snap = str(tmp_path_factory.mktemp("config1_q8"))
    ec.write(snap, int8_dense=True)
    cpu_ids, cpu_lg, _ = _run(CPU_ENGINE, snap, ["--no-vulkan"], os.path.join(snap, "cpu_logits.bin"))
    dump = os.path.join(snap, "blocks.bin")
    ids, lg, out = _run(GPU_ENGINE, snap, [], os.path.join(snap, "gpu_block_logits.bin"), {"COLI_VK_DUMP": dump})
    assert "dense offload" in out and "block fusion ENABLED" in out, out[-3000:]
    # replay every block call of the engine's loop through fp32 projections
    # around the oracle mixers, with the container's weights
    W = ec.open_tensors(snap)
    c = ec.CFG
    full = [i for i, t in enumerate(c["layer_types"]) if t == "full_attention"]
    lin = [i for i, t in enumerate(c["layer_types"]) if t != "full_attention"]
    orc = Oracle()
    eps = c["rms_norm_eps"]
    H, KH, hd = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
    rot = int(hd * c["partial_rotary_factor"])
    kv, gstate = {}, {}
    worst, kinds = {}, {}

    def w(li, name):
        return np.asarray(W[f"model.layers.{li}.{name}"], np.float32)

    def gqa_block(kvi, x, pos_base, max_t):
        li = full[kvi]
        S = x.shape[0]
        xb = bf(x)
        qg = bf(xb @ bf(w(li, "self_attn.q_proj.weight")).T).reshape(S, H, 2 * hd)
        k = bf(xb @ bf(w(li, "self_attn.k_proj.weight")).T).reshape(S, KH, hd)
        v = bf(xb @ bf(w(li, "self_attn.v_proj.weight")).T).reshape(S, KH, hd)
        Kc, Vc = kv.setdefault(kvi, (np.zeros((KH, max_t, hd), np.float32), np.zeros((KH, max_t, hd), np.float32)))
        orc.gqa_prologue(qg, k, v, w(li, "self_attn.q_norm.weight"), w(li, "self_attn.k_norm.weight"), pos_base,
                         Kc, Vc, rot=rot, theta=c["rope_theta"], eps=eps)
        ctx = orc.gqa_attend(qg, Kc, Vc, pos_base)
        return bf(ctx.reshape(S, H * hd)) @ bf(w(li, "self_attn.o_proj.weight")).T

    def gdn_block(gi, x):
        li = lin[gi]
        kd, vh, vd = c["linear_key_head_dim"], c["linear_num_value_heads"], c["linear_value_head_dim"]
        cd = 2 * c["linear_num_key_heads"] * kd + vh * vd
        st = gstate.setdefault(gi, (np.zeros((vh, kd, vd), np.float32), np.zeros((4, cd), np.float32)))
        f = lambda n: np.ascontiguousarray(bf(x) @ bf(w(li, n)).T, np.float32)   # noqa: E731
        ab = lambda n: np.ascontiguousarray(x @ w(li, n).T, np.float32)   # noqa: E731
        y = orc.gdn_seq(f("linear_attn.in_proj_qkv.weight"), f("linear_attn.in_proj_z.weight"),
                        ab("linear_attn.in_proj_a.weight"), ab("linear_attn.in_proj_b.weight"),
                        w(li, "linear_attn.conv1d.weight"), w(li, "linear_attn.A_log"),
                        w(li, "linear_attn.dt_bias"), w(li, "linear_attn.norm.weight"), st[1], st[0],
                        KH=c["linear_num_key_heads"], KD=kd, eps=eps)
        return bf(y.reshape(x.shape[0], -1)) @ bf(w(li, "linear_attn.out_proj.weight")).T

    def tail(li, resid, delta, r):
        # each step of the route tail against its own device inputs: the
        # residual add against the oracle block, the post-norm of the device's
        # residual, the router over the device's normed rows
        _check("resid_out", r["resid_out"], resid + delta, worst)
        nrm = _rms_zc(r["resid_out"], w(li, "post_attention_layernorm.weight"), eps)
        _check("nrm_out", r["nrm_out"], nrm, worst)
        _check("router logits", r["pr_out"], r["nrm_out"] @ w(li, "mlp.gate.weight").T, worst)

    for rec in ec.read_dump(dump):
        kind, layer, r = rec[0], rec[1], rec[2] if len(rec) > 2 else None
        kinds[kind] = kinds.get(kind, 0) + 1
        if kind == "gqa_full":
            _check("gqa block", r["out"], gqa_block(layer, r["x"], r["pos_base"], r["max_t"]), worst)
        elif kind == "gqa_full_route":
            li = r["ln_layer"]
            x = _rms_zc(r["resid"], w(li, "input_layernorm.weight"), eps)
            delta = gqa_block(layer, x, r["pos_base"], r["max_t"])
            _check("gqa block (route)", r["resid_out"] - r["resid"], delta, worst)
            tail(li, r["resid"], delta, r)
        elif kind == "gdn_full":
            _check("gdn block", r["out"], gdn_block(layer, r["x"]), worst)
        elif kind == "gdn_full_route":
            delta = gdn_block(layer, r["x"])
            _check("gdn block (route)", r["resid_out"] - r["resid"], delta, worst)
            tail(r["ln_layer"], r["resid"], delta, r)
    match = sum(a == b for a, b in zip(ids, cpu_ids))
    c0 = cosine(lg[0], cpu_lg[0])
    record("engine blocks (int8-exact dense)", {"calls": kinds, "worst": worst, "ids_matching": match,
                                                "prefill_logit_cos": c0})
    # every layer ran as a device block: prefill (1 call per layer) + 31 decode steps
    assert kinds.get("gqa_full_route", 0) + kinds.get("gqa_full", 0) == 32, kinds
    assert kinds.get("gdn_full", 0) + kinds.get("gdn_full_route", 0) == 3 * 32, kinds
    assert len(ids) == len(cpu_ids)
