"""Host-side pieces of the engine integration (no GPU): the Vulkan-ABI
adapter library exports the whole interface the engine links against, the
config-1 container's int8 round trip is exact under the engine's own
quantisation, and the adapter's dump records read back."""
import ctypes
import os
import struct

import numpy as np

import engine_container as ec

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ADAPTER = os.path.join(ROOT, "qwen3.c_b200", "lib", "libcoli_vk_cuda.so")

# Every function c/backend_vulkan.h declares (the interface c/qwen.c is built
# against with -DCOLI_VULKAN); names only.
VK_ABI = """alloc_priority attention_absorb attention_absorb_project attn_qprep available decode_prof
eg_gather_available eg_table_init eg_table_set eg_table_set_shared eg_xs_bind expert_group
expert_group_issue expert_group_issue_id expert_group_issue_pipe expert_group_take expert_group_take_pipe
final_norm_weight gate_up gdn gdn_available gdn_ba_weight gdn_conv_ensure gdn_conv_weight gdn_full
gdn_full_available gdn_full_route gdn_full_route_pipe gdn_full_seq gdn_project gdn_reset gdn_state_ensure
gqa gqa_available gqa_full gqa_full_available gqa_full_route gqa_full_route_pipe gqa_norm_weight
gqa_project init kv_ensure kv_reset kv_row layer_norm_weight matmul matmul_argmax matmul_pair mem_budget
mem_info moe_ix_available moe_route_available route_cache_stats shutdown stream_add stream_available
stream_begin stream_copy_resid stream_end stream_ix_hist stream_ix_pending stream_moe_fused
stream_norm_argmax stream_nrm tensor_bytes tensor_ensure tensor_free""".split()


def _adapter():
    if not os.path.exists(ADAPTER):
        import subprocess
        from conftest import load_pkg
        load_pkg().build()
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "qwen3.c_b200", "engine"),
                        os.path.join(ROOT, "qwen3.c_b200", "lib", "libcoli_vk_cuda.so")], check=True)
    return ctypes.CDLL(ADAPTER)


def test_adapter_exports_the_whole_vulkan_abi():
    assert len(VK_ABI) == 67
    lib = _adapter()
    missing = [n for n in VK_ABI if not hasattr(lib, "coli_vk_" + n)]
    assert not missing, missing


def test_adapter_without_device_reports_unavailable():
    """On a host without a GPU the adapter's init fails cleanly, which is
    the engine's signal to run everything on its CPU path."""
    lib = _adapter()
    lib.coli_vk_init.argtypes = [ctypes.c_char_p]
    try:
        import torch
        if torch.cuda.is_available():
            return
    except ImportError:
        pass
    assert lib.coli_vk_init(b"unused.spv") == 0
    assert lib.coli_vk_available() == 0
    assert lib.coli_vk_stream_available() == 0 and lib.coli_vk_eg_gather_available() == 0


def test_int8_round_trip_is_exact_under_the_engines_quantisation():
    """quant_rows fmt 1 (c/qwen.c:266-275) of an already round-tripped row
    gives back the same int8 values and scales."""
    rng = np.random.default_rng(5)
    w = rng.standard_normal((64, 2048), dtype=np.float32) * np.float32(0.02)
    w1 = ec._q8_roundtrip(w)

    def quant(x):
        amax = np.abs(x).max(axis=1, keepdims=True)
        sc = (amax / np.float32(127.0)).astype(np.float32)
        return np.clip(np.rint(x / sc), -127, 127).astype(np.int8), sc
    q1, s1 = quant(w1)
    q0, s0 = quant(w)
    np.testing.assert_array_equal(q1, q0)
    np.testing.assert_allclose(s1, s0, rtol=2e-7)


def test_container_tensor_table():
    names = {n: (dt, shp) for n, dt, shp, _ in ec._tensors(ec.CFG)}
    assert names["model.embed_tokens.weight"] == ("F32", (248320, 2048))
    assert names["model.layers.3.self_attn.q_proj.weight"] == ("F32", (16 * 2 * 256, 2048))
    assert names["model.layers.0.linear_attn.in_proj_qkv.weight"] == ("F32", (8192, 2048))
    assert names["model.layers.0.mlp.experts.7.down_proj.weight"] == ("I8", (2048, 512))
    assert names["model.layers.0.mlp.experts.7.down_proj.weight.qs"] == ("F32", (2048,))
    assert "lm_head.weight" not in names      # tied to the embedding
    assert sum(1 for t in ec.CFG["layer_types"] if t == "full_attention") == 1


def test_dump_records_read_back(tmp_path):
    p = tmp_path / "d.bin"
    rng = np.random.default_rng(1)
    k, v = rng.standard_normal(256, dtype=np.float32), rng.standard_normal(256, dtype=np.float32)
    S, H, KH, hd = 2, 16, 2, 256
    q = rng.standard_normal(S * H * 2 * hd, dtype=np.float32)
    ctx = rng.standard_normal(S * H * hd, dtype=np.float32)
    with open(p, "wb") as f:
        f.write(struct.pack("<4i", 1, 0, 7, 256) + k.tobytes() + v.tobytes())
        f.write(struct.pack("<8i", 2, 0, S, H, KH, hd, 64, 9) + struct.pack("<f", 0.0625) + q.tobytes() + ctx.tobytes())
    recs = ec.read_dump(str(p))
    assert recs[0][0] == "kv" and recs[0][2] == 7
    np.testing.assert_array_equal(recs[0][3], k)
    kind, layer, c = recs[1]
    assert kind == "gqa" and c["S"] == S and c["T"] == 9 and c["scale"] == np.float32(0.0625)
    np.testing.assert_array_equal(c["ctx"].ravel(), ctx)
