"""Failure paths of the backend, made without faulting the GPU
(c/backend_vulkan.c:1115-1126 shape guards, :1800-1802 "not done" returns,
:1836 a lost device makes every later call return 0):

* bad shapes and arguments on the entry points return 0 with a reason and
  leave the backend usable;
* an injected allocation failure (host-side hook) makes the call that
  needed the memory return 0, and the next call succeeds;
* a device-side wait that runs out: the cross-rank barrier on one GPU with a
  peer that never arrives (a flag nothing sets) and a 50 ms limit. The kernel
  gives up, the next synchronising call returns 0 with "timed out", every
  later call returns 0, and coli_cuda_init brings the backend back.
"""
import ctypes

import numpy as np
import pytest

from conftest import load_pkg
from helpers import CD, CONVK, KD, KH_G, VD, VH_G, assert_close, gdn_inputs, gdn_params
from oracle import Oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    pkg = load_pkg()
    pkg.build()
    b = pkg.Backend(0)
    yield b
    b.shutdown()


def _zero(rc, lib, what):
    assert rc == 0, f"{what} accepted"
    msg = lib.coli_cuda_last_error().decode()
    assert msg and msg != "ok", what
    assert lib.coli_cuda_available() == 1, f"{what} killed the backend: {msg}"
    return msg


def test_bad_shapes_rejected(be):
    lib = be.lib
    fp = ctypes.POINTER(ctypes.c_float)
    buf = np.zeros(1 << 16, np.float32)
    p = buf.ctypes.data_as(fp)
    _zero(lib.coli_cuda_kv_ensure(60, 1, 2, 64, 128), lib, "head dim 128")
    _zero(lib.coli_cuda_kv_ensure(200, 1, 2, 64, 256), lib, "layer out of range")
    assert lib.coli_cuda_kv_ensure(60, 2, 2, 64, 256) == 1
    _zero(lib.coli_cuda_gqa(60, p, p, 1, 12, 2, 256, 64, 0, 10, 0.0625), lib, "H != 8 KH")
    _zero(lib.coli_cuda_gqa(60, p, p, 1, 16, 2, 256, 64, 3, 10, 0.0625), lib, "st0 != 0")
    _zero(lib.coli_cuda_gqa(60, p, p, 5, 16, 2, 256, 64, 0, 70, 0.0625), lib, "T beyond max_t")
    _zero(lib.coli_cuda_kv_row(60, 2, 0, p, p), lib, "request beyond the batch")
    _zero(lib.coli_cuda_kv_rows(60, 0, 120, 10, p, p), lib, "rows beyond the cache")
    _zero(lib.coli_cuda_gqa_decode_dev(60, 3, None, None, None, None, None, 16, 2, 256, 64,
                                       ctypes.c_float(1e-6), ctypes.c_float(1e7), 1), lib, "batch beyond the cache")
    _zero(lib.coli_cuda_gdn_state_ensure(61, 0, 32, 128, 128), lib, "GDN batch 0")
    assert lib.coli_cuda_gdn_state_ensure(61, 1, VH_G, KD, VD) == 1
    _zero(lib.coli_cuda_gdn(61, p, p, p, p, p, p, p, p, 16, 128, 30, 128, ctypes.c_float(1e-6)), lib,
          "VH != 2 KH")
    _zero(lib.coli_cuda_gdn_decode(61, 1, p, p, p, p, p, 16, 128, 32, 128, ctypes.c_float(1e-6)), lib,
          "decode without conv history")
    h = ctypes.c_void_p()
    _zero(lib.coli_cuda_tensor_ensure(ctypes.byref(h), buf.ctypes.data, None, 2, 64, 8, 0), lib, "int4 format")
    _zero(lib.coli_cuda_tensor_ensure(ctypes.byref(h), buf.ctypes.data, None, 0, 12, 8, 0), lib,
          "I not a multiple of 8")
    assert lib.coli_cuda_tensor_ensure(ctypes.byref(h), buf.ctypes.data, None, 0, 64, 8, 0) == 1
    _zero(lib.coli_cuda_matmul_dev(h, ctypes.c_void_p(buf.ctypes.data + 4), 1, ctypes.c_void_p(buf.ctypes.data), 0),
          lib, "unaligned x")
    lib.coli_cuda_tensor_free(h)
    _zero(lib.coli_cuda_peer_barrier(None, 2, 0, 1), lib, "null flags")
    assert lib.coli_cuda_sync() == 1


def test_injected_allocation_failure(be):
    lib = be.lib
    lib.coli_cuda_debug_fail_alloc(0)
    msg = _zero(lib.coli_cuda_kv_ensure(62, 1, 2, 4096, 256), lib, "allocation")
    assert "refused" in msg
    assert lib.coli_cuda_kv_ensure(62, 1, 2, 4096, 256) == 1    # the hook fires once
    lib.coli_cuda_debug_fail_alloc(1)                             # K succeeds, V is refused
    _zero(lib.coli_cuda_kv_ensure(63, 1, 2, 4096, 256), lib, "second allocation")
    lib.coli_cuda_debug_fail_alloc(-1)
    assert lib.coli_cuda_kv_ensure(63, 1, 2, 4096, 256) == 1
    assert lib.coli_cuda_sync() == 1


def test_device_wait_times_out_then_reinit(be):
    lib = be.lib
    assert lib.coli_cuda_set_wait_limit(50_000_000) == 1          # 50 ms
    mine, _ = be.ipc_alloc(64)
    peer, _ = be.ipc_alloc(64)      # stands for rank 1's flag array; nothing ever writes rank 1's slot
    try:
        assert lib.coli_cuda_peer_barrier((ctypes.c_void_p * 2)(mine, peer), 2, 0, 1) == 1
        assert lib.coli_cuda_sync() == 0
        assert "timed out" in lib.coli_cuda_last_error().decode()
        assert lib.coli_cuda_available() == 0
        assert lib.coli_cuda_gdn_available() == 0
    finally:
        assert lib.coli_cuda_init(0) == 1, lib.coli_cuda_last_error()
        assert lib.coli_cuda_set_wait_limit(0) == 1
    # the backend computes again: one GDN decode step against the oracle
    orc = Oracle()
    cfg = "failure_reinit"
    prm = gdn_params(cfg)
    be.gdn_setup(64, 1, prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["gnorm"])
    state = np.zeros((VH_G, KD, VD), np.float32)
    ring = np.zeros((CONVK, CD), np.float32)
    be.gdn_state_set(64, 0, state)
    be.gdn_conv_set(64, 0, ring)
    ins = gdn_inputs(cfg, 1)
    y = be.gdn_decode(64, ins["qkv"], ins["z"], ins["a"], ins["b"])
    want = orc.gdn_seq(ins["qkv"], ins["z"], ins["a"], ins["b"], prm["conv_w"], prm["A_log"], prm["dt_bias"],
                       prm["gnorm"], ring, state, KH=KH_G, KD=KD)
    assert_close(y, want, what="after re-init")
