"""ctypes binding of libcoli_cuda.so — the C ABI in include/backend_cuda.h.

This is the Python-side stub a maintainer would use to drive the backend
(the engine itself calls the C ABI directly). Host-pointer calls take fp32
numpy arrays; *_dev calls take device pointers (ints), e.g. from
torch.Tensor.data_ptr(). Every call that returns 0 raises BackendError with
coli_cuda_last_error(): there is no CPU fallback.
"""
import ctypes
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "lib", "libcoli_cuda.so")
HEADER = os.path.join(ROOT, "include", "backend_cuda.h")

_i, _f, _vp = ctypes.c_int, ctypes.c_float, ctypes.c_void_p
_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int)
_sz = ctypes.POINTER(ctypes.c_size_t)

# argtypes per exported function (kept in the header's order)
SIGNATURES = {
    "coli_cuda_init": ([_i], _i),
    "coli_cuda_shutdown": ([], None),
    "coli_cuda_available": ([], _i),
    "coli_cuda_mem_info": ([_sz, _sz], None),
    "coli_cuda_last_error": ([], ctypes.c_char_p),
    "coli_cuda_set_wait_limit": ([ctypes.c_ulonglong], _i),
    "coli_cuda_debug_fail_alloc": ([_i], None),
    "coli_cuda_sync": ([], _i),
    "coli_cuda_get_stream": ([], _vp),
    "coli_cuda_set_stream": ([_vp], _i),
    "coli_cuda_ktimer_enable": ([_i], _i),
    "coli_cuda_ktimer_read": ([_i, ctypes.POINTER(ctypes.c_double), _ip], _i),
    "coli_cuda_launch_count": ([], ctypes.c_longlong),
    "coli_cuda_gdn_available": ([], _i),
    "coli_cuda_gqa_available": ([], _i),
    "coli_cuda_gqa_full_available": ([], _i),
    "coli_cuda_gdn_full_available": ([], _i),
    "coli_cuda_kv_ensure": ([_i] * 5, _i),
    "coli_cuda_kv_row": ([_i, _i, _i, _fp, _fp], _i),
    "coli_cuda_kv_rows": ([_i, _i, _i, _i, _fp, _fp], _i),
    "coli_cuda_kv_read": ([_i, _i, _i, _i, _fp, _fp], _i),
    "coli_cuda_kv_reset": ([], None),
    "coli_cuda_kv_rows_dev": ([_i] * 4 + [_vp, _vp, _i], _i),
    "coli_cuda_kv_device_ptr": ([_i, ctypes.POINTER(_vp), ctypes.POINTER(_vp)], _i),
    "coli_cuda_gqa_norm_weight": ([_i, _fp, _fp, _i], _i),
    "coli_cuda_gqa": ([_i, _fp, _fp] + [_i] * 7 + [_f], _i),
    "coli_cuda_gqa_step": ([_i] * 4 + [_fp] * 4 + [_i] * 4 + [_f, _f], _i),
    "coli_cuda_gqa_step_dev": ([_i] * 4 + [_vp] * 4 + [_i] * 4 + [_f, _f, _i], _i),
    "coli_cuda_gqa_decode": ([_i, _i, _fp, _fp, _fp, _ip, _fp] + [_i] * 4 + [_f, _f], _i),
    "coli_cuda_gqa_decode_dev": ([_i, _i, _vp, _vp, _vp, _vp, _vp] + [_i] * 4 + [_f, _f, _i], _i),
    "coli_cuda_gqa_decode_noalloc": ([_i, _i, _vp, _vp, _vp, _vp, _vp] + [_i] * 4 + [_f, _f, _i], _i),
    "coli_cuda_gqa_prefill_heads_dev": ([_i] * 4 + [_vp] * 4 + [_i] * 4 + [_f, _f, _i, _i, _i], _i),
    "coli_cuda_gdn_prefill_heads_dev": ([_i, _i, _i] + [_vp] * 5 + [_i] * 4 + [_f, _i, _i, _i], _i),
    "coli_cuda_ipc_alloc": ([ctypes.c_size_t, ctypes.POINTER(_vp), _vp], _i),
    "coli_cuda_ipc_free": ([_vp, ctypes.c_size_t], _i),
    "coli_cuda_ipc_open": ([_vp, ctypes.POINTER(_vp)], _i),
    "coli_cuda_ipc_close": ([_vp], _i),
    "coli_cuda_peer_barrier": ([ctypes.POINTER(_vp), _i, _i, ctypes.c_uint], _i),
    "coli_cuda_gqa_prefill_heads_gather_dev": ([_i] * 4 + [_vp] * 3 + [ctypes.POINTER(_vp), _i, _i] + [_i] * 4
                                               + [_f, _f, _i, _i, _i], _i),
    "coli_cuda_gdn_prefill_heads_gather_dev": ([_i, _i, _i] + [_vp] * 4 + [ctypes.POINTER(_vp), _i, _i]
                                               + [_i] * 4 + [_f, _i, _i, _i], _i),
    "coli_cuda_gdn_state_ensure": ([_i] * 5, _i),
    "coli_cuda_gdn_conv_ensure": ([_i] * 4, _i),
    "coli_cuda_gdn_conv_weight": ([_i, _fp, _i, _i], _i),
    "coli_cuda_gdn_params": ([_i, _fp, _fp, _fp, _i, _i], _i),
    "coli_cuda_gdn_reset": ([], None),
    "coli_cuda_gdn_state_get": ([_i, _i, _fp], _i),
    "coli_cuda_gdn_state_set": ([_i, _i, _fp], _i),
    "coli_cuda_gdn_conv_get": ([_i, _i, _fp], _i),
    "coli_cuda_gdn_conv_set": ([_i, _i, _fp], _i),
    "coli_cuda_gdn": ([_i] + [_fp] * 8 + [_i] * 4 + [_f], _i),
    "coli_cuda_gdn_decode": ([_i, _i] + [_fp] * 5 + [_i] * 4 + [_f], _i),
    "coli_cuda_gdn_decode_dev": ([_i, _i] + [_vp] * 5 + [_i] * 4 + [_f, _i], _i),
    "coli_cuda_gdn_prefill": ([_i, _i, _i] + [_fp] * 5 + [_i] * 4 + [_f], _i),
    "coli_cuda_gdn_prefill_dev": ([_i, _i, _i] + [_vp] * 5 + [_i] * 4 + [_f, _i], _i),
    "coli_cuda_tensor_ensure": ([ctypes.POINTER(_vp), _vp, _fp, _i, _i, _i, _i], _i),
    "coli_cuda_tensor_free": ([_vp], None),
    "coli_cuda_tensor_bytes": ([_vp], ctypes.c_size_t),
    "coli_cuda_matmul": ([ctypes.POINTER(_vp), _fp, _fp, _vp, _fp] + [_i] * 5, _i),
    "coli_cuda_matmul_dev": ([_vp, _vp, _i, _vp, _i], _i),
    "coli_cuda_matmul_multi_dev": ([ctypes.POINTER(_vp), _i, _vp, _i, ctypes.POINTER(_vp), _i], _i),
    "coli_cuda_gqa_project": ([_i, _fp, _vp, _fp] + [_i] * 7 + [_f, _i], _i),
    "coli_cuda_gdn_project": ([_i] + [_fp] * 7 + [_vp, _fp] + [_i] * 4 + [_f, _i], _i),
    "coli_cuda_gqa_full": ([_i, _fp, _i, _vp, _vp, _vp, _vp, _fp] + [_i] * 7 + [_f, _f, _i], _i),
    "coli_cuda_gdn_full": ([_i, _fp, _i, _vp, _vp, _fp, _vp, _fp] + [_i] * 6 + [_f, _i], _i),
    "coli_cuda_gdn_full_seq": ([_i, _fp, _i, _i, _vp, _vp, _fp, _vp, _fp] + [_i] * 6 + [_f, _i], _i),
    "coli_cuda_gdn_full_ab": ([_i, _fp, _i, _i] + [_vp] * 5 + [_fp] + [_i] * 6 + [_f, _i], _i),
    "coli_cuda_moe_route_available": ([], _i),
    "coli_cuda_st_open": ([ctypes.c_char_p], _i),
    "coli_cuda_st_close": ([_i], None),
    "coli_cuda_st_info": ([_i, ctypes.c_char_p, ctypes.POINTER(ctypes.c_longlong), _ip, _ip], _i),
    "coli_cuda_st_read_f32": ([_i, ctypes.c_char_p, _fp, ctypes.c_longlong], ctypes.c_longlong),
    "coli_cuda_st_dense": ([_i, ctypes.c_char_p, ctypes.POINTER(_vp)], _i),
    "coli_cuda_layer_norm_weight": ([_i, _fp, _fp, _i], _i),
    "coli_cuda_gqa_full_route": ([_i, _fp, _i] + [_vp] * 5 + [_i, _fp, _fp, _fp] + [_i] * 7 + [_f, _f, _i, _i], _i),
    "coli_cuda_gdn_full_route": ([_i, _fp, _fp, _i, _vp, _vp, _fp, _vp, _vp, _i, _fp, _fp, _fp] + [_i] * 6
                                 + [_f, _i, _i], _i),
}


def header_symbols(path=HEADER):
    """Function names declared in include/backend_cuda.h."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"\b(coli_cuda_\w+)\s*\(", text)


class BackendError(RuntimeError):
    pass


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_fp)


def load_library(path=LIB_PATH):
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} is missing: build it with `python qwen3.c_b200/build.py` "
            "(the backend has no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


class Backend:
    """Thin, checked wrapper over the C ABI (one process, one device)."""

    def __init__(self, device=0, path=LIB_PATH):
        self.lib = load_library(path)
        self._ok(self.lib.coli_cuda_init(device), "coli_cuda_init")

    # ------------------------------------------------------------------ util
    def last_error(self):
        return self.lib.coli_cuda_last_error().decode()

    def _ok(self, rc, what):
        if rc != 1:
            raise BackendError(f"{what}: {self.last_error()}")

    def sync(self):
        self._ok(self.lib.coli_cuda_sync(), "coli_cuda_sync")

    def shutdown(self):
        self.lib.coli_cuda_shutdown()

    def mem_info(self):
        a, b = ctypes.c_size_t(), ctypes.c_size_t()
        self.lib.coli_cuda_mem_info(ctypes.byref(a), ctypes.byref(b))
        return a.value, b.value

    def set_stream(self, stream_ptr):
        self._ok(self.lib.coli_cuda_set_stream(stream_ptr), "coli_cuda_set_stream")

    def get_stream(self):
        return self.lib.coli_cuda_get_stream()

    K_GQA_SPLIT, K_GDN_DECODE, K_GQA_PREFILL, K_GDN_PREFILL, K_GQA_COMBINE = range(5)

    def ktimer_enable(self, on=True):
        self._ok(self.lib.coli_cuda_ktimer_enable(int(on)), "ktimer_enable")

    def ktimer_read(self, kernel):
        ms, n = ctypes.c_double(), ctypes.c_int()
        self._ok(self.lib.coli_cuda_ktimer_read(kernel, ctypes.byref(ms), ctypes.byref(n)), "ktimer_read")
        return ms.value, n.value

    def launch_count(self):
        return self.lib.coli_cuda_launch_count()

    # ------------------------------------------------------------------ KV
    def kv_ensure(self, layer, batch, KH, max_t, hd=256):
        self._ok(self.lib.coli_cuda_kv_ensure(layer, batch, KH, max_t, hd), "kv_ensure")

    def kv_rows(self, layer, req, row0, k, v):
        k, kp = _f32(k)
        v, vp = _f32(v)
        n = k.shape[0]
        self._ok(self.lib.coli_cuda_kv_rows(layer, req, row0, n, kp, vp), "kv_rows")

    def kv_row(self, layer, req, row, k, v):
        k, kp = _f32(k)
        v, vp = _f32(v)
        self._ok(self.lib.coli_cuda_kv_row(layer, req, row, kp, vp), "kv_row")

    def kv_read(self, layer, req, row0, n, hd=256):
        k = np.zeros((n, hd), np.float32)
        v = np.zeros((n, hd), np.float32)
        self._ok(self.lib.coli_cuda_kv_read(layer, req, row0, n, k.ctypes.data_as(_fp),
                                            v.ctypes.data_as(_fp)), "kv_read")
        return k, v

    def kv_rows_dev(self, layer, req, row0, n, k_ptr, v_ptr, dtype=1):
        self._ok(self.lib.coli_cuda_kv_rows_dev(layer, req, row0, n, k_ptr, v_ptr, dtype), "kv_rows_dev")

    def kv_reset(self):
        self.lib.coli_cuda_kv_reset()

    def kv_device_ptr(self, layer):
        k, v = _vp(), _vp()
        self._ok(self.lib.coli_cuda_kv_device_ptr(layer, ctypes.byref(k), ctypes.byref(v)), "kv_device_ptr")
        return k.value, v.value

    def gqa_norm_weight(self, layer, qnw, knw):
        qnw, qp = _f32(qnw)
        knw, kp = _f32(knw)
        self._ok(self.lib.coli_cuda_gqa_norm_weight(layer, qp, kp, qnw.shape[0]), "gqa_norm_weight")

    # ------------------------------------------------------------------ GQA
    def gqa(self, layer, q, T, max_t, scale=None):
        q, qp = _f32(q)
        S, H, two_hd = q.shape
        hd = two_hd // 2
        KH = H // 8
        scale = 1.0 / np.sqrt(hd) if scale is None else scale
        ctx = np.zeros((S, H, hd), np.float32)
        self._ok(self.lib.coli_cuda_gqa(layer, qp, ctx.ctypes.data_as(_fp), S, H, KH, hd, max_t, 0,
                                        T, scale), "gqa")
        return ctx

    def gqa_step(self, layer, req, pos_base, qg, k, v, rot=64, eps=1e-6, theta=1e7):
        qg, qp = _f32(qg)
        k, kp = _f32(k)
        v, vp = _f32(v)
        S, H, two_hd = qg.shape
        hd = two_hd // 2
        ctx = np.zeros((S, H, hd), np.float32)
        self._ok(self.lib.coli_cuda_gqa_step(layer, req, S, pos_base, qp, kp, vp,
                                             ctx.ctypes.data_as(_fp), H, k.shape[1], hd, rot, eps,
                                             theta), "gqa_step")
        return ctx

    def gqa_decode(self, layer, qg, k, v, pos, rot=64, eps=1e-6, theta=1e7):
        qg, qp = _f32(qg)
        k, kp = _f32(k)
        v, vp = _f32(v)
        pos = np.ascontiguousarray(pos, dtype=np.int32)
        B, H, two_hd = qg.shape
        hd = two_hd // 2
        ctx = np.zeros((B, H, hd), np.float32)
        self._ok(self.lib.coli_cuda_gqa_decode(layer, B, qp, kp, vp, pos.ctypes.data_as(_ip),
                                               ctx.ctypes.data_as(_fp), H, k.shape[1], hd, rot,
                                               eps, theta), "gqa_decode")
        return ctx

    def gqa_decode_dev(self, layer, B, qg, k, v, pos, ctx, H=16, KH=2, hd=256, rot=64, eps=1e-6,
                       theta=1e7, dtype=1):
        self._ok(self.lib.coli_cuda_gqa_decode_dev(layer, B, qg, k, v, pos, ctx, H, KH, hd, rot, eps,
                                                   theta, dtype), "gqa_decode_dev")

    def gqa_decode_noalloc(self, layer, B, qg, k, v, pos, ctx, H=16, KH=2, hd=256, rot=64,
                           eps=1e-6, theta=1e7, dtype=1):
        self._ok(self.lib.coli_cuda_gqa_decode_noalloc(layer, B, qg, k, v, pos, ctx, H, KH, hd, rot,
                                                       eps, theta, dtype), "gqa_decode_noalloc")

    def gqa_prefill_heads_dev(self, layer, req, S, pos_base, qg, k, v, ctx, h0, nh, H=16, KH=2,
                              hd=256, rot=64, eps=1e-6, theta=1e7, dtype=1):
        self._ok(self.lib.coli_cuda_gqa_prefill_heads_dev(layer, req, S, pos_base, qg, k, v, ctx, H,
                                                          KH, hd, rot, eps, theta, dtype, h0, nh),
                 "gqa_prefill_heads_dev")

    # ---- head-sharded prefill with the all-gather fused into the output kernels
    IPC_HANDLE_BYTES = 64

    def ipc_alloc(self, nbytes):
        """cudaMalloc'd, zeroed device buffer and its IPC handle (bytes)."""
        ptr = _vp()
        handle = ctypes.create_string_buffer(self.IPC_HANDLE_BYTES)
        self._ok(self.lib.coli_cuda_ipc_alloc(nbytes, ctypes.byref(ptr), handle), "ipc_alloc")
        return ptr.value, handle.raw

    def ipc_free(self, ptr, nbytes):
        self._ok(self.lib.coli_cuda_ipc_free(ptr, nbytes), "ipc_free")

    def ipc_open(self, handle):
        ptr = _vp()
        buf = ctypes.create_string_buffer(bytes(handle), self.IPC_HANDLE_BYTES)
        self._ok(self.lib.coli_cuda_ipc_open(buf, ctypes.byref(ptr)), "ipc_open")
        return ptr.value

    def ipc_close(self, ptr):
        self._ok(self.lib.coli_cuda_ipc_close(ptr), "ipc_close")

    @staticmethod
    def _ptr_array(ptrs):
        return (_vp * len(ptrs))(*ptrs)

    def peer_barrier(self, flags, rank, epoch):
        self._ok(self.lib.coli_cuda_peer_barrier(self._ptr_array(flags), len(flags), rank, epoch),
                 "peer_barrier")

    def gqa_prefill_heads_gather_dev(self, layer, req, S, pos_base, qg, k, v, dsts, rank, h0, nh, H=16,
                                     KH=2, hd=256, rot=64, eps=1e-6, theta=1e7, dtype=1):
        self._ok(self.lib.coli_cuda_gqa_prefill_heads_gather_dev(
            layer, req, S, pos_base, qg, k, v, self._ptr_array(dsts), len(dsts), rank, H, KH, hd, rot,
            eps, theta, dtype, h0, nh), "gqa_prefill_heads_gather_dev")

    def gdn_prefill_heads_gather_dev(self, layer, req, S, qkv, z, a, b, dsts, rank, kh0, nkh, KH=16,
                                     KD=128, VH=32, VD=128, eps=1e-6, dtype=1):
        self._ok(self.lib.coli_cuda_gdn_prefill_heads_gather_dev(
            layer, req, S, qkv, z, a, b, self._ptr_array(dsts), len(dsts), rank, KH, KD, VH, VD, eps,
            dtype, kh0, nkh), "gdn_prefill_heads_gather_dev")

    def gdn_prefill_heads_dev(self, layer, req, S, qkv, z, a, b, y, kh0, nkh, KH=16, KD=128,
                              VH=32, VD=128, eps=1e-6, dtype=1):
        self._ok(self.lib.coli_cuda_gdn_prefill_heads_dev(layer, req, S, qkv, z, a, b, y, KH, KD, VH,
                                                          VD, eps, dtype, kh0, nkh),
                 "gdn_prefill_heads_dev")

    def gqa_step_dev(self, layer, req, S, pos_base, qg, k, v, ctx, H=16, KH=2, hd=256, rot=64,
                     eps=1e-6, theta=1e7, dtype=1):
        self._ok(self.lib.coli_cuda_gqa_step_dev(layer, req, S, pos_base, qg, k, v, ctx, H, KH, hd,
                                                 rot, eps, theta, dtype), "gqa_step_dev")

    # ------------------------------------------------------------------ GDN
    def gdn_setup(self, layer, batch, conv_w, A_log, dt_bias, gnorm, KH=16, KD=128, VH=32, VD=128,
                  conv_k=4):
        CD = 2 * KH * KD + VH * VD
        self._ok(self.lib.coli_cuda_gdn_state_ensure(layer, batch, VH, KD, VD), "gdn_state_ensure")
        self._ok(self.lib.coli_cuda_gdn_conv_ensure(layer, batch, conv_k, CD), "gdn_conv_ensure")
        conv_w, cp = _f32(conv_w)
        self._ok(self.lib.coli_cuda_gdn_conv_weight(layer, cp, conv_k, CD), "gdn_conv_weight")
        A_log, ap = _f32(A_log)
        dt_bias, dp = _f32(dt_bias)
        gnorm, gp = _f32(gnorm)
        self._ok(self.lib.coli_cuda_gdn_params(layer, ap, dp, gp, VH, VD), "gdn_params")

    def gdn_reset(self):
        self.lib.coli_cuda_gdn_reset()

    def gdn_state_get(self, layer, req, VH=32, KD=128, VD=128):
        s = np.zeros((VH, KD, VD), np.float32)
        self._ok(self.lib.coli_cuda_gdn_state_get(layer, req, s.ctypes.data_as(_fp)), "gdn_state_get")
        return s

    def gdn_state_set(self, layer, req, state):
        state, sp = _f32(state)
        self._ok(self.lib.coli_cuda_gdn_state_set(layer, req, sp), "gdn_state_set")

    def gdn_conv_get(self, layer, req, conv_k=4, CD=8192):
        r = np.zeros((conv_k, CD), np.float32)
        self._ok(self.lib.coli_cuda_gdn_conv_get(layer, req, r.ctypes.data_as(_fp)), "gdn_conv_get")
        return r

    def gdn_conv_set(self, layer, req, ring):
        ring, rp = _f32(ring)
        self._ok(self.lib.coli_cuda_gdn_conv_set(layer, req, rp), "gdn_conv_set")

    def gdn(self, layer, qn, kn, v, z, decay, beta, gnorm, KH=16, KD=128, VH=32, VD=128, eps=1e-6):
        arrs = [_f32(x) for x in (qn, kn, v, z, decay, beta, gnorm)]
        y = np.zeros(VH * VD, np.float32)
        self._ok(self.lib.coli_cuda_gdn(layer, *[p for _, p in arrs], y.ctypes.data_as(_fp), KH, KD,
                                        VH, VD, eps), "gdn")
        return y

    def gdn_decode(self, layer, qkv, z, a, b, KH=16, KD=128, VH=32, VD=128, eps=1e-6):
        arrs = [_f32(x) for x in (qkv, z, a, b)]
        B = arrs[0][0].shape[0]
        y = np.zeros((B, VH * VD), np.float32)
        self._ok(self.lib.coli_cuda_gdn_decode(layer, B, *[p for _, p in arrs], y.ctypes.data_as(_fp),
                                               KH, KD, VH, VD, eps), "gdn_decode")
        return y

    def gdn_decode_dev(self, layer, B, qkv, z, a, b, y, KH=16, KD=128, VH=32, VD=128, eps=1e-6,
                       dtype=1):
        self._ok(self.lib.coli_cuda_gdn_decode_dev(layer, B, qkv, z, a, b, y, KH, KD, VH, VD, eps,
                                                   dtype), "gdn_decode_dev")

    def gdn_prefill(self, layer, req, qkv, z, a, b, KH=16, KD=128, VH=32, VD=128, eps=1e-6):
        arrs = [_f32(x) for x in (qkv, z, a, b)]
        S = arrs[0][0].shape[0]
        y = np.zeros((S, VH * VD), np.float32)
        self._ok(self.lib.coli_cuda_gdn_prefill(layer, req, S, *[p for _, p in arrs],
                                                y.ctypes.data_as(_fp), KH, KD, VH, VD, eps),
                 "gdn_prefill")
        return y

    def gdn_prefill_dev(self, layer, req, S, qkv, z, a, b, y, KH=16, KD=128, VH=32, VD=128,
                        eps=1e-6, dtype=1):
        self._ok(self.lib.coli_cuda_gdn_prefill_dev(layer, req, S, qkv, z, a, b, y, KH, KD, VH, VD,
                                                    eps, dtype), "gdn_prefill_dev")


class DenseTensor:
    """A resident dense weight W [O][I] (bf16 on the device), the handle the
    block-level calls take. fmt 0 = fp32 weights, 1 = int8 with per-row scales."""

    def __init__(self, be, w, scales=None, fmt=0):
        self.be = be
        self.O, self.I = w.shape
        self.h = _vp()
        if fmt == 0:
            w = np.ascontiguousarray(w, np.float32)
            sp = None
        else:
            w = np.ascontiguousarray(w, np.int8)
            scales, sp = _f32(scales)
        be._ok(be.lib.coli_cuda_tensor_ensure(ctypes.byref(self.h), w.ctypes.data, sp, fmt, self.I, self.O, 0),
               "tensor_ensure")

    @property
    def nbytes(self):
        return self.be.lib.coli_cuda_tensor_bytes(self.h)

    def free(self):
        if self.h:
            self.be.lib.coli_cuda_tensor_free(self.h)
            self.h = _vp()


def _block_methods():
    """Block-level calls (projections + mixer + out-projection) on Backend."""

    def matmul(self, t, x):
        """y = x W^T with a DenseTensor t; x [S][I] fp32 host."""
        x, xp = _f32(x)
        S = x.shape[0] if x.ndim > 1 else 1
        y = np.zeros((S, t.O), np.float32)
        self._ok(self.lib.coli_cuda_matmul(ctypes.byref(t.h), y.ctypes.data_as(_fp), xp, None, None, 0, S, t.I,
                                           t.O, 0), "matmul")
        return y

    def gqa_full(self, layer, x, gq, gk, gv, go, pos_base, H=16, KH=2, hd=256, rot=64, max_t=None, eps=1e-6,
                 theta=1e7):
        x, xp = _f32(x)
        S, D = x.shape
        out = np.zeros((S, go.O), np.float32)
        self._ok(self.lib.coli_cuda_gqa_full(layer, xp, D, gq.h, gk.h, gv.h, go.h, out.ctypes.data_as(_fp), S, H, KH,
                                             hd, rot, pos_base, max_t or (pos_base + S), eps, theta, go.O),
                 "gqa_full")
        return out

    def gdn_full_seq(self, layer, x, params, gqkv, gz, gout, KH=16, KD=128, VH=32, VD=128, eps=1e-6):
        """S tokens (S = 1 goes through coli_cuda_gdn_full); params [S][2*VH+VD]."""
        x, xp = _f32(x)
        S, D = x.shape
        params, pp = _f32(params)
        out = np.zeros((S, gout.O), np.float32)
        CD = 2 * KH * KD + VH * VD
        if S == 1:
            rc = self.lib.coli_cuda_gdn_full(layer, xp, D, gqkv.h, gz.h, pp, gout.h, out.ctypes.data_as(_fp), KH, KD,
                                             VH, VD, CD, 4, eps, gout.O)
        else:
            rc = self.lib.coli_cuda_gdn_full_seq(layer, xp, S, D, gqkv.h, gz.h, pp, gout.h,
                                                 out.ctypes.data_as(_fp), KH, KD, VH, VD, CD, 4, eps, gout.O)
        self._ok(rc, "gdn_full")
        return out

    def matmul_multi_dev(self, tensors, x, S, ys, y_bf16=0):
        """Device pointers: x bf16 [S][I], ys[i] [S][O_i]; one launch for S <= 16."""
        n = len(tensors)
        th = (_vp * n)(*[t.h for t in tensors])
        yh = (_vp * n)(*ys)
        self._ok(self.lib.coli_cuda_matmul_multi_dev(th, n, x, S, yh, y_bf16), "matmul_multi_dev")

    def gdn_full_ab(self, layer, x, gqkv, gz, ga, gb, gout, KH=16, KD=128, VH=32, VD=128, eps=1e-6):
        """S tokens with the a / b projections on the device (no params rows)."""
        x, xp = _f32(x)
        S, D = x.shape
        out = np.zeros((S, gout.O), np.float32)
        CD = 2 * KH * KD + VH * VD
        rc = self.lib.coli_cuda_gdn_full_ab(layer, xp, S, D, gqkv.h, gz.h, ga.h, gb.h, gout.h, out.ctypes.data_as(_fp),
                                            KH, KD, VH, VD, CD, 4, eps, gout.O)
        self._ok(rc, "gdn_full_ab")
        return out

    def matmul_dev(self, t, x, S, y, y_bf16=0):
        """Device pointers: x bf16 [S][I], y [S][O]."""
        self._ok(self.lib.coli_cuda_matmul_dev(t.h, x, S, y, y_bf16), "matmul_dev")

    def layer_norm_weight(self, layer, in_ln, post_ln):
        a, ap = _f32(in_ln)
        b, bp = _f32(post_ln)
        self._ok(self.lib.coli_cuda_layer_norm_weight(layer, ap, bp, a.shape[0]), "layer_norm_weight")

    def gqa_full_route(self, layer, resid, gq, gk, gv, go, router, ln_layer, pos_base, H=16, KH=2, hd=256, rot=64,
                       max_t=None, eps=1e-6, theta=1e7):
        resid, rp = _f32(resid)
        S, D = resid.shape
        ro, nr = np.zeros((S, D), np.float32), np.zeros((S, D), np.float32)
        pr = np.zeros((S, router.O), np.float32)
        self._ok(self.lib.coli_cuda_gqa_full_route(layer, rp, D, gq.h, gk.h, gv.h, go.h, router.h, ln_layer,
                                                   ro.ctypes.data_as(_fp), nr.ctypes.data_as(_fp),
                                                   pr.ctypes.data_as(_fp), S, H, KH, hd, rot, pos_base,
                                                   max_t or (pos_base + S), eps, theta, go.O, router.O),
                 "gqa_full_route")
        return ro, nr, pr

    def gdn_full_route(self, layer, x_in, resid, params, gqkv, gz, gout, router, ln_layer, KH=16, KD=128, VH=32,
                       VD=128, eps=1e-6):
        x_in, xp = _f32(x_in)
        resid, rp = _f32(resid)
        params, pp = _f32(params)
        D = x_in.shape[-1]
        ro, nr = np.zeros(D, np.float32), np.zeros(D, np.float32)
        pr = np.zeros(router.O, np.float32)
        CD = 2 * KH * KD + VH * VD
        self._ok(self.lib.coli_cuda_gdn_full_route(layer, xp, rp, D, gqkv.h, gz.h, pp, gout.h, router.h, ln_layer,
                                                   ro.ctypes.data_as(_fp), nr.ctypes.data_as(_fp),
                                                   pr.ctypes.data_as(_fp), KH, KD, VH, VD, CD, 4, eps, gout.O,
                                                   router.O), "gdn_full_route")
        return ro, nr, pr

    for f in (matmul, matmul_dev, matmul_multi_dev, gqa_full, gdn_full_seq, gdn_full_ab, layer_norm_weight,
              gqa_full_route, gdn_full_route):
        setattr(Backend, f.__name__, f)


_block_methods()
