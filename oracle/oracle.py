"""ctypes bindings for the CPU checkers — TEST INFRASTRUCTURE ONLY.

`Oracle` wraps oracle/liboracle.so (the fp32 restatement of the reference's
token-mixer arithmetic, oracle/oracle.c). `Reference` wraps
oracle/_ref/libqwenref.so (the reference's own c/qwen.c compiled unmodified
through oracle/ref_harness.c). Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs use this module; the CUDA backend never does.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_f32p = ctypes.POINTER(ctypes.c_float)
_c_int, _c_float = ctypes.c_int, ctypes.c_float


def _p(a):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_f32p)


def build():
    """Compile liboracle.so (and _ref where the reference sources exist)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", HERE], check=True)


class Oracle:
    def __init__(self, path=None):
        path = path or os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        self.lib = lib = ctypes.CDLL(path)
        lib.orc_gqa_prologue.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p] + [_c_int] * 5 + \
            [_c_float, _c_float, _c_int, _f32p, _f32p, _c_int]
        lib.orc_gqa_attend.argtypes = [_f32p] * 4 + [_c_int] * 6 + [_c_float]
        lib.orc_gdn_step.argtypes = [_f32p] * 11 + [_c_int] * 5 + [_c_float]
        lib.orc_gdn_seq.argtypes = [_f32p] * 11 + [_c_int] * 6 + [_c_float]
        lib.orc_gdn_recur.argtypes = [_f32p] * 9 + [_c_int] * 4 + [_c_float]
        lib.orc_threads.restype = _c_int
        lib.orc_set_threads.argtypes = [_c_int]

    def threads(self):
        return self.lib.orc_threads()

    def set_threads(self, n):
        self.lib.orc_set_threads(n)

    def gqa_prologue(self, qg, k, v, qnw, knw, pos_base, Kc, Vc, rot=64, theta=1e7, eps=1e-6):
        """In place: qg [S,H,2hd] normed+roped; k [S,KH,hd] normed+roped;
        cache Kc/Vc [KH,max_t,hd] rows pos_base.. written."""
        S, H, two_hd = qg.shape
        hd = two_hd // 2
        KH, max_t = Kc.shape[0], Kc.shape[1]
        self.lib.orc_gqa_prologue(_p(qg), _p(k), _p(v), _p(qnw), _p(knw), S, H, KH, hd, rot,
                                  theta, eps, pos_base, _p(Kc), _p(Vc), max_t)

    def gqa_attend(self, qg, Kc, Vc, pos_base, scale=None):
        S, H, two_hd = qg.shape
        hd = two_hd // 2
        KH, max_t = Kc.shape[0], Kc.shape[1]
        scale = 1.0 / np.sqrt(np.float32(hd)) if scale is None else scale
        ctx = np.zeros((S, H, hd), np.float32)
        self.lib.orc_gqa_attend(_p(qg), _p(Kc), _p(Vc), _p(ctx), S, H, KH, hd, max_t, pos_base,
                                float(scale))
        return ctx

    def gdn_seq(self, qkv, z, a, b, conv_w, A_log, dt_bias, gnorm, ring, state, KH, KD, eps=1e-6):
        """S tokens for one request; ring [K,CD] and state [VH,KD,VD] update in place."""
        S = qkv.shape[0]
        VH, _, VD = state.shape
        K = ring.shape[0]
        y = np.zeros((S, VH * VD), np.float32)
        self.lib.orc_gdn_seq(_p(qkv), _p(z), _p(a), _p(b), _p(conv_w), _p(A_log), _p(dt_bias),
                             _p(gnorm), _p(ring), _p(state), _p(y), S, KH, KD, VH, VD, K, eps)
        return y

    def gdn_recur(self, qn, kn, v, z, decay, beta, gnorm, state, KH, eps=1e-6):
        """Post-norm recurrence only; state [VH,KD,VD] updated in place."""
        VH, KD, VD = state.shape
        y = np.zeros(VH * VD, np.float32)
        self.lib.orc_gdn_recur(_p(qn), _p(kn), _p(v), _p(z), _p(decay), _p(beta), _p(gnorm),
                               _p(state), _p(y), KH, KD, VH, VD, eps)
        return y


class Reference:
    """The reference's own functions (attention(), gdn_step(), matmul())."""

    def __init__(self, path=None):
        path = path or os.path.join(HERE, "_ref", "libqwenref.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = lib = ctypes.CDLL(path)
        lib.ref_attention.argtypes = [_f32p, _f32p] + [_c_int] * 6 + [_c_float] * 3 + [_f32p] * 8 + [_c_int]
        lib.ref_gdn_steps.argtypes = [_f32p, _f32p] + [_c_int] * 7 + [_c_float] + [_f32p] * 11
        lib.ref_matmul.argtypes = [_f32p, _f32p, _f32p, _c_int, _c_int, _c_int]
        lib.ref_threads.restype = _c_int

    @staticmethod
    def available(path=None):
        return os.path.exists(path or os.path.join(HERE, "_ref", "libqwenref.so"))

    def threads(self):
        return self.lib.ref_threads()

    def matmul(self, x, W):
        S, I = x.shape
        O = W.shape[0]
        y = np.zeros((S, O), np.float32)
        self.lib.ref_matmul(_p(y), _p(x), _p(W), S, I, O)
        return y

    def attention(self, x, pos_base, H, KH, hd, Wq, Wk, Wv, Wo, qn, kn, Kc, Vc,
                  partial_rotary=0.25, theta=1e7, eps=1e-6):
        S, D = x.shape
        out = np.zeros((S, Wo.shape[0]), np.float32)
        self.lib.ref_attention(_p(x), _p(out), S, pos_base, D, H, KH, hd, partial_rotary, theta,
                               eps, _p(Wq), _p(Wk), _p(Wv), _p(Wo), _p(qn), _p(kn), _p(Kc),
                               _p(Vc), Kc.shape[1])
        return out

    def gdn_steps(self, x, KH, KD, VH, VD, K, Wqkv, Wz, Wa, Wb, conv, A_log, dt_bias, gnorm,
                  Wout, state, ring, eps=1e-6):
        S, D = x.shape
        out = np.zeros((S, D), np.float32)
        self.lib.ref_gdn_steps(_p(x), _p(out), S, D, KH, KD, VH, VD, K, eps, _p(Wqkv), _p(Wz),
                               _p(Wa), _p(Wb), _p(conv), _p(A_log), _p(dt_bias), _p(gnorm),
                               _p(Wout), _p(state), _p(ring))
        return out
