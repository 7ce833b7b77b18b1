"""The 40 token-mixing layers of Qwen3.5-35B-A3B on the CUDA backend.

Layer i is gated full attention iff (i+1) % 4 == 0 (c/qwen.c:398), so the
stack is 30 GatedDeltaNet + 10 gated GQA layers. Only the token mixers run:
the projections, residual/norm and MoE around them belong to the engine, so
every layer here reads synthetic, already-projected activations (random
weights of the real shapes for the per-layer parameters). The KV caches and
GDN states are resident per layer, as the engine would hold them.

MixerStack (the benchmark form) has two modes, each on one GPU of a
multi-GPU job (one process per GPU):
  decode   a batch of requests, each rank owning its own block of requests
           (sharding.request_shard); no collective on the data path.
  prefill  one long prompt, each rank computing a block of heads of every
           layer (sharding.head_shard); the layer outputs are gathered either
           by the output kernels themselves, storing into every rank's
           buffer over NVLink (fused=True, peer.PeerBuffer, one device-side
           barrier per layer), or by an NCCL all-gather after each layer.
BlockStack is the same 40 layers with their projections and the residual
stream flowing from layer to layer (the engine's loop without the MoE), for
parity checks through the host-buffer block ABI.
"""
import torch

from . import peer, sharding

H, KH, HD, ROT, EPS, THETA = 16, 2, 256, 64, 1e-6, 1e7
GKH, GKD, GVH, GVD = 16, 128, 32, 128
CD = 2 * GKH * GKD + GVH * GVD
KV_BASE, GDN_BASE = 40, 40        # backend layer slots used by the stack


def is_full(i):
    return (i + 1) % 4 == 0


class MixerStack:
    def __init__(self, be, n_layers=40, seed=0):
        self.be = be
        self.n = n_layers
        self.kinds = ["gqa" if is_full(i) else "gdn" for i in range(n_layers)]
        self.g = torch.Generator(device="cuda").manual_seed(seed)

    def _rand(self, *shape, std=1.0):
        return torch.randn(*shape, generator=self.g, device="cuda") * std

    def _gdn_params(self, slot, batch, n_vheads):
        be, lib = self.be, self.be.lib
        import ctypes
        fp = ctypes.POINTER(ctypes.c_float)
        conv = self._rand(CD, 4, std=0.3).cpu().numpy()
        alog = (torch.rand(GVH, generator=self.g, device="cuda") * 2.7726).cpu().numpy()
        dtb = self._rand(GVH).cpu().numpy()
        gn = (1 + self._rand(GVD, std=0.1)).cpu().numpy()
        be._ok(lib.coli_cuda_gdn_state_ensure(slot, batch, n_vheads, GKD, GVD), "gdn_state_ensure")
        be._ok(lib.coli_cuda_gdn_conv_ensure(slot, batch, 4, CD), "gdn_conv_ensure")
        be._ok(lib.coli_cuda_gdn_conv_weight(slot, conv.ctypes.data_as(fp), 4, CD), "gdn_conv_weight")
        be._ok(lib.coli_cuda_gdn_params(slot, alog.ctypes.data_as(fp), dtb.ctypes.data_as(fp),
                                        gn.ctypes.data_as(fp), GVH, GVD), "gdn_params")

    def _norm_w(self, slot):
        self.be.gqa_norm_weight(slot, self._rand(HD, std=0.1).cpu().numpy(),
                                self._rand(HD, std=0.1).cpu().numpy())

    # ------------------------------------------------------------ decode
    def setup_decode(self, batch, context):
        """Caches of `batch` requests holding `context - 1` random rows each;
        every decode step appends row context-1 (the step is repeatable)."""
        self.B, self.T = batch, context
        be = self.be
        src_k = self._rand(KH * context, HD).bfloat16()
        src_v = self._rand(KH * context, HD).bfloat16()
        kvi = gi = 0
        for kind in self.kinds:
            if kind == "gqa":
                be.kv_ensure(KV_BASE + kvi, batch, KH, context)
                self._norm_w(KV_BASE + kvi)
                for r in range(batch):
                    be.kv_rows_dev(KV_BASE + kvi, r, 0, KH * context, src_k.data_ptr(),
                                   src_v.data_ptr(), 1)
                kvi += 1
            else:
                self._gdn_params(GDN_BASE + gi, batch, GVH)
                gi += 1
        be.gdn_reset()
        B = batch
        self.qg = self._rand(B, H, 2 * HD).bfloat16()
        self.k = self._rand(B, KH, HD).bfloat16()
        self.v = (self._rand(B, KH, HD) / 16).bfloat16()
        self.pos = torch.full((B,), context - 1, dtype=torch.int32, device="cuda")
        self.ctx = torch.empty(B, H, HD, dtype=torch.bfloat16, device="cuda")
        self.qkv = self._rand(B, CD).bfloat16()
        self.z = self._rand(B, GVH * GVD).bfloat16()
        self.a = self._rand(B, GVH).bfloat16()
        self.b = self._rand(B, GVH).bfloat16()
        self.y = torch.empty(B, GVH * GVD, dtype=torch.bfloat16, device="cuda")
        be.sync()

    def decode_step(self):
        be, B = self.be, self.B
        kvi = gi = 0
        for kind in self.kinds:
            if kind == "gqa":
                be.gqa_decode_dev(KV_BASE + kvi, B, self.qg.data_ptr(), self.k.data_ptr(),
                                  self.v.data_ptr(), self.pos.data_ptr(), self.ctx.data_ptr(),
                                  H, KH, HD, ROT, EPS, THETA, 1)
                kvi += 1
            else:
                be.gdn_decode_dev(GDN_BASE + gi, B, self.qkv.data_ptr(), self.z.data_ptr(),
                                  self.a.data_ptr(), self.b.data_ptr(), self.y.data_ptr(),
                                  GKH, GKD, GVH, GVD, EPS, 1)
                gi += 1

    def decode_bytes_per_request(self):
        """Algorithmic HBM bytes of one decode step for one request."""
        n_gqa = sum(k == "gqa" for k in self.kinds)
        n_gdn = self.n - n_gqa
        return n_gqa * (2048 * self.T + 2048 + 16384 + 8192) + n_gdn * 4_423_808

    # ------------------------------------------------------------ prefill
    def setup_prefill(self, S, world=1, rank=0, fused=False):
        """One prompt of S tokens; this rank computes heads of its shard.
        fused: gather the layer outputs in the kernels (peer stores) rather
        than with NCCL."""
        self.S, self.world, self.rank = S, world, rank
        self.fused = fused and world > 1
        self.h0, self.h1 = sharding.head_shard(H, world, rank)
        self.k0, self.k1 = sharding.kv_heads_for(self.h0, self.h1, H // KH)
        self.g0, self.g1 = sharding.head_shard(GKH, world, rank)
        be = self.be
        kvi = gi = 0
        for kind in self.kinds:
            if kind == "gqa":
                be.kv_ensure(KV_BASE + kvi, 1, self.k1 - self.k0, S)
                self._norm_w(KV_BASE + kvi)
                kvi += 1
            else:
                self._gdn_params(GDN_BASE + gi, 1, 2 * (self.g1 - self.g0))
                gi += 1
        be.gdn_reset()
        self.pqg = self._rand(S, H, 2 * HD).bfloat16()
        self.pk = self._rand(S, KH, HD).bfloat16()
        self.pv = self._rand(S, KH, HD).bfloat16()
        self.pqkv = self._rand(S, CD).bfloat16()
        self.pz = self._rand(S, GVH * GVD).bfloat16()
        self.pa = self._rand(S, GVH).bfloat16()
        self.pb = self._rand(S, GVH).bfloat16()
        nh, nv = self.h1 - self.h0, 2 * (self.g1 - self.g0)
        self.pctx = torch.empty(S, nh, HD, dtype=torch.bfloat16, device="cuda")
        self.py = torch.empty(S, nv * GVD, dtype=torch.bfloat16, device="cuda")
        if self.fused:
            # two buffers per kind, alternating by layer: a rank may store layer
            # L+1 while a slower peer still reads layer L's output; the barrier
            # after every layer keeps ranks within one layer of each other
            self.gq_bufs = [peer.PeerBuffer(be, world * S * nh * HD * 2, world, rank) for _ in range(2)]
            self.gd_bufs = [peer.PeerBuffer(be, world * S * nv * GVD * 2, world, rank) for _ in range(2)]
            self.pbar = peer.PeerBarrier(be, world, rank)
        else:
            self.ctx_all = torch.empty(world, S, nh, HD, dtype=torch.bfloat16, device="cuda")
            self.y_all = torch.empty(world, S, nv * GVD, dtype=torch.bfloat16, device="cuda")
        be.sync()

    def close_prefill(self):
        """Release the peer buffers of a fused setup (collective)."""
        if getattr(self, "fused", False):
            for b in self.gq_bufs + self.gd_bufs:
                b.close()
            self.pbar.close()
            self.fused = False

    def prefill(self, gather=True):
        """All layers' mixers over the prompt; with world > 1 each layer's
        per-rank output is all-gathered (rank-major [world][S][heads][dim])."""
        import torch.distributed as dist
        be, S = self.be, self.S
        sharded = self.world > 1
        kvi = gi = 0
        for kind in self.kinds:
            if kind == "gqa":
                if self.fused:
                    be.gqa_prefill_heads_gather_dev(KV_BASE + kvi, 0, S, 0, self.pqg.data_ptr(),
                                                    self.pk.data_ptr(), self.pv.data_ptr(),
                                                    self.gq_bufs[kvi % 2].ptrs, self.rank, self.h0,
                                                    self.h1 - self.h0)
                    self.pbar()
                elif sharded:
                    be.gqa_prefill_heads_dev(KV_BASE + kvi, 0, S, 0, self.pqg.data_ptr(),
                                             self.pk.data_ptr(), self.pv.data_ptr(),
                                             self.pctx.data_ptr(), self.h0, self.h1 - self.h0)
                else:
                    be.gqa_step_dev(KV_BASE + kvi, 0, S, 0, self.pqg.data_ptr(), self.pk.data_ptr(),
                                    self.pv.data_ptr(), self.pctx.data_ptr())
                if sharded and gather and not self.fused:
                    dist.all_gather_into_tensor(self.ctx_all, self.pctx)
                kvi += 1
            else:
                if self.fused:
                    be.gdn_prefill_heads_gather_dev(GDN_BASE + gi, 0, S, self.pqkv.data_ptr(),
                                                    self.pz.data_ptr(), self.pa.data_ptr(),
                                                    self.pb.data_ptr(), self.gd_bufs[gi % 2].ptrs,
                                                    self.rank, self.g0, self.g1 - self.g0)
                    self.pbar()
                elif sharded:
                    be.gdn_prefill_heads_dev(GDN_BASE + gi, 0, S, self.pqkv.data_ptr(),
                                             self.pz.data_ptr(), self.pa.data_ptr(),
                                             self.pb.data_ptr(), self.py.data_ptr(), self.g0,
                                             self.g1 - self.g0)
                else:
                    be.gdn_prefill_dev(GDN_BASE + gi, 0, S, self.pqkv.data_ptr(), self.pz.data_ptr(),
                                       self.pa.data_ptr(), self.pb.data_ptr(), self.py.data_ptr())
                if sharded and gather and not self.fused:
                    dist.all_gather_into_tensor(self.y_all, self.py)
                gi += 1

    def prefill_flops_bytes(self):
        """Whole-job algorithmic work of one prefill: GQA FLOPs (causal) and
        GDN bytes (S x 32,896 + 2 MiB state per layer)."""
        n_gqa = sum(k == "gqa" for k in self.kinds)
        n_gdn = self.n - n_gqa
        return n_gqa * 8192.0 * self.S * (self.S + 1), n_gdn * (self.S * 32896 + 2 * 1024 * 1024)


# ------------------------------------------------------------ whole blocks
D_MODEL = 2048


def block_weights(seed, i):
    """Random weights of the real shapes for model layer i (N(0, 0.02)
    matrices; small vectors as a freshly initialised layer has them), a pure
    function of (seed, i) so a checker can regenerate them."""
    import numpy as np
    rng = np.random.default_rng([seed, i])
    w = lambda *s: (rng.standard_normal(s, dtype=np.float32) * np.float32(0.02))   # noqa: E731
    if is_full(i):
        return dict(q=w(H * 2 * HD, D_MODEL), k=w(KH * HD, D_MODEL), v=w(KH * HD, D_MODEL),
                    o=w(D_MODEL, H * HD), qn=np.zeros(HD, np.float32), kn=np.zeros(HD, np.float32),
                    in_ln=np.zeros(D_MODEL, np.float32))
    return dict(qkv=w(CD, D_MODEL), z=w(GVH * GVD, D_MODEL), a=w(GVH, D_MODEL), b=w(GVH, D_MODEL),
                out=w(D_MODEL, GVH * GVD), conv=(rng.standard_normal((CD, 4), dtype=np.float32) * np.float32(0.3)),
                A_log=np.log(rng.uniform(1.0, 16.0, GVH)).astype(np.float32), dt_bias=np.ones(GVH, np.float32),
                gnorm=np.ones(GVD, np.float32), in_ln=np.zeros(D_MODEL, np.float32))


def rmsnorm_zc(x, w, eps=EPS):
    """x * rsqrt(mean x^2 + eps) * (1 + w), mean square in double (c/qwen.c:326-330)."""
    import numpy as np
    x = np.asarray(x, np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    return (x * (1.0 / np.sqrt((ms + eps).astype(np.float32))) * (1.0 + w)).astype(np.float32)


def gdn_params_rows(wt, xn):
    """The engine's per-token [decay | beta | gnorm] rows from the tiny a / b
    projections it keeps on the host (c/qwen.c:681-686, 1356-1368)."""
    import numpy as np
    a, b = xn @ wt["a"].T, xn @ wt["b"].T
    sp = np.where(a + wt["dt_bias"] > 20, a + wt["dt_bias"], np.log1p(np.exp(a + wt["dt_bias"])))
    decay = np.exp(-np.exp(wt["A_log"]) * sp).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-b))).astype(np.float32)
    return np.concatenate([decay, beta, np.broadcast_to(wt["gnorm"], (xn.shape[0], GVD))], axis=1).astype(np.float32)


class BlockStack:
    """The token-mixing blocks of the 40-layer stack with data flowing between
    layers, as in the engine's layer loop minus the MoE (c/qwen.c:1347-1387):
    x_{i+1} = x_i + block_i(rmsnorm_zc(x_i, in_ln_i)), each block = its
    projections + mixer + out-projection on the device (coli_cuda_gqa_full /
    coli_cuda_gdn_full_seq), weights bf16-resident, KV / state carried across
    calls. Host buffers in and out per block (the engine-facing ABI)."""

    def __init__(self, be, n_layers=40, seed=0, max_t=4096):
        from .coli_cuda import DenseTensor
        self.be, self.n, self.seed, self.max_t = be, n_layers, seed, max_t
        self.t = []
        kvi = gi = 0
        for i in range(n_layers):
            wt = block_weights(seed, i)
            if is_full(i):
                be.kv_ensure(KV_BASE + kvi, 1, KH, max_t)
                be.gqa_norm_weight(KV_BASE + kvi, wt["qn"], wt["kn"])
                self.t.append({n: DenseTensor(be, wt[n]) for n in ("q", "k", "v", "o")})
                kvi += 1
            else:
                be.gdn_setup(GDN_BASE + gi, 1, wt["conv"], wt["A_log"], wt["dt_bias"], wt["gnorm"])
                self.t.append({n: DenseTensor(be, wt[n]) for n in ("qkv", "z", "out")})
                gi += 1
        be.gdn_reset()
        self.pos = 0

    def forward(self, x):
        """S new tokens through all layers; returns (per-layer normed inputs,
        per-layer block outputs, final residual)."""
        be, ins, outs = self.be, [], []
        kvi = gi = 0
        for i in range(self.n):
            wt = block_weights(self.seed, i)
            xn = rmsnorm_zc(x, wt["in_ln"])
            t = self.t[i]
            if is_full(i):
                o = be.gqa_full(KV_BASE + kvi, xn, t["q"], t["k"], t["v"], t["o"], self.pos, max_t=self.max_t)
                kvi += 1
            else:
                o = be.gdn_full_seq(GDN_BASE + gi, xn, gdn_params_rows(wt, xn), t["qkv"], t["z"], t["out"])
                gi += 1
            ins.append(xn)
            outs.append(o)
            x = x + o
        self.pos += x.shape[0]
        return ins, outs, x

    def close(self):
        for t in self.t:
            for d in t.values():
                d.free()
