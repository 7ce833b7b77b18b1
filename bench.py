"""Benchmark of the qwen3.c token-mixer hot path on B200.

Headline (BASELINE metric "decode attn-layer tok/s @32k ctx"): one gated GQA
decode step of one full-attention layer for a batch of 64 requests, each at
context 32768 (Qwen3.5-35B-A3B shapes: 16 Q / 2 KV heads, head_dim 256, bf16
KV cache resident in HBM). One "step" = every request decodes one token
through the layer's attention (q/k norm + RoPE + KV append + split-KV
attention + gate). value = requests*GPUs / step time (tokens/s for the layer).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Multi-GPU: launched by torchrun, one rank per GPU; decode shards by request
(each rank owns its own 64 requests and their KV cache, no collective on the
data path) -> weak scaling. Timing: CUDA events on the launching stream,
barrier + synchronize on both sides, max over ranks.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B_REQ = 64          # requests per GPU
T_CTX = 32768       # context length (cache rows per request, incl. the new token)
H, KH, HD, ROT = 16, 2, 256, 64
EPS, THETA = 1e-6, 1e7
GDN_B = 256         # secondary: GatedDeltaNet decode batch
GDN_BYTES_PER_REQ = 4_194_304 + 196_608 + 24_704 + 8_192


def _pkg():
    import __graft_entry__ as ge
    return ge._pkg()


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d.get("bf16_tflops"), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clock and clock-event reasons of this process's GPU, polled through
    NVML every ~2 ms from a thread while the timed region runs (so even a
    region of a few milliseconds gets samples); nvidia-smi at 100 ms when
    NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, local_rank):
        self.local = local_rank
        self.sm, self.reasons, self.smax = [], set(), None
        self._stop = threading.Event()
        self.t = None

    def _handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        # NVML numbers every GPU of the machine; find this process's device by
        # its PCI bus id (NVML writes the domain with 8 digits, CUDA with 4)
        want = str(getattr(torch.cuda.get_device_properties(self.local), "pci_bus_id", "")).lower()
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            bus = pynvml.nvmlDeviceGetPciInfo(h).busId
            bus = (bus.decode() if isinstance(bus, bytes) else str(bus)).lower()
            if want and bus.endswith(want.split(":", 1)[-1]):
                return h
        return pynvml.nvmlDeviceGetHandleByIndex(self.local)

    def _poll(self, h):
        import pynvml
        bits = [(n, getattr(pynvml, c, 0)) for n, c in self.REASONS]
        while not self._stop.is_set():
            try:
                self.sm.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                for n, b in bits:
                    if r & b:
                        self.reasons.add(n)
            except Exception:
                break
            time.sleep(0.002)

    def __enter__(self):
        try:
            import pynvml
            h = self._handle()
            self.smax = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._poll, args=(h,), daemon=True)
            self.t.start()
        except Exception:
            self.t = None
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.t:
            self.t.join(timeout=2)

    def brief(self):
        """Median SM clock and reasons over a short timed region (a leg)."""
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None,
                "reasons": sorted(self.reasons), "samples": len(self.sm)}

    def summary(self):
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.smax,
                "reasons": sorted(self.reasons), "samples": len(self.sm), "source": "nvml, 2 ms polling"}


def _local_rank():
    return int(os.environ.get("LOCAL_RANK", "0"))


def dist_setup():
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(ws, x):
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------- CPU legs
def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_port_baseline(n_req=8):
    """Oracle port (c/qwen.c:598-663 restated) on the host cores: one decode
    token per request at context T_CTX, requests one after another (the
    reference engine is single-sequence)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle
    synth = _pkg().synth
    orc = Oracle()
    Kc = synth.bf16_round(synth.normal(1, (KH, T_CTX, HD)))
    Vc = synth.bf16_round(synth.normal(2, (KH, T_CTX, HD)))
    qn, kn = synth.normal(3, (HD,), std=0.1), synth.normal(4, (HD,), std=0.1)
    t0 = time.perf_counter()
    for r in range(n_req):
        qg = synth.normal(10 + r, (1, H, 2 * HD))
        k, v = synth.normal(100 + r, (1, KH, HD)), synth.normal(200 + r, (1, KH, HD))
        orc.gqa_prologue(qg, k, v, qn, kn, T_CTX - 1, Kc, Vc)
        orc.gqa_attend(qg, Kc, Vc, T_CTX - 1)
    dt = time.perf_counter() - t0
    cores = orc.threads()
    # the same work on one thread (the reference's shipped build has no OpenMP)
    orc.set_threads(1)
    n1 = 2
    t1 = time.perf_counter()
    for r in range(n1):
        qg = synth.normal(10 + r, (1, H, 2 * HD))
        k, v = synth.normal(100 + r, (1, KH, HD)), synth.normal(200 + r, (1, KH, HD))
        orc.gqa_prologue(qg, k, v, qn, kn, T_CTX - 1, Kc, Vc)
        orc.gqa_attend(qg, Kc, Vc, T_CTX - 1)
    one = n1 / (time.perf_counter() - t1)
    orc.set_threads(cores)
    return {"value": n_req / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "cpu_model": cpu_model(), "value_1_thread": one,
            "sample": f"{n_req} requests x 1 decode token at context {T_CTX} (oracle/oracle.c "
                      f"prologue+attend, OpenMP over heads as in c/qwen.c:640); 1-thread figure "
                      f"from {n1} requests"}


def reference_arm(args):
    """The reference's own attention() (c/qwen.c:581-666, compiled unmodified
    into oracle/_ref) on the host cores, same workload shape; falls back to the
    oracle port if the reference library was not built."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Reference
    synth = _pkg().synth
    if not Reference.available():
        res = cpu_port_baseline()
        kind, cores = "port", res["cores"]
        step_fn = None
    else:
        kind = "reference"
    D = 2048
    per_step = 1
    times = []
    if kind == "reference":
        ref = Reference()
        cores = ref.threads()
        Wq = synth.normal(1, (H * 2 * HD, D), std=0.02)
        Wk = synth.normal(2, (KH * HD, D), std=0.02)
        Wv = synth.normal(3, (KH * HD, D), std=0.02)
        Wo = synth.normal(4, (D, H * HD), std=0.02)
        qn, kn = synth.normal(5, (HD,), std=0.1), synth.normal(6, (HD,), std=0.1)
        Kc = synth.normal(7, (KH, T_CTX, HD))
        Vc = synth.normal(8, (KH, T_CTX, HD))

        def step_fn(i):
            for r in range(per_step):
                x = synth.normal(1000 + i * per_step + r, (1, D))
                ref.attention(x, T_CTX - 1, H, KH, HD, Wq, Wk, Wv, Wo, qn, kn, Kc, Vc)
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            step_fn(i)
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
        value = per_step * len(times) / sum(times)
        sample = (f"{per_step} requests per step x 1 decode token at context {T_CTX}; each "
                  "attention() call includes its q/k/v/o projections (D=2048)")
    else:
        value = res["value"]
        sample = res["sample"]
    line = {"metric": "decode attn-layer tok/s @32k ctx", "value": value, "unit": "tok/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": workload_config(),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": kind,
                             "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def workload_config():
    return {"workload": "gated GQA decode step, one full-attention layer (BASELINE config 2)",
            "requests_per_gpu": B_REQ, "context": T_CTX, "q_heads": H, "kv_heads": KH,
            "head_dim": HD, "kv_cache": "bf16 resident", "l2": "inputs larger than L2 (4.3 GB KV per step)"}


# ----------------------------------------------------------------- our arm
def run_ours(args, ws, rank, local):
    import torch
    pkg = _pkg()
    be = pkg.Backend(local)
    torch.cuda.set_device(local)
    st = torch.cuda.Stream()          # a real stream: the backend launches on it, events time it
    torch.cuda.set_stream(st)
    be.set_stream(st.cuda_stream)
    peak_hbm, peak_tc, peak_kind = _peaks()
    if args.only:  # one secondary leg alone (profiling runs)
        fn = {"gdn": run_gdn_secondary, "prefill": run_prefill_secondary,
              "gdnprefill": run_gdn_prefill_secondary, "stack": run_stack_decode,
              "stackprefill": run_stack_prefill, "linear": run_linear,
              "gqagrid": run_gqa_grid, "gdngrid": run_gdn_grid}[args.only]
        res = fn(be, args, st, peak_tc if args.only in ("prefill", "stackprefill") else peak_hbm)
        if rank == 0:
            print(json.dumps(res))
        return

    # ---- state: a 64-request bf16 KV cache at 32k context, random contents
    layer = 0
    be.kv_ensure(layer, B_REQ, KH, T_CTX)
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    qn = (torch.randn(HD, generator=g, device="cuda") * 0.1).cpu().numpy()
    kn = (torch.randn(HD, generator=g, device="cuda") * 0.1).cpu().numpy()
    be.gqa_norm_weight(layer, qn, kn)
    rows = torch.empty(KH * T_CTX, HD, dtype=torch.bfloat16, device="cuda")
    rows2 = torch.empty_like(rows)
    for r in range(B_REQ):
        rows.normal_(generator=g)
        rows2.normal_(generator=g)
        be.kv_rows_dev(layer, r, 0, KH * T_CTX, rows.data_ptr(), rows2.data_ptr(), 1)
    del rows, rows2
    qg = torch.randn(B_REQ, H, 2 * HD, generator=g, device="cuda").bfloat16()
    k = torch.randn(B_REQ, KH, HD, generator=g, device="cuda").bfloat16()
    v = (torch.randn(B_REQ, KH, HD, generator=g, device="cuda") / 16).bfloat16()
    pos = torch.full((B_REQ,), T_CTX - 1, dtype=torch.int32, device="cuda")
    ctx = torch.empty(B_REQ, H, HD, dtype=torch.bfloat16, device="cuda")
    be.sync()

    def step():
        be.gqa_decode_dev(layer, B_REQ, qg.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(),
                          ctx.data_ptr(), H, KH, HD, ROT, EPS, THETA, 1)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    launches0 = be.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(st)
        for _ in range(args.steps):
            step()
        e1.record(st)
        torch.cuda.synchronize()
    be.sync()
    ms_local = e0.elapsed_time(e1)
    launches = be.launch_count() - launches0
    # Per-kernel times for the roofline come from a second pass with the
    # library's event timer on (events between the launches stop the
    # programmatic overlap of prologue, split and combine, so the headline
    # pass above runs without them).
    nk = max(10, min(args.steps, 200))
    be.ktimer_enable(True)
    be.ktimer_read(be.K_GQA_SPLIT)
    be.ktimer_read(be.K_GQA_COMBINE)
    for _ in range(nk):
        step()
    be.sync()
    be.ktimer_enable(False)
    split_ms, split_n = be.ktimer_read(be.K_GQA_SPLIT)
    comb_ms, comb_n = be.ktimer_read(be.K_GQA_COMBINE)
    barrier(ws)
    ms = max_over_ranks(ws, ms_local)
    ms_step = ms / args.steps
    value = ws * B_REQ / (ms_step / 1e3)

    # roofline of the dominant kernel (split-KV attention): algorithmic bytes =
    # the K and V rows every request reads: B * KH * T * hd * 2 B * 2
    split_bytes = B_REQ * KH * T_CTX * HD * 2 * 2
    split_avg_s = split_ms / max(split_n, 1) / 1e3
    achieved = split_bytes / split_avg_s / 1e9
    step_bytes = B_REQ * (2048 * T_CTX + 2048 + 16384 + 8192)

    # ---- e2e through the public host API (pinned fp32 host buffers)
    e2e = run_e2e(be, layer, args, st) if not args.quick else None
    secondary = {}
    if not args.quick:
        be.kv_reset()
        legs = [("gdn_decode", lambda: run_gdn_secondary(be, args, st, peak_hbm)),
                ("gqa_prefill", lambda: run_prefill_secondary(be, args, st, peak_tc)),
                ("gdn_prefill", lambda: run_gdn_prefill_secondary(be, args, st, peak_hbm)),
                ("gqa_decode_grid", lambda: run_gqa_grid(be, args, st, peak_hbm)),
                ("gdn_decode_grid", lambda: run_gdn_grid(be, args, st, peak_hbm))]
        if not args.no_stack:
            legs += [("stack_decode", lambda: run_stack_decode(be, args, st, peak_hbm)),
                     ("stack_prefill", lambda: run_stack_prefill(be, args, st, peak_tc))]
        for name, fn in legs:
            try:
                secondary.update(fn())
            except Exception as e:   # a failed leg is reported, the headline line still prints
                secondary[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
            be.kv_reset()
            be.gdn_reset()

    if rank != 0:
        return
    line = {
        "metric": "decode attn-layer tok/s @32k ctx", "value": value, "unit": "tok/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random bf16 KV cache and activations)",
        "config": dict(workload_config(), parallelism=f"requests sharded over {ws} GPU(s), no collective"),
        "roofline": {"bound": "hbm", "kernel": "gqa_split_kernel", "achieved": achieved,
                     "peak": peak_hbm, "unit": "GB/s", "frac": achieved / peak_hbm,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6650 GB/s",
                     "traffic": traffic_from_profile(), "bytes_per_launch": split_bytes,
                     "avg_launch_us": split_avg_s * 1e6,
                     "step_frac": step_bytes / (ms_step / 1e3) / 1e9 / peak_hbm},
        "kernels_ms_per_step": {"gqa_split": split_ms / max(split_n, 1),
                                "gqa_combine": comb_ms / max(comb_n, 1)},
        "e2e": e2e,
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
        "secondary": secondary,
    }
    if not args.no_cpu:
        line["cpu_baseline"] = cpu_port_baseline()
    print(json.dumps(line))


def traffic_from_profile():
    """DRAM bytes per launch of gqa_split_kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "gqa_split_decode_b64_t32k.md")
    if not os.path.exists(p):
        return None
    for ln in open(p):
        if ln.startswith("traffic_bytes_per_launch:"):
            return float(ln.split(":")[1])
    return None


def run_e2e(be, layer, args, st):
    import torch
    n = max(10, args.steps // 10)
    qg = torch.randn(B_REQ, H, 2 * HD).pin_memory()
    k = torch.randn(B_REQ, KH, HD).pin_memory()
    v = (torch.randn(B_REQ, KH, HD) / 16).pin_memory()
    pos = torch.full((B_REQ,), T_CTX - 1, dtype=torch.int32).pin_memory()
    ctx = torch.empty(B_REQ, H, HD).pin_memory()
    import ctypes
    fp = ctypes.POINTER(ctypes.c_float)
    ip = ctypes.POINTER(ctypes.c_int)

    def call():
        rc = be.lib.coli_cuda_gqa_decode(
            layer, B_REQ, ctypes.cast(qg.data_ptr(), fp), ctypes.cast(k.data_ptr(), fp),
            ctypes.cast(v.data_ptr(), fp), ctypes.cast(pos.data_ptr(), ip),
            ctypes.cast(ctx.data_ptr(), fp), H, KH, HD, ROT, EPS, THETA)
        if rc != 1:
            raise RuntimeError(be.last_error())
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(n):
        call()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    h2d = qg.numel() * 4 + k.numel() * 4 + v.numel() * 4 + pos.numel() * 4
    d2h = ctx.numel() * 4
    return {"value": B_REQ / (ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms, "steps": n,
            "api": "coli_cuda_gqa_decode (fp32 host buffers, pinned)"}


def run_gdn_secondary(be, args, st, peak_hbm):
    """GatedDeltaNet decode at batch 256, bf16 activations."""
    import torch
    KHg, KD, VHg, VD = 16, 128, 32, 128
    CD = 2 * KHg * KD + VHg * VD
    g = torch.Generator(device="cuda").manual_seed(99)
    be.gdn_setup(0, GDN_B, (torch.randn(CD, 4, generator=g, device="cuda") * 0.3).cpu().numpy(),
                 (torch.rand(VHg, generator=g, device="cuda") * 2.77).cpu().numpy(),
                 torch.randn(VHg, generator=g, device="cuda").cpu().numpy(),
                 (1 + 0.1 * torch.randn(VD, generator=g, device="cuda")).cpu().numpy())
    qkv = torch.randn(GDN_B, CD, generator=g, device="cuda").bfloat16()
    z = torch.randn(GDN_B, VHg * VD, generator=g, device="cuda").bfloat16()
    a = torch.randn(GDN_B, VHg, generator=g, device="cuda").bfloat16()
    b = torch.randn(GDN_B, VHg, generator=g, device="cuda").bfloat16()
    y = torch.empty(GDN_B, VHg * VD, dtype=torch.bfloat16, device="cuda")
    n = max(20, args.steps // 5)

    def step():
        be.gdn_decode_dev(0, GDN_B, qkv.data_ptr(), z.data_ptr(), a.data_ptr(), b.data_ptr(),
                          y.data_ptr(), 16, 128, 32, 128, 1e-6, 1)
    for _ in range(max(3, args.warmup)):
        step()
    be.sync()
    be.ktimer_enable(True)
    be.ktimer_read(be.K_GDN_DECODE)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(n):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    be.ktimer_enable(False)
    kms, kn = be.ktimer_read(be.K_GDN_DECODE)
    ms = e0.elapsed_time(e1) / n
    bytes_ = GDN_B * GDN_BYTES_PER_REQ
    kavg = kms / max(kn, 1)
    return {"gdn_decode": {"metric": "GDN decode tok/s (one layer)", "batch": GDN_B,
                           "value": GDN_B / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms,
                           "kernel_us": kavg * 1e3,
                           "achieved_GBs": bytes_ / (kavg / 1e3) / 1e9,
                           "frac_of_hbm": bytes_ / (kavg / 1e3) / 1e9 / peak_hbm,
                           "bytes_per_step": bytes_}}


def _time(st, fn, n):
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(n):
        fn()
    e1.record(st)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n


def _time_graph(st, fn, n, reps=3):
    """Device time per call of fn with the n calls captured in one CUDA graph
    and the graph replayed: at a few microseconds per step a Python loop of
    library calls measures the host, not the GPU (a serving loop replays
    its decode step as a graph for the same reason). None when the capture
    fails; the caller then keeps the eager figure."""
    import torch
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st, capture_error_mode="thread_local"):
            for _ in range(n):
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            g.replay()
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (reps * n)
        del g
        return ms
    except Exception as e:   # noqa: BLE001 -- reported, the eager number stands
        print(f"graph capture failed: {type(e).__name__}: {e}", file=sys.stderr)
        torch.cuda.synchronize()
        return None


def _graph_entry(st, fn, n, ms_eager):
    """ms per step (graph replay where it captured, else eager) and the
    fields that say which."""
    ms_g = _time_graph(st, fn, n)
    if ms_g is None:
        return ms_eager, {"timing": "eager launches (graph capture failed)"}
    return ms_g, {"timing": f"CUDA graph of {n} steps, replayed", "ms_per_step_eager": ms_eager}


def run_gqa_grid(be, args, st, peak_hbm):
    """BASELINE config 2's grid: GQA decode at batch {1, 16, 64} x context
    {4096, 32768} (one layer, bf16 cache; the headline is the 64 x 32768 point)."""
    import torch
    out = {}
    g = torch.Generator(device="cuda").manual_seed(5)
    layer = 5
    for T in (4096, 32768):
        for B in (1, 16, 64):
            be.kv_ensure(layer, B, KH, T)
            be.gqa_norm_weight(layer, (0.1 * torch.randn(HD, generator=g, device="cuda")).cpu().numpy(),
                               (0.1 * torch.randn(HD, generator=g, device="cuda")).cpu().numpy())
            rows = torch.randn(KH * T, HD, generator=g, device="cuda").bfloat16()
            for r in range(B):
                be.kv_rows_dev(layer, r, 0, KH * T, rows.data_ptr(), rows.data_ptr(), 1)
            qg = torch.randn(B, H, 2 * HD, generator=g, device="cuda").bfloat16()
            k = torch.randn(B, KH, HD, generator=g, device="cuda").bfloat16()
            v = (torch.randn(B, KH, HD, generator=g, device="cuda") / 16).bfloat16()
            pos = torch.full((B,), T - 1, dtype=torch.int32, device="cuda")
            ctx = torch.empty(B, H, HD, dtype=torch.bfloat16, device="cuda")
            be.sync()

            def step():
                be.gqa_decode_dev(layer, B, qg.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(),
                                  ctx.data_ptr(), H, KH, HD, ROT, EPS, THETA, 1)
            for _ in range(5):
                step()
            be.sync()
            n = 50 if B * T >= 64 * 4096 else 200
            ms, how = _graph_entry(st, step, n, _time(st, step, n))
            bytes_ = B * (2048 * T + 2048 + 16384 + 8192)
            out[f"gqa_decode_B{B}_T{T}"] = {"value": B / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms,
                                            "GBs": bytes_ / (ms / 1e3) / 1e9,
                                            "frac_of_hbm": bytes_ / (ms / 1e3) / 1e9 / peak_hbm,
                                            "l2_note": "inputs larger than L2" if bytes_ > 126e6 else
                                            "working set fits L2 (repeated steps re-read it from L2)",
                                            **how}
            del rows
            be.kv_reset()
    return {"gqa_decode_grid": out}


def run_gdn_grid(be, args, st, peak_hbm):
    """BASELINE config 3's grid: GatedDeltaNet decode at batch {1, 64, 256}."""
    import torch
    KHg, KD, VHg, VD = 16, 128, 32, 128
    CD = 2 * KHg * KD + VHg * VD
    out = {}
    g = torch.Generator(device="cuda").manual_seed(6)
    for B in (1, 64, 256):
        be.gdn_setup(6, B, (torch.randn(CD, 4, generator=g, device="cuda") * 0.3).cpu().numpy(),
                     (torch.rand(VHg, generator=g, device="cuda") * 2.77).cpu().numpy(),
                     torch.randn(VHg, generator=g, device="cuda").cpu().numpy(),
                     (1 + 0.1 * torch.randn(VD, generator=g, device="cuda")).cpu().numpy())
        qkv = torch.randn(B, CD, generator=g, device="cuda").bfloat16()
        z = torch.randn(B, VHg * VD, generator=g, device="cuda").bfloat16()
        a = torch.randn(B, VHg, generator=g, device="cuda").bfloat16()
        b = torch.randn(B, VHg, generator=g, device="cuda").bfloat16()
        y = torch.empty(B, VHg * VD, dtype=torch.bfloat16, device="cuda")

        def step():
            be.gdn_decode_dev(6, B, qkv.data_ptr(), z.data_ptr(), a.data_ptr(), b.data_ptr(), y.data_ptr(),
                              16, 128, 32, 128, 1e-6, 1)
        for _ in range(5):
            step()
        be.sync()
        ms, how = _graph_entry(st, step, 100, _time(st, step, 100))
        bytes_ = B * GDN_BYTES_PER_REQ
        out[f"gdn_decode_B{B}"] = {"value": B / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms,
                                   "GBs": bytes_ / (ms / 1e3) / 1e9,
                                   "frac_of_hbm": bytes_ / (ms / 1e3) / 1e9 / peak_hbm,
                                   "l2_note": "state larger than L2" if bytes_ > 126e6 else
                                   "state fits L2 (repeated steps re-read it from L2)", **how}
    return {"gdn_decode_grid": out}


def run_prefill_secondary(be, args, st, peak_tc):
    """Causal gated-GQA prefill of one layer, S in {8192,
    32768}, batch 1, bf16 q/k/v ~ N(0,1): prologue + tcgen05 flash kernel."""
    import torch
    out = {}
    layer = 1
    for S in [int(x) for x in args.lengths.split(",")]:
        be.kv_ensure(layer, 1, KH, S)
        g = torch.Generator(device="cuda").manual_seed(S)
        be.gqa_norm_weight(layer, (0.1 * torch.randn(HD, generator=g, device="cuda")).cpu().numpy(),
                           (0.1 * torch.randn(HD, generator=g, device="cuda")).cpu().numpy())
        qg = torch.randn(S, H, 2 * HD, generator=g, device="cuda").bfloat16()
        k = torch.randn(S, KH, HD, generator=g, device="cuda").bfloat16()
        v = torch.randn(S, KH, HD, generator=g, device="cuda").bfloat16()
        ctx = torch.empty(S, H, HD, dtype=torch.bfloat16, device="cuda")

        def step():
            be.gqa_step_dev(layer, 0, S, 0, qg.data_ptr(), k.data_ptr(), v.data_ptr(),
                            ctx.data_ptr(), H, KH, HD, ROT, EPS, THETA, 1)
        for _ in range(3):
            step()
        be.sync()
        reps = 10 if S <= 8192 else 4
        be.ktimer_enable(True)
        be.ktimer_read(be.K_GQA_PREFILL)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(_local_rank()) as clk:
            e0.record(st)
            for _ in range(reps):
                step()
            e1.record(st)
            torch.cuda.synchronize()
        be.ktimer_enable(False)
        kms, kn = be.ktimer_read(be.K_GQA_PREFILL)
        ms = e0.elapsed_time(e1) / reps
        flops = 8192.0 * S * (S + 1)
        kavg = kms / max(kn, 1)
        out[f"gqa_prefill_{S}"] = {
            "metric": "GQA prefill tok/s (one layer, causal)", "S": S, "value": S / (ms / 1e3),
            "unit": "tok/s", "ms_per_call": ms, "kernel_ms": kavg,
            "achieved_TFLOPs": flops / (kavg / 1e3) / 1e12,
            "frac_of_bf16_peak": flops / (kavg / 1e3) / 1e12 / peak_tc, "clocks": clk.brief()}
        del qg, k, v, ctx
        be.kv_reset()
    return out


def run_gdn_prefill_secondary(be, args, st, peak_hbm):
    """GatedDeltaNet chunk-64 prefill of one layer, batch 1,
    bf16 inputs, zero initial state and conv history, fp32 state.
    Algorithmic bytes = S x 32,896 (qkv, z, a, b in; y out; bf16) + 2 MiB state."""
    import torch
    KHg, KD, VHg, VD = 16, 128, 32, 128
    CD = 2 * KHg * KD + VHg * VD
    out = {}
    g = torch.Generator(device="cuda").manual_seed(7)
    be.gdn_setup(2, 1, (torch.randn(CD, 4, generator=g, device="cuda") * 0.3).cpu().numpy(),
                 (torch.rand(VHg, generator=g, device="cuda") * 2.77).cpu().numpy(),
                 torch.randn(VHg, generator=g, device="cuda").cpu().numpy(),
                 (1 + 0.1 * torch.randn(VD, generator=g, device="cuda")).cpu().numpy())
    nkh = args.gdn_kheads or KHg          # K heads this GPU owns (a head shard when < 16)
    if nkh != KHg:
        assert be.lib.coli_cuda_gdn_state_ensure(2, 1, 2 * nkh, KD, VD) == 1
    for S in [int(x) for x in args.lengths.split(",")]:
        qkv = torch.randn(S, CD, generator=g, device="cuda").bfloat16()
        z = torch.randn(S, VHg * VD, generator=g, device="cuda").bfloat16()
        a = torch.randn(S, VHg, generator=g, device="cuda").bfloat16()
        b = torch.randn(S, VHg, generator=g, device="cuda").bfloat16()
        y = torch.empty(S, 2 * nkh * VD, dtype=torch.bfloat16, device="cuda")

        def call():
            if nkh == KHg:
                be.gdn_prefill_dev(2, 0, S, qkv.data_ptr(), z.data_ptr(), a.data_ptr(), b.data_ptr(),
                                   y.data_ptr(), KHg, KD, VHg, VD, 1e-6, 1)
            else:
                be.gdn_prefill_heads_dev(2, 0, S, qkv.data_ptr(), z.data_ptr(), a.data_ptr(),
                                         b.data_ptr(), y.data_ptr(), 0, nkh)

        def step():
            be.gdn_reset()
            call()
        for _ in range(2):
            step()
        be.sync()
        reps = 10 if S <= 8192 else 5
        be.ktimer_enable(True)
        be.ktimer_read(be.K_GDN_PREFILL)
        # back-to-back calls in one event pair (the state carried from call to
        # call, as consecutive prompts or layers would): single calls after
        # an idle gap measured 5-10 % apart from run to run on this pool
        be.gdn_reset()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(_local_rank()) as clk:
            e0.record(st)
            for _ in range(reps):
                call()
            e1.record(st)
            torch.cuda.synchronize()
        be.ktimer_enable(False)
        be.ktimer_read(be.K_GDN_PREFILL)
        ms = e0.elapsed_time(e1) / reps
        bytes_ = (S * 32896 + 2 * 1024 * 1024) * nkh // KHg
        out[f"gdn_prefill_{S}" + (f"_kheads{nkh}" if nkh != KHg else "")] = {
            "metric": "GDN chunked prefill tok/s (one layer)", "S": S, "k_heads": nkh,
            "value": S / (ms / 1e3),
            "unit": "tok/s", "ms_per_call": ms, "achieved_GBs": bytes_ / (ms / 1e3) / 1e9,
            "frac_of_hbm": bytes_ / (ms / 1e3) / 1e9 / peak_hbm, "clocks": clk.brief()}
        del qkv, z, a, b, y
    return out


def _dist():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def run_stack_decode(be, args, st, peak_hbm):
    """BASELINE config 5 (i): the 40-layer mixer stack (30 GDN + 10 gated GQA)
    decoding one token for a batch of 256 requests at context 32768, sharded
    by request over the GPUs (no collective on the data path). 256 requests do
    not fit one GPU (~175 GiB of KV + state), so one GPU runs 128 and the
    per-request rate is what scales."""
    import torch
    pkg = _pkg()
    ws, rank = _dist()
    total = args.stack_batch
    b0, b1 = pkg.sharding.request_shard(total, ws, rank)
    B = min(b1 - b0, 128)
    stack = pkg.stack.MixerStack(be, seed=1000 + rank)
    stack.setup_decode(B, T_CTX)
    for _ in range(max(3, args.warmup // 4)):
        stack.decode_step()
    torch.cuda.synchronize()
    barrier(ws)
    n = max(5, args.steps // 50)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(n):
        stack.decode_step()
    e1.record(st)
    torch.cuda.synchronize()
    ms = pkg.sharding.max_over_ranks(e0.elapsed_time(e1) / n)
    reqs = B * ws
    bytes_ = stack.decode_bytes_per_request() * B
    return {"stack_decode": {
        "metric": "40-layer mixer stack decode tok/s", "requests_total": reqs,
        "requests_per_gpu": B, "context": T_CTX, "n_gpus": ws, "value": reqs / (ms / 1e3),
        "unit": "tok/s", "ms_per_step": ms, "per_gpu_GBs": bytes_ / (ms / 1e3) / 1e9,
        "frac_of_hbm": bytes_ / (ms / 1e3) / 1e9 / peak_hbm, "steps": n}}


def run_linear(be, args, st, peak_hbm):
    """Dense projections of one block (hidden 2048, BASELINE config 1 shapes) on
    the tcgen05 linear kernel: decode (S = 1, 64: weight streaming, HBM bound)
    and prefill (S = 4096: tensor bound). Six copies of each weight are
    rotated so every call streams its weights from HBM (> L2)."""
    import torch
    import numpy as np
    pkg = _pkg()
    _, peak_tc, _ = _peaks()
    shapes = {"gqa_q_gate": (8192, 2048), "gqa_o": (2048, 4096), "gdn_qkv": (8192, 2048),
              "gdn_z": (4096, 2048), "gdn_out": (2048, 4096)}
    out = {}
    rng = np.random.default_rng(3)
    for name, (O, I) in shapes.items():
        ts = [pkg.coli_cuda.DenseTensor(be, (rng.standard_normal((O, I), dtype=np.float32) * 0.02))
              for _ in range(6)]
        for S in (1, 64, 4096):
            x = torch.randn(S, I, device="cuda").bfloat16()
            y = torch.empty(S, O, device="cuda", dtype=torch.bfloat16)
            for i in range(6):
                be.matmul_dev(ts[i], x.data_ptr(), S, y.data_ptr(), 1)
            reps = 30 if S < 4096 else 10
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            be.sync()
            e0.record(st)
            for i in range(reps):
                be.matmul_dev(ts[i % 6], x.data_ptr(), S, y.data_ptr(), 1)
            e1.record(st)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / reps * 1e3
            wbytes = O * I * 2 + S * (I + O) * 2
            out[f"{name}_S{S}"] = {"O": O, "I": I, "S": S, "us": us,
                                   "GBs": wbytes / us / 1e3, "frac_of_hbm": wbytes / us / 1e3 / peak_hbm,
                                   "TFLOPs": 2.0 * S * O * I / us / 1e6,
                                   "frac_of_bf16": 2.0 * S * O * I / us / 1e6 / peak_tc}
        for t in ts:
            t.free()
    # a decode step's input projections as the block calls issue them: one
    # launch for all weights of the layer (q|gate, k, v; qkv, z, a, b)
    for name, Os in {"gqa_in_S1_multi": (8192, 512, 512), "gdn_in_S1_multi": (8192, 4096, 32, 32)}.items():
        I = 2048
        sets = [[pkg.coli_cuda.DenseTensor(be, rng.standard_normal((O, I), dtype=np.float32) * 0.02) for O in Os]
                for _ in range(6)]
        x = torch.randn(1, I, device="cuda").bfloat16()
        ys = [torch.empty(1, O, device="cuda", dtype=torch.bfloat16) for O in Os]
        yp = [y.data_ptr() for y in ys]
        for i in range(6):
            be.matmul_multi_dev(sets[i], x.data_ptr(), 1, yp, 1)
        reps = 30
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        be.sync()
        e0.record(st)
        for i in range(reps):
            be.matmul_multi_dev(sets[i % 6], x.data_ptr(), 1, yp, 1)
        e1.record(st)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / reps * 1e3
        wbytes = sum(O * I * 2 + (I + O) * 2 for O in Os)
        out[name] = {"O": list(Os), "I": I, "S": 1, "us": us, "GBs": wbytes / us / 1e3,
                     "frac_of_hbm": wbytes / us / 1e3 / peak_hbm}
        for ts in sets:
            for t in ts:
                t.free()
    return {"linear": out}


def run_stack_prefill(be, args, st, peak_tc):
    """BASELINE config 5 (ii): prefill of one 32k-token prompt through the
    40-layer mixer stack, heads sharded over the GPUs; each layer's output is
    gathered by the output kernels' peer stores over NVLink (or, with
    --nccl-gather, by an NCCL all-gather after the layer)."""
    import torch
    pkg = _pkg()
    ws, rank = _dist()
    S = int(args.lengths.split(",")[-1])
    stack = pkg.stack.MixerStack(be, seed=7)
    fused = ws > 1 and not args.nccl_gather
    stack.setup_prefill(S, ws, rank, fused=fused)
    stack.prefill()
    torch.cuda.synchronize()
    barrier(ws)
    reps = 2
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        be.gdn_reset()
        stack.prefill()
    e1.record(st)
    torch.cuda.synchronize()
    ms = pkg.sharding.max_over_ranks(e0.elapsed_time(e1) / reps)
    flops, gdn_bytes = stack.prefill_flops_bytes()
    stack.close_prefill()
    return {"stack_prefill": {
        "metric": "40-layer mixer stack prefill tok/s", "S": S, "n_gpus": ws,
        "value": S / (ms / 1e3), "unit": "tok/s", "ms": ms,
        "gqa_TFLOP": flops / 1e12, "gdn_GB": gdn_bytes / 1e9,
        "parallelism": f"heads sharded over {ws} GPU(s); layer outputs gathered by "
                       + ("peer stores in the output kernels + a device barrier per layer" if fused
                          else "NCCL all-gather per layer")}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--requests", type=int, default=B_REQ, help="decode requests per GPU")
    ap.add_argument("--context", type=int, default=T_CTX, help="decode context length")
    ap.add_argument("--quick", action="store_true",
                    help="headline kernel only (no e2e / secondary / CPU legs), for profiling")
    ap.add_argument("--only", choices=["gdn", "prefill", "gdnprefill", "stack", "stackprefill", "linear",
                                       "gqagrid", "gdngrid"],
                    default=None,
                    help="run one secondary leg alone and print its JSON (profiling)")
    ap.add_argument("--lengths", default="8192,32768", help="prefill lengths of the secondary legs")
    ap.add_argument("--gdn-kheads", type=int, default=0,
                    help="GDN prefill leg: K heads owned by this GPU (e.g. 2 = one rank of an 8-way head shard)")
    ap.add_argument("--stack-batch", type=int, default=256, help="stack decode requests (all GPUs)")
    ap.add_argument("--no-stack", action="store_true", help="skip the 40-layer stack legs of the default run")
    ap.add_argument("--nccl-gather", action="store_true",
                    help="stack prefill: gather layer outputs with NCCL instead of the fused peer stores")
    args = ap.parse_args()
    globals()["B_REQ"], globals()["T_CTX"] = args.requests, args.context
    if args.quick:
        args.no_cpu = True
    if args.warmup < 3:
        args.warmup = 3
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            reference_arm(args)
        return
    ws, rank, local = dist_setup()
    run_ours(args, ws, rank, local)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
