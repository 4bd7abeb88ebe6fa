"""Benchmark: GGUF block-quantized decode GEMV and prefill GEMM on B200.

Headline (one "step" = one decode token, M = 1, through L = 32 Llama-3-8B-shaped
layers, each with 7 projections):
  q, o  [4096 x 4096]  Q4_K     k [1024 x 4096]  Q4_K     v [1024 x 4096]  Q6_K
  gate, up [14336 x 4096] Q4_K  down [4096 x 14336] Q6_K          (138.9 MB / layer)
Weights are N(0, 0.02) quantized on the host by planejaja_b200.quantize (seed
1000 + projection index), activations N(0, 1) (seed 2000 + activation index);
synthetic data and random-init weights stand in for the Llama checkpoints.  The
32 layers are distinct device copies (4.44 GB), so every step streams far more
than the 126 MB L2 and consecutive steps never hit in L2.

Per layer, one fused GEMV launch per shared activation: q|k|v (attention
input), o, gate|up (FFN input), down -- 4 launches (down's K = 14336
activations quantised by a separate preparation kernel, the others on chip).
A step is captured once as a CUDA graph and replayed.

metric  : decode GEMV HBM GB/s = (weight bytes + fp32 activations + fp32
          outputs) of the whole step / step time (max over ranks), all ranks.
e2e     : the same step through the C-ABI calls with host buffers: pinned-host
          -> device copy of the step's activation vectors, the GEMVs, device ->
          pinned-host copies of all outputs of all layers (each layer's outputs
          copied by a second stream as soon as the layer is done, overlapped
          with the later layers), stream sync.
roofline: dominant kernel = the fused M = 1 Q4_K gate|up launch (2 x [14336 x
          4096], 66.19 MB), timed alone with CUDA events over the 32 layer
          copies; bound = HBM, peak = MEASURED_PEAKS.json hbm_gbs.  "kernels"
          gives the same for each of the step's four launches.
workloads (N = 1): the other configurations, one record each -- Llama-3-8B at
          M = 4 and 16, the same step with v and down in the reference's own
          Q6_K layout (NODESTOR, dequant_q6k.comp), Llama-2-7B Q4_0, and the
          Llama-2-70B FFN (gate|up [28672 x 8192], down [8192 x 28672], Q4_K)
          at M = 1 and 16.
prefill : the tcgen05 GEMM on Q4_K [14336 x 4096] and Q6_K [4096 x 14336] (both
          layouts) at M = 128 / 512 / 2048 tokens, TFLOP/s against the measured
          bf16 peak.
cpu_baseline: the CPU oracle (C restatement of the reference's dequant +
          cpu_matmul_f32) on one layer, all host threads, rows walked
          contiguously; cpu_baseline_single: the reference's own loop order on
          one pinned core (dequant, transpose to [K x N], cpu_matmul_f32 with
          stride-N reads of B).

--gpus N > 1 (torchrun, one process per GPU): the headline is N independent
replicas of the Llama-3-8B step (weak scaling: an 8B model fits one GPU and is
served by replicas; no collective).  The tensor-parallel forms are
"tp_workloads" (strong scaling): every projection row-sharded across the ranks,
each GEMV storing its output rows into every rank's buffer over NVLink (the
all-gather fused into the GEMV, nsq_gemv_multi_xchg) -- the Llama-3-8B step and
the Llama-2-70B FFN at M = 1 and 16 -- plus the 70B FFN with an NCCL all_gather
after each GEMV instead.

--impl reference times that CPU path alone (the reference is Rust/Vulkan;
neither toolchain nor a Vulkan driver exists on the box) on the same workload,
a bounded sample per step.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import multiprocessing
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, KV, FFN = 4096, 1024, 14336
# Workloads: projections (name, N_out, K, ggml_type) of one layer, which
# activation feeds each, the fused launches (activation index, names).
WORKLOADS = {
    "l3-8b": {
        "spec": [("q", HIDDEN, HIDDEN, 12), ("k", KV, HIDDEN, 12), ("v", KV, HIDDEN, 14), ("o", HIDDEN, HIDDEN, 12),
                 ("gate", FFN, HIDDEN, 12), ("up", FFN, HIDDEN, 12), ("down", HIDDEN, FFN, 14)],
        "act_of": {"q": 0, "k": 0, "v": 0, "o": 1, "gate": 2, "up": 2, "down": 3},
        "act_k": [HIDDEN, HIDDEN, HIDDEN, FFN],
        "groups": [(0, ["q", "k", "v"]), (1, ["o"]), (2, ["gate", "up"]), (3, ["down"])],
        "layers": 32,
        "metric": "decode GEMV HBM GB/s (Llama-3-8B Q4_K_M, M={m})",
        "desc": "llama3-8b Q4_K_M decode, M={m}, {layers} layers x 7 projections per step",
    },
    # Llama-2-7B, Q4_0 everywhere (q, k, v, o [4096 x 4096], gate / up
    # [11008 x 4096], down [4096 x 11008]; 113.8 MB per layer)
    "l2-7b": {
        "spec": [("q", 4096, 4096, 2), ("k", 4096, 4096, 2), ("v", 4096, 4096, 2), ("o", 4096, 4096, 2),
                 ("gate", 11008, 4096, 2), ("up", 11008, 4096, 2), ("down", 4096, 11008, 2)],
        "act_of": {"q": 0, "k": 0, "v": 0, "o": 1, "gate": 2, "up": 2, "down": 3},
        "act_k": [4096, 4096, 4096, 11008],
        "groups": [(0, ["q", "k", "v"]), (1, ["o"]), (2, ["gate", "up"]), (3, ["down"])],
        "layers": 32,
        "metric": "decode GEMV HBM GB/s (Llama-2-7B Q4_0, M={m})",
        "desc": "llama2-7b Q4_0 decode, M={m}, {layers} layers x 7 projections per step",
    },
    # Llama-2-70B FFN, Q4_K (gate/up [28672 x 8192], down [8192 x 28672])
    "l2-70b-ffn": {
        "spec": [("gate", 28672, 8192, 12), ("up", 28672, 8192, 12), ("down", 8192, 28672, 12)],
        "act_of": {"gate": 0, "up": 0, "down": 1},
        "act_k": [8192, 28672],
        "groups": [(0, ["gate", "up"]), (1, ["down"])],
        "layers": 8,
        "metric": "decode GEMV HBM GB/s (Llama-2-70B FFN Q4_K, M={m})",
        "desc": "llama2-70b FFN Q4_K decode, M={m}, {layers} layers x 3 projections per step",
    },
}
LAYER_SPEC = WORKLOADS["l3-8b"]["spec"]
ACT_OF = WORKLOADS["l3-8b"]["act_of"]
ACT_K = WORKLOADS["l3-8b"]["act_k"]
GROUPS = WORKLOADS["l3-8b"]["groups"]
WORKLOAD = "l3-8b"
M_TOK = 1
SEED_W, SEED_X = 1000, 2000
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
METRIC = "decode GEMV HBM GB/s (Llama-3-8B Q4_K_M, M=1)"
UNIT = "GB/s"
PREFILL_SHAPES = [("Q4_K", 14336, 4096, 12, 0), ("Q6_K", 4096, 14336, 14, 0), ("Q6_K_nodestor", 4096, 14336, 14, 1)]
PREFILL_M = [128, 512, 2048]
POOL = None  # spawn-started process pool for host-side quantisation (before any GPU call)
_HOST_CACHE = {}


def select_workload(name: str, m: int) -> None:
    """Rebinds the module-level workload description (before any leg runs)."""
    global LAYER_SPEC, ACT_OF, ACT_K, GROUPS, WORKLOAD, M_TOK, METRIC
    w = WORKLOADS[name]
    LAYER_SPEC, ACT_OF, ACT_K, GROUPS = w["spec"], w["act_of"], w["act_k"], w["groups"]
    WORKLOAD, M_TOK = name, m
    METRIC = w["metric"].format(m=m)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def workload_bytes(name: str, m: int):
    """(weight, activation, output) bytes of one layer of a workload."""
    from planejaja_b200.formats import fmt
    spec = WORKLOADS[name]["spec"]
    w = sum(fmt(t).tensor_bytes(n, k) for _, n, k, t in spec)
    x = sum(m * k * 4 for _, n, k, t in spec)
    y = sum(m * n * 4 for _, n, k, t in spec)
    return w, x, y


def layer_bytes_total():
    return workload_bytes(WORKLOAD, M_TOK)


def _quant_job(job):
    from planejaja_b200 import quantize as Q
    key, n, k, t, seed, layout, rows = job
    return key, Q.synthetic_weights(n, k, t, seed=seed, q6k_layout=layout, rows=rows)


def host_weights(name: str, q6k_layout: int = 0, world: int = 1, rank: int = 0):
    """Quantized bytes of one layer, {projection: uint8 array}; with world > 1
    only this rank's row shard of each matrix (a contiguous byte range)."""
    key = (name, q6k_layout, world, rank)
    if key in _HOST_CACHE:
        return _HOST_CACHE[key]
    jobs = []
    for i, (nm, n, k, t) in enumerate(WORKLOADS[name]["spec"]):
        rows = None if world == 1 else (rank * n // world, (rank + 1) * n // world)
        jobs.append((nm, n, k, t, SEED_W + i, q6k_layout if t in (13, 14) else 0, rows))
    out = dict(POOL.map(_quant_job, jobs)) if POOL is not None else dict(map(_quant_job, jobs))
    _HOST_CACHE[key] = out
    return out


def host_layer():
    """Quantized bytes of one layer of the selected workload."""
    return host_weights(WORKLOAD)


def host_acts(name: str = None, m: int = None):
    from planejaja_b200 import quantize as Q
    name, m = name or WORKLOAD, m or M_TOK
    return [Q.synthetic_activations(m, k, seed=SEED_X + i).reshape(-1)
            for i, k in enumerate(WORKLOADS[name]["act_k"])]


class ClockSampler:
    """Samples SM clock and throttle reasons with NVML in a background thread."""

    def __init__(self, index: int, period: float = 0.005):
        self.index, self.period = index, period
        self.samples, self.reasons = [], set()
        self._stop = threading.Event()
        self._t = None
        self.max_mhz = None

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
        except Exception:
            self.nv = None
            return self
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def _run(self):
        nv = self.nv
        names = {
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, bit in names.items():
                    if r & bit:
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


# --------------------------------------------------------------------------- CPU (oracle) legs
def cpu_leg(layer, acts, rows_frac: float = 1.0, reps: int = 1, threads: int = 0, min_seconds: float = 0.0):
    """Time the oracle's dequant + cpu_matmul_f32 composition over (a row
    sample of) one layer, rows walked contiguously, `reps` times or until
    `min_seconds` have passed; returns (GB/s, bytes, seconds, threads)."""
    from oracle import oracle as O
    from planejaja_b200.formats import fmt
    O.build()
    th = threads or O.num_threads()
    jobs = []
    for name, n, k, t in LAYER_SPEC:
        rb = fmt(t).row_bytes(k)
        nr = max(1, int(n * rows_frac))
        jobs.append((layer[name][: nr * rb], t, acts[ACT_OF[name]], nr, k))
    nbytes = sum(j[0].nbytes + j[4] * 4 + j[3] * 4 for j in jobs)
    w0, t0_, x0, _, k0 = jobs[0]
    O.quant_matmul(w0[: fmt(t0_).row_bytes(k0)], t0_, x0, 1, k0, threads=th)  # warm
    t0 = time.perf_counter()
    done = 0
    while done < reps or time.perf_counter() - t0 < min_seconds:
        for w, t, x, nr, k in jobs:
            O.quant_matmul(w, t, x, nr, k, threads=th)
        done += 1
    dt = time.perf_counter() - t0
    return nbytes * done / dt / 1e9, nbytes * done, dt, th


def cpu_leg_reference_loop(layer, acts):
    """The reference's own CPU path, single-threaded and pinned to one core:
    each matrix dequantized to f32 (Q4_K through the AVX2 restatement of
    simd_x86.rs, the other formats through their scalar restatements),
    transposed to the [K x N] layout cpu_matmul_f32 takes, then
    cpu_matmul_f32's i-j-l loop with stride-N reads of B
    (pipeline.rs:1256-1268).  Returns the record for the bench line."""
    from oracle import oracle as O
    O.build()
    old = os.sched_getaffinity(0)
    core = min(old)
    os.sched_setaffinity(0, {core})
    try:
        t_dq = t_tr = t_mm = 0.0
        nbytes = 0
        for name, n, k, t in LAYER_SPEC:
            w, x = layer[name], acts[ACT_OF[name]]
            s = time.perf_counter()
            wf = O.dequant_q4_k_avx2(w) if t == 12 else O.dequant(w, t)
            t_dq += time.perf_counter() - s
            s = time.perf_counter()
            b = np.ascontiguousarray(wf.reshape(n, k).T)
            t_tr += time.perf_counter() - s
            s = time.perf_counter()
            O.matmul_f32(x.reshape(-1, k), b, x.size // k, k, n)
            t_mm += time.perf_counter() - s
            nbytes += w.nbytes + x.nbytes + (x.size // k) * n * 4
            del wf, b
    finally:
        os.sched_setaffinity(0, old)
    total = t_dq + t_tr + t_mm
    return {"value": round(nbytes / total / 1e9, 4), "unit": UNIT, "cores": 1, "kind": "port",
            "loop": "reference order: dequant, transpose to [K x N], cpu_matmul_f32 i-j-l with stride-N B reads",
            "pinned": f"sched_setaffinity to core {core}",
            "sample": f"one whole layer ({nbytes / 1e6:.1f} MB of weights and activations)",
            "dequant_s": round(t_dq, 3), "transpose_s": round(t_tr, 3), "matmul_s": round(t_mm, 3)}


def run_reference(args, rank, world):
    """--impl reference: the CPU restatement of the reference path, timed on the host."""
    if rank != 0:
        return
    layer, acts = host_layer(), host_acts()
    for _ in range(args.warmup):
        cpu_leg(layer, acts, rows_frac=args.ref_frac)
    vals, secs = [], 0.0
    for _ in range(args.steps):
        v, nb, dt, th = cpu_leg(layer, acts, rows_frac=args.ref_frac)
        vals.append(v)
        secs += dt
    w, x, y = layer_bytes_total()
    value = float(np.mean(vals))
    out = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * secs / max(1, args.steps), 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOADS[WORKLOAD]["desc"].format(m=M_TOK, layers=1),
                   "sample": f"{args.ref_frac:.4f} of the rows of each of the {len(LAYER_SPEC)} matrices of one "
                             f"layer per step",
                   "layers_per_step": 1, "batch": M_TOK},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": th, "kind": "port",
                         "loop": "rows walked contiguously (each W row dequantized once, its dot product in "
                                 "cpu_matmul_f32's order), all host threads; the reference's own loop is "
                                 "single-threaded with stride-N reads and slower",
                         "sample": f"{args.ref_frac:.4f} of one layer's rows per step "
                                   f"({(w * args.ref_frac) / 1e6:.1f} MB of weights)"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


# --------------------------------------------------------------------------- GPU legs
class Ctx:
    """Per-rank GPU context shared by the legs."""

    def __init__(self, world, rank, local_rank):
        import torch
        from planejaja_b200.engine import CudaEngine
        self.world, self.rank, self.local_rank = world, rank, local_rank
        self.dev = torch.device("cuda", local_rank)
        torch.cuda.set_device(self.dev)
        self.eng = CudaEngine(local_rank)
        self.lib = self.eng.lib
        self.launches = 0

    def barrier(self):
        import torch.distributed as dist
        if self.world > 1:
            dist.barrier(device_ids=[self.local_rank])

    def max_over_ranks(self, v):
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())


class DecodeStep:
    """One decode step of a workload on this rank: L distinct layer copies, one
    fused GEMV launch per shared activation, captured as one CUDA graph.

    mode "single": every matrix whole on this GPU (N = 1, or one replica per
    rank); "p2p": rows sharded over the ranks, all-gather fused into the GEMV;
    "nccl": rows sharded, an NCCL all_gather after each GEMV."""

    def __init__(self, ctx, name, m, L, mode="single", q6k_layout=0, graph=True):
        import torch
        import torch.distributed as dist
        from planejaja_b200 import _lib
        from planejaja_b200.formats import fmt
        self.ctx, self.name, self.m, self.L, self.mode = ctx, name, m, L, mode
        wl = WORKLOADS[name]
        self.spec, self.groups, self.act_k = wl["spec"], wl["groups"], wl["act_k"]
        eng, lib, dev = ctx.eng, ctx.lib, ctx.dev
        world, rank = (ctx.world, ctx.rank) if mode != "single" else (1, 0)
        self.world = world
        hw = host_weights(name, q6k_layout, world, rank)
        self.type_of = {nm: t for nm, n, k, t in self.spec}
        self.n_of = {nm: n for nm, n, k, t in self.spec}
        self.layout_of = {nm: (q6k_layout if t in (13, 14) else 0) for nm, n, k, t in self.spec}
        rows_of = {nm: n // world for nm, n, k, t in self.spec}
        base = {nm: eng.upload(hw[nm]) for nm in hw}
        del hw
        self.layers = [{nm: (rows_of[nm], b if li == 0 else b.clone()) for nm, b in base.items()} for li in range(L)]
        self.acts_h = host_acts(name, m)
        self.acts = [torch.from_numpy(a).to(dev) for a in self.acts_h]
        M = m

        def flat_views(sizes):
            flat = torch.empty(L * sum(M * n for _, n in sizes), dtype=torch.float32, device=dev)
            views, off = [], 0
            for _ in range(L):
                d = {}
                for nm, n in sizes:
                    d[nm] = flat[off:off + M * n]
                    off += M * n
                views.append(d)
            return flat, views

        self.outs_local_flat, self.outs_local = flat_views([(nm, rows_of[nm]) for nm, n, k, t in self.spec])
        self.ws = eng.workspace(lib.nsq_gemv_workspace_size(M, max(self.act_k)))
        self.exchange = None
        if mode == "p2p":
            from planejaja_b200.sharded import Exchange, OutputLayout, xsegments
            layout = OutputLayout()
            for li in range(L):
                for nm, n, k, t in self.spec:
                    layout.add((li, nm), M, n)
            self.exchange = Exchange(layout.nbytes)
            self.out_dev = torch.as_tensor(self.exchange.view(0, (layout.nbytes // 4,)))
        elif mode == "nccl":
            self.outs_full_flat, self.outs_full = flat_views([(nm, n) for nm, n, k, t in self.spec])
            self.out_dev = self.outs_full_flat
        else:
            self.out_dev = self.outs_local_flat
        self.calls = []  # per layer, per fused launch: (activation index, names, ctypes array)
        for li in range(L):
            per = []
            for a, names in self.groups:
                if mode == "p2p":
                    arr = xsegments([(self.layers[li][nm][1].data_ptr(), self.type_of[nm], self.layout_of[nm],
                                      rows_of[nm], rank * rows_of[nm], self.n_of[nm],
                                      layout.offsets[(li, nm)][0]) for nm in names])
                else:
                    arr = (_lib.Segment * len(names))()
                    for i, nm in enumerate(names):
                        arr[i] = _lib.Segment(self.layers[li][nm][1].data_ptr(), self.type_of[nm], self.layout_of[nm],
                                              rows_of[nm], self.outs_local[li][nm].data_ptr())
                per.append((a, names, arr))
            self.calls.append(per)
        wb = sum(fmt(t).tensor_bytes(n, k) for _, n, k, t in self.spec)
        xb = sum(M * k * 4 for _, n, k, t in self.spec)
        yb = sum(M * n * 4 for _, n, k, t in self.spec)
        self.step_bytes = (wb + xb + yb) * L  # the whole job's bytes (all ranks together when sharded)
        self.weight_bytes = wb * L
        self.n_launch = 0
        self.graph = None
        self._dist = dist
        self.step()
        torch.cuda.synchronize()
        if graph:
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                self.step()
            torch.cuda.current_stream(dev).wait_stream(s)
            torch.cuda.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=s):
                self.step()
            torch.cuda.synchronize()

    def launch(self, li, gi, st):
        """One fused launch (layer li, launch gi) on stream st."""
        lib, M = self.ctx.lib, self.m
        a, names, arr = self.calls[li][gi]
        if self.mode == "p2p":
            rc = lib.nsq_gemv_multi_xchg(ctypes.cast(arr, ctypes.c_void_p), len(names), self.acts[a].data_ptr(), M,
                                         self.act_k[a], self.exchange.comm, self.ws.data_ptr(), self.ws.numel(), st)
        else:
            rc = lib.nsq_gemv_multi(ctypes.cast(arr, ctypes.c_void_p), len(names), self.acts[a].data_ptr(), M,
                                    self.act_k[a], self.ws.data_ptr(), self.ws.numel(), st)
        assert rc == 0, rc

    def step(self, after_layer=None):
        import torch
        st = torch.cuda.current_stream(self.ctx.dev).cuda_stream
        k0 = self.ctx.lib.nsq_kernel_launches()  # libnsq's own kernels (NCCL's are not counted)
        for li in range(self.L):
            for gi, (a, names, arr) in enumerate(self.calls[li]):
                self.launch(li, gi, st)
                if self.mode == "nccl":
                    for nm in names:
                        self._dist.all_gather_into_tensor(self.outs_full[li][nm], self.outs_local[li][nm])
            if after_layer is not None:
                after_layer(li)
        if self.mode == "p2p":
            self.exchange.wait(st)  # the step ends when every rank's rows have landed here
        self.n_launch = self.ctx.lib.nsq_kernel_launches() - k0

    def run(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self.step()

    def time(self, steps, warmup):
        """ms per step, CUDA events, max over ranks (barrier + sync on both sides)."""
        import torch
        ctx = self.ctx
        for _ in range(warmup):
            self.run()
        torch.cuda.synchronize()
        ctx.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            self.run()
        e1.record()
        torch.cuda.synchronize()
        ctx.barrier()
        torch.cuda.synchronize()
        ctx.launches += self.n_launch * steps
        return ctx.max_over_ranks(e0.elapsed_time(e1)) / steps

    def _e2e_graph(self, out_pin):
        """One step captured with its outputs streamed back to pinned host memory
        layer by layer: after each layer's launches a second stream copies that
        layer's outputs while the compute stream goes on with the next layer."""
        import torch
        dev = self.ctx.dev
        per_layer = self.out_dev.numel() // self.L
        s, side = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        events = [torch.cuda.Event() for _ in range(self.L)]

        def after_layer(li):
            events[li].record(s)
            side.wait_event(events[li])
            with torch.cuda.stream(side):
                sl = slice(li * per_layer, (li + 1) * per_layer)
                out_pin[sl].copy_(self.out_dev[sl], non_blocking=True)

        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            side.wait_stream(s)  # the copy stream joins the capture
            self.step(after_layer)
            s.wait_stream(side)  # every copy is part of the step
        torch.cuda.synchronize()
        return g

    def time_e2e(self, steps, warmup):
        """The same step with pinned-host inputs copied in and all outputs read back, per step.
        Single-GPU steps copy each layer's outputs back as soon as the layer is done,
        overlapped with the later layers (one graph); sharded steps copy the whole
        output once the step's exchanges have landed."""
        import torch
        ctx, dev = self.ctx, self.ctx.dev
        acts_pin = [torch.from_numpy(a).pin_memory() for a in self.acts_h]
        out_pin = torch.empty(self.out_dev.numel(), dtype=torch.float32).pin_memory()
        overlapped = self.mode == "single" and self.graph is not None and self.out_dev.numel() % self.L == 0
        g = self._e2e_graph(out_pin) if overlapped else None

        def e2e_step():
            for a, src in enumerate(acts_pin):
                self.acts[a].copy_(src, non_blocking=True)
            if g is not None:
                g.replay()
            else:
                self.run()
                out_pin.copy_(self.out_dev, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()

        for _ in range(warmup):
            e2e_step()
        ctx.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        ctx.launches += self.n_launch * steps
        ms = ctx.max_over_ranks(e0.elapsed_time(e1)) / steps
        return ms, sum(a.numel() * 4 for a in acts_pin), out_pin.numel() * 4

    def kernel_alone(self, gi, reps_min=256):
        """One of the step's launches (index gi of a layer) alone, rotating over
        the layer copies: (us per launch, algorithmic bytes per launch)."""
        import torch
        from planejaja_b200.formats import fmt
        st = torch.cuda.current_stream(self.ctx.dev).cuda_stream
        a, names, _ = self.calls[0][gi]
        k = self.act_k[a]
        nbytes = sum(fmt(self.type_of[nm]).tensor_bytes(self.n_of[nm] // self.world, k) +
                     self.m * (self.n_of[nm] // self.world) * 4 for nm in names) + self.m * k * 4
        for li in range(self.L):
            self.launch(li, gi, st)
        torch.cuda.synchronize()
        reps = max(4, reps_min // self.L) * self.L
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            self.launch(i % self.L, gi, st)
        e1.record()
        torch.cuda.synchronize()
        self.ctx.launches += reps
        return e0.elapsed_time(e1) / reps * 1e3, nbytes

    def close(self):
        import torch
        self.graph = None
        torch.cuda.synchronize()
        if self.exchange is not None:
            # no rank may unmap its buffer while a peer can still store into it
            self.ctx.barrier()
            self.exchange.close()
            self.exchange = None
        self.layers = self.calls = None
        torch.cuda.empty_cache()


def workload_record(ctx, name, m, mode, steps, warmup, q6k_layout=0, hbm_peak=None):
    st = DecodeStep(ctx, name, m, WORKLOADS[name]["layers"], mode=mode, q6k_layout=q6k_layout)
    try:
        ms = st.time(steps, warmup)
        world = ctx.world
        # replicas: every rank streams the whole step; sharded: the step's bytes once
        total = st.step_bytes * (world if mode == "single" else 1)
        gbs = total / (ms * 1e-3) / 1e9
        rec = {"metric": WORKLOADS[name]["metric"].format(m=m), "value": round(gbs, 2), "unit": UNIT,
               "ms_per_step": round(ms, 4), "layers": st.L,
               "weight_bytes_per_step": st.weight_bytes, "q6k_layout": "nodestor" if q6k_layout else "ggml"}
        if hbm_peak:
            rec["frac_of_measured_hbm_per_gpu"] = round(gbs / world / hbm_peak, 4)
        if mode != "single":
            rec["scaling"] = "strong"
            rec["parallelism"] = (f"tp{world} row-sharded, all-gather fused into the GEMV (NVLink peer stores)"
                                  if mode == "p2p" else f"tp{world} row-sharded + NCCL all_gather per projection")
        return rec
    finally:
        st.close()


def prefill_records(ctx, bf16_peak, peak_kind, shapes=PREFILL_SHAPES, ms_list=PREFILL_M, reps=20):
    """tcgen05 GEMM TFLOP/s per (format, M), rotating over 4 weight copies."""
    import torch
    from planejaja_b200.formats import fmt
    eng, lib, dev = ctx.eng, ctx.lib, ctx.dev
    st = torch.cuda.current_stream(dev).cuda_stream
    out = []
    for label, n, k, t, lay in shapes:
        from planejaja_b200 import quantize as Q
        w0 = eng.upload(Q.synthetic_weights(n, k, t, seed=SEED_W + 4, q6k_layout=lay))
        ws = [w0] + [w0.clone() for _ in range(3)]
        for pm in ms_list:
            xp = torch.randn(pm, k, device=dev).to(torch.bfloat16)
            yp = torch.empty(pm, n, dtype=torch.bfloat16, device=dev)
            for i in range(3):
                assert lib.nsq_gemm_bf16(ws[i].data_ptr(), t, lay, xp.data_ptr(), yp.data_ptr(), pm, n, k, st) == 0
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(reps):
                lib.nsq_gemm_bf16(ws[i % 4].data_ptr(), t, lay, xp.data_ptr(), yp.data_ptr(), pm, n, k, st)
            e1.record()
            torch.cuda.synchronize()
            ctx.launches += reps
            ms = e0.elapsed_time(e1) / reps
            tf = 2.0 * pm * n * k / (ms * 1e-3) / 1e12
            out.append({"weights": f"{label} [{n}x{k}]", "M": pm, "tflops": round(tf, 1), "ms": round(ms, 4),
                        "frac": round(tf / bf16_peak, 4), "peak_tflops": bf16_peak, "peak_kind": peak_kind})
        del ws, w0
    torch.cuda.empty_cache()
    return out


# Single-kernel cases for profilers (bench.py --case NAME): a few launches of
# one kernel on one GPU, nothing timed.  (weights, ggml type, layout, N, K, M, kind)
CASES = {
    "gemv_gate_up_m1": ("2 x [14336 x 4096] Q4_K (Llama-3-8B gate|up)", 12, 0, 14336, 4096, 1, "gemv2"),
    "gemv_down_m1": ("[4096 x 14336] Q6_K (Llama-3-8B down)", 14, 0, 4096, 14336, 1, "gemv"),
    "gemv_down_nodestor_m1": ("[4096 x 14336] Q6_K NODESTOR layout", 14, 1, 4096, 14336, 1, "gemv"),
    "gemv_tc_70b_gate_up_m16": ("2 x [28672 x 8192] Q4_K at M = 16, tcgen05", 12, 0, 28672, 8192, 16, "gemv2"),
    "gemv_mma_70b_gate_up_m16": ("2 x [28672 x 8192] Q4_K at M = 16, mma.sync", 12, 0, 28672, 8192, 16, "gemv2_mma"),
    "gemm_q4k_m128": ("Q4_K [14336 x 4096], M = 128", 12, 0, 14336, 4096, 128, "gemm"),
    "gemm_q4k_m2048": ("Q4_K [14336 x 4096], M = 2048", 12, 0, 14336, 4096, 2048, "gemm"),
    "gemm_q6k_m512": ("Q6_K [4096 x 14336], M = 512", 14, 0, 4096, 14336, 512, "gemm"),
}


def run_case(name, reps):
    """Launches one case `reps` times (after one warm-up launch) on cuda:0."""
    import torch
    from planejaja_b200 import _lib
    from planejaja_b200 import quantize as Q
    from planejaja_b200.engine import CudaEngine
    desc, t, lay, n, k, m, kind = CASES[name]
    eng = CudaEngine(0)
    if kind == "gemv2_mma":  # the mma.sync kernel: switch the tcgen05 path off
        os.environ["NSQ_TC_MIN_M"] = "17"
        eng.lib.nsq_reload_tuning()
    w = eng.upload(Q.synthetic_weights(n, k, t, seed=SEED_W, q6k_layout=lay))
    w2 = w.clone() if kind.startswith("gemv2") else None
    for i in range(reps + 1):
        if kind == "gemm":
            x = torch.randn(m, k, device="cuda").to(torch.bfloat16) if i == 0 else x
            eng.gemm_bf16(w, t, x, n, k, lay)
        else:
            x = torch.from_numpy(host_acts_like(m, k)).cuda() if i == 0 else x
            if w2 is not None:
                eng.gemv_multi([(w, t, n, lay), (w2, t, n, lay)], x, k)
            else:
                eng.gemv(w, t, x, n, k, lay)
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    print(f"case {name}: {desc}, {reps + 1} launches", flush=True)


def host_acts_like(m, k):
    from planejaja_b200 import quantize as Q
    return Q.synthetic_activations(m, k, seed=SEED_X)


def run_gpu(args, rank, world, local_rank):
    import torch
    from planejaja_b200.formats import fmt

    ctx = Ctx(world, rank, local_rank)
    hbm_peak, bf16_peak, peak_kind = peaks()
    headline_mode = "single" if (world == 1 or not args.tp) else args.exchange
    result = {}
    with ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ else local_rank) as clk:
        step = DecodeStep(ctx, WORKLOAD, M_TOK, args.layers, mode=headline_mode, graph=not args.no_graph)
        ms = step.time(args.steps, args.warmup)
        total = step.step_bytes * (world if headline_mode == "single" else 1)
        value = total / (ms * 1e-3) / 1e9
        e2e_ms, h2d, d2h = step.time_e2e(args.steps, args.warmup)
        e2e_value = total / (e2e_ms * 1e-3) / 1e9
        wb, xb, yb = workload_bytes(WORKLOAD, M_TOK)
        result.update({
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak" if headline_mode == "single" else "strong", "vs_baseline": None,
            "dtype": "int8x2-dp4a/f32",
            "data": "synthetic (N(0,0.02) weights quantized on host; N(0,1) activations)",
            "config": {"workload": WORKLOADS[WORKLOAD]["desc"].format(m=M_TOK, layers=args.layers),
                       "layers": args.layers, "batch": M_TOK, "weight_bytes_per_step": wb * args.layers,
                       "parallelism": ("single GPU" if world == 1 else
                                       f"{world} independent replicas, one per GPU (no collective)"
                                       if headline_mode == "single" else
                                       f"tp{world} row-sharded, all-gather fused into the GEMV"),
                       "l2": f"inputs larger than L2: {args.layers} distinct layer copies, "
                             f"{wb * args.layers / 1e9:.2f} GB per step per replica",
                       "cuda_graph": step.graph is not None},
            "frac_of_nominal_8tbs": round(value / world / NOMINAL_HBM_GBS, 4),
            "frac_of_measured_hbm_per_gpu": round(value / world / hbm_peak, 4),
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms, 4)},
        })

        # ---- the step's launches alone; the dominant one (gate|up) is the roofline kernel
        if not args.skip_roofline and headline_mode == "single":
            kernels = {}
            for gi, (a, names) in enumerate(step.groups):
                us, nb = step.kernel_alone(gi)
                kernels["|".join(names)] = {"us_per_launch": round(us, 3), "bytes_per_launch": nb,
                                            "gbs": round(nb / (us * 1e-6) / 1e9, 1),
                                            "frac": round(nb / (us * 1e-6) / 1e9 / hbm_peak, 4)}
            result["kernels"] = kernels
            gk = [g for g in kernels if "gate" in g.split("|")][0]
            g = kernels[gk]
            gt = step.type_of["gate"]
            rows = step.n_of["gate"]
            KG = step.act_k[step.groups[[i for i, (_, nm) in enumerate(step.groups) if "gate" in nm][0]][0]]
            traffic = None
            tp = os.path.join(ROOT, "profiles", "traffic.json")
            if os.path.exists(tp) and M_TOK == 1 and world == 1:
                keys = {"l3-8b": "gemv_fused_q4k_m1_gate_up", "l2-7b": "gemv_fused_q40_m1_gate_up"}
                tr = json.load(open(tp))
                traffic = tr.get(keys.get(WORKLOAD, ""))
            result["roofline"] = {
                "bound": "hbm",
                "kernel": f"gemv_fused_kernel<M={M_TOK},{fmt(gt).name}> gate|up 2 x [{rows}x{KG}] (FFN input projection)",
                "achieved": g["gbs"], "peak": hbm_peak, "unit": "GB/s", "frac": g["frac"], "peak_kind": peak_kind,
                "frac_of_nominal_8tbs": round(g["gbs"] / NOMINAL_HBM_GBS, 4),
                "bytes_per_launch": g["bytes_per_launch"], "us_per_launch": g["us_per_launch"],
                "traffic": traffic,
                "traffic_source": ("dram__bytes_read.sum + dram__bytes_write.sum of one launch, copied from the ncu "
                                   "capture summarised in profiles/traffic.json (same kernel, not this run)")
                if traffic else None}
        n_head_launch = step.n_launch
        step.close()
        del step

        # ---- the other configurations
        if not args.no_sub and world == 1:
            subs = {}
            for key, (name, m, lay) in {"l3-8b_q6k_nodestor_m1": ("l3-8b", 1, 1), "l3-8b_m4": ("l3-8b", 4, 0),
                                        "l3-8b_m16": ("l3-8b", 16, 0), "l2-7b_m1": ("l2-7b", 1, 0),
                                        "l2-70b-ffn_m1": ("l2-70b-ffn", 1, 0),
                                        "l2-70b-ffn_m16": ("l2-70b-ffn", 16, 0)}.items():
                subs[key] = workload_record(ctx, name, m, "single", args.sub_steps, args.warmup, lay, hbm_peak)
            result["workloads"] = subs
            if not args.skip_roofline:
                result["prefill"] = prefill_records(ctx, bf16_peak, peak_kind)
        if not args.no_sub and world > 1:
            tps = {}
            for key, (name, m, mode) in {"tp_l3-8b_m1": ("l3-8b", 1, "p2p"),
                                         "tp_l2-70b-ffn_m1": ("l2-70b-ffn", 1, "p2p"),
                                         "tp_l2-70b-ffn_m16": ("l2-70b-ffn", 16, "p2p"),
                                         "tp_l2-70b-ffn_m1_nccl": ("l2-70b-ffn", 1, "nccl")}.items():
                tps[key] = workload_record(ctx, name, m, mode, args.sub_steps, args.warmup, 0, hbm_peak)
            result["tp_workloads"] = tps
    result["clocks"] = clk.summary()
    result["gpu_launches"] = n_head_launch * args.steps  # the headline's timed region
    result["gpu_launches_per_step"] = n_head_launch
    result["gpu_launches_all_legs"] = ctx.launches
    assert ctx.eng.device_status() == 0, "a bounded device wait timed out"

    # ---- CPU baselines (rank 0, N = 1)
    if rank == 0 and world == 1 and not args.skip_cpu:
        layer, acts_h = host_layer(), host_acts()
        v, nb, dt, th = cpu_leg(layer, acts_h, rows_frac=args.cpu_frac, reps=args.cpu_reps,
                                min_seconds=args.cpu_seconds)
        result["cpu_baseline"] = {"value": round(v, 3), "unit": UNIT, "cores": th, "kind": "port",
                                  "loop": "rows walked contiguously (each W row dequantized once, its dot product "
                                          "in cpu_matmul_f32's order), all host threads",
                                  "sample": f"oracle dequant + cpu_matmul_f32 over {args.cpu_frac:.3f} of the rows "
                                            f"of one layer's 7 matrices, repeated for >= {args.cpu_seconds:.0f} s "
                                            f"({nb / 1e6:.1f} MB in {dt:.1f} s)"}
        result["cpu_baseline_single"] = cpu_leg_reference_loop(layer, acts_h)
    if rank == 0:
        print(json.dumps(result), flush=True)


def main():
    global POOL
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--sub-steps", type=int, default=20, help="timed steps of each extra workload record")
    ap.add_argument("--impl", default="nsq", choices=["nsq", "reference"])
    ap.add_argument("--layers", type=int, default=None, help="layer copies per step (default: the workload's)")
    ap.add_argument("--workload", default="l3-8b", choices=sorted(WORKLOADS))
    ap.add_argument("--tokens", type=int, default=1, help="tokens per decode step, M (1..16)")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="headline only (no extra workloads, no prefill)")
    ap.add_argument("--tp", action="store_true",
                    help="N > 1: headline tensor parallel (row-sharded) instead of independent replicas")
    ap.add_argument("--skip-roofline", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--cpu-frac", type=float, default=1.0)
    ap.add_argument("--cpu-reps", type=int, default=1)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-frac", type=float, default=0.25)
    ap.add_argument("--case", choices=sorted(CASES), default=None,
                    help="run only this single-kernel case a few times (for profilers), print nothing else")
    ap.add_argument("--case-reps", type=int, default=2)
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="tensor-parallel all-gather: fused into the GEMV (p2p) or NCCL all_gather")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    select_workload(args.workload, args.tokens)
    if args.layers is None:
        args.layers = WORKLOADS[args.workload]["layers"]

    if args.case:
        run_case(args.case, args.case_reps)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    # host-side quantisation in spawned workers, started before any GPU call
    ncpu = len(os.sched_getaffinity(0))
    POOL = multiprocessing.get_context("spawn").Pool(max(1, min(8, ncpu // max(1, world))))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
            return
        if world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local_rank))
        try:
            run_gpu(args, rank, world, local_rank)
        finally:
            if world > 1:
                import torch.distributed as dist
                dist.destroy_process_group()
    finally:
        POOL.close()
        POOL.join()


if __name__ == "__main__":
    main()
