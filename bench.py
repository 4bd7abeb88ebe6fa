"""Benchmark: Llama-3-8B-shaped Q4_K_M decode over GGUF blocks on B200.

Workload (one "step" = one decode token, M = 1, through a stack of L = 32
Llama-3-8B-shaped layers, each with 7 projections):
  q, o  [4096 x 4096]  Q4_K     k [1024 x 4096]  Q4_K     v [1024 x 4096]  Q6_K
  gate, up [14336 x 4096] Q4_K  down [4096 x 14336] Q6_K          (138.9 MB / layer)
Weights are N(0, 0.02) quantized on the host by planejaja_b200.quantize (seed
1000), activations N(0, 1) (seed 2000); synthetic data, random-init weights.
The 32 layers are distinct device copies (4.44 GB), so every step streams far
more than the 126 MB L2 and consecutive steps never hit in L2.

Per layer, one fused GEMV launch per shared activation: q|k|v (attention
input), o, gate|up (FFN input), down -- 4 kernels, activations quantized on
chip.  A step is captured once as a CUDA graph and replayed.

With --gpus N > 1 (torchrun, one process per GPU): every projection is
row-sharded across the ranks (each rank holds N_out / N rows of each matrix)
and each GEMV stores its output rows into every rank's output buffer over
NVLink (the all-gather a tensor-parallel decode needs, fused into the GEMV;
nsq_gemv_multi_xchg), strong scaling, total work fixed.  --exchange nccl
runs the GEMV followed by an NCCL all_gather per projection instead.

--workload l2-7b: Llama-2-7B in Q4_0 (q, k, v, o [4096 x 4096], gate / up
[11008 x 4096], down [4096 x 11008]; 32 layer copies, 3.64 GB per step), the
7 projections of a layer in the same 4 fused launches.

--workload l2-70b-ffn --tokens {1,16}: the Llama-2-70B FFN (gate|up [28672 x 8192]
Q4_K, down [8192 x 28672] Q4_K; 8 layer copies, 3.17 GB), the row-sharded
configuration measured at 1/2/4/8 GPUs.

metric  : decode GEMV HBM GB/s = (weight bytes + fp32 activations + fp32
          outputs) of the whole step / step time (max over ranks), all ranks.
e2e     : the same step through the C-ABI engine calls with host buffers:
          pinned-host -> device copy of the step's activation vectors (the
          inputs every layer copy reads), the GEMVs, one device ->
          pinned-host copy of all outputs of all layers (one contiguous
          buffer), stream sync per step.
roofline: dominant kernel = the fused M = 1 Q4_K gate|up launch (FFN input
          projection, 2 x [14336 x 4096], 66.06 MB), timed alone with CUDA
          events rotating over the 32 layer copies; bound = HBM, peak =
          MEASURED_PEAKS.json hbm_gbs.
prefill : the tcgen05 GEMM on Q4_K [14336 x 4096] at M = 512 tokens, TFLOP/s.
cpu_baseline: the CPU oracle (C restatement of the reference's dequant +
          cpu_matmul_f32 composition) on one layer, all host threads.

--impl reference times that CPU path alone (the reference is Rust/Vulkan;
neither toolchain nor a Vulkan driver exists on the box) on the same
workload, a bounded sample per step.
"""
from __future__ import annotations

import argparse
import ctypes
import json
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


def layer_bytes_total():
    from planejaja_b200.formats import fmt
    w = sum(fmt(t).tensor_bytes(n, k) for _, n, k, t in LAYER_SPEC)
    x = sum(M_TOK * k * 4 for _, n, k, t in LAYER_SPEC)
    y = sum(M_TOK * n * 4 for _, n, k, t in LAYER_SPEC)
    return w, x, y


def host_layer():
    """Quantized bytes of one layer, {name: uint8 array [N * row_bytes]}."""
    from planejaja_b200 import quantize as Q
    return {name: Q.synthetic_weights(n, k, t, seed=SEED_W + i)
            for i, (name, n, k, t) in enumerate(LAYER_SPEC)}


def host_acts():
    from planejaja_b200 import quantize as Q
    return [Q.synthetic_activations(M_TOK, k, seed=SEED_X + i).reshape(-1) for i, k in enumerate(ACT_K)]


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
    sample of) one layer, `reps` times or until `min_seconds` have passed;
    returns (GB/s, bytes, seconds, threads)."""
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
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOADS[WORKLOAD]["desc"].format(m=M_TOK, layers=1),
                   "sample": f"{args.ref_frac:.4f} of the rows of each of the {len(LAYER_SPEC)} matrices of one "
                             f"layer per step",
                   "layers_per_step": 1, "batch": M_TOK},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": th, "kind": "port",
                         "sample": f"{args.ref_frac:.4f} of one layer's rows per step "
                                   f"({(w * args.ref_frac) / 1e6:.1f} MB of weights)"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


# --------------------------------------------------------------------------- GPU leg
def run_gpu(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from planejaja_b200 import _lib
    from planejaja_b200.engine import CudaEngine
    from planejaja_b200.formats import fmt

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    eng = CudaEngine(local_rank)
    lib = eng.lib
    L = args.layers

    layer = host_layer()
    acts_h = host_acts()

    # shard rows (contiguous byte ranges) and upload; layer copies are device clones
    shards = {}
    for name, n, k, t in LAYER_SPEC:
        rb = fmt(t).row_bytes(k)
        assert n % world == 0
        rows = n // world
        shards[name] = (rows, eng.upload(layer[name][rank * rows * rb:(rank + 1) * rows * rb]))
    layers = []
    for li in range(L):
        layers.append({name: (rows, buf if li == 0 else buf.clone()) for name, (rows, buf) in shards.items()})
    acts = [torch.from_numpy(a).to(dev) for a in acts_h]
    M = M_TOK
    def flat_views(sizes):
        # one contiguous device buffer per step's outputs (one read-back per step)
        flat = torch.empty(L * sum(M * n for _, n in sizes), dtype=torch.float32, device=dev)
        views, off = [], 0
        for _ in range(L):
            d = {}
            for name, n in sizes:
                d[name] = flat[off:off + M * n]
                off += M * n
            views.append(d)
        return flat, views

    outs_local_flat, outs_local = flat_views([(name, rows) for name, (rows, _) in layers[0].items()])
    # scratch for prepared activations when they do not fit on chip (M > 4 or long rows)
    ws = eng.workspace(lib.nsq_gemv_workspace_size(M, max(ACT_K)))
    ws_ptr, ws_n = ws.data_ptr(), ws.numel()
    p2p = world > 1 and args.exchange == "p2p"
    exchange = None
    if p2p:
        # full outputs of every projection live in the exchange buffer; each
        # GEMV stores its rows into every rank's buffer (all-gather fused)
        from planejaja_b200.sharded import Exchange, OutputLayout, xsegments
        layout = OutputLayout()
        for li in range(L):
            for name, n, k, t in LAYER_SPEC:
                layout.add((li, name), M, n)
        exchange = Exchange(layout.nbytes)
        outs_full = [{name: exchange.view(layout.offsets[(li, name)][0], (M * n,)) for name, n, k, t in LAYER_SPEC}
                     for li in range(L)]
    elif world > 1:
        outs_full_flat, outs_full = flat_views([(name, n) for name, n, k, t in LAYER_SPEC])
    else:
        outs_full_flat, outs_full = outs_local_flat, outs_local
    # one fused launch per shared activation (q|k|v, o, gate|up, down for Llama-3-8B)
    TYPE_OF = {name: t for name, n, k, t in LAYER_SPEC}
    N_OF = {name: n for name, n, k, t in LAYER_SPEC}
    seg_arrays = []
    xseg_arrays = []
    for li in range(L):
        per, xper = [], []
        for a, names in GROUPS:
            arr = (_lib.Segment * len(names))()
            for i, nm in enumerate(names):
                rows, w = layers[li][nm]
                arr[i] = _lib.Segment(w.data_ptr(), TYPE_OF[nm], 0, rows, outs_local[li][nm].data_ptr())
            per.append((a, names, arr))
            if p2p:
                xper.append((a, names, xsegments([(layers[li][nm][1].data_ptr(), TYPE_OF[nm], 0, layers[li][nm][0],
                                                   rank * layers[li][nm][0], N_OF[nm],
                                                   layout.offsets[(li, nm)][0]) for nm in names])))
        seg_arrays.append(per)
        xseg_arrays.append(xper)
    n_launch = 0

    def step():
        nonlocal n_launch
        n_launch = 0
        st = torch.cuda.current_stream(dev).cuda_stream
        if p2p:
            for li in range(L):
                for a, names, arr in xseg_arrays[li]:
                    rc = lib.nsq_gemv_multi_xchg(ctypes.cast(arr, ctypes.c_void_p), len(names), acts[a].data_ptr(),
                                                 M, ACT_K[a], exchange.comm, ws_ptr, ws_n, st)
                    assert rc == 0, rc
                    n_launch += 1
            exchange.wait(st)  # the step ends when every rank's rows have landed here
            n_launch += 1
            return
        for li in range(L):
            for a, names, arr in seg_arrays[li]:
                rc = lib.nsq_gemv_multi(ctypes.cast(arr, ctypes.c_void_p), len(names), acts[a].data_ptr(), M,
                                        ACT_K[a], ws_ptr, ws_n, st)
                assert rc == 0, rc
                n_launch += 1
                if world > 1:
                    for nm in names:
                        dist.all_gather_into_tensor(outs_full[li][nm], outs_local[li][nm])

    # warm + capture (single GPU: the whole step as one CUDA graph)
    step()
    torch.cuda.synchronize()
    graph = None
    if not args.no_graph:
        # the whole step, NCCL all-gathers included for N > 1, as one graph
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            step()
        torch.cuda.synchronize()
    launches_per_step = n_launch

    def run_step():
        if graph is not None:
            graph.replay()
        else:
            step()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ else local_rank) as clk:
        ev0.record()
        for _ in range(args.steps):
            run_step()
        ev1.record()
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    wb, xb, yb = layer_bytes_total()
    step_bytes = (wb + xb + yb) * L
    value = step_bytes / (ms * 1e-3) / 1e9

    # ---- e2e: host buffers through the C-ABI calls, copies inside the timed region
    # the step's inputs are its activation vectors (every layer copy reads
    # the same ones); its result is every output of every layer, read back
    # in one copy from the contiguous output buffer
    acts_pin = [torch.from_numpy(a).pin_memory() for a in acts_h]
    if p2p:
        out_dev = torch.as_tensor(exchange.view(0, (layout.nbytes // 4,)))
    else:
        out_dev = outs_full_flat
    out_pin = torch.empty(out_dev.numel(), dtype=torch.float32).pin_memory()
    h2d = sum(a.numel() * 4 for a in acts_pin)
    d2h = out_pin.numel() * 4

    def e2e_step():
        for a, src in enumerate(acts_pin):
            acts[a].copy_(src, non_blocking=True)
        run_step()
        out_pin.copy_(out_dev, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    e2e_value = step_bytes / (e2e_ms * 1e-3) / 1e9

    hbm_peak, bf16_peak, peak_kind = peaks()
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "int8x2-dp4a/f32",
        "data": "synthetic (N(0,0.02) weights quantized on host; N(0,1) activations)",
        "config": {"workload": WORKLOADS[WORKLOAD]["desc"].format(m=M, layers=L),
                   "layers": L, "batch": 1, "weight_bytes_per_step": wb * L,
                   "parallelism": (f"tp{world} row-sharded, all-gather fused into the GEMV (NVLink peer stores)"
                                   if p2p else f"tp{world} row-sharded + NCCL all-gather") if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2: {L} distinct layer copies, {wb * L / 1e9:.2f} GB per step",
                   "cuda_graph": graph is not None},
        "frac_of_nominal_8tbs": round(value / NOMINAL_HBM_GBS, 4),
        "gpu_launches": launches_per_step * args.steps,
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 4)},
    }
    clocks = clk.summary()

    # ---- dominant kernel alone: the fused Q4_K gate|up launch (FFN input
    # projection, 2 x [14336 x 4096]) over the layer copies
    if not args.skip_roofline:
        rows, _ = layers[0]["gate"]
        gt = TYPE_OF["gate"]
        gname = fmt(gt).name
        gi = [i for i, (a, names) in enumerate(GROUPS) if "gate" in names][0]
        ga = GROUPS[gi][0]
        KG = ACT_K[ga]
        gbytes = 2 * fmt(gt).tensor_bytes(rows, KG) + M * KG * 4 + 2 * M * rows * 4
        st = torch.cuda.current_stream(dev).cuda_stream
        gu = [seg_arrays[li][gi][2] for li in range(L)]
        reps = max(4, 256 // L) * L
        for i in range(L):
            lib.nsq_gemv_multi(ctypes.cast(gu[i], ctypes.c_void_p), 2, acts[ga].data_ptr(), M, KG, ws_ptr, ws_n, st)
        torch.cuda.synchronize()
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record()
        for i in range(reps):
            lib.nsq_gemv_multi(ctypes.cast(gu[i % L], ctypes.c_void_p), 2, acts[ga].data_ptr(), M, KG, ws_ptr, ws_n,
                               st)
        k1.record()
        torch.cuda.synchronize()
        kms = k0.elapsed_time(k1) / reps
        achieved = gbytes / (kms * 1e-3) / 1e9
        traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tp):
            keys = {"l3-8b": "gemv_fused_q4k_m1_gate_up", "l2-7b": "gemv_fused_q40_m1_gate_up"}
            key = keys.get(WORKLOAD) if M == 1 and world == 1 else None
            traffic = json.load(open(tp)).get(key) if key else None
        result["roofline"] = {"bound": "hbm",
                              "kernel": f"gemv_fused_kernel<M={M},{gname}> gate|up 2 x [{rows}x{KG}] (FFN input projection)",
                              "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                              "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
                              "frac_of_nominal_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
                              "bytes_per_launch": gbytes, "us_per_launch": round(kms * 1e3, 3),
                              "traffic": traffic}

        # ---- prefill GEMM (tcgen05) on the gate matrix (Q4_K [14336 x 4096] for Llama-3-8B) at M = 512
        import torch as T
        pm = args.prefill_m
        wq = layers[0]["gate"][1]
        xp = T.randn(pm, KG, device=dev).to(T.bfloat16)
        yp = T.empty(pm, rows, dtype=T.bfloat16, device=dev)
        for _ in range(3):
            lib.nsq_gemm_bf16(wq.data_ptr(), gt, 0, xp.data_ptr(), yp.data_ptr(), pm, rows, KG, st)
        torch.cuda.synchronize()
        p0, p1 = T.cuda.Event(enable_timing=True), T.cuda.Event(enable_timing=True)
        preps = 20
        p0.record()
        for i in range(preps):
            lib.nsq_gemm_bf16(layers[i % L]["gate"][1].data_ptr(), gt, 0, xp.data_ptr(), yp.data_ptr(), pm, rows,
                              KG, st)
        p1.record()
        torch.cuda.synchronize()
        pms = p0.elapsed_time(p1) / preps
        tflops = 2.0 * pm * rows * KG / (pms * 1e-3) / 1e12
        result["prefill"] = {"kernel": f"gemm_tc_kernel<{gname}> (tcgen05, bf16, fp32 TMEM accumulate)",
                             "shape": f"M={pm} N={rows} K={KG}", "tflops": round(tflops, 1),
                             "ms": round(pms, 4), "peak_tflops": bf16_peak, "peak_kind": peak_kind,
                             "frac": round(tflops / bf16_peak, 4)}
    result["clocks"] = clocks
    assert eng.device_status() == 0, "a bounded device wait timed out"

    # ---- CPU baseline: oracle on one layer, all host threads (rank 0, N = 1)
    if rank == 0 and world == 1 and not args.skip_cpu:
        v, nb, dt, th = cpu_leg(layer, acts_h, rows_frac=args.cpu_frac, reps=args.cpu_reps,
                                min_seconds=args.cpu_seconds)
        result["cpu_baseline"] = {"value": round(v, 3), "unit": UNIT, "cores": th, "kind": "port",
                                  "sample": f"oracle dequant + cpu_matmul_f32 over {args.cpu_frac:.3f} of the rows "
                                            f"of one layer's 7 matrices, repeated for >= {args.cpu_seconds:.0f} s "
                                            f"({nb / 1e6:.1f} MB in {dt:.1f} s)"}
    if rank == 0:
        print(json.dumps(result), flush=True)
    graph = None
    if exchange is not None:
        # no rank may unmap its buffer while a peer can still store into it
        torch.cuda.synchronize()
        barrier()
        exchange.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="nsq", choices=["nsq", "reference"])
    ap.add_argument("--layers", type=int, default=None, help="layer copies per step (default: the workload's)")
    ap.add_argument("--workload", default="l3-8b", choices=sorted(WORKLOADS))
    ap.add_argument("--tokens", type=int, default=1, help="tokens per decode step, M (1..16)")
    ap.add_argument("--prefill-m", type=int, default=512)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--skip-roofline", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--cpu-frac", type=float, default=1.0)
    ap.add_argument("--cpu-reps", type=int, default=1)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-frac", type=float, default=0.25)
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="N > 1: all-gather fused into the GEMV (p2p) or NCCL all_gather per projection")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    select_workload(args.workload, args.tokens)
    if args.layers is None:
        args.layers = WORKLOADS[args.workload]["layers"]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
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


if __name__ == "__main__":
    main()
