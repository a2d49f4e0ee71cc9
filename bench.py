#!/usr/bin/env python
"""Benchmark of the quantized-GEMV hot path (BASELINE config c2).

Workload ("step"): one decode token's FFN GEMVs of the Qwen2.5-0.5B shape with
Q4_K weights - 24 layers x {gate 4864x896, up 4864x896, down 896x4864} = 72
fused GEMVs over 72 distinct resident weight matrices (159.7 MB per step, above
the 126 MB L2, so every step streams its weights from HBM).  Each GEMV
quantizes its fp32 input to Q8_0 on the device and runs the fused integer
GEMV, exactly the work of the reference's matmul_q_fused (src/quant.c:441).
Weights and activations are seeded synthetic data (no checkpoints offline).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

value  : whole-job GB/s of algorithmic bytes (packed weights + fp32 x + fp32
         out), inputs resident in HBM, CUDA events on the launching stream, max
         over ranks.  The 72 GEMVs of a step run as one engine program
         (quantr_program_run: activation quantizer + persistent GEMV engine),
         replayed as a CUDA graph; per_call_value times the same step as 72
         separate quantr_gemv_dev calls.
e2e    : the same metric with HOST buffers through the C-ABI program call:
         every step copies its inputs from pinned host memory and its outputs
         back inside the CUDA-event region, steps pipelined over two buffer
         sets and copy-in / compute / copy-out streams as a serving loop runs
         them.  e2e_dropin: the reference's own entry point, 72 synchronous
         matmul_q_fused_batch calls with host arrays per step (weights
         registered once, like the reference's load-time mmap).
batch_sweep : the rest of the c2 sweep (batch 4 and 16 by default, --sweep)
         on the same weights, timed like `value`; jobs of 2+ tokens run on
         the tensor-core kernel.
c1_q8_0 : BASELINE config c1 (Q8_0 5632x2048 GEMV, batch 1), 16 distinct
         copies per replay so every replay streams from HBM (--no-c1 skips),
         with its own CPU baseline (the reference's matmul_q_fused).
decode_c3, moe_c4, decode_c5 : BASELINE configs c3 (TinyLlama decode, batch
         1), c4 (one Qwen1.5-MoE layer with shared expert, 64 tokens) and c5
         (Qwen3-30B-A3B decode, 64 sequences), each with its CPU baseline.
int8_compute : the compute-bound int8 case (one c5 expert, 1024 tokens per
         GEMV) in TOP/s against the int8 tensor peak measured in-process.
sharded : the two multi-GPU forms (row-sharded head GEMV with all-gather,
         expert-parallel MoE with all-to-all dispatch) with parity flags.
N > 1  : every rank runs its own replica of the step on its GPU (the GEMV
         metric shards by independent work; no collective on the data path),
         so scaling is weak.
--impl reference : the reference's own quant.c (oracle/_ref, the fastest
         build this host runs, all host threads) on the same workload, rank 0.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "quantr-in-c_b200")
sys.path.insert(0, PKG)

import synth  # noqa: E402

METRIC = "quantized GEMV HBM GB/s (% of 8 TB/s); decode tok/s at 1/2/4/8 B200 vs host CPU"
HIDDEN, FFN, LAYERS = 896, 4864, 24
Q8_0, Q4_K, Q6_K = 8, 12, 14
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) of one k_program launch of the c2 step at batch 1
# (24 layers), from the ncu --set full capture of that launch summarised under
# profiles/ (k_program_c2_full.txt): 159,962,112 read + 4,132,864 written
# (algorithmic: 159,694,848 weight bytes + 0.64 MB x + 1.02 MB out per step).
# Reported only for that configuration.
NCU_TRAFFIC_C2_B1 = 164094976
NCU_TRAFFIC_SOURCE = "ncu --set full capture of k_program, c2 step at batch 1, 24 layers (profiles/k_program_c2_full.txt)"


def cudart_lib(device):
    """The CUDA runtime library through ctypes, current device set, or None."""
    cands = ["libcudart.so.12", os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "lib64", "libcudart.so.12")]
    for name in cands:
        try:
            L = ctypes.CDLL(name)
        except OSError:
            continue
        vp = ctypes.c_void_p
        L.cudaSetDevice.argtypes = [ctypes.c_int]
        L.cudaMemcpyAsync.argtypes = [vp, vp, ctypes.c_size_t, ctypes.c_int, vp]
        L.cudaEventRecord.argtypes = [vp, vp]
        L.cudaStreamWaitEvent.argtypes = [vp, vp, ctypes.c_uint]
        L.cudaEventCreateWithFlags.argtypes = [ctypes.POINTER(vp), ctypes.c_uint]
        L.cudaEventDestroy.argtypes = [vp]
        if L.cudaSetDevice(device) != 0:
            return None
        return L
    return None


def cuda_ok(rc, what):
    if rc != 0:
        raise RuntimeError(f"CUDA runtime call failed ({what}): error {rc}")

def row_bytes(t, d):
    return (d // synth.BLOCK_ELEMS[t]) * synth.BLOCK_BYTES[t]


def step_shapes(layers):
    """(type, n, d, input-kind) per GEMV of one step, in model order."""
    out = []
    for _ in range(layers):
        out += [(Q4_K, FFN, HIDDEN, "x"), (Q4_K, FFN, HIDDEN, "x"), (Q4_K, HIDDEN, FFN, "h")]
    return out


def gemv_bytes(t, n, d, B):
    return n * row_bytes(t, d) + 4 * d * B + 4 * n * B


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        self.proc.wait()
        rows = [r.split(", ") for r in open(self.path).read().strip().splitlines() if r.strip()]
        os.unlink(self.path)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip() == "Active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------- CPU reference --

def cpu_reference_run(layers, B, steps, warmup, budget_s=None):
    """Times the reference's matmul_q_fused on this host (oracle/_ref build).

    Returns (GB/s, seconds, steps done, threads, variant, kind)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    threads = os.cpu_count() or 1
    os.environ.setdefault("OMP_PROC_BIND", "close")
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    import oracle  # test infrastructure: the CPU baseline leg only
    variant = oracle.best_cpu_variant()
    if oracle.ref_available(variant):
        lib, kind = oracle.RefLib(variant), "reference"
    else:
        lib, kind, variant = oracle.Oracle(), "port", "restatement"
    rng = synth.rng_for(11)
    shapes = step_shapes(layers)
    ws = [synth.matrix(rng, t, n, d) for t, n, d, _ in shapes]
    xs = {d: synth.activations(rng, B, d) for d in (HIDDEN, FFN)}
    f = lib.fn["matmul_q_fused"]
    import ctypes
    outs = {n: np.empty(n, np.float32) for n in (HIDDEN, FFN)}

    def one_step():
        for (t, n, d, _), w in zip(shapes, ws):
            for b in range(B):
                f(outs[n].ctypes.data_as(ctypes.c_void_p), xs[d][b].ctypes.data_as(ctypes.c_void_p),
                  w.ctypes.data_as(ctypes.c_void_p), t, n, d, threads)

    for _ in range(warmup):
        one_step()
    done = 0
    t0 = time.perf_counter()
    while True:
        one_step()
        done += 1
        el = time.perf_counter() - t0
        if budget_s is None and done >= steps:
            break
        if budget_s is not None and (el >= budget_s or done >= 100000) and done >= 3:
            break
    el = time.perf_counter() - t0
    nbytes = sum(gemv_bytes(t, n, d, B) for t, n, d, _ in shapes)
    return nbytes * done / el / 1e9, el, done, threads, variant, kind


def cpu_c1_run(budget_s):
    """The reference's matmul_q_fused on the c1 shape (Q8_0 5632x2048, batch
    1) on this host, over 16 distinct weight copies like the GPU line.
    Returns (GB/s, calls, threads, variant, kind)."""
    import ctypes
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    threads = os.cpu_count() or 1
    import oracle  # test infrastructure: the CPU baseline leg only
    variant = oracle.best_cpu_variant()
    if oracle.ref_available(variant):
        lib, kind = oracle.RefLib(variant), "reference"
    else:
        lib, kind, variant = oracle.Oracle(), "port", "restatement"
    rng = synth.rng_for(12)
    n, d = 5632, 2048
    w0 = synth.matrix(rng, Q8_0, n, d)
    ws = [w0.copy() for _ in range(16)]
    x = synth.activations(rng, 1, d)[0]
    out = np.empty(n, np.float32)
    f = lib.fn["matmul_q_fused"]
    P = ctypes.c_void_p
    f(out.ctypes.data_as(P), x.ctypes.data_as(P), ws[0].ctypes.data_as(P), Q8_0, n, d, threads)
    done = 0
    t0 = time.perf_counter()
    while done < 3 or (time.perf_counter() - t0 < budget_s and done < 100000):
        f(out.ctypes.data_as(P), x.ctypes.data_as(P), ws[done % 16].ctypes.data_as(P), Q8_0, n, d, threads)
        done += 1
    el = time.perf_counter() - t0
    return gemv_bytes(Q8_0, n, d, 1) * done / el / 1e9, done, threads, variant, kind


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    gbs, el, done, threads, variant, kind = cpu_reference_run(args.layers, args.batch, args.steps, args.warmup)
    sample = (f"{done} full steps ({3 * args.layers} GEMVs each) of the workload, reference src/quant.c "
              f"{variant} build, OpenMP threads={threads}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": done, "warmup": args.warmup, "ms_per_step": round(el / done * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": config_dict(args),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if kind == "reference" and variant != "scalar":
        line["note"] = ("the reference's Q4_K kernel reads fp16 scales as integers (src/quant.c:302-303), so "
                        "its values are wrong, but its memory traffic and instruction mix are the same")
    print(json.dumps(line), flush=True)


def config_dict(args):
    return {
        "workload": (f"c2: Qwen2.5-0.5B FFN GEMVs, Q4_K weights, {args.layers} layers x "
                     f"(gate {FFN}x{HIDDEN}, up {FFN}x{HIDDEN}, down {HIDDEN}x{FFN}), batch {args.batch}, "
                     "Q8_0 activations quantized on the fly"),
        "type": "Q4_K", "batch": args.batch, "layers": args.layers,
        "weight_bytes_per_step": sum(n * row_bytes(t, d) for t, n, d, _ in step_shapes(args.layers)),
        "l2": "inputs larger than L2: 159.7 MB of distinct weights cycled per step vs 126 MB L2",
        "launch": ("one engine program per step (72 independent GEMVs: quantizer launch + persistent "
                   "engine launch, programmatic dependent launch), replayed as a CUDA graph"),
        "parallelism": f"replicas x{args.gpus}",
    }


# ------------------------------------------------------------------- ours --

def ours_arm(args):
    import torch
    import torch.distributed as dist

    import quantr

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    L = quantr.lib()
    assert L.quantr_gpu_init(local) == 0
    dev = torch.device("cuda", local)
    B = args.batch
    shapes = step_shapes(args.layers)
    rng = synth.rng_for(11)
    host_w = [synth.matrix(rng, t, n, d) for t, n, d, _ in shapes]
    dev_w = [torch.from_numpy(w).to(dev) for w in host_w]
    # All inputs and all outputs of a step are slices of one buffer each, so
    # the end-to-end run moves them with one copy per direction.
    x_sizes = [B * (HIDDEN if k == "x" else FFN) for _, _, _, k in shapes]
    o_sizes = [B * n for _, n, _, _ in shapes]
    xall = torch.from_numpy(np.concatenate([synth.activations(rng, 1, sz)[0] for sz in x_sizes])).to(dev)
    oall = torch.empty(sum(o_sizes), device=dev)
    xin = [v.view(B, -1) for v in torch.split(xall, x_sizes)]
    outs = [v.view(B, -1) for v in torch.split(oall, o_sizes)]
    ws_bytes = max(quantr.workspace_bytes(d, B) for _, _, d, _ in shapes)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    nbytes = sum(gemv_bytes(t, n, d, B) for t, n, d, _ in shapes)

    # One engine program holds the step's 72 independent GEMVs.
    prog = quantr.Program([(w.data_ptr(), t, n, d, B, x.data_ptr(), d, o.data_ptr(), n)
                           for (t, n, d, _), w, x, o in zip(shapes, dev_w, xin, outs)])

    def step(stream):
        prog.run(stream)

    def step_per_call(stream):
        for (t, n, d, _), w, x, o in zip(shapes, dev_w, xin, outs):
            quantr.gemv_dev(o.data_ptr(), n, x.data_ptr(), d, w.data_ptr(), t, n, d, B, ws.data_ptr(), ws_bytes,
                            stream)

    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        c0 = quantr.launch_count()
        step(s.cuda_stream)  # eager warm-up: sets kernel attributes before capture
        launches_per_step = quantr.launch_count() - c0
        step_per_call(s.cuda_stream)
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            step(s.cuda_stream)
        graph_pc = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_pc, stream=s):
            step_per_call(s.cuda_stream)
    torch.cuda.synchronize()
    assert quantr.device_status(0) == 0

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    # Clock soak: untimed replays so the sampler sees the GPU under this load
    # for ~1.5 s around the (much shorter) timed region.
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < 1.5:
        for _ in range(50):
            graph.replay()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        ev0.record(s)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(s)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    assert quantr.device_status(0) == 0
    gbs = world * nbytes * args.steps / (ms / 1e3) / 1e9
    per_gpu = nbytes * args.steps / (ms / 1e3) / 1e9

    # The same step as 72 separate GEMV calls (one engine launch pair each).
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            graph_pc.replay()
        ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev2.record(s)
        for _ in range(args.steps):
            graph_pc.replay()
        ev3.record(s)
    torch.cuda.synchronize()
    per_call_gbs = nbytes * args.steps / (ev2.elapsed_time(ev3) / 1e3) / 1e9

    # The rest of the c2 batch sweep (batch 1, 4 and 16): the same 72 weights
    # at the other batch sizes, device-resident inputs, CUDA-graph replays
    # timed with CUDA events like `value` (rank-local; reported per GPU).
    def time_program(shp, ws_dev, Bs):
        """ms per replay of one program over (type, n, d) shapes and weights."""
        xs = [torch.from_numpy(synth.activations(rng, Bs, d)).to(dev) for _, _, d, *_ in shp]
        os_ = [torch.empty(Bs, n, device=dev) for _, n, _, *_ in shp]
        pr = quantr.Program([(w.data_ptr(), t, n, d, Bs, x.data_ptr(), d, o.data_ptr(), n)
                             for (t, n, d, *_), w, x, o in zip(shp, ws_dev, xs, os_)])
        with torch.cuda.stream(s):
            pr.run(s.cuda_stream)
            s.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                pr.run(s.cuda_stream)
            for _ in range(args.warmup):
                g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(args.steps):
                g.replay()
            e1.record(s)
        torch.cuda.synchronize()
        assert quantr.device_status(0) == 0
        del g
        pr.close()
        return e0.elapsed_time(e1) / args.steps

    sweep = {}
    for Bs in args.sweep:
        if Bs == B:
            continue
        t_ms = time_program(shapes, dev_w, Bs)
        nb = sum(gemv_bytes(t, n, d, Bs) for t, n, d, _ in shapes)
        sweep[str(Bs)] = {"GB/s": round(nb / (t_ms / 1e3) / 1e9, 2), "ms_per_step": round(t_ms, 5),
                          "tok_per_s": round(Bs / (t_ms / 1e3), 1),
                          "path": "tensor cores (tcgen05.mma kind::i8)" if Bs >= 2 else "dp4a engine"}

    # BASELINE config c1: the Q8_0 GEMV at the TinyLlama FFN shape (5632 x
    # 2048, quants uniform in [-127, 127], scale max|w|/127 of w ~ N(0, 0.02)),
    # batch 1; 16 distinct copies per replay (196 MB, above L2) as one program.
    c1 = None
    if not args.no_c1:
        c1_shapes = [(Q8_0, 5632, 2048)] * 16
        w1 = torch.from_numpy(synth.q8_0_matrix(rng, 5632, 2048)).to(dev)
        c1_w = [w1.clone() for _ in c1_shapes]  # distinct addresses: every replay streams 196 MB
        t_ms = time_program(c1_shapes, c1_w, 1)
        nb = sum(gemv_bytes(t, n, d, 1) for t, n, d in c1_shapes)
        c1 = {"GB/s": round(nb / (t_ms / 1e3) / 1e9, 2), "us_per_gemv": round(t_ms * 1e3 / len(c1_shapes), 3),
              "frac_of_peak": round(nb / (t_ms / 1e3) / 1e9 / load_peaks()[0], 4),
              "workload": "c1: 16 distinct Q8_0 5632x2048 GEMVs per replay (196 MB > L2), batch 1"}
        del c1_w
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            gbs_c, done, threads, variant, kind = cpu_c1_run(min(5.0, args.cpu_seconds))
            c1["cpu_baseline"] = {"value": round(gbs_c, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                                  "sample": (f"{done} matmul_q_fused calls on the c1 shape over 16 distinct weight "
                                             f"copies, reference src/quant.c {variant} build")}

    # End to end with HOST buffers, (a) through the C-ABI program call: every
    # step copies all 72 inputs from pinned host memory to the device, runs
    # the program, and copies all outputs back to pinned host memory.  Steps
    # are pipelined the way a serving loop runs them: two buffer sets (one
    # program bound to each) and three streams (copy in, compute, copy out),
    # so step i's copy-in and step i-1's copy-out overlap computation.  CUDA
    # events bracket the first copy-in and the last copy-out.
    h2d = xall.numel() * 4
    d2h = oall.numel() * 4
    hx_pin = torch.empty(xall.numel(), dtype=torch.float32).pin_memory()
    hx_pin.copy_(torch.from_numpy(synth.activations(rng, 1, xall.numel())[0]))
    xall2, oall2 = torch.empty_like(xall), torch.empty_like(oall)
    xin2 = [v.view(B, -1) for v in torch.split(xall2, x_sizes)]
    outs2 = [v.view(B, -1) for v in torch.split(oall2, o_sizes)]
    prog2 = quantr.Program([(w.data_ptr(), t, n, d, B, x.data_ptr(), d, o.data_ptr(), n)
                            for (t, n, d, _), w, x, o in zip(shapes, dev_w, xin2, outs2)])
    sets = [(xall, oall, prog), (xall2, oall2, prog2)]
    ho_pin = [torch.empty(oall.numel(), dtype=torch.float32).pin_memory() for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    # The per-step copies and stream/event calls go straight to the CUDA
    # runtime (about 1 us of host time each; torch's wrappers cost several
    # times that, which made the host, not the GPU, set the pace of a 41 us
    # step).  Falls back to torch's calls where the runtime library is absent.
    rt = cudart_lib(dev.index or 0)
    if rt is not None:
        vp = ctypes.c_void_p
        rev = {}
        for key in ("in", "comp", "out"):
            rev[key] = []
            for _ in range(2):
                h = vp()
                cuda_ok(rt.cudaEventCreateWithFlags(ctypes.byref(h), 2), "cudaEventCreateWithFlags")  # no timing
                rev[key].append(h)
        sin, scomp, sout = vp(s_in.cuda_stream), vp(s.cuda_stream), vp(s_out.cuda_stream)
        xptr = [vp(xall.data_ptr()), vp(xall2.data_ptr())]
        optr = [vp(oall.data_ptr()), vp(oall2.data_ptr())]
        hxp, hop = vp(hx_pin.data_ptr()), [vp(t.data_ptr()) for t in ho_pin]

    def e2e_pipe(nsteps):
        for i in range(nsteps):
            j = i % 2
            xa, oa, pr = sets[j]
            if rt is not None:
                cuda_ok(rt.cudaStreamWaitEvent(sin, rev["comp"][j], 0), "wait")  # step i-2 has read this input
                cuda_ok(rt.cudaMemcpyAsync(xptr[j], hxp, h2d, 1, sin), "copy in")
                cuda_ok(rt.cudaEventRecord(rev["in"][j], sin), "record")
                cuda_ok(rt.cudaStreamWaitEvent(scomp, rev["in"][j], 0), "wait")
                cuda_ok(rt.cudaStreamWaitEvent(scomp, rev["out"][j], 0), "wait")  # step i-2's outputs are out
                pr.run(s.cuda_stream)
                cuda_ok(rt.cudaEventRecord(rev["comp"][j], scomp), "record")
                cuda_ok(rt.cudaStreamWaitEvent(sout, rev["comp"][j], 0), "wait")
                cuda_ok(rt.cudaMemcpyAsync(hop[j], optr[j], d2h, 2, sout), "copy out")
                cuda_ok(rt.cudaEventRecord(rev["out"][j], sout), "record")
                continue
            s_in.wait_event(ev_comp[j])  # step i-2 has read this input buffer
            with torch.cuda.stream(s_in):
                xa.copy_(hx_pin, non_blocking=True)
                ev_in[j].record(s_in)
            s.wait_event(ev_in[j])
            s.wait_event(ev_out[j])  # step i-2's outputs are copied out
            pr.run(s.cuda_stream)
            ev_comp[j].record(s)
            s_out.wait_event(ev_comp[j])
            with torch.cuda.stream(s_out):
                ho_pin[j].copy_(oa, non_blocking=True)
                ev_out[j].record(s_out)

    e2e_pipe(max(2, args.warmup))
    torch.cuda.synchronize()
    e2e_runs = []
    for _ in range(3):  # median of three repeats (host-copy bandwidth varies between boxes and runs)
        if world > 1:
            dist.barrier()
        ev4, ev5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev4.record(s_in)
        e2e_pipe(args.steps)
        ev5.record(s_out)
        torch.cuda.synchronize()
        te = torch.tensor([ev4.elapsed_time(ev5)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_runs.append(world * nbytes * args.steps / (float(te.item()) / 1e3) / 1e9)
    assert quantr.device_status(0) == 0
    e2e_gbs = statistics.median(e2e_runs)
    if rt is not None:
        for hs in rev.values():
            for h in hs:
                rt.cudaEventDestroy(h)
    prog2.close()

    # (b) through the reference's own entry point, one synchronous
    # matmul_q_fused_batch per GEMV with host arrays (weights registered once,
    # like the reference's load-time mmap).
    for w in host_w:
        quantr.register_weights(w)
    hx = [synth.activations(rng, B, HIDDEN if k == "x" else FFN) for _, _, _, k in shapes]

    def e2e_step():
        for (t, n, d, _), w, x in zip(shapes, host_w, hx):
            quantr.matmul_q_fused_batch(x, w, t, n, d)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_dropin_gbs = world * nbytes * args.steps / float(te.item()) / 1e9
    for w in host_w:
        quantr.unregister_weights(w)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs_c, el, done, threads, variant, kind = cpu_reference_run(args.layers, B, 0, 1, budget_s=args.cpu_seconds)
        cpu = {"value": round(gbs_c, 3), "unit": "GB/s", "cores": threads, "kind": kind,
               "sample": (f"{done} full steps ({len(shapes)} GEMVs each, {el:.1f} s) of the same workload, "
                          f"reference src/quant.c {variant} build")}

    sharded = None
    if not args.no_sharded:
        own_group = world == 1 and not dist.is_initialized()
        if own_group:  # the forms run their collectives over a one-rank group
            import datetime
            import socket
            with socket.socket() as so:
                so.bind(("127.0.0.1", 0))
                port = so.getsockname()[1]
            dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                                    timeout=datetime.timedelta(seconds=120), device_id=dev)
        sharded = sharded_forms(args, dev, world, rank)
        if own_group:
            dist.destroy_process_group()
    decode = c5 = c4 = i8 = None
    if rank == 0 and world == 1 and not args.no_int8:
        i8 = int8_compute(args, dev, s)
    if not args.no_decode:
        # c3 decode on every GPU (N > 1: one replica per rank, no collective
        # on the data path); rank 0 reports the aggregate from the slowest rank.
        decode = decode_c3(args, dev, s, cpu=(rank == 0 and world == 1))
        if world > 1:
            ms_all = [None] * world
            dist.all_gather_object(ms_all, decode["ms_per_token"])
            decode["ranks"] = world
            decode["per_rank_ms_per_token"] = ms_all
            decode["tok_per_s_aggregate"] = round(world * 1e3 / max(ms_all), 1)
            decode["aggregate_how"] = "N replicas (one sequence each), N x 1000 / max over ranks of ms per token"
        if rank != 0:
            decode = None
    if rank == 0 and world == 1 and not args.no_c4:
        c4 = moe_c4(args, dev, s)
    if rank == 0 and world == 1 and not args.no_c5:
        c5 = decode_c5(args, dev, s)

    peak, peak_kind = load_peaks()
    if rank == 0:
        c2_b1 = B == 1 and args.layers == LAYERS
        line = {
            "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": config_dict(args),
            "pct_of_8TBs_per_gpu": round(100.0 * per_gpu / NOMINAL_HBM_GBS, 2),
            "gemv_steps_per_s": round(world * args.steps / (ms / 1e3), 1),
            "roofline": {"bound": "hbm", "achieved": round(per_gpu, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(per_gpu / peak, 4), "peak_source": peak_kind,
                         "traffic": NCU_TRAFFIC_C2_B1 if c2_b1 else None,
                         "traffic_source": NCU_TRAFFIC_SOURCE if c2_b1 else None,
                         "kernel": "k_program (persistent GEMV engine) + k_quant_tasks, one launch pair per step"},
            "per_call_value": round(per_call_gbs, 3),
            "per_call_note": "same step as 72 quantr_gemv_dev calls (one quantizer + engine launch each)",
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "repeats": [round(v, 1) for v in e2e_runs],
                    "api": ("quantr_program_run with all step inputs copied from pinned host memory and all "
                            "outputs copied back inside the timed region (CUDA events); steps pipelined over two "
                            "buffer sets and copy-in / compute / copy-out streams; per-step copies and stream/event "
                            + ("calls through the CUDA runtime (ctypes)" if rt is not None else "calls through torch"))},
            "e2e_dropin": {"value": round(e2e_dropin_gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                           "d2h_bytes_per_step": d2h,
                           "api": "72 synchronous matmul_q_fused_batch calls per step with host arrays"},
            "batch_sweep": sweep,
            "c1_q8_0": c1,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "decode_c3": decode,
            "moe_c4": c4,
            "decode_c5": c5,
            "int8_compute": i8,
            "sharded": sharded,
        }
        print(json.dumps(line), flush=True)
    del graph, graph_pc
    prog.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------ sharded forms --

def sharded_forms(args, dev, world, rank):
    """The two multi-GPU forms of quantr-in-c_b200/shard.py, timed at this N
    (at N = 1 they run without collectives) with a bit-exactness flag against
    the one-GPU result computed on rank 0:
      tp_head  c3's output head (32000 x 2048 Q6_K, batch 1) row-sharded, one
               all-gather per call (strong scaling: fixed rows);
      ep_moe   c5's MoE layer (128 experts top-8, dim 2048, I 768, Q4_K),
               64 tokens per rank (weak scaling), experts split 128/N,
               all-to-all dispatch of Q8_0 activations + return of per-pair
               outputs, selection-order combine.
    Times are CUDA events over `steps` calls after warm-up, max over ranks."""
    import torch
    import torch.distributed as dist

    import quantr
    import shard
    be = shard.CudaBackend(dev)
    rng = synth.rng_for(77)
    out = {}

    def max_ms(ms_local):
        t = torch.tensor([ms_local], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, n):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return max_ms(e0.elapsed_time(e1) / n)

    # --- tensor-parallel head GEMV ---
    n, d, t = 32000, 2048, Q6_K
    w = synth.matrix(rng, t, n, d)
    x = torch.from_numpy(synth.activations(rng, 1, d)).to(dev)
    g = shard.RowShardedGemv(w, t, n, d, be)
    res = g(x).clone()
    # One call (GEMV shard + all-gather) captured as a CUDA graph, as a decode
    # loop replays it; released before the process group goes away.
    cs = torch.cuda.Stream(dev)
    cs.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(cs):
        g(x)
    torch.cuda.current_stream(dev).wait_stream(cs)
    torch.cuda.synchronize()
    tp_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(tp_graph, stream=cs):
        g(x)
    ms_call = timed(tp_graph.replay, args.steps)
    del tp_graph
    ag_in = torch.zeros(g.npad, device=dev)
    ag_out = torch.zeros(world * g.npad, device=dev)
    ms_ag = timed(lambda: dist.all_gather_into_tensor(ag_out, ag_in) if world > 1 else None, args.steps)
    ok = True
    if rank == 0:
        full = torch.zeros(1, n, device=dev)
        wd = be.upload(w)
        be.gemv(full, n, x, wd, t, n, d)
        ok = bool(torch.equal(full.view(torch.int32), res.contiguous().view(torch.int32)))
    flag = torch.tensor([1 if ok else 0], device=dev)
    if world > 1:
        dist.broadcast(flag, 0)
    wbytes = n * row_bytes(t, d)
    out["tp_head"] = {"shape": f"{n}x{d} Q6_K, batch 1, rows split {world} ways", "us_per_call": round(ms_call * 1e3, 2),
                      "timing": "CUDA graph of one call (GEMV shard + all-gather), CUDA events, max over ranks",
                      "all_gather_us": round(ms_ag * 1e3, 2) if world > 1 else 0.0,
                      "GBs_aggregate": round(wbytes / (ms_call / 1e3) / 1e9, 1),
                      "bit_exact_vs_1gpu": bool(flag.item()), "collective": "all_gather_into_tensor (NCCL)"}

    # --- expert-parallel MoE layer ---
    E, k, dim, hid, tq = 128, 8, 2048, 768, Q4_K
    T_rank = 64
    mats = [np.stack([synth.matrix(rng, tq, hid, dim) for _ in range(E)]),
            np.stack([synth.matrix(rng, tq, hid, dim) for _ in range(E)]),
            np.stack([synth.matrix(rng, tq, dim, hid) for _ in range(E)])]
    xb_all = synth.activations(rng, T_rank * world, dim)
    lg_all = rng.standard_normal((T_rank * world, E), dtype=np.float32)
    moe = shard.ExpertShardedMoE(E, k, dim, hid, mats[0], tq, mats[1], tq, mats[2], tq, be)
    r0 = rank * T_rank
    xb = torch.from_numpy(xb_all[r0:r0 + T_rank]).to(dev)
    lg = torch.from_numpy(lg_all[r0:r0 + T_rank]).to(dev)
    mo, _, _ = moe(xb, logits=lg)
    ms_moe = timed(lambda: moe(xb, logits=lg), max(5, args.steps // 4))
    parts = [torch.empty_like(mo) for _ in range(world)] if world > 1 else [mo]
    if world > 1:
        dist.all_gather(parts, mo)
    ok = True
    if rank == 0:
        full_moe = shard.ExpertShardedMoE.__new__(shard.ExpertShardedMoE)
        # the one-GPU block on every rank's tokens: all experts here
        xa = torch.from_numpy(xb_all).to(dev)
        la = torch.from_numpy(lg_all).to(dev)
        ew = [torch.from_numpy(np.ascontiguousarray(m_).reshape(-1)).to(dev) for m_ in mats]
        ewts = [quantr.ExpertWeights(m_.data_ptr(), mats[i][0].nbytes, None, tq) for i, m_ in enumerate(ew)]
        T_all = T_rank * world
        ref = torch.empty(T_all, dim, device=dev)
        wsb = quantr.moe_workspace_bytes(T_all, E, k, dim, hid)
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        quantr.moe_dev(ref.data_ptr(), dim, xa.data_ptr(), dim, T_all, E, k, *ewts, dim, hid, ws.data_ptr(), wsb,
                       logits=la.data_ptr(), ldl=E, stream=torch.cuda.current_stream(dev).cuda_stream)
        torch.cuda.synchronize()
        ok = bool(torch.equal(torch.cat(parts).view(torch.int32), ref.view(torch.int32)))
        del full_moe
    flag = torch.tensor([1 if ok else 0], device=dev)
    if world > 1:
        dist.broadcast(flag, 0)
    st = moe.stats
    ebytes = E * (2 * hid * row_bytes(tq, dim) + dim * row_bytes(tq, hid))
    out["ep_moe"] = {"shape": f"c5 MoE layer: E={E} top-{k}, dim {dim}, I {hid}, Q4_K; {T_rank} tokens per rank, "
                              f"experts split {world} ways",
                     "us_per_layer": round(ms_moe * 1e3, 2),
                     "tokens_per_s_aggregate": round(T_rank * world / (ms_moe / 1e3), 1),
                     "expert_GBs_aggregate": round(ebytes / (ms_moe / 1e3) / 1e9, 1),
                     "pairs_sent_rank0": st.get("pairs_sent"), "dispatch_bytes_rank0": st.get("dispatch_bytes"),
                     "return_bytes_rank0": st.get("return_bytes"),
                     "bit_exact_vs_1gpu": bool(flag.item()),
                     "collective": "all_to_all_single x4 (counts, Q8_0 rows, expert ids, per-pair outputs; NCCL)"}
    return out


# ------------------------------------------------------------- decode --

def cpu_forward_run(spec, model_seed, prompt, positions, budget_s):
    """Times the reference's own forward_runtime on this host: the unmodified
    reference (oracle/_ref/libquantr_ref_forward_avx512.so, all host threads)
    on the same model, feeding `prompt` at positions 0.. until `positions`
    forward calls or `budget_s` seconds.  Returns (s per call, calls, threads,
    kind)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    threads = os.cpu_count() or 1
    import forward  # test infrastructure: the CPU baseline leg only
    import model_synth as ms
    model = ms.build(spec, seed=model_seed)
    if forward.reference_available("avx512"):
        r, kind = forward.Reference(model, variant="avx512", threads=threads, backend=2), "reference"
    else:
        r, kind = forward.Restated(model, threads=threads), "port"
    r.forward(int(prompt[0]), 0)  # warm-up (page-in)
    t0 = time.perf_counter()
    done = 0
    while done < positions and (done < 2 or time.perf_counter() - t0 < budget_s):
        r.forward(int(prompt[done % len(prompt)]), done)
        done += 1
    el = time.perf_counter() - t0
    r.close()
    return el / done, done, threads, kind


def decode_c3(args, dev, s, cpu=True):
    """BASELINE config c3 on the device decoder: TinyLlama-1.1B shape, 512
    prompt tokens prefilled, then greedy decode.  Decode time per token is
    the difference of two CUDA-event-timed generate runs (512 + K and 512 + 0
    positions), so the prefill cancels; the KV context runs 512..511+K."""
    import torch

    import model_synth as ms
    import quantr
    spec = ms.tinyllama()
    t0 = time.perf_counter()
    model = ms.build(spec, seed=1)
    t_build = time.perf_counter() - t0
    t0 = time.perf_counter()
    dec = quantr.Decoder(model)
    torch.cuda.synchronize()
    t_load = time.perf_counter() - t0
    info = dec.info()
    n_prompt, K = 512, args.decode_steps
    prompt_h = ms.prompt(spec, n_prompt, seed=7)
    prompt = torch.from_numpy(prompt_h).to(dev)
    out = torch.empty(max(K, 1), 1, dtype=torch.int32, device=dev)

    def timed(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            e0.record(s)
            dec.generate_dev(prompt.data_ptr(), n_prompt, steps, out.data_ptr(), s.cuda_stream)
            e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    timed(8)  # warm-up
    reps = []
    for _ in range(3):
        t_full, t_pre = timed(K), timed(0)
        reps.append(((t_full - t_pre) / K, t_pre / n_prompt))
    ms_tok = statistics.median(r[0] for r in reps)
    ms_pos_prefill = statistics.median(r[1] for r in reps)
    assert quantr.device_status(0) == 0
    toks_dev = out[:K, 0].cpu().numpy()
    # End to end through the host API: prompt from host memory in, tokens out.
    t0 = time.perf_counter()
    toks_host = dec.generate(prompt_h, K)[0]
    t_e2e = time.perf_counter() - t0
    same = bool(np.array_equal(toks_dev, toks_host))
    kv_bytes = info["kv_bytes_per_position"] * (n_prompt + (K + 1) / 2.0)  # average context
    bytes_tok = info["weight_bytes_per_step"] + kv_bytes
    gbs = bytes_tok / (ms_tok / 1e3) / 1e9
    peak, peak_kind = load_peaks()
    res = {
        "workload": ("c3: TinyLlama-1.1B shape (22 layers, dim 2048, 32/4 heads, head_dim 64, FFN 5632, vocab "
                     "32000, RoPE 10000), Q4_K linears, Q6_K head, Q8_0 embedding, fp32 KV; 512 prompt tokens "
                     f"then {K} greedy tokens, batch 1; seeded random weights"),
        "tok_per_s": round(1e3 / ms_tok, 1), "ms_per_token": round(ms_tok, 4),
        "prefill_us_per_position": round(ms_pos_prefill * 1e3, 2),
        "bytes_per_token": int(bytes_tok), "achieved_GBs": round(gbs, 1),
        "hbm_frac": round(gbs / peak, 4), "pct_of_8TBs": round(100 * gbs / NOMINAL_HBM_GBS, 2),
        "launches_per_token": info["launches_per_decode_step"],
        "e2e": {"tok_per_s": round(K / t_e2e, 2), "positions_per_s": round((n_prompt + K) / t_e2e, 1),
                "api": (f"quantr_decoder_generate with host prompt in / host tokens out: {n_prompt} prefill "
                        f"positions + {K} greedy tokens in {t_e2e * 1e3:.1f} ms wall")},
        "tokens_device_equal_host": same,
        "model_build_s": round(t_build, 2), "decoder_create_s": round(t_load, 2),
        "device_bytes": info["device_bytes"],
    }
    dec.close()
    if cpu and not args.no_cpu_baseline:
        sec, done, threads, kind = cpu_forward_run(spec, 1, prompt_h[0], 1000, args.cpu_seconds)
        res["cpu_baseline"] = {"value": round(1.0 / sec, 3), "unit": "tok/s", "cores": threads, "kind": kind,
                               "sample": (f"{done} forward_runtime calls at positions 0..{done - 1} on the same "
                                          f"model ({sec * 1e3:.0f} ms each)")}
    return res


def _cudart():
    """The CUDA runtime torch loaded (for raw device-to-device copies)."""
    import ctypes
    import glob

    import torch
    libdir = os.path.join(os.path.dirname(torch.__file__), "lib")
    for cand in sorted(glob.glob(os.path.join(libdir, "libcudart.so*"))) + \
            sorted(glob.glob("/usr/local/cuda/lib64/libcudart.so*")):
        try:
            return ctypes.CDLL(cand)
        except OSError:
            pass
    raise OSError("libcudart not found")


def decode_c5(args, dev, s):
    """BASELINE config c5 on the device decoder: Qwen3-30B-A3B shape (48
    layers, hidden 2048, 32/4 heads of head_dim 128, 128 experts top-8 of
    768, vocab 151936, all Q4_K), 64 sequences each with a seeded 1024-token
    KV context (cache filled with N(0, 1) values; the decode step's cost does
    not depend on them), then greedy decode steps at positions 1024, 1025, ...
    Time per step = CUDA events over `steps` step calls after warm-up."""
    import ctypes

    import torch

    import model_synth as ms
    import quantr
    spec = ms.qwen3_moe(seq_len=1024 + max(8, args.c5_steps + 8))
    t0 = time.perf_counter()
    model = ms.build(spec, seed=5)
    t_build = time.perf_counter() - t0
    B, ctx = 64, 1024
    t0 = time.perf_counter()
    dec = quantr.Decoder(model, batch=B)
    torch.cuda.synchronize()
    t_load = time.perf_counter() - t0
    info = dec.info()
    kptr, vptr, kv_bytes = dec.kv()
    g = torch.Generator(device=dev)
    g.manual_seed(55)
    chunk = 1 << 28  # floats per fill
    buf = torch.empty(chunk, dtype=torch.float32, device=dev)
    rt = _cudart()
    for base in (kptr, vptr):
        off = 0
        while off < kv_bytes:
            n = min(chunk * 4, kv_bytes - off)
            buf.normal_(generator=g)
            assert rt.cudaMemcpy(ctypes.c_void_p(base + off), ctypes.c_void_p(buf.data_ptr()), ctypes.c_size_t(n),
                                 3) == 0
            off += n
    del buf
    torch.cuda.synchronize()
    tok = torch.from_numpy(ms.prompt(spec, 1, seed=8, batch=B)[:, 0].copy()).to(dev)
    pos = torch.full((B,), ctx, dtype=torch.int32, device=dev)

    def steps(n):
        with torch.cuda.stream(s):
            for _ in range(n):
                dec.step_dev(tok.data_ptr(), pos.data_ptr(), None, 0, tok.data_ptr(), s.cuda_stream)
                pos.add_(1)

    steps(args.warmup)
    torch.cuda.synchronize()
    pos.fill_(ctx)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
    steps(args.c5_steps)
    with torch.cuda.stream(s):
        e1.record(s)
    torch.cuda.synchronize()
    st = quantr.device_status(0)
    ms_step = e0.elapsed_time(e1) / args.c5_steps
    # Bytes per step: dense weights + the head + every expert (each is chosen
    # by at least one of the 64 tokens with probability 1 - (120/128)^64 =
    # 0.984) + the KV rows read (64 sequences at context ctx + step).
    ebytes = spec.n_layers * spec.expert_count * (
        2 * spec.hidden_dim * ms.row_bytes(ms.Q4_K, spec.dim) + spec.dim * ms.row_bytes(ms.Q4_K, spec.hidden_dim))
    kv_step = info["kv_bytes_per_position"] * B * (ctx + (args.c5_steps + 1) / 2.0)
    bytes_step = info["weight_bytes_per_step"] + ebytes + kv_step
    gbs = bytes_step / (ms_step / 1e3) / 1e9
    peak, _ = load_peaks()
    res = {
        "workload": ("c5: Qwen3-30B-A3B shape (48 layers, hidden 2048, 32/4 heads, head_dim 128, 128 experts "
                     "top-8 x 768, vocab 151936), all Q4_K, fp32 KV; 64 sequences, each at a seeded 1024-token "
                     f"context, {args.c5_steps} greedy steps; seeded random weights"),
        "tok_per_s": round(B / (ms_step / 1e3), 1), "ms_per_step": round(ms_step, 3),
        "bytes_per_step": int(bytes_step), "achieved_GBs": round(gbs, 1), "hbm_frac": round(gbs / peak, 4),
        "kv_bytes_per_step": int(kv_step), "launches_per_step": info["launches_per_decode_step"],
        "device_status": st, "model_build_s": round(t_build, 1), "decoder_create_s": round(t_load, 1),
        "device_bytes": info["device_bytes"] + 2 * kv_bytes,
    }
    dec.close()
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import forward  # test infrastructure: the CPU baseline leg only
        threads = os.cpu_count() or 1
        r = forward.Restated(model, threads=threads)
        r.forward(5, 0)
        t0 = time.perf_counter()
        done = 0
        while done < 2 or (time.perf_counter() - t0 < args.cpu_seconds and done < 64):
            r.forward(5 + done, done + 1)
            done += 1
        sec = (time.perf_counter() - t0) / done
        r.close()
        res["cpu_baseline"] = {"value": round(1.0 / sec, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                               "sample": (f"{done} restated forward_runtime calls (head_dim 128 is not expressible "
                                          f"in the reference; oracle/forward_oracle.c) at positions 1..{done} of one "
                                          f"sequence, {sec:.2f} s each")}
    del model
    return res


def moe_c4(args, dev, s):
    """BASELINE config c4: one Qwen1.5-MoE-A2.7B-shape MoE layer for 64 tokens
    - router logits N(0, 1), 60 experts top-4 (intermediate 1408, gate/up Q5_K,
    down Q6_K) through quantr_moe_dev, then the shared expert (5632, same
    types) with its sigmoid gate through quantr_moe_shared_dev - as one CUDA
    graph, CUDA events over `steps` replays."""
    import torch

    import quantr
    rng = synth.rng_for(44)
    T, E, k, dim, hid, sh = 64, 60, 4, 2048, 1408, 5632
    Q5_K = 13
    w1 = torch.from_numpy(np.stack([synth.matrix(rng, Q5_K, hid, dim) for _ in range(E)])).to(dev)
    w3 = torch.from_numpy(np.stack([synth.matrix(rng, Q5_K, hid, dim) for _ in range(E)])).to(dev)
    w2 = torch.from_numpy(np.stack([synth.matrix(rng, Q6_K, dim, hid) for _ in range(E)])).to(dev)
    s1 = torch.from_numpy(synth.matrix(rng, Q5_K, sh, dim)).to(dev)
    s3 = torch.from_numpy(synth.matrix(rng, Q5_K, sh, dim)).to(dev)
    s2 = torch.from_numpy(synth.matrix(rng, Q6_K, dim, sh)).to(dev)
    gate = torch.from_numpy((rng.standard_normal(dim, dtype=np.float32) * np.float32(0.02)).astype(np.float32)).to(dev)
    xb = torch.from_numpy(synth.activations(rng, T, dim)).to(dev)
    lg = torch.from_numpy(rng.standard_normal((T, E), dtype=np.float32)).to(dev)
    out = torch.empty(T, dim, device=dev)
    wsb = quantr.moe_workspace_bytes(T, E, k, dim, hid)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    ew = [quantr.ExpertWeights(t.data_ptr(), t[0].numel(), None, ty) for t, ty in ((w1, Q5_K), (w3, Q5_K),
                                                                                    (w2, Q6_K))]
    sel = torch.empty(T, k, dtype=torch.int32, device=dev)

    def layer(stream):
        quantr.moe_dev(out.data_ptr(), dim, xb.data_ptr(), dim, T, E, k, *ew, dim, hid, ws.data_ptr(), wsb,
                       logits=lg.data_ptr(), ldl=E, sel=sel.data_ptr(), stream=stream)
        quantr.moe_shared_dev(out.data_ptr(), dim, xb.data_ptr(), dim, T, gate.data_ptr(), s1.data_ptr(), Q5_K,
                              s3.data_ptr(), Q5_K, s2.data_ptr(), Q6_K, dim, sh, stream)

    with torch.cuda.stream(s):
        layer(s.cuda_stream)  # plans (allocating) before capture
        s.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=s):
            layer(s.cuda_stream)
        for _ in range(args.warmup):
            gr.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(args.steps):
            gr.replay()
        e1.record(s)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    chosen = np.unique(sel.cpu().numpy())
    rb1, rb2 = w1[0].numel(), w2[0].numel()
    bytes_layer = len(chosen) * (2 * rb1 + rb2) + s1.numel() + s3.numel() + s2.numel() + 4 * dim
    gbs = bytes_layer / (us / 1e6) / 1e9
    peak, _ = load_peaks()
    res = {"workload": ("c4: Qwen1.5-MoE-A2.7B-shape MoE layer, 64 tokens, router logits N(0,1), 60 experts "
                        "top-4 x 1408 (gate/up Q5_K, down Q6_K) + shared expert 5632 with sigmoid gate"),
           "us_per_layer": round(us, 2), "tokens_per_s": round(T / (us / 1e6), 1),
           "experts_chosen": int(len(chosen)), "bytes_per_layer": int(bytes_layer), "achieved_GBs": round(gbs, 1),
           "hbm_frac": round(gbs / peak, 4),
           "device_status": quantr.device_status(0)}
    if not args.no_cpu_baseline:
        # The reference's matmul_q_fused for the layer's GEMVs (per token: 4
        # experts x 3 plus the shared expert's 3; routing and softmax omitted).
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import ctypes

        import oracle
        variant = oracle.best_cpu_variant()
        lib = oracle.RefLib(variant) if oracle.ref_available(variant) else oracle.Oracle()
        f = lib.fn["matmul_q_fused"]
        threads = os.cpu_count() or 1
        hw = [t.cpu().numpy() for t in (w1, w3, w2)]
        hs = [t.cpu().numpy() for t in (s1, s3, s2)]
        xh = xb.cpu().numpy()
        selh = sel.cpu().numpy()
        o1 = np.empty(max(hid, sh), np.float32)
        o2 = np.empty(dim, np.float32)
        P = ctypes.c_void_p
        t0 = time.perf_counter()
        done = 0
        while done < T and (done < 2 or time.perf_counter() - t0 < args.cpu_seconds):
            x = xh[done]
            for e in selh[done]:
                f(o1.ctypes.data_as(P), x.ctypes.data_as(P), hw[0][e].ctypes.data_as(P), Q5_K, hid, dim, threads)
                f(o1.ctypes.data_as(P), x.ctypes.data_as(P), hw[1][e].ctypes.data_as(P), Q5_K, hid, dim, threads)
                f(o2.ctypes.data_as(P), o1.ctypes.data_as(P), hw[2][e].ctypes.data_as(P), Q6_K, dim, hid, threads)
            f(o1.ctypes.data_as(P), x.ctypes.data_as(P), hs[0].ctypes.data_as(P), Q5_K, sh, dim, threads)
            f(o1.ctypes.data_as(P), x.ctypes.data_as(P), hs[1].ctypes.data_as(P), Q5_K, sh, dim, threads)
            f(o2.ctypes.data_as(P), o1.ctypes.data_as(P), hs[2].ctypes.data_as(P), Q6_K, dim, sh, threads)
            done += 1
        sec = (time.perf_counter() - t0) / done
        res["cpu_baseline"] = {"value": round(1.0 / sec, 2), "unit": "tokens/s", "cores": threads,
                               "kind": "reference" if oracle.ref_available(variant) else "port",
                               "sample": (f"{done} tokens of the layer's 15 matmul_q_fused calls each "
                                          f"({variant} build; routing omitted), {sec * 1e3:.1f} ms per token")}
    del gr
    return res


def int8_compute(args, dev, s):
    """The compute-bound int8 case: one c5 expert's three projections (W1, W3
    768x2048 and W2 2048x768, Q4_K) with 1024 tokens each, one program (the
    tensor-core kernel, 64-token slices re-reading the weights from L2).
    Reports int8 TOP/s (2*n*d*tokens per GEMV) against this GPU's dense int8
    peak measured in the same process (cuBLASLt through torch._int_mm)."""
    import torch

    import quantr
    rng = synth.rng_for(88)
    T, hid, dim = 1024, 768, 2048
    shapes = [(Q4_K, hid, dim), (Q4_K, hid, dim), (Q4_K, dim, hid)]
    ws = [torch.from_numpy(synth.matrix(rng, t, n, d)).to(dev) for t, n, d in shapes]
    xs = [torch.from_numpy(synth.activations(rng, T, d)).to(dev) for _, _, d in shapes]
    os_ = [torch.empty(T, n, device=dev) for _, n, _ in shapes]
    pr = quantr.Program([(w.data_ptr(), t, n, d, T, x.data_ptr(), d, o.data_ptr(), n)
                         for (t, n, d), w, x, o in zip(shapes, ws, xs, os_)])
    with torch.cuda.stream(s):
        pr.run(s.cuda_stream)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            pr.run(s.cuda_stream)
        for _ in range(args.warmup):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(args.steps):
            g.replay()
        e1.record(s)
    torch.cuda.synchronize()
    st = quantr.device_status(0)
    ms = e0.elapsed_time(e1) / args.steps
    del g
    info = pr.info()
    pr.close()
    ops = sum(2.0 * n * d * T for _, n, d in shapes)
    tops = ops / (ms / 1e3) / 1e12
    peak = int8_peak(dev.index if dev.index is not None else 0)
    return {"workload": ("one c5 expert (W1, W3 768x2048, W2 2048x768, Q4_K) with 1024 tokens per GEMV, one "
                         "program on the tensor cores (64-token slices)"),
            "us_per_program": round(ms * 1e3, 2), "int8_tops": round(tops, 2), "int8_peak_tops": round(peak, 1),
            "frac_of_int8_peak": round(tops / peak, 4), "items": info["items"], "device_status": st,
            "peak_how": "torch._int_mm 8192^3 int8 GEMM (cuBLASLt), best of 20, same process"}


def profile_case(name, steps):
    """A small case of one configuration for ncu captures (a few GB on the
    device at most), `steps` runs of it:
      c1  one program of 16 Q8_0 5632x2048 GEMVs, batch 1 (196 MB);
      c3  decode steps of the c3 shape (2 layers) at position 512, batch 1;
      c4  the c4 MoE layer (60 experts top-4, 64 tokens) through quantr_moe_dev;
      c5  decode steps of the c5 layer shape (2 layers, vocab 1024, 64
          sequences at position 1024, KV cache zeros);
      int8  the int8_compute line's program (one c5 expert, 1024 tokens).
    Prints the device status only."""
    import torch

    import model_synth as ms
    import quantr
    assert quantr.lib().quantr_gpu_init(0) == 0
    dev = torch.device("cuda", 0)
    s = torch.cuda.current_stream().cuda_stream
    if name == "c1":
        rng = synth.rng_for(7)
        w = torch.from_numpy(synth.matrix(rng, Q8_0, 5632, 2048)).to(dev)
        ws = [w.clone() for _ in range(16)]
        xs = [torch.from_numpy(synth.activations(rng, 1, 2048)).to(dev) for _ in ws]
        os_ = [torch.empty(1, 5632, device=dev) for _ in ws]
        pr = quantr.Program([(wi.data_ptr(), Q8_0, 5632, 2048, 1, x.data_ptr(), 2048, o.data_ptr(), 5632)
                             for wi, x, o in zip(ws, xs, os_)])
        for _ in range(steps):
            pr.run(s)
        torch.cuda.synchronize()
        pr.close()
        print(json.dumps({"profile_case": name, "steps": steps, "device_status": quantr.device_status(0)}))
        return
    if name == "c4":
        rng = synth.rng_for(44)
        T, E, k, dim, hid = 64, 60, 4, 2048, 1408
        Q5_K = 13
        w1 = torch.from_numpy(np.stack([synth.matrix(rng, Q5_K, hid, dim) for _ in range(E)])).to(dev)
        w3 = torch.from_numpy(np.stack([synth.matrix(rng, Q5_K, hid, dim) for _ in range(E)])).to(dev)
        w2 = torch.from_numpy(np.stack([synth.matrix(rng, Q6_K, dim, hid) for _ in range(E)])).to(dev)
        xb = torch.from_numpy(synth.activations(rng, T, dim)).to(dev)
        lg = torch.from_numpy(rng.standard_normal((T, E), dtype=np.float32)).to(dev)
        out = torch.empty(T, dim, device=dev)
        wsb = quantr.moe_workspace_bytes(T, E, k, dim, hid)
        wsp = torch.empty(wsb, dtype=torch.uint8, device=dev)
        ew = [quantr.ExpertWeights(t.data_ptr(), t[0].numel(), None, ty) for t, ty in ((w1, Q5_K), (w3, Q5_K),
                                                                                        (w2, Q6_K))]
        for _ in range(steps):
            quantr.moe_dev(out.data_ptr(), dim, xb.data_ptr(), dim, T, E, k, *ew, dim, hid, wsp.data_ptr(), wsb,
                           logits=lg.data_ptr(), ldl=E, stream=s)
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": name, "steps": steps, "device_status": quantr.device_status(0)}))
        return
    if name == "int8":  # the int8_compute line's program: one c5 expert, 1024 tokens per GEMV
        rng = synth.rng_for(88)
        T, hid, dimx = 1024, 768, 2048
        shapes = [(Q4_K, hid, dimx), (Q4_K, hid, dimx), (Q4_K, dimx, hid)]
        ws = [torch.from_numpy(synth.matrix(rng, t, n, d)).to(dev) for t, n, d in shapes]
        xs = [torch.from_numpy(synth.activations(rng, T, d)).to(dev) for _, _, d in shapes]
        os_ = [torch.empty(T, n, device=dev) for _, n, _ in shapes]
        pr = quantr.Program([(w.data_ptr(), t, n, d, T, x.data_ptr(), d, o.data_ptr(), n)
                             for (t, n, d), w, x, o in zip(shapes, ws, xs, os_)])
        for _ in range(steps):
            pr.run(s)
        torch.cuda.synchronize()
        pr.close()
        print(json.dumps({"profile_case": name, "steps": steps, "device_status": quantr.device_status(0)}))
        return
    if name == "c3":  # decode steps of the c3 shape (2 layers) at position 512, batch 1
        spec = ms.tinyllama(layers=2)
        model = ms.build(spec, seed=1)
        dec = quantr.Decoder(model)
        tok = torch.tensor([5], dtype=torch.int32, device="cuda")
        pos = torch.full((1,), 512, dtype=torch.int32, device="cuda")
        for _ in range(steps):
            dec.step_dev(tok.data_ptr(), pos.data_ptr(), None, 0, tok.data_ptr(), s)
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": name, "steps": steps, "device_status": quantr.device_status(0)}))
        dec.close()
        return
    if name != "c5":
        raise ValueError(name)
    spec = ms.qwen3_moe(layers=2, vocab=1024, seq_len=1040)
    model = ms.build(spec, seed=5)
    B = 64
    dec = quantr.Decoder(model, batch=B)
    tok = torch.from_numpy(ms.prompt(spec, 1, seed=8, batch=B)[:, 0].copy()).cuda()
    pos = torch.full((B,), 1024, dtype=torch.int32, device="cuda")
    for _ in range(steps):
        dec.step_dev(tok.data_ptr(), pos.data_ptr(), None, 0, tok.data_ptr(), s)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": name, "steps": steps, "device_status": quantr.device_status(0)}))
    dec.close()


def int8_peak(device=0):
    """Dense int8 tensor throughput of this GPU (TOP/s): torch._int_mm (a cuBLASLt
    int8 x int8 -> int32 GEMM) of 8192^3, best of 20 after warm-up, CUDA events.
    The denominator for tensor-pipe fractions of int8 work."""
    import torch
    dev = torch.device("cuda", device)
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = None
    for _ in range(20):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    return 2.0 * n ** 3 / (best / 1e3) / 1e12


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-c1", action="store_true", help="skip the c1 Q8_0 GEMV line")
    ap.add_argument("--no-decode", action="store_true", help="skip the c3 decode line")
    ap.add_argument("--no-sharded", action="store_true", help="skip the tensor/expert-parallel forms")
    ap.add_argument("--no-c4", action="store_true", help="skip the c4 MoE layer line")
    ap.add_argument("--no-c5", action="store_true", help="skip the c5 decode line (48 layers, 17 GB of weights)")
    ap.add_argument("--no-int8", action="store_true", help="skip the compute-bound int8 line")
    ap.add_argument("--c5-steps", type=int, default=16)
    ap.add_argument("--decode-steps", type=int, default=128)
    ap.add_argument("--profile-case", choices=["c1", "c3", "c4", "c5", "int8"], default=None,
                    help="run a small case of a configuration for ncu captures and exit")
    ap.add_argument("--int8-peak", action="store_true",
                    help="only measure the GPU's dense int8 tensor throughput (cuBLASLt GEMM) and print it")
    ap.add_argument("--sweep", type=lambda v: [int(b) for b in v.split(",") if b], default=[4, 16],
                    help="other batch sizes timed on the same weights (comma list; empty to skip)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_case:
        profile_case(args.profile_case, args.steps)
        return
    if args.int8_peak:
        print(json.dumps({"int8_dense_tops": round(int8_peak(), 1),
                          "how": "torch._int_mm 8192^3 int8 GEMM (cuBLASLt), best of 20, CUDA events"}))
        return
    if args.impl == "reference":
        reference_arm(args)
    else:
        ours_arm(args)


if __name__ == "__main__":
    main()
