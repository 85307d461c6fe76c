#!/usr/bin/env python
"""Benchmark of the 3.5-bit decode GEMV path (libq35 on B200).

One step = the seven projections of one LLaMA-70B decoder layer (q 8192->8192,
k/v 8192->1024, o 8192->8192, gate/up 8192->28672, down 28672->8192) at batch M=1:
int8 activations x 3.5-bit packed weights -> exact int32 accumulators and fp32
dequantized outputs, everything resident in HBM.  The metric is algorithmic GB/s:
  bytes(3.5-bit) = ceil(K*N*7/16) + 8N + M*K + 8*M*N    (weights, scale+offset, x, C+y)
  bytes(INT4)    = K*N/2 + 4N + M*K + 8*M*N
The same run also measures the rest of the projection sweep (M in {1,4,16,64}, 3.5-bit
and INT4) and reports it under "sweep".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the CPU restatement of the reference's Fortran kernels
(matmul_3p5bit_awq + dequantize_output_3p5bit) on the host cores: the reference's own
Fortran needs gfortran, which the image lacks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "3.5-bit decode GEMV GB/s (LLaMA-70B layer projections, batch 1)"
UNIT = "GB/s"
SHAPES = [("q", 8192, 8192), ("k", 8192, 1024), ("v", 8192, 1024), ("o", 8192, 8192),
          ("gate", 8192, 28672), ("up", 8192, 28672), ("down", 28672, 8192)]
BATCHES = [1, 4, 16, 64]


def algo_bytes(fmt: int, M: int, K: int, N: int) -> int:
    if fmt == 0:
        return (K * N * 7 + 15) // 16 + 8 * N + M * K + 8 * M * N
    return K * N // 2 + 4 * N + M * K + 8 * M * N


def config(extra=None):
    c = {"workload": "LLaMA-70B decoder-layer projections q,k,v,o,gate,up,down "
                     "(8192->8192, 8192->1024 x2, 8192->8192, 8192->28672 x2, 28672->8192), "
                     "3.5-bit asym per-column weights, int8 activations, batch M=1",
         "weights": "N(0,0.02^2) fp32 generated and quantized on the device (seed 0)",
         "activations": "int8 uniform [-127,127] (seed 0)",
         "l2": "inputs larger than L2: 3 weight copies (3 x 375 MB) rotated between steps "
               "and between launches of one shape (L2 126 MB)"}
    if extra:
        c.update(extra)
    return c


# ----------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) < 10:
                continue
            if self.uuid and self.uuid not in p[1]:
                continue
            try:
                rows.append((float(p[2]), float(p[3]), float(p[4]), p[6:10]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        busy = [r for r in rows if r[2] > 200.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in busy for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in busy), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(busy)}


# ----------------------------------------------------------------------------------
def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


def cpu_baseline(seconds: float = 12.0, frac_cols: int = 8):
    """The oracle (C restatement of matmul_3p5bit_awq + dequantize_output_3p5bit, gcc
    -O3 -march=native, OpenMP over columns, all host threads) on a column sample of the
    same step: every projection with N/frac_cols columns, M=1."""
    import numpy as np
    from oracle import oracle as orc
    orc.build(native=True)
    L = orc.lib(native=True)
    threads = os.cpu_count() or 1
    L.orc_set_threads(threads)
    data = []
    for i, (nm, K, N) in enumerate(SHAPES):
        n = N // frac_cols
        wq = np.empty((K // 2, n), np.int8, order="F")
        L.orc_gen_int8(wq.ctypes.data, wq.size, 0, 100 + i)
        A = np.empty((1, K), np.int8, order="F")
        L.orc_gen_int8(A.ctypes.data, A.size, 0, 200 + i)
        s = np.ones(n, np.float32)
        o = np.zeros(n, np.float32)
        C_ = np.zeros((1, n), np.int32, order="F")
        Y = np.zeros((1, n), np.float32, order="F")
        data.append((K, n, A, wq, s, o, C_, Y))
    nbytes = sum(algo_bytes(0, 1, K, n) for K, n, *_ in data)

    def step():
        for K, n, A, wq, s, o, C_, Y in data:
            L.orc_matmul_3p5bit_awq(A, wq, s, o, C_, 1, n, K, 0)
            L.orc_dequantize_output_3p5bit(C_, s, o, Y, 1, n)

    step()
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or reps < 1:
        step()
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return {"value": nbytes / dt / 1e9, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"M=1, each of the 7 projections with N/{frac_cols} columns "
                      f"({nbytes/1e6:.1f} MB algorithmic), {reps} reps",
            "ms_per_sample": dt * 1e3, "note": "gfortran absent: C restatement of the "
                                               "reference loops stands in for the Fortran build"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    from oracle import oracle as orc
    orc.build(native=True)
    L = orc.lib(native=True)
    threads = os.cpu_count() or 1
    L.orc_set_threads(threads)
    frac = 64
    data = []
    for i, (nm, K, N) in enumerate(SHAPES):
        n = N // frac
        wq = np.empty((K // 2, n), np.int8, order="F")
        L.orc_gen_int8(wq.ctypes.data, wq.size, 0, 100 + i)
        A = np.empty((1, K), np.int8, order="F")
        L.orc_gen_int8(A.ctypes.data, A.size, 0, 200 + i)
        data.append((K, n, A, wq, np.ones(n, np.float32), np.zeros(n, np.float32),
                     np.zeros((1, n), np.int32, order="F"), np.zeros((1, n), np.float32, order="F")))
    nbytes = sum(algo_bytes(0, 1, K, n) for K, n, *_ in data)

    def step():
        for K, n, A, wq, s, o, C_, Y in data:
            L.orc_matmul_3p5bit_awq(A, wq, s, o, C_, 1, n, K, 0)
            L.orc_dequantize_output_3p5bit(C_, s, o, Y, 1, n)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    v = nbytes / dt / 1e9
    sample = (f"per step: M=1, each of the 7 projections with N/{frac} columns "
              f"({nbytes/1e6:.2f} MB algorithmic)")
    out = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "int8xint4/int3->int32",
           "data": "synthetic", "impl": "reference", "config": config(),
           "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                            "sample": sample},
           "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "the reference's Fortran cannot be compiled here (no gfortran); the timed "
                   "code is the C restatement of matmul_3p5bit_awq + dequantize_output_3p5bit"}
    print(json.dumps(out), flush=True)


# ----------------------------------------------------------------------------------
def run_ours(args):
    import ctypes as C
    import numpy as np
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import Context, QuantizedMatrix

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    L = _lib.load()
    ctx = Context(local)
    stream = torch.cuda.ExternalStream(ctx.stream, device=f"cuda:{local}")
    SETS = 3   # weight copies rotated between launches: 3 x 375 MB, so no launch hits L2

    # weights for both formats, generated + quantized + repacked on the device
    mats = {}
    for fmt in (0, 1):
        for st in range(SETS):
            for i, (nm, K, N) in enumerate(SHAPES):
                h = C.c_void_p()
                _lib.check(L.q35_weights_generate(ctx.h, fmt, N, K, st, 10 * i + fmt + 1, 0.02, C.byref(h)),
                           "weights_generate")
                qm = QuantizedMatrix.from_handle(ctx, h, K, N, fmt)
                mats[(fmt, st, nm)] = qm
    maxM = max(BATCHES)
    xs, outs = {}, {}
    for i, (nm, K, N) in enumerate(SHAPES):
        x = torch.empty(maxM * K, dtype=torch.int8, device="cuda")
        _lib.check(L.q35_gen_int8_dev(x.data_ptr(), x.numel(), 0, 1000 + i, None))
        xs[nm] = x
        outs[nm] = (torch.empty(maxM * N, dtype=torch.int32, device="cuda"),
                    torch.empty(maxM * N, dtype=torch.float32, device="cuda"))
    torch.cuda.synchronize()

    def launch(fmt, st, M, nm):
        Cd, Yd = outs[nm]
        mats[(fmt, st, nm)].gemm_dev(xs[nm].data_ptr(), M, Cd.data_ptr(), Yd.data_ptr())

    def layer_steps(fmt, M):            # one graph = SETS steps (one per weight copy)
        for st in range(SETS):
            for nm, _, _ in SHAPES:
                launch(fmt, st, M, nm)

    def shape_launches(nm, reps):       # one graph = reps launches of one shape, rotating copies
        for r in range(reps):
            launch(0, r % SETS, 1, nm)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def time_graph(g, n_replays, warmup):
        for _ in range(warmup):
            g.launch()
        ctx.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n_replays):
            g.launch()
        e1.record(stream)
        ctx.synchronize()
        ms = e0.elapsed_time(e1)
        if dist is not None:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def graph_of(fn):
        fn()                      # first run outside capture: workspace sized, attributes set
        ctx.synchronize()
        return ctx.capture(fn)

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        if not uuid.startswith("GPU-"):
            uuid = "GPU-" + uuid
    except Exception:
        pass

    hbm, peak_kind = peaks()
    step_bytes = sum(algo_bytes(0, 1, K, N) for _, K, N in SHAPES)
    g_main = graph_of(lambda: layer_steps(0, 1))
    replays = max(1, args.steps // SETS)
    steps_timed = replays * SETS
    with ClockSampler(uuid) as clk:
        ms_total = time_graph(g_main, replays, max(1, args.warmup // SETS))
        ms_step = ms_total / steps_timed
        # per-shape launch durations (roofline): graphs of 12 launches of one shape
        per_shape = {}
        ktime, kbytes = 0.0, 0
        for nm, K, N in SHAPES:
            g = graph_of(lambda nm=nm: shape_launches(nm, 12))
            t = time_graph(g, max(2, args.steps // 40), 2) / (12 * max(2, args.steps // 40))
            g.close()
            bb = algo_bytes(0, 1, K, N)
            per_shape[nm] = {"us": t * 1e3, "GBps": bb / (t * 1e-3) / 1e9}
            ktime += t
            kbytes += bb
        sweep = {}
        for fmt in (0, 1):
            for M in BATCHES:
                if fmt == 0 and M == 1:
                    continue
                g = graph_of(lambda fmt=fmt, M=M: layer_steps(fmt, M))
                n = max(2, args.steps // 12)
                s_ms = time_graph(g, n, 1) / (n * SETS)
                g.close()
                b = sum(algo_bytes(fmt, M, K, N) for _, K, N in SHAPES)
                sweep[f"{'q35' if fmt == 0 else 'int4'}_m{M}"] = {
                    "GBps": b / (s_ms * 1e-3) / 1e9, "us_per_layer": s_ms * 1e3}
    clocks = clk.summary()
    ctx.device_error()

    value_rank = step_bytes / (ms_step * 1e-3) / 1e9
    value = value_rank * world
    sweep["q35_m1"] = {"GBps": value_rank, "us_per_layer": ms_step * 1e3}
    # dominant kernel: gemv_kernel<3.5-bit, MT=1>; its largest launches (gate/up/down,
    # 82% of a step's bytes) are represented by the gate launch, the shape of the ncu capture
    achieved = per_shape["gate"]["GBps"]
    achieved_all = kbytes / (ktime * 1e-3) / 1e9
    traffic = None
    tf = os.path.join(ROOT, "profiles", "gemv_q35_gate_m1_traffic.json")
    if os.path.exists(tf):
        try:
            traffic = json.load(open(tf)).get("dram_bytes_per_launch")
        except Exception:
            traffic = None

    # e2e through the C ABI with host buffers (q35_matmul_cached: H2D of x, D2H of C and y)
    hA = {nm: np.asfortranarray(xs[nm][:K].cpu().numpy().reshape(1, K)) for nm, K, _ in SHAPES}
    hC = {nm: np.zeros((1, N), np.int32, order="F") for nm, _, N in SHAPES}
    hY = {nm: np.zeros((1, N), np.float32, order="F") for nm, _, N in SHAPES}

    def e2e_step(st):
        for nm, K, N in SHAPES:
            _lib.check(L.q35_matmul_cached(ctx.h, mats[(0, st, nm)].h, hA[nm].ctypes.data, 1,
                                           hC[nm].ctypes.data, hY[nm].ctypes.data), "matmul_cached")

    for i in range(max(args.warmup, 3)):
        e2e_step(i % SETS)
    e_steps = max(args.steps // 4, 12)
    barrier()
    t0 = time.perf_counter()
    for i in range(e_steps):
        e2e_step(i % SETS)
    e_dt = (time.perf_counter() - t0) / e_steps
    if dist is not None:
        t = torch.tensor([e_dt], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_dt = float(t.item())
    e2e = {"value": step_bytes / e_dt / 1e9 * world, "unit": UNIT,
           "h2d_bytes_per_step": sum(K for _, K, _ in SHAPES),
           "d2h_bytes_per_step": sum(8 * N for _, _, N in SHAPES),
           "api": "q35_matmul_cached per projection (host int8 A in, host int32 C + fp32 Out back), "
                  "synchronous, wall clock"}

    result = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
              "steps": steps_timed, "warmup": args.warmup, "ms_per_step": ms_step,
              "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
              "dtype": "int8 x 3.5-bit -> int32 (+fp32 dequant)", "data": "synthetic",
              "config": config({"parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                                "timing": "CUDA graph of 3 steps (one per weight copy) replayed; "
                                          "CUDA events on the library stream"}),
              "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                           "frac": achieved / hbm, "peak_kind": peak_kind,
                           "traffic": traffic,
                           "kernel": "gemv_kernel<3.5-bit, MT=1>, gate launch 8192->28672 "
                                     "(algorithmic 103.2 MB per launch / CUDA-event launch time)",
                           "frac_vs_8TBps": achieved / 8000.0,
                           "achieved_all_7_shapes": achieved_all,
                           "algo_bytes_per_launch": algo_bytes(0, 1, 8192, 28672)},
              "e2e": e2e,
              "gpu_launches": steps_timed * len(SHAPES),
              "clocks": clocks, "per_shape_m1": per_shape, "sweep": sweep}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            result["cpu_baseline"] = cpu_baseline()
        except Exception as e:  # reported, not fatal
            result["cpu_baseline"] = {"value": None, "error": str(e)}
    if rank == 0:
        print(json.dumps(result), flush=True)
    g_main.close()
    for qm in mats.values():
        qm.close()
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_case(args):
    """A few launches of one projection (for profiler captures): --case name:fmt:M."""
    import ctypes as C
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import Context, QuantizedMatrix
    nm, fmt, M = args.case.split(":")
    fmt, M = int(fmt), int(M)
    K, N = {n: (k, c) for n, k, c in SHAPES}[nm]
    L = _lib.load()
    ctx = Context(0)
    h = C.c_void_p()
    _lib.check(L.q35_weights_generate(ctx.h, fmt, N, K, 0, 1, 0.02, C.byref(h)), "weights_generate")
    qm = QuantizedMatrix.from_handle(ctx, h, K, N, fmt)
    x = torch.empty(M * K, dtype=torch.int8, device="cuda")
    _lib.check(L.q35_gen_int8_dev(x.data_ptr(), x.numel(), 0, 2, None))
    Cd = torch.empty(M * N, dtype=torch.int32, device="cuda")
    Yd = torch.empty(M * N, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    for _ in range(args.warmup + args.steps):
        qm.gemm_dev(x.data_ptr(), M, Cd.data_ptr(), Yd.data_ptr())
    ctx.synchronize()
    print(json.dumps({"case": args.case, "launches": args.warmup + args.steps,
                      "algo_bytes_per_launch": algo_bytes(fmt, M, K, N)}))
    qm.close()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--case", default=None, help="profile helper: name:fmt:M, e.g. gate:0:1")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.case:
        run_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
