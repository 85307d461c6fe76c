#!/usr/bin/env python
"""Benchmark of asicForTranAI's quantized decode path on B200 (libq35).

Headline (value): the 3.5-bit decode GEMV over one LLaMA-70B decoder layer's seven
projections (q 8192->8192, k/v 8192->1024, o 8192->8192, gate/up 8192->28672,
down 28672->8192) at batch M=1, int8 activations x 3.5-bit packed weights -> exact
int32 accumulators and fp32 dequantized outputs, everything resident in HBM.  With N
GPUs every rank runs its tensor-parallel shard of the layer (q/k/v/gate/up split by
columns, o/down by rows) and value = all ranks' bytes / the slowest rank's time.
The metric is algorithmic GB/s:
  bytes(3.5-bit) = ceil(K*N*7/16) + 8N + M*K + 8*M*N    (weights, scale+offset, x, C+y)
  bytes(INT4)    = K*N/2 + 4N + M*K + 8*M*N
The same run reports:
  sweep    the projection sweep, M in {1,4,16,64} x {3.5-bit, INT4} (M >= 5 runs on the
           tensor-core engine, M <= 4 on the CUDA-core GEMV);
  prefill  the M=2048 GEMMs gate (8192->28672) and down (28672->8192) on the tensor
           cores (int8 TOP/s; one GPU only);
  decode   LLaMA-70B-shape greedy decode (prompt 512, 512 steps) at batch 1 and 16,
           tensor-parallel over the N GPUs (one int32 all-reduce after o and after
           down), and on one GPU the LLaMA-13B shape (prompt 128, 256 steps) at batch
           1 and 8; random-init 3.5-bit weights; tok/s and the fraction of the
           weight-streaming roofline;
  e2e      the headline through the reference-facing C ABI with host buffers.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--sections gemv,prefill,decode]

The nvidia-smi clock samples of the timed region go to clocks_<pid>.csv under
$Q35_CLOCKS_DIR (default: the temporary directory); their median and reasons are in the line.

--impl reference times the CPU restatement of the reference's Fortran kernels
(matmul_3p5bit_awq + dequantize_output_3p5bit) on the host cores: the reference's own
Fortran needs gfortran, which the image lacks.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "3.5-bit decode GEMV GB/s (LLaMA-70B layer projections, batch 1)"
UNIT = "GB/s"
SHAPES = [("q", 8192, 8192), ("k", 8192, 1024), ("v", 8192, 1024), ("o", 8192, 8192),
          ("gate", 8192, 28672), ("up", 8192, 28672), ("down", 28672, 8192)]
ROW_SPLIT = {"o", "down"}          # row-parallel projections; the rest split by columns
# the same layer as the decode model issues it: q|k|v and gate|up share their input, so each
# pair/triple is one matrix (columns concatenated) and one launch
FUSED = [("qkv", 8192, 10240), ("o", 8192, 8192), ("gate_up", 8192, 57344), ("down", 28672, 8192)]
BATCHES = [1, 4, 16, 64]
NOMINAL_INT8_TOPS = 4500.0         # B200 dense int8, NVIDIA's figure


def algo_bytes(fmt: int, M: int, K: int, N: int) -> int:
    if fmt == 0:
        return (K * N * 7 + 15) // 16 + 8 * N + M * K + 8 * M * N
    return K * N // 2 + 4 * N + M * K + 8 * M * N


def shard(shapes, world):
    """Each rank's (name, K, N) of the tensor-parallel split of the layer."""
    return [(nm, K // world, N) if nm in ROW_SPLIT else (nm, K, N // world) for nm, K, N in shapes]


def config(world, extra=None):
    c = {"workload": "LLaMA-70B decoder-layer projections q,k,v,o,gate,up,down "
                     "(8192->8192, 8192->1024 x2, 8192->8192, 8192->28672 x2, 28672->8192), "
                     "3.5-bit asym per-column weights, int8 activations, batch M=1",
         "weights": "N(0,0.02^2) fp32 generated and quantized on the device (seed 0)",
         "activations": "int8 uniform [-127,127] (seed 0)",
         "l2": "inputs larger than L2: 3 weight copies (3 x 375 MB per GPU at N=1) rotated between "
               "steps and between launches of one shape (L2 126 MB)",
         "parallelism": (f"tensor parallel x{world}: q,k,v,gate,up split by columns, o,down by rows"
                         if world > 1 else "single GPU")}
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
        out_dir = os.environ.get("Q35_CLOCKS_DIR") or tempfile.gettempdir()
        self.path = os.path.join(out_dir, f"clocks_{os.getpid()}.csv")

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


CPU_SAMPLE_COLS = 8       # both CPU legs run every projection with N/8 of its columns
CPU_THREAD_MODEL = ("OpenMP over output columns on all host threads (the reference's matmul_3p5bit_awq "
                    "loops are `do concurrent`, which gfortran runs on one thread)")


def _cpu_sample(L, frac_cols):
    import numpy as np
    data = []
    for i, (nm, K, N) in enumerate(SHAPES):
        n = N // frac_cols
        wq = np.empty((K // 2, n), np.int8, order="F")
        L.orc_gen_int8(wq.ctypes.data, wq.size, 0, 100 + i)
        A = np.empty((1, K), np.int8, order="F")
        L.orc_gen_int8(A.ctypes.data, A.size, 0, 200 + i)
        data.append((K, n, A, wq, np.ones(n, np.float32), np.zeros(n, np.float32),
                     np.zeros((1, n), np.int32, order="F"), np.zeros((1, n), np.float32, order="F")))
    return data


def _cpu_step(L, data):
    for K, n, A, wq, s, o, C_, Y in data:
        L.orc_matmul_3p5bit_awq(A, wq, s, o, C_, 1, n, K, 0)
        L.orc_dequantize_output_3p5bit(C_, s, o, Y, 1, n)


def _cpu_rate(L, data, seconds):
    nbytes = sum(algo_bytes(0, 1, K, n) for K, n, *_ in data)
    _cpu_step(L, data)
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or reps < 1:
        _cpu_step(L, data)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return nbytes / dt / 1e9, dt, reps, nbytes


def cpu_baseline(seconds: float = 12.0, frac_cols: int = CPU_SAMPLE_COLS):
    """The oracle (C restatement of matmul_3p5bit_awq + dequantize_output_3p5bit, gcc
    -O3 -march=native, OpenMP over columns, all host threads) on a column sample of the
    same step: every projection with N/frac_cols columns, M=1.  The same sample on one
    thread, the reference's own thread model, is reported beside it."""
    from oracle import oracle as orc
    orc.build(native=True)
    L = orc.lib(native=True)
    threads = os.cpu_count() or 1
    data = _cpu_sample(L, frac_cols)
    L.orc_set_threads(1)
    v1, dt1, _, _ = _cpu_rate(L, data, 3.0)
    L.orc_set_threads(threads)
    v, dt, reps, nbytes = _cpu_rate(L, data, seconds)
    return {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"M=1, each of the 7 projections with N/{frac_cols} columns "
                      f"({nbytes/1e6:.1f} MB algorithmic), {reps} reps",
            "ms_per_sample": dt * 1e3, "thread_model": CPU_THREAD_MODEL,
            "single_thread": {"value": v1, "unit": UNIT, "cores": 1, "ms_per_sample": dt1 * 1e3},
            "gemv_8192x8192_m1": cpu_kernels_8192(L, threads),
            "note": "gfortran absent: C restatement of the reference loops stands in for the Fortran build"}


def cpu_kernels_8192(L, threads, seconds=1.5):
    """The reference's three CPU kernels on one 8192 x 8192 GEMV at M=1 (ms per call and
    algorithmic GB/s): matmul_3p5bit_awq + dequantize_output_3p5bit and matmul_int4_awq +
    dequantize_output on one thread (their loops are `do concurrent`, one thread under
    gfortran), and matmul_int4_simd (matmul_simd_optimized.f90, OpenMP over columns) on all
    host threads -- the C restatements of the oracle."""
    import numpy as np
    K = N = 8192
    A = np.empty((1, K), np.int8, order="F")
    L.orc_gen_int8(A.ctypes.data, A.size, 0, 300)
    wq = np.empty((K // 2, N), np.int8, order="F")
    L.orc_gen_int8(wq.ctypes.data, wq.size, 0, 301)
    s = np.ones(N, np.float32)
    o = np.zeros(N, np.float32)
    C_ = np.zeros((1, N), np.int32, order="F")
    Y = np.zeros((1, N), np.float32, order="F")
    kernels = {
        "q35_awq_dequant": (1, 0, lambda: (L.orc_matmul_3p5bit_awq(A, wq, s, o, C_, 1, N, K, 0),
                                           L.orc_dequantize_output_3p5bit(C_, s, o, Y, 1, N))),
        "int4_awq_dequant": (1, 1, lambda: (L.orc_matmul_int4_awq(A, wq, s, C_, 1, N, K),
                                            L.orc_dequantize_output(C_, s, Y, 1, N))),
        "int4_simd_dequant": (threads, 1, lambda: (L.orc_matmul_int4_simd(A, wq, s, C_, 1, N, K),
                                                   L.orc_dequantize_output(C_, s, Y, 1, N))),
    }
    out = {}
    for name, (th, fmt, fn) in kernels.items():
        L.orc_set_threads(th)
        fn()
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds or reps < 2:
            fn()
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        out[name] = {"ms": dt * 1e3, "GBps": algo_bytes(fmt, 1, K, N) / dt / 1e9, "threads": th}
    L.orc_set_threads(threads)
    return out


def run_reference(args):
    """The reference arm: the C restatement of the reference's matmul_3p5bit_awq +
    dequantize_output_3p5bit on rank 0's host cores (OpenMP over columns, all threads), on
    the same column sample as cpu_baseline; other ranks exit without work."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as orc
    orc.build(native=True)
    L = orc.lib(native=True)
    threads = os.cpu_count() or 1
    L.orc_set_threads(threads)
    frac = CPU_SAMPLE_COLS
    data = _cpu_sample(L, frac)
    nbytes = sum(algo_bytes(0, 1, K, n) for K, n, *_ in data)
    for _ in range(args.warmup):
        _cpu_step(L, data)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _cpu_step(L, data)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    v = nbytes / dt / 1e9
    sample = (f"per step: M=1, each of the 7 projections with N/{frac} columns "
              f"({nbytes/1e6:.2f} MB algorithmic)")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    out = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "int8xint4/int3->int32",
           "data": "synthetic", "impl": "reference", "config": config(world),
           "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                            "sample": sample, "thread_model": CPU_THREAD_MODEL},
           "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "the reference's Fortran cannot be compiled here (no gfortran); the timed "
                   "code is the C restatement of matmul_3p5bit_awq + dequantize_output_3p5bit "
                   "on the host cores of rank 0"}
    print(json.dumps(out), flush=True)


# ----------------------------------------------------------------------------------
class Harness:
    """Per-process state of a run: rank, context, the torch process group used for
    barriers and the max-over-ranks of timings, the library's TP group."""

    def __init__(self):
        import torch
        self.torch = torch
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dist = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
            self.dist = dist
        from asicfortranai_b200.quantized import Context
        self.ctx = Context(self.local)
        self.stream = torch.cuda.ExternalStream(self.ctx.stream, device=f"cuda:{self.local}")
        self.tp = None
        if self.world > 1:
            from asicfortranai_b200.tp import TPGroup
            self.tp = TPGroup.from_torch(self.ctx, self.dist, timeout_s=120)

    def barrier(self):
        self.torch.cuda.synchronize()
        if self.dist is not None:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, v: float) -> float:
        if self.dist is None:
            return v
        t = self.torch.tensor([v], device="cuda", dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(self, v: float) -> float:
        if self.dist is None:
            return v
        t = self.torch.tensor([v], device="cuda", dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def time_ms(self, fn, n, warmup):
        """CUDA-event time of n calls of fn (enqueued on the library stream), max over ranks."""
        torch = self.torch
        for _ in range(warmup):
            fn()
        self.ctx.synchronize()
        self.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for _ in range(n):
            fn()
        e1.record(self.stream)
        self.ctx.synchronize()
        return self.max_over_ranks(e0.elapsed_time(e1))

    def uuid(self):
        try:
            u = str(self.torch.cuda.get_device_properties(self.local).uuid)
            return u if u.startswith("GPU-") else "GPU-" + u
        except Exception:
            return None


def tp_parity(H):
    """At N > 1, before anything is timed: the tensor-parallel path at this N, bit for bit
    against the same path on one GPU (rank 0 builds the unsharded twin), whose arithmetic
    the test suite checks against the oracle at these widths.  Integer partial sums are
    order free, so TP=N must equal one GPU exactly (transformer_layer.f90:415-417, 550,
    557 under the row split).  Checks:
      * the fused exchange of a row-parallel projection, x += dequant(sum over ranks of C),
        over NVLink peer memory (rows x N = 1x1024, 16x1024, 5x2048) and NCCL (64x8192),
        three calls each, against the sums of every rank's seeded partials;
      * the LLaMA-70B widths with two layers and vocabulary 32000 (the benchmarked model's
        random-init weights): prefill logits of a 16-token prompt, 32 greedy decode steps
        (logits and tokens; one row: the exchange fused with the next RMSNorm), 16 top-p
        tokens (p = 0.9, sampled over the gathered vocabulary shards), and a 16-sequence
        batch (tensor-core matmuls, several-row exchange) for 4 tokens.
    Returns the JSON summary; every rank learns the outcome."""
    import numpy as np
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.llama_model import LLAMA70B, LLaMAModel
    L, ctx, rank, world = _lib.load(), H.ctx, H.rank, H.world
    t0 = time.time()
    res = {"tp": world, "exchange": {}, "reference": "the same model on one GPU (rank 0), bit for bit"}
    ok = True
    for rows, N in ((1, 1024), (16, 1024), (5, 2048), (64, 8192)):
        rng = np.random.default_rng(100 + rows)
        Cs = [rng.integers(-2**20, 2**20, size=(rows, N), dtype=np.int32) for _ in range(world)]
        sc = rng.random(N, dtype=np.float32) * np.float32(1e-3)
        off = rng.standard_normal(N).astype(np.float32)
        x0 = rng.standard_normal((rows, N)).astype(np.float32)
        tot = sum(c.astype(np.int64) for c in Cs).astype(np.int32)
        want = x0 + (tot.astype(np.float32) + off) * sc
        dC = torch.from_numpy(Cs[rank]).cuda()
        dx = torch.from_numpy(x0).cuda()
        ds, do = torch.from_numpy(sc).cuda(), torch.from_numpy(off).cuda()
        e_ok = True
        for _ in range(3):
            dC.copy_(torch.from_numpy(Cs[rank]))
            dx.copy_(torch.from_numpy(x0))
            torch.cuda.synchronize()
            _lib.check(L.q35_tp_allreduce_dequant(H.tp.h, ctx.h, dC.data_ptr(), rows, N, ds.data_ptr(),
                                                  do.data_ptr(), dx.data_ptr()), "tp_allreduce_dequant")
            ctx.synchronize()
            e_ok &= bool(np.array_equal(dx.cpu().numpy().view(np.uint32), want.view(np.uint32)))
        res["exchange"][f"{rows}x{N}"] = e_ok
        ok &= e_ok
    ctx.device_error()

    cfg1 = dict(LLAMA70B, n_layers=2, max_seq=64, max_batch=1, wformat=0, rope_mode=0)
    cfgb = dict(cfg1, max_batch=16)
    rng = np.random.default_rng(7)
    prompt = rng.integers(1, cfg1["vocab"] + 1, size=16).astype(np.int32)
    prompts = rng.integers(1, cfg1["vocab"] + 1, size=(16, 4)).astype(np.int32)

    def run(tp):
        m = LLaMAModel(ctx, cfg1, tp=tp)
        m.init_random(0, 0.02)
        out = {"prefill": m.forward_llama(prompt)}
        toks, lgs = [int(m.last_tokens()[0])], []
        for _ in range(32):
            nxt, lg = m.decode_step(want_logits=True)
            toks.append(int(nxt[0]))
            lgs.append(lg[0].copy())
        out["greedy"], out["decode_logits"] = np.array(toks), np.stack(lgs)
        m.reset_kv_cache()
        m.set_sampling("top_p", top_p=0.9, seed=5)
        out["top_p"] = m.generate(prompt[None, :], 16)[0]
        m.close()
        mb = LLaMAModel(ctx, cfgb, tp=tp)
        mb.init_random(0, 0.02)
        out["batch16"] = np.stack(mb.generate(prompts, 4))
        mb.close()
        ctx.synchronize()
        return out

    got = run(H.tp)
    torch.cuda.empty_cache()
    checks = {}
    if rank == 0:
        ref = run(None)
        for k in ("prefill", "decode_logits"):
            checks[k] = bool(np.array_equal(got[k].view(np.uint32), ref[k].view(np.uint32)))
        for k in ("greedy", "top_p", "batch16"):
            checks[k] = bool(np.array_equal(got[k], ref[k]))
        ok &= all(checks.values())
        torch.cuda.empty_cache()
    flag = torch.tensor([0.0 if ok else 1.0], device="cuda", dtype=torch.float64)
    H.dist.all_reduce(flag)
    res["model"] = ("LLaMA-70B widths (hidden 8192, 64/8 heads, FFN 28672, vocab 32000), 2 layers, "
                    "random-init 3.5-bit; prefill 16 tokens, 32 greedy steps, 16 top-p tokens, batch 16 x 4 tokens")
    res["checks"] = checks
    res["ok"] = float(flag.item()) == 0.0
    res["seconds"] = time.time() - t0
    return res


def gemv_section(H, args):
    """Headline + projection sweep + e2e; every rank runs its shard of the layer."""
    import ctypes as C
    import numpy as np
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import QuantizedMatrix
    L, ctx, world = _lib.load(), H.ctx, H.world
    shapes = shard(SHAPES, world)
    SETS = 3   # weight copies rotated between launches, so no launch hits L2
    mats = {}
    for fmt in (0, 1):
        for st in range(SETS):
            for i, (nm, K, N) in enumerate(shapes):
                h = C.c_void_p()
                _lib.check(L.q35_weights_generate(ctx.h, fmt, N, K, 100 * H.rank + st, 10 * i + fmt + 1, 0.02,
                                                  C.byref(h)), "weights_generate")
                mats[(fmt, st, nm)] = QuantizedMatrix.from_handle(ctx, h, K, N, fmt)
    maxM = max(BATCHES)
    xs, outs = {}, {}
    for i, (nm, K, N) in enumerate(shapes):
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
            for nm, _, _ in shapes:
                launch(fmt, st, M, nm)

    def shape_launches(nm, reps):       # one graph = reps launches of one shape
        for r in range(reps):
            launch(0, r % SETS, 1, nm)

    def graph_of(fn):
        fn()                      # first run outside capture: workspace sized, attributes set
        ctx.synchronize()
        return ctx.capture(fn)

    def step_range(s0, n):              # steps s0 .. s0+n-1, step i on weight copy i % SETS
        for i in range(s0, s0 + n):
            for nm, _, _ in shapes:
                launch(0, i % SETS, 1, nm)

    rank_bytes = sum(algo_bytes(0, 1, K, N) for _, K, N in shapes)
    step_bytes = H.sum_over_ranks(rank_bytes)
    # exactly W warm-up steps, then exactly K timed steps, each a CUDA graph of its steps
    g_warm = graph_of(lambda: step_range(0, args.warmup))
    g_main = graph_of(lambda: step_range(args.warmup, args.steps))
    steps_timed = args.steps
    res = {"steps_timed": steps_timed}
    with ClockSampler(H.uuid()) as clk:
        g_warm.launch()
        ms_total = H.time_ms(g_main.launch, 1, 0)
        ms_step = ms_total / steps_timed
        per_shape = {}
        for nm, K, N in shapes:
            g = graph_of(lambda nm=nm: shape_launches(nm, 12))
            n = max(2, args.steps // 40)
            t = H.time_ms(g.launch, n, 2) / (12 * n)
            g.close()
            bb = algo_bytes(0, 1, K, N)
            per_shape[nm] = {"K": K, "N": N, "us": t * 1e3, "GBps": bb / (t * 1e-3) / 1e9}
        sweep = {}
        for fmt in (0, 1):
            for M in BATCHES:
                if fmt == 0 and M == 1:
                    continue
                g = graph_of(lambda fmt=fmt, M=M: layer_steps(fmt, M))
                n = max(2, args.steps // 12)
                s_ms = H.time_ms(g.launch, n, 1) / (n * SETS)
                g.close()
                b = H.sum_over_ranks(sum(algo_bytes(fmt, M, K, N) for _, K, N in shapes))
                sweep[f"{'q35' if fmt == 0 else 'int4'}_m{M}"] = {
                    "GBps": b / (s_ms * 1e-3) / 1e9, "us_per_layer": s_ms * 1e3,
                    "engine": "tensor cores (tcgen05 kind::i8)" if M >= 5 else "CUDA cores (dp4a)"}
        # the model's launch structure (fused q|k|v and gate|up), M = 1
        fshapes = shard(FUSED, world)
        fmats = {}
        for st in range(SETS):
            for i, (nm, K, N) in enumerate(fshapes):
                h = C.c_void_p()
                _lib.check(L.q35_weights_generate(ctx.h, 0, N, K, 100 * H.rank + st, 50 + i, 0.02, C.byref(h)),
                           "weights_generate")
                fmats[(st, nm)] = QuantizedMatrix.from_handle(ctx, h, K, N, 0)
        fx = {}
        for i, (nm, K, N) in enumerate(fshapes):
            x = torch.empty(K, dtype=torch.int8, device="cuda")
            _lib.check(L.q35_gen_int8_dev(x.data_ptr(), x.numel(), 0, 2000 + i, None))
            fx[nm] = (x, torch.empty(N, dtype=torch.int32, device="cuda"), torch.empty(N, dtype=torch.float32, device="cuda"))
        torch.cuda.synchronize()

        def fused_steps():
            for st in range(SETS):
                for nm, _, _ in fshapes:
                    x, Cd, Yd = fx[nm]
                    fmats[(st, nm)].gemm_dev(x.data_ptr(), 1, Cd.data_ptr(), Yd.data_ptr())

        g = graph_of(fused_steps)
        n = max(2, args.steps // 6)
        f_ms = H.time_ms(g.launch, n, 1) / (n * SETS)
        g.close()
        fb = H.sum_over_ranks(sum(algo_bytes(0, 1, K, N) for _, K, N in fshapes))
        res["layer_fused_m1"] = {"GBps": fb / (f_ms * 1e-3) / 1e9, "us_per_layer": f_ms * 1e3,
                                 "launches": [f"{nm} {K}->{N}" for nm, K, N in fshapes]}
        for qm in fmats.values():
            qm.close()
    res["clocks"] = clk.summary()
    ctx.device_error()
    res["value"] = step_bytes / (ms_step * 1e-3) / 1e9
    res["ms_per_step"] = ms_step
    sweep["q35_m1"] = {"GBps": res["value"], "us_per_layer": ms_step * 1e3, "engine": "CUDA cores (dp4a)"}
    res["sweep"], res["per_shape_m1"] = sweep, per_shape

    # e2e through the C ABI with page-locked host buffers: q35_matmul_cached called as the
    # Fortran drop-in matmul_int4_cublas_cached calls it (A in, fp32 Out back, no int32 C;
    # matmul_cublas.f90:279-325), H2D of x and D2H of y straight to and from the caller's
    # buffers
    keep = []

    def pinned(n, dt):
        t = torch.empty(n, dtype=dt, pin_memory=True)
        keep.append(t)
        return t.numpy()

    hA, hY = {}, {}
    for nm, K, N in shapes:
        hA[nm] = pinned(K, torch.int8)
        hA[nm][:] = xs[nm][:K].cpu().numpy()
        hY[nm] = pinned(N, torch.float32)

    def e2e_step(st):
        for nm, K, N in shapes:
            _lib.check(L.q35_matmul_cached(ctx.h, mats[(0, st, nm)].h, hA[nm].ctypes.data, 1,
                                           None, hY[nm].ctypes.data), "matmul_cached")

    for i in range(max(args.warmup, 3)):
        e2e_step(i % SETS)
    e_steps = max(args.steps // 4, 12)
    H.barrier()
    t0 = time.perf_counter()
    for i in range(e_steps):
        e2e_step(i % SETS)
    e_dt = H.max_over_ranks((time.perf_counter() - t0) / e_steps)
    res["e2e"] = {"value": step_bytes / e_dt / 1e9, "unit": UNIT,
                  "h2d_bytes_per_step": sum(K for _, K, _ in shapes),
                  "d2h_bytes_per_step": sum(4 * N for _, _, N in shapes),
                  "api": "q35_matmul_cached per projection as matmul_int4_cublas_cached calls it (page-locked "
                         "host int8 A in, host fp32 Out back), synchronous, wall clock, max over ranks"}
    g_main.close()
    g_warm.close()
    for qm in mats.values():
        qm.close()
    return res


def prefill_section(H, args):
    """M=2048 GEMMs on the tensor cores (3.5-bit weights, 2 copies rotated: > L2)."""
    import ctypes as C
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import QuantizedMatrix
    L, ctx = _lib.load(), H.ctx
    M = 2048
    out = {}
    for i, (nm, K, N) in enumerate((("gate", 8192, 28672), ("down", 28672, 8192))):
        mats = []
        for st in range(2):
            h = C.c_void_p()
            _lib.check(L.q35_weights_generate(ctx.h, 0, N, K, st, 500 + i, 0.02, C.byref(h)), "weights_generate")
            mats.append(QuantizedMatrix.from_handle(ctx, h, K, N, 0))
        x = torch.empty(M * K, dtype=torch.int8, device="cuda")
        _lib.check(L.q35_gen_int8_dev(x.data_ptr(), x.numel(), 0, 600 + i, None))
        Cd = torch.empty(M * N, dtype=torch.int32, device="cuda")
        Yd = torch.empty(M * N, dtype=torch.float32, device="cuda")
        it = [0]

        def one():
            mats[it[0] % 2].gemm_dev(x.data_ptr(), M, Cd.data_ptr(), Yd.data_ptr())
            it[0] += 1

        n = 10
        ms = H.time_ms(one, n, 3) / n
        ops = 2.0 * M * K * N
        out[nm] = {"M": M, "K": K, "N": N, "ms": ms, "TOPS": ops / (ms * 1e-3) / 1e12}
        for qm in mats:
            qm.close()
        del x, Cd, Yd
    # int8 tensor-core reference throughput on this GPU: cuBLASLt int8 GEMM through torch
    try:
        a = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device="cuda")
        b = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device="cuda")
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = 1e9
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        lib_tops = 2.0 * 8192 ** 3 / (best * 1e-3) / 1e12
        del a, b
    except Exception as e:   # reported, not fatal
        lib_tops = None
        out["int8_library_error"] = str(e)
    out["int8_library_TOPS"] = lib_tops
    out["int8_nominal_TOPS"] = NOMINAL_INT8_TOPS
    for nm in ("gate", "down"):
        out[nm]["frac_of_nominal"] = out[nm]["TOPS"] / NOMINAL_INT8_TOPS
        if lib_tops:
            out[nm]["frac_of_library"] = out[nm]["TOPS"] / lib_tops
    out["note"] = ("int8 ops = 2*M*K*N; the kernel decodes the 3.5-bit weights in shared memory and runs "
                   "tcgen05.mma kind::i8; 'library' = torch._int_mm (cuBLASLt int8) 8192^3 on the same GPU")
    torch.cuda.empty_cache()
    return out


def decode_section(H, args):
    """Greedy decode, random-init 3.5-bit weights, TP over the run's GPUs."""
    import numpy as np
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.llama_model import LLAMA13B, LLAMA70B, LLaMAModel
    hbm, _ = peaks()
    L, ctx, world = _lib.load(), H.ctx, H.world
    runs = [("llama70b", LLAMA70B, 512, 512, 1), ("llama70b", LLAMA70B, 512, 512, 16)]
    if world == 1:
        runs += [("llama13b", LLAMA13B, 128, 256, 1), ("llama13b", LLAMA13B, 128, 256, 8)]
    out = {}
    for name, base, prompt, steps, b in runs:
        cfg = dict(base, max_seq=prompt + steps, max_batch=b, wformat=0, rope_mode=0)
        t0 = time.time()
        m = LLaMAModel(ctx, cfg, tp=H.tp)
        m.init_random(0, 0.02)
        ctx.synchronize()
        t_init = time.time() - t0
        rng = np.random.default_rng(1)
        prompts = rng.integers(1, cfg["vocab"] + 1, size=(b, prompt)).astype(np.int32)
        m.reset_kv_cache()
        H.barrier()
        t0 = time.perf_counter()
        for s in range(b):
            m.forward_next_token(prompts[s], seq=s)
        t_prefill = H.max_over_ranks(time.perf_counter() - t0)
        m.decode_step()                       # first step builds the CUDA graph
        ctx.synchronize()
        ms = H.time_ms(lambda: _lib.check(L.q35_model_decode_steps_async(m.h, steps - 1), "decode"), 1, 0)
        ms_step = ms / (steps - 1)
        ctx.device_error()
        # bytes streamed per step by one rank: its weights (without the embedding table,
        # of which a step reads one row) and its KV cache at the mean position
        hidden, Vg = cfg["hidden"], cfg["vocab"]
        w_rank = m.weight_bytes - 4 * Vg * hidden
        kvh = cfg["n_kv_heads"] // world
        mean_pos = prompt + steps / 2
        kv_rank = cfg["n_layers"] * 2 * kvh * cfg["head_dim"] * 4 * mean_pos * b
        bytes_rank = w_rank + kv_rank
        roof_tok_s = b / (bytes_rank / (hbm * 1e9))
        tok_s = b * 1000.0 / ms_step
        out[f"{name}_b{b}"] = {
            "tp": world, "batch": b, "prompt": prompt, "steps": steps, "ms_per_step": ms_step,
            "tok_s": tok_s, "weight_GB_per_rank": w_rank / 1e9, "kv_GB_per_rank_mean": kv_rank / 1e9,
            "roofline_tok_s": roof_tok_s, "roofline_frac": tok_s / roof_tok_s,
            "hbm_GBps_per_rank": bytes_rank / (ms_step * 1e-3) / 1e9,
            "prefill_s": t_prefill, "prefill_tok_s": b * prompt / t_prefill, "init_s": t_init}
        m.close()
        torch.cuda.empty_cache()
    out["note"] = ("tok/s = batch x steps / CUDA-event time of the graph-replayed decode steps (max over "
                   "ranks); roofline = batch / (bytes one rank streams per step / measured HBM GB/s): its "
                   "weights except the embedding table, plus its KV cache at the mean position; prefill is "
                   "one forward per sequence, wall clock")
    return out


def run_ours(args):
    H = Harness()
    sections = set(args.sections.split(","))
    hbm, peak_kind = peaks()
    result = None
    parity = None
    if H.world > 1 and not args.no_parity:
        parity = tp_parity(H)
        if not parity["ok"]:
            if H.rank == 0:
                print(json.dumps({"metric": METRIC, "value": None, "unit": UNIT, "n_gpus": H.world,
                                  "parity": parity, "error": "tensor-parallel parity failed; nothing timed"}),
                      flush=True)
            raise SystemExit(1)
    if "gemv" in sections:
        g = gemv_section(H, args)
        achieved = g["per_shape_m1"]["gate"]["GBps"]
        traffic = None
        # DRAM bytes of one gate launch from the ncu capture summarised in the profile
        tf = os.path.join(ROOT, "profiles", "gemv_q35_gate_m1.md")
        if os.path.exists(tf) and H.world == 1:
            mt = re.search(r"dram_bytes_per_launch[^|]*\|\s*(\d+)", open(tf).read())
            traffic = int(mt.group(1)) if mt else None
        gate = g["per_shape_m1"]["gate"]
        result = {"metric": METRIC, "value": g["value"], "unit": UNIT, "n_gpus": H.world,
                  "steps": g["steps_timed"], "warmup": args.warmup, "ms_per_step": g["ms_per_step"],
                  "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                  "dtype": "int8 x 3.5-bit -> int32 (+fp32 dequant)", "data": "synthetic",
                  "config": config(H.world, {"timing": "W warm-up steps then the K timed steps, each set "
                                                       "one CUDA graph (step i on weight copy i mod 3); "
                                                       "CUDA events on the library stream, max over ranks"}),
                  "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                               "frac": achieved / hbm, "peak_kind": peak_kind, "traffic": traffic,
                               "kernel": f"gemv_kernel<3.5-bit, MT=1>, gate launch {gate['K']}->{gate['N']} "
                                         "(algorithmic bytes per launch / CUDA-event launch time)",
                               "frac_vs_8TBps": achieved / 8000.0,
                               "algo_bytes_per_launch": algo_bytes(0, 1, gate["K"], gate["N"])},
                  "e2e": g["e2e"], "gpu_launches": g["steps_timed"] * len(SHAPES),
                  "clocks": g["clocks"], "per_shape_m1": g["per_shape_m1"], "sweep": g["sweep"],
                  "layer_fused_m1": g["layer_fused_m1"]}
        if parity is not None:
            result["parity"] = parity
    if "prefill" in sections and H.world == 1:
        pf = prefill_section(H, args)
        if result is not None:
            result["prefill"] = pf
        elif H.rank == 0:
            print(json.dumps({"prefill": pf}), flush=True)
    if "decode" in sections:
        dc = decode_section(H, args)
        if result is not None:
            result["decode"] = dc
        elif H.rank == 0:
            print(json.dumps({"decode": dc}), flush=True)
    if result is not None and H.rank == 0 and H.world == 1 and not args.no_cpu_baseline:
        try:
            result["cpu_baseline"] = cpu_baseline()
        except Exception as e:  # reported, not fatal
            result["cpu_baseline"] = {"value": None, "error": str(e)}
    if result is not None and H.rank == 0:
        print(json.dumps(result), flush=True)
    if H.tp is not None:
        H.tp.close()
    H.ctx.close()
    if H.dist is not None:
        H.dist.barrier()
        H.dist.destroy_process_group()


def run_case(args):
    """A few launches of one projection (for profiler captures): --case name:fmt:M."""
    import ctypes as C
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import Context, QuantizedMatrix
    nm, fmt, M = args.case.split(":")
    fmt, M = int(fmt), int(M)
    K, N = {n: (k, c) for n, k, c in SHAPES + [("prefill_gate", 8192, 28672), ("prefill_down", 28672, 8192)]}[nm]
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
    ctx.device_error()
    print(json.dumps({"case": args.case, "launches": args.warmup + args.steps,
                      "algo_bytes_per_launch": algo_bytes(fmt, M, K, N)}))
    qm.close()
    ctx.close()


def run_decode_case(args):
    """LLaMA-70B-shape decode steps with fewer layers (for profiler captures):
    --decode-case layers:batch:prompt:steps.  Random-init 3.5-bit weights, one prefill per
    sequence, the first decode step (which builds the step's CUDA graph), then `steps`
    graph-replayed decode steps."""
    import numpy as np
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.llama_model import LLAMA70B, LLaMAModel
    from asicfortranai_b200.quantized import Context
    layers, b, prompt, steps = (int(v) for v in args.decode_case.split(":"))
    L = _lib.load()
    ctx = Context(0)
    cfg = dict(LLAMA70B, n_layers=layers, max_seq=prompt + steps + 1, max_batch=b, wformat=0, rope_mode=0)
    m = LLaMAModel(ctx, cfg)
    m.init_random(0, 0.02)
    rng = np.random.default_rng(1)
    prompts = rng.integers(1, cfg["vocab"] + 1, size=(b, prompt)).astype(np.int32)
    for s in range(b):
        m.forward_next_token(prompts[s], seq=s)
    m.decode_step()
    _lib.check(L.q35_model_decode_steps_async(m.h, steps), "decode")
    ctx.synchronize()
    ctx.device_error()
    print(json.dumps({"decode_case": args.decode_case, "tokens": m.last_tokens().tolist()}))
    m.close()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--sections", default="gemv,prefill,decode",
                    help="comma list of gemv (headline, sweep, e2e), prefill, decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the tensor-parallel parity check at N > 1")
    ap.add_argument("--case", default=None, help="profile helper: name:fmt:M, e.g. gate:0:1")
    ap.add_argument("--decode-case", default=None,
                    help="profile helper: LLaMA-70B-shape decode, layers:batch:prompt:steps, e.g. 4:1:512:20")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.case:
        run_case(args)
    elif args.decode_case:
        run_decode_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
