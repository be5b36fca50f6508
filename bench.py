"""Benchmark for the B200 LARQL quantized-matvec backend (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Default workload `c2_q4k` = the Q4_K cells of BASELINE.json configs[1]: weights
4096x4096, 14336x4096, 4096x14336, 128256x4096 (LARQL Q4_K, 148 B / 256 values,
quantized on the device by the bit-exact port of `quantize_q4_k` from f32
~ N(0, 0.02)), x ~ N(0, 1) f32 at batch 1, 4 and 8.  One step = all 12 matvecs
(381 MB of weights read per batch size, 1.14 GB per step — larger than the
126 MB L2, so every step streams the weights from HBM).  The same sweep in
Q4_0 (18 B / 32), GGUF Q8_0 (34 B / 32) and Q6_K (210 B / 256), quantized on the
device by the bit-exact ports of `quantize_q4_0` / `quantize_q8_0` /
`quantize_q6_k`, is timed the same way and reported under "formats"
(--formats q4k drops it).

metric = algorithmic bytes (weight bytes + 4*K*B + 4*N*B per matvec) / time.
At N > 1 GPUs each matrix is row-sharded across the ranks and the row-shard
outputs are all-gathered over NCCL every step (strong scaling).
"""
from __future__ import annotations

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
sys.path.insert(0, os.path.join(ROOT, "encoding-experiment_b200"))

SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]  # (rows N, cols K)
BATCHES = [1, 4, 8]


def workload_cells(name: str):
    """-> (description, [(rows, cols, copies)], batches).

    c2_q4k  BASELINE configs[1], Q4_K cells (default): 4 shapes x batch 1/4/8.
    c1_q4k  BASELINE configs[0]: one 11008x4096 Q4_K matvec, batch 1; 10 weight
            copies (260 MB) are read round-robin so the step exceeds the 126 MB L2.
    cell:NxKxB  a single matvec cell (profiling).
    (c5_gate and gate:B run only the gate walk; see run_gate_only.)
    """
    if name == "c2_q4k":
        return "c2_q4k (BASELINE configs[1], Q4_K cells)", [(n, k, 1) for n, k in SHAPES], BATCHES
    if name == "c1_q4k":
        return "c1_q4k (BASELINE configs[0], 10 rotating weight copies)", [(11008, 4096, 10)], [1]
    if name.startswith("cell:"):
        n, k, b = (int(v) for v in name[5:].split("x"))
        return f"cell {n}x{k} batch {b}", [(n, k, 1)], [b]
    raise SystemExit(f"unknown workload {name}")


def algo_bytes(rows: int, cols: int, batch: int) -> int:
    return rows * cols // 256 * 148 + 4 * cols * batch + 4 * rows * batch


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU, read through NVML every ~2 ms by a thread.

    Only samples taken between mark_start() and mark_end() — the timed region — enter summary().
    Falls back to `nvidia-smi -lms 50` when NVML cannot be loaded."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, gpu_index: int, period_s: float = 0.002):
        self.gpu_index, self.period = gpu_index, period_s
        self.samples = []  # (t, sm_mhz, reason_names, power_w)
        self.sm_max = None
        self.window = (None, None)
        self.stop = threading.Event()
        self.source = None

    def _uuid(self):
        import torch
        u = str(torch.cuda.get_device_properties(self.gpu_index).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u

    def __enter__(self):
        try:
            import pynvml as N
            N.nvmlInit()
            self.N = N
            self.h = N.nvmlDeviceGetHandleByUUID(self._uuid())
            self.sm_max = float(N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM))
            self.bits = [(name, getattr(N, const)) for name, const in self.REASONS]
            self.source = "nvml"
            self.t = threading.Thread(target=self._run_nvml, daemon=True)
        except Exception:
            self.source = "nvidia-smi"
            self.t = threading.Thread(target=self._run_smi, daemon=True)
        self.t.start()
        return self

    def _run_nvml(self):
        N, h = self.N, self.h
        while not self.stop.is_set():
            try:
                t = time.perf_counter()
                sm = float(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM))
                r = N.nvmlDeviceGetCurrentClocksEventReasons(h)
                pw = N.nvmlDeviceGetPowerUsage(h) / 1000.0
                self.samples.append((t, sm, [n for n, b in self.bits if r & b], pw))
            except Exception:
                pass
            time.sleep(self.period)

    def _run_smi(self):
        fields = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                  "clocks_event_reasons.sw_power_cap")
        try:
            p = subprocess.Popen(["nvidia-smi", f"--id={self._uuid()}", f"--query-gpu={fields}",
                                  "--format=csv,noheader,nounits", "-lms", "50"],
                                 stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            return
        for ln in p.stdout:
            parts = [x.strip() for x in ln.split(",")]
            try:
                sm, mx, pw = float(parts[0]), float(parts[1]), float(parts[2])
            except (ValueError, IndexError):
                continue
            self.sm_max = mx
            names = [n for (n, _), v in zip(self.REASONS, parts[3:7]) if v.lower() == "active"]
            self.samples.append((time.perf_counter(), sm, names, pw))
            if self.stop.is_set():
                break
        p.terminate()

    def mark_start(self):
        self.window = (time.perf_counter(), None)

    def mark_end(self):
        self.window = (self.window[0], time.perf_counter())

    def __exit__(self, *a):
        self.stop.set()
        self.t.join(timeout=5)

    def summary(self):
        t0, t1 = self.window
        inside = [s for s in self.samples if t0 is not None and t1 is not None and t0 <= s[0] <= t1]
        sm = [s[1] for s in inside]
        reasons = sorted({n for s in inside for n in s[2]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.sm_max,
                "reasons": reasons, "samples": len(sm),
                "power_w_max": max((s[3] for s in inside), default=None), "source": self.source,
                "window_ms": round((t1 - t0) * 1e3, 1) if t0 is not None and t1 is not None else None}


def dist_setup():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def cpu_q4k_baseline(threads: int, frac: int, min_seconds: float):
    """The oracle port of q4k_matvec.rs:31-87 on the host cores over a row slice of every sweep cell."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cells = []
    for (n, k) in SHAPES:
        rows = max(8, n // frac)
        rng = np.random.default_rng(abs(hash((n, k))) % (2 ** 31))
        w = O.quantize_q4_k(rng.standard_normal(rows * k, dtype=np.float32) * np.float32(0.02))
        x = rng.standard_normal(8 * k, dtype=np.float32)
        cells.append((rows, k, w, x))
    total_bytes, t_total = 0, 0.0
    t_start = time.perf_counter()
    reps = 0
    while True:
        for (rows, k, w, x) in cells:
            for b in BATCHES:
                t0 = time.perf_counter()
                for bi in range(b):
                    O.matvec_mt("q4k", w, np.ascontiguousarray(x[bi * k:(bi + 1) * k]), rows, k, threads)
                t_total += time.perf_counter() - t0
                total_bytes += algo_bytes(rows, k, b)
        reps += 1
        if time.perf_counter() - t_start >= min_seconds:
            break
    return total_bytes / t_total / 1e9, reps, t_total


def _reference_cells(threads: int):
    """Every Q4_K sweep cell at full size for the reference arm: W ~ N(0, 0.02) f32 quantized by the oracle's
    quantize_q4_k (q4_common.rs:104-170), generated and quantized in 4 M-value chunks on the host threads."""
    from concurrent.futures import ThreadPoolExecutor
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cells = []
    for (n, k) in SHAPES:
        per = max(1, (1 << 22) // k)

        def make(r0, n=n, k=k, per=per):
            rc = min(per, n - r0)
            g = np.random.default_rng([n, k, r0])
            return O.quantize_q4_k(g.standard_normal(rc * k, dtype=np.float32) * np.float32(0.02))

        with ThreadPoolExecutor(threads) as ex:
            w = np.concatenate(list(ex.map(make, range(0, n, per))))
        cells.append((n, k, w))
    x = np.random.default_rng(77).standard_normal(max(BATCHES) * max(k for _, k in SHAPES), dtype=np.float32)
    return cells, x


def run_reference(args, world, rank):
    """--impl reference: the reference CPU path on the same workload as our arm — every Q4_K cell of the sweep at
    full size, batch 1 / 4 / 8 as that many trait calls (q4k_matvec takes one vector) — computed by the oracle
    port of q4k_matvec.rs:31-87 (the Rust crate cannot be built here) with its rows split over all host threads.
    Steps run until K are done or 120 s of timed work have passed (at least 3)."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    t_setup = time.perf_counter()
    cells, x = _reference_cells(threads)
    t_setup = time.perf_counter() - t_setup
    step_bytes = sum(algo_bytes(n, k, b) for (n, k, _) in cells for b in BATCHES)

    def step():
        t0 = time.perf_counter()
        for b in BATCHES:
            for (n, k, w) in cells:
                for bi in range(b):
                    O.matvec_mt("q4k", w, np.ascontiguousarray(x[bi * k:(bi + 1) * k]), n, k, threads)
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        step()
    times, spent = [], 0.0
    while len(times) < args.steps and (spent < 120.0 or len(times) < 3):
        times.append(step())
        spent += times[-1]
    sec = sum(times) / len(times)
    value = step_bytes / sec / 1e9
    line = {
        "impl": "reference", "metric": "Q4_K matvec HBM GB/s", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": len(times), "steps_requested": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 2), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "q4k x f32", "data": "synthetic",
        "config": {"workload": "c2_q4k (BASELINE configs[1], Q4_K cells)", "matrices": [[n, k, 1] for n, k in SHAPES],
                   "batches": BATCHES},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port", "host": host_cpu(),
                         "sample": f"every Q4_K sweep cell at full size per step ({step_bytes / 1e6:.0f} MB); oracle "
                                   "restatement of q4k_matvec.rs:31-87, rows split over the host threads; weights "
                                   f"generated and quantized on the host in {t_setup:.0f} s (not timed)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


FORMATS = {  # name -> (C-ABI format, bytes per block, values per block, device quantizer, label)
    "q4k": (1, 148, 256, "quantize_q4_k_dev", "Q4_K"),
    "q4_0": (0, 18, 32, "quantize_q4_0_dev", "Q4_0"),
    "q8_0": (5, 34, 32, "quantize_q8_0_dev", "Q8_0"),
    "q6k": (3, 210, 256, "quantize_q6_k_dev", "Q6_K"),
    # GGUF-144 Q4_K: the reference has no encoder that round-trips through its decoder (ggml.rs:228-273), so the
    # timed weights are random bytes with a fixed finite d / dmin in every super-block
    "q4k_gguf": (8, 144, 256, None, "Q4_K_GGUF"),
    # GGUF-144 Q4_K in llama.cpp's layout (the reference's Metal q4kf kernels): random bytes the same way
    "q4k_llama": (9, 144, 256, None, "Q4_K_GGUF_LLAMA"),
}


def fmt_algo_bytes(fmt: str, rows: int, cols: int, batch: int) -> int:
    _, bpb, vpb, _, _ = FORMATS[fmt]
    return rows * cols // vpb * bpb + 4 * cols * batch + 4 * rows * batch


GATE = dict(L=34, F=10240, D=2560, k=10, batches=(1, 64, 1024))


def gate_cpu_baseline(min_seconds: float):
    """The reference's gate KNN after warmup() (f32 dot + top-k, oracle port) on 1 host core, timed over a
    2-layer sample and scaled to the 34-layer walk of one query."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    F, D, L = GATE["F"], GATE["D"], GATE["L"]
    rng = np.random.default_rng(5)
    layers = [(rng.standard_normal(F * D, dtype=np.float32) * np.float32(0.02)).astype(np.float16).astype(np.float32)
              for _ in range(2)]
    q = rng.standard_normal(D, dtype=np.float32)
    n, t0 = 0, time.perf_counter()
    while True:
        for g in layers:
            O.gate_knn_f32(g, q, F, D, GATE["k"])
            n += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    per_layer = (time.perf_counter() - t0) / n
    return 1.0 / (per_layer * L), n, per_layer


def run_gate_walk(args, world, rank, local, be, stream, dev):
    """34 layers x 10240 gate rows x 2560 f16 ~ N(0, 0.02), queries ~ N(0, 1),
    top-10 per (layer, query).  N > 1: each rank holds 10240 / N rows of every layer; per-rank top-10 lists
    are all-gathered over NCCL and merged on every rank."""
    import torch
    import torch.distributed as dist
    import larql_cuda as Lc
    Ln, F, D, k = GATE["L"], GATE["F"], GATE["D"], GATE["k"]
    Fr = F // world
    g = torch.empty(Ln * Fr * D, dtype=torch.float16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(9000 + rank)
    for l in range(Ln):
        g[l * Fr * D:(l + 1) * Fr * D] = (torch.randn(Fr * D, generator=gen, device=dev) * 0.02).half()
    wt = be.register_weight(g, Lc.FMT_F16_HALFRS, Ln * Fr, D)
    del g
    torch.cuda.synchronize()
    hbm, peak_kind = peaks()
    tflops_peak = 1627.1
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tflops_peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        pass
    out = {"config": "BASELINE configs[4]: 34 x 10240 x 2560 f16 gates ~ N(0,0.02), queries ~ N(0,1), top-10; "
                     "gates generated on the device",
           "kernel": "batch 1-4: gate_gemv_kernel (CUDA cores, f32 dots of the f16 rows) + gate_merge; larger batches: "
                     "gate_query_prep + gate_tc_kernel (tcgen05 kind::f16, M128 N256) + gate_merge"
                     + (" + NCCL all-gather of per-rank top-10 + topk_merge_lists" if world > 1 else ""),
           "batches": {}}
    offs = torch.tensor([r * Fr for r in range(world)], dtype=torch.int32, device=dev)
    steps = max(3, min(args.steps, 20))
    for B in GATE["batches"]:
        q = torch.randn(B, D, generator=gen, device=dev)
        oi = torch.empty(Ln * B * k, dtype=torch.int32, device=dev)
        osc = torch.empty(Ln * B * k, dtype=torch.float32, device=dev)
        gi = torch.empty(world * Ln * B * k, dtype=torch.int32, device=dev) if world > 1 else None
        gs = torch.empty(world * Ln * B * k, dtype=torch.float32, device=dev) if world > 1 else None
        mi = torch.empty(Ln * B * k, dtype=torch.int32, device=dev) if world > 1 else None
        ms_ = torch.empty(Ln * B * k, dtype=torch.float32, device=dev) if world > 1 else None

        def walk():
            be.gate_topk_dev(wt, Ln, Fr, q, B, k, oi, osc, stream=stream.cuda_stream)
            if world > 1:
                with torch.cuda.stream(stream):
                    dist.all_gather_into_tensor(gi, oi)
                    dist.all_gather_into_tensor(gs, osc)
                be.topk_merge_dev(gi, gs, world, Ln * B, k, k, mi, ms_, offsets=offs, stream=stream.cuda_stream)

        for _ in range(max(3, args.warmup)):
            walk()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            walk()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        gate_bytes = Ln * F * D * 2 + 4 * B * D + 8 * Ln * B * k
        flops = 2.0 * B * Ln * F * D
        ent = {"ms_per_batch": round(ms, 4), "queries_per_s": round(B / (ms * 1e-3), 1),
               "GBps": round(gate_bytes / (ms * 1e-3) / 1e9, 1), "TFLOPs": round(flops / (ms * 1e-3) / 1e12, 2)}
        if B <= 64:
            ent["roofline"] = {"bound": "hbm", "achieved": ent["GBps"], "peak": hbm, "unit": "GB/s",
                               "frac": round(ent["GBps"] / hbm / world, 4), "peak_kind": peak_kind,
                               "algo_bytes": gate_bytes}
        else:
            ent["roofline"] = {"bound": "tensor", "achieved": ent["TFLOPs"], "peak": tflops_peak, "unit": "TFLOP/s",
                               "frac": round(ent["TFLOPs"] / tflops_peak / world, 4), "peak_kind": "measured bf16",
                               "algo_flops": flops,
                               "note": "algorithmic flops count each product once; the kernel issues two f16 MMAs "
                                       "per product (query hi and lo planes)"}
        # e2e: pinned host queries in, (index, score) lists out, every step
        qh = q.cpu().pin_memory()
        ih = torch.empty(Ln * B * k, dtype=torch.int32).pin_memory()
        sh = torch.empty(Ln * B * k, dtype=torch.float32).pin_memory()
        src_i, src_s = (mi, ms_) if world > 1 else (oi, osc)

        def e2e():
            with torch.cuda.stream(stream):
                q.copy_(qh, non_blocking=True)
            walk()
            with torch.cuda.stream(stream):
                ih.copy_(src_i, non_blocking=True)
                sh.copy_(src_s, non_blocking=True)
            stream.synchronize()

        e2e()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            e2e()
        es = (time.perf_counter() - t0) / steps
        if world > 1:
            t = torch.tensor([es], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            es = float(t.item())
        ent["e2e"] = {"value": round(B / es, 1), "unit": "queries/s", "h2d_bytes_per_step": 4 * B * D,
                      "d2h_bytes_per_step": 8 * Ln * B * k}
        out["batches"][str(B)] = ent
    if rank == 0 and world == 1 and not args.no_cpu:
        qps, n, per_layer = gate_cpu_baseline(8.0)
        out["cpu_baseline"] = {"value": round(qps, 3), "unit": "queries/s", "cores": 1, "kind": "port",
                               "sample": f"{n} layer scans of 10240 x 2560 pre-decoded f32 rows, one query "
                                         f"({per_layer * 1e3:.1f} ms each, x34 layers); oracle port of the "
                                         "reference's post-warmup() gate_knn (f32 dot, AVX2/FMA when present)"}
    wt.release()
    return out


def run_gate_q4(args, world, rank, local, be, stream, dev):
    """gate_knn_q4 / gate_knn_adaptive's Q4 branch (gate.rs:672-731) at the configs[4] shape: 34 layers x 10240
    Q4_0 gate rows x 2560 (quantized on the device from N(0, 0.02)), one query ~ N(0, 1), top-10 by |score| per
    layer: quantize_to_q8, one Q4_0 x Q8 matvec over every layer's rows, candidate + merge selection."""
    import torch
    import larql_cuda as Lc
    Ln, F, D, k = GATE["L"], GATE["F"], GATE["D"], GATE["k"]
    q4 = torch.empty(Ln * F * D // 32 * 18, dtype=torch.uint8, device=dev)
    gen = torch.Generator(device=dev).manual_seed(9100)
    lb = F * D // 32 * 18
    for l in range(Ln):
        wf = torch.randn(F * D, generator=gen, device=dev) * 0.02
        torch.cuda.synchronize()
        be.quantize_q4_0_dev(wf, q4[l * lb:(l + 1) * lb])
        be.sync()
        del wf
    wt = be.register_weight(q4, Lc.FMT_Q4_0, Ln * F, D)
    w_host = q4.cpu().numpy()  # for the host entry point, which finds a weight by (host pointer, length)
    del q4
    q = torch.randn(1, D, generator=gen, device=dev)
    oi = torch.empty(Ln * k, dtype=torch.int32, device=dev)
    osc = torch.empty(Ln * k, dtype=torch.float32, device=dev)
    for _ in range(max(3, args.warmup)):
        be.gate_topk_q4_dev(wt, Ln, F, q, 1, k, oi, osc, stream=stream.cuda_stream)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    n0 = Lc.launch_count()
    with torch.cuda.graph(graph, stream=stream):
        be.gate_topk_q4_dev(wt, Ln, F, q, 1, k, oi, osc, stream=stream.cuda_stream)
    launches = Lc.launch_count() - n0
    steps = max(10, min(args.steps, 50))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(steps):
            graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    graph = None
    ms = e0.elapsed_time(e1) / steps
    algo = Ln * lb + 4 * D + 8 * Ln * k
    hbm, peak_kind = peaks()
    gbs = algo / (ms * 1e-3) / 1e9
    # e2e: host query in, host (index, score) lists out, through the synchronous host entry point
    qh = q.cpu().numpy()
    be.gate_knn_q4(w_host, Ln, F, D, qh, k)  # places the host weight once (registry by pointer, length)
    t0 = time.perf_counter()
    for _ in range(steps):
        be.gate_knn_q4(w_host, Ln, F, D, qh, k)
    es = (time.perf_counter() - t0) / steps
    out = {"config": "gate_knn_q4 at the configs[4] shape: 34 x 10240 x 2560 Q4_0 gates (quantized on the device from "
                     "N(0, 0.02)), one query, top-10 by |score| per layer; one CUDA graph per query",
           "ms_per_query": round(ms, 4), "queries_per_s": round(1e3 / ms, 1), "GBps": round(gbs, 1),
           "gpu_launches_per_query": launches,
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(gbs / hbm, 4), "peak_kind": peak_kind, "algo_bytes": algo},
           "e2e": {"value": round(1.0 / es, 1), "unit": "queries/s", "h2d_bytes_per_step": 4 * D,
                   "d2h_bytes_per_step": 8 * Ln * k, "api": "larql_cuda_gate_topk_q4 (host query / lists)"}}
    wt.release()
    return out


DECODE = dict(layers=32, hidden=4096, inter=14336, nq=32, nkv=8, hd=128, seq=2048, theta=500000.0)


def run_lm_head_sharded(args, world, rank, local, be, stream, dev):
    """The lm-head KNN with the 128256-row Q4_0 head row-sharded over N GPUs: each rank takes the top 10 logits of
    its vocabulary rows (quantize_to_q8, Q4_0 x Q8 matvec, logit top-k), the (id, logit) lists are all-gathered over
    NCCL and the top 10 of the N x 10 candidates by signed logit (ties by lower id) is the head's.  One CUDA graph
    per query, timed with CUDA events, max over ranks."""
    import torch
    import torch.distributed as dist
    N, K, k = 128256, 4096, 10
    per = (N + world - 1) // world
    r0, r1 = rank * per, min(N, (rank + 1) * per)
    g = torch.Generator(device=dev).manual_seed(4242 + rank)
    wf = torch.randn((r1 - r0) * K, generator=g, device=dev, dtype=torch.float32) * 0.02
    q4 = torch.empty((r1 - r0) * K // 32 * 18, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    be.quantize_q4_0_dev(wf, q4)
    be.sync()
    del wf
    import larql_cuda as Lc
    wt = be.register_weight(q4, Lc.FMT_Q4_0, r1 - r0, K)
    del q4
    x = torch.randn(K, generator=torch.Generator(device=dev).manual_seed(99), device=dev, dtype=torch.float32)
    ids = torch.empty(k, dtype=torch.int32, device=dev)
    vals = torch.empty(k, dtype=torch.float32, device=dev)
    packed = torch.empty(2 * k, dtype=torch.float32, device=dev)   # [logits | ids as bits]: one collective
    gathered = torch.empty(world * 2 * k, dtype=torch.float32, device=dev)
    gvals = torch.empty(world * k, dtype=torch.float32, device=dev)
    pos = torch.empty(k, dtype=torch.int32, device=dev)
    top = torch.empty(k, dtype=torch.float32, device=dev)
    final = torch.empty(k, dtype=torch.int32, device=dev)

    def query():
        be.lm_head_knn_dev(wt, x, k, ids, vals, stream=stream.cuda_stream)
        with torch.cuda.stream(stream):
            packed[:k].copy_(vals)
            packed[k:].copy_((ids + r0).view(torch.float32))
            dist.all_gather_into_tensor(gathered, packed)
            gvals.copy_(gathered.view(world, 2, k)[:, 0, :].reshape(-1))
        # the top k of the candidates by signed logit; positions map back to vocabulary ids
        be.logit_topk_dev(gvals, world * k, k, pos, top, stream=stream.cuda_stream)
        with torch.cuda.stream(stream):
            final.copy_(gathered.view(world, 2, k)[:, 1, :].reshape(-1).view(torch.int32)[pos.long()])

    for _ in range(max(3, args.warmup)):
        query()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        query()
    torch.cuda.synchronize()
    dist.barrier()
    iters = max(10, min(args.steps, 50))
    for _ in range(3):
        with torch.cuda.stream(stream):
            graph.replay()
    stream.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(iters):
            graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    del graph  # a graph holding NCCL calls goes before the process group
    t = torch.tensor([e0.elapsed_time(e1) * 1e3 / iters], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = float(t.item())
    hbm, peak_kind = peaks()
    algo = N * (K // 32) * 18 + 4 * K * world + 4 * N
    wt.release()
    return {"config": f"lm_head_knn_backend Q4 branch, {N} x {K} Q4_0 head row-sharded over {world} GPUs, top {k}: "
                      "per rank quantize_to_q8 + Q4_0 x Q8 matvec + logit top-k, one NCCL all-gather of the packed "
                      "(logit, id) lists, logit top-k of the candidates; one CUDA graph per query",
            "us_per_query": round(us, 2), "queries_per_s": round(1e6 / us, 1),
            "GBps": round(algo / (us * 1e-6) / 1e9, 1),
            "roofline": {"bound": "hbm", "achieved": round(algo / (us * 1e-6) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(algo / (us * 1e-6) / 1e9 / hbm / world, 4), "peak_kind": peak_kind,
                         "algo_bytes": algo, "note": "frac is per GPU (aggregate rate / N / peak)"}}


def run_lm_head(args, world, rank, local, be, stream, dev):
    """lm_head_knn_backend's Q4 branch (walk.rs:549-583) on the configs[1] lm-head shape: a 128256 x 4096 Q4_0 lm
    head (quantized on the device from N(0, 0.02)), one N(0, 1) query, top 10 logits.  One query = device
    quantize_to_q8, the Q4_0 x Q8 matvec and the two-launch logit top-k, replayed from one CUDA graph; the 296 MB
    head is larger than L2, so every query streams it from HBM."""
    import torch
    import larql_cuda as L
    N, K, k = 128256, 4096, 10
    g = torch.Generator(device=dev).manual_seed(4242)
    wf = torch.randn(N * K, generator=g, device=dev, dtype=torch.float32) * 0.02
    q4 = torch.empty(N * K // 32 * 18, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    be.quantize_q4_0_dev(wf, q4)
    be.sync()
    del wf
    wt = be.register_weight(q4, 0, N, K)
    w_host = q4.cpu().numpy()  # for the host entry point, which finds a weight by (host pointer, length)
    del q4
    x = torch.randn(K, generator=g, device=dev, dtype=torch.float32)
    ids = torch.empty(k, dtype=torch.int32, device=dev)
    vals = torch.empty(k, dtype=torch.float32, device=dev)
    for _ in range(3):
        be.lm_head_knn_dev(wt, x, k, ids, vals, stream=stream.cuda_stream)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    n0 = L.launch_count()
    with torch.cuda.graph(graph, stream=stream):
        be.lm_head_knn_dev(wt, x, k, ids, vals, stream=stream.cuda_stream)
    launches = L.launch_count() - n0
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        with torch.cuda.stream(stream):
            graph.replay()
    iters = max(10, args.steps)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(iters):
            graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / iters
    algo = N * (K // 32) * 18 + 4 * K + 4 * N
    hbm, peak_kind = peaks()
    gbs = algo / (us * 1e-6) / 1e9
    # e2e: host query in, host ids / logits out, through the synchronous host entry point
    import ctypes as C
    qh = x.cpu().pin_memory()
    ih = np.empty(k, np.uint32)
    vh = np.empty(k, np.float32)
    cnt = C.c_size_t(0)
    wt_host = be.register_weight(w_host, 0, N, K)  # placed once, as the registry does on a first call

    def e2e_call():
        L.check(L.lib().larql_cuda_lm_head_knn(be.ctx, w_host.ctypes.data, w_host.nbytes, N, K, qh.data_ptr(), k,
                                               ih.ctypes.data, vh.ctypes.data, C.byref(cnt)))

    for _ in range(3):
        e2e_call()
    t0 = time.perf_counter()
    for _ in range(iters):
        e2e_call()
    e2e_qps = iters / (time.perf_counter() - t0)
    graph = None
    wt.release()
    wt_host.release()
    del w_host
    out = {"config": f"lm_head_knn_backend Q4 branch: {N} x {K} Q4_0 lm head (configs[1] lm-head shape), one "
                     f"query, top {k}; one CUDA graph per query (quantize_to_q8, Q4_0 x Q8 matvec, logit top-k)",
           "us_per_query": round(us, 2), "queries_per_s": round(1e6 / us, 1), "GBps": round(gbs, 1),
           "gpu_launches_per_query": launches,
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(gbs / hbm, 4), "peak_kind": peak_kind, "algo_bytes": algo},
           "e2e": {"value": round(e2e_qps, 1), "unit": "queries/s", "h2d_bytes_per_step": 4 * K,
                   "d2h_bytes_per_step": 8 * k, "api": "larql_cuda_lm_head_knn (host query / ids / logits)"}}
    if rank == 0 and not args.no_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        rows = N // 64
        rng = np.random.default_rng(6)
        wq = O.quantize_q4_0(rng.standard_normal(rows * K, dtype=np.float32) * np.float32(0.02))
        q8, s8 = O.quantize_to_q8(rng.standard_normal(K, dtype=np.float32))
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 5.0:
            O.q4_0_matvec_q8(wq, q8, s8, rows, K)
            n += 1
        per_query = (time.perf_counter() - t0) / n * 64
        out["cpu_baseline"] = {"value": round(1.0 / per_query, 3), "unit": "queries/s", "cores": 1, "kind": "port",
                               "sample": f"{n} Q4_0 x Q8 matvecs over 1/64 of the lm-head rows (5 s), scaled to "
                                         "the whole head; oracle restatement of q4_dot.c:169-199 (top-k not "
                                         "counted)"}
    return out


def run_decode(args, world, rank, local, be, stream, dev):
    """one token through 32 distinct random-init Llama-style Q4_K layers (hidden 4096,
    32 / 8 heads of 128, SwiGLU 14336, RMSNorm eps 1e-5, RoPE theta 500000) at position 2048 over a 2048-token
    f16 KV cache ~ N(0, 1) per layer.  Weights ~ N(0, 0.02) quantized on the device; norms 1 + N(0, 0.02)."""
    import torch
    import torch.distributed as dist
    import larql_cuda as Lc
    D = dict(DECODE, layers=args.decode_layers)
    H, I, nq, nkv, hd, seq = D["hidden"], D["inter"], D["nq"], D["nkv"], D["hd"], D["seq"]
    qd, kvd = nq * hd, nkv * hd
    # every rank builds the same model (same seeds); at world > 1 each registers its head / FFN shard
    # (larql_cuda_layer_register_shard) and the O / down partial sums are all-reduced over NCCL
    gen = torch.Generator(device=dev).manual_seed(4242)
    sharded = world > 1
    kvd_l = kvd // world

    def q4k(rows, cols):
        wf = torch.randn(rows * cols, generator=gen, device=dev) * 0.02
        q = torch.empty(rows * cols // 256 * 148, dtype=torch.uint8, device=dev)
        torch.cuda.synchronize()
        be.quantize_q4_k_dev(wf, q)
        be.sync()
        return q

    be.kv_init(D["layers"], seq + 64, nkv // world, hd)
    handles = []
    for l in range(D["layers"]):
        w = {"q": q4k(qd, H), "k": q4k(kvd, H), "v": q4k(kvd, H), "o": q4k(H, qd), "gate": q4k(I, H),
             "up": q4k(I, H), "down": q4k(H, I)}
        n1 = 1.0 + torch.randn(H, generator=gen, device=dev) * 0.02
        n2 = 1.0 + torch.randn(H, generator=gen, device=dev) * 0.02
        if sharded:
            handles.append(be.layer_register_shard(w, n1, n2, H, I, nq, nkv, rank, world, hd, eps=1e-5))
        else:
            handles.append(be.layer_register(w, n1, n2, H, I, nq, nkv, hd, eps=1e-5))
        kc = torch.randn(seq * kvd, generator=gen, device=dev).half()
        vc = torch.randn(seq * kvd, generator=gen, device=dev).half()
        if sharded:  # this rank's KV heads
            kc = kc.view(seq, kvd)[:, rank * kvd_l:(rank + 1) * kvd_l].contiguous()
            vc = vc.view(seq, kvd)[:, rank * kvd_l:(rank + 1) * kvd_l].contiguous()
        be.kv_populate_f16_dev(l, kc, vc, seq)
        del w, kc, vc
    torch.cuda.synchronize()
    x0 = torch.randn(H, generator=gen, device=dev)
    x = x0.clone()
    red = torch.zeros(H, dtype=torch.float32, device=dev)
    # the O / down partial sums are all-reduced by the library's one-shot peer-memory kernel (NVLink /
    # NVSwitch), or by NCCL when LARQL_BENCH_TP_REDUCE=nccl or the peer mapping is unavailable
    reducer = "nccl"
    if sharded and os.environ.get("LARQL_BENCH_TP_REDUCE", "p2p") == "p2p":
        try:
            hs = [None] * world
            dist.all_gather_object(hs, be.p2p_init(rank, world, H))
            be.p2p_connect(hs)
            reducer = "p2p"
        except Exception as ex:  # noqa: BLE001
            print(f"peer all-reduce unavailable ({ex}); using NCCL", file=sys.stderr)
        flag = torch.tensor([1 if reducer == "p2p" else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)  # every rank takes the same path
        reducer = "p2p" if int(flag.item()) == 1 else "nccl"

    def reduce(buf, n, st):  # all-reduce of the O / down partial sums, on the token's stream
        if reducer == "p2p":
            be.p2p_allreduce_dev(buf, n, stream=st)
        else:
            with torch.cuda.stream(stream):
                dist.all_reduce(red)
        return 0

    def token():
        if sharded:
            be.decode_token_sharded_dev(handles, x, seq, D["theta"], red, reduce, stream=stream.cuda_stream)
        else:
            be.decode_token_dev(handles, x, seq, D["theta"], stream=stream.cuda_stream)

    for _ in range(2):
        token()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    n0 = Lc.launch_count()
    with torch.cuda.graph(graph, stream=stream):
        token()
    launches = Lc.launch_count() - n0
    torch.cuda.synchronize()
    steps = max(5, min(args.steps, 50))
    for _ in range(max(3, args.warmup)):
        with torch.cuda.stream(stream):
            graph.replay()
    stream.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        with torch.cuda.stream(stream):
            graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if sharded:  # the slowest rank's time
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    token_bytes = D["layers"] * (((qd + 2 * kvd) * H + H * qd + 2 * I * H + H * I) // 256 * 148
                                 + (seq + 1) * kvd * 2 * 2)
    hbm, peak_kind = peaks()
    cfg = ("BASELINE configs[2]: 32" if D["layers"] == 32 else
           f"profiling case (NOT the BASELINE config): {D['layers']}")
    out = {"config": cfg + " distinct Llama-style Q4_K layers (4096, 32/8 x 128, SwiGLU 14336), "
                     "one token at position 2048 over 2048-token f16 KV caches; one CUDA graph per token"
                     + (f"; heads and FFN rows sharded over {world} GPUs, "
                        + ("one-shot peer-memory all-reduce" if reducer == "p2p" else "NCCL all-reduce")
                        + " after O and down" if sharded else ""),
           "tokens_per_s": round(1e3 / ms, 1), "ms_per_token": round(ms, 4), "gpu_launches_per_token": launches,
           "roofline": {"bound": "hbm", "achieved": round(token_bytes / (ms * 1e-3) / 1e9, 1), "peak": hbm,
                        "unit": "GB/s", "frac": round(token_bytes / (ms * 1e-3) / 1e9 / hbm, 4),
                        "peak_kind": peak_kind, "algo_bytes_per_token": token_bytes,
                        "ideal_tokens_per_s": round(hbm * 1e9 / token_bytes, 1)}}
    if not sharded:
        # e2e: decode_token with a host x in and the host residual out; the cache length is rewound each step
        xh = x0.cpu().numpy()
        be.kv_set_length(seq)
        be.decode_token(handles, xh, D["theta"])
        t0 = time.perf_counter()
        for _ in range(steps):
            be.kv_set_length(seq)
            be.decode_token(handles, xh, D["theta"])
        es = (time.perf_counter() - t0) / steps
        out["e2e"] = {"value": round(1.0 / es, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * H,
                      "d2h_bytes_per_step": 4 * H, "api": "larql_cuda_decode_token (host x / out, synchronous)"}
        # the same token as one persistent launch (larql_cuda_decode_set_persistent), timed the same way
        be.decode_set_persistent(True)
        try:
            be.kv_set_length(seq)
            token()  # uploads the layers' tensor maps outside the capture
            stream.synchronize()
            pgraph = torch.cuda.CUDAGraph()
            n0 = Lc.launch_count()
            with torch.cuda.graph(pgraph, stream=stream):
                token()
            plaunch = Lc.launch_count() - n0
            for _ in range(max(3, args.warmup)):
                with torch.cuda.stream(stream):
                    pgraph.replay()
            stream.synchronize()
            e0.record(stream)
            for _ in range(steps):
                with torch.cuda.stream(stream):
                    pgraph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            pms = e0.elapsed_time(e1) / steps
            del pgraph
            out["persistent_kernel"] = {
                "tokens_per_s": round(1e3 / pms, 1), "ms_per_token": round(pms, 4), "gpu_launches_per_token": plaunch,
                "frac": round(token_bytes / (pms * 1e-3) / 1e9 / hbm, 4),
                "note": "one cooperative launch per token (decode_persist.cu), opt-in; the per-kernel pipeline above "
                        "is the default"}
        finally:
            be.decode_set_persistent(False)
    else:
        # e2e: the captured sharded token with x copied in from pinned host memory and the residual copied back
        xh = x0.cpu().pin_memory()
        xo = torch.empty(H, dtype=torch.float32).pin_memory()
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(steps):
            with torch.cuda.stream(stream):
                x.copy_(xh, non_blocking=True)
                graph.replay()
                xo.copy_(x, non_blocking=True)
            stream.synchronize()
        es = (time.perf_counter() - t0) / steps
        t = torch.tensor([es], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        es = float(t.item())
        out["e2e"] = {"value": round(1.0 / es, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * H,
                      "d2h_bytes_per_step": 4 * H,
                      "api": "larql_cuda_decode_token_sharded_dev in a CUDA graph, pinned host x / out"}
    del graph  # a graph holding NCCL calls goes before the process group
    torch.cuda.synchronize()
    for h in handles:
        be.layer_release(h)
    be.kv_init(1, 1, nkv // world, hd)  # drop the caches
    return out


def host_cpu():
    """The host CPU model and the threads this process may use (for the CPU baselines)."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    model = ln.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        usable = len(os.sched_getaffinity(0))
    except AttributeError:
        usable = os.cpu_count()
    return {"cpu_model": model, "nproc": usable, "logical_cpus": os.cpu_count()}


C1 = dict(rows=11008, cols=4096, copies=10)


def run_c1(args, world, rank, local, be, stream, dev):
    """one 11008 x 4096 Q4_K matvec at batch 1.  Copy 0 of W is the configs[0] matrix itself
    (numpy PCG64 seed 0, f32 ~ N(0, 0.02)), quantized on the device by the bit-exact port of quantize_q4_k; nine
    more copies from other seeds are read round-robin so that one step (10 launches, 261 MB of weights) is larger
    than the 126 MB L2.  x ~ N(0, 1) f32 (seed 1).  Reported: the step rate, the cold-L2 time of one launch with
    its roofline, e2e through larql_cuda_matvec with pinned host x / y, and (rank 0, N = 1) the oracle port of
    q4k_matvec.rs:31-87 on one host core over the whole configs[0] matrix."""
    import torch
    import larql_cuda as L
    N, K, copies = C1["rows"], C1["cols"], C1["copies"]
    x = torch.from_numpy(np.random.default_rng(1).standard_normal(K, dtype=np.float32)).to(dev)
    y = torch.empty(copies * N, dtype=torch.float32, device=dev)
    wts, w0_host = [], None
    for cp in range(copies):
        if cp == 0:
            wf = torch.from_numpy(np.random.default_rng(0).standard_normal(N * K, dtype=np.float32)
                                  * np.float32(0.02)).to(dev)
        else:
            g = torch.Generator(device=dev).manual_seed(31337 + cp)
            wf = torch.randn(N * K, generator=g, device=dev, dtype=torch.float32) * 0.02
        q = torch.empty(N * K // 256 * 148, dtype=torch.uint8, device=dev)
        torch.cuda.synchronize()
        be.quantize_q4_k_dev(wf, q)
        be.sync()
        del wf
        if cp == 0:
            w0_host = q.cpu().numpy()
        wts.append(be.register_weight(q, L.FMT_Q4_K, N, K))
        del q
    torch.cuda.synchronize()

    def step():
        for cp in range(copies):
            be.matvec_dev(wts[cp], x, y[cp * N:(cp + 1) * N], batch=1, stream=stream.cuda_stream)

    for _ in range(2):
        step()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    n0 = L.launch_count()
    with torch.cuda.graph(graph, stream=stream):
        step()
    launches = L.launch_count() - n0
    steps = max(10, args.steps)
    for _ in range(max(3, args.warmup)):
        with torch.cuda.stream(stream):
            graph.replay()
    stream.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(steps):
            graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    per_launch = algo_bytes(N, K, 1)
    hbm, peak_kind = peaks()
    # one launch with cold L2 (a 256 MB buffer written, then another read, before it), median of 10
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    flush_rd = torch.ones(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    times = []
    for r in range(12):
        with torch.cuda.stream(stream):
            flush.fill_(float(r))
            flush_rd.sum()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        be.matvec_dev(wts[0], x, y[:N], batch=1, stream=stream.cuda_stream)
        ev1.record(stream)
        stream.synchronize()
        if r >= 2:
            times.append(ev0.elapsed_time(ev1) * 1e3)
    del flush, flush_rd
    us = statistics.median(times)
    gbs = per_launch / (us * 1e-6) / 1e9
    # e2e: pinned host x in, host y out, through the synchronous public entry point, every launch
    xh = x.cpu().pin_memory()
    yh = torch.empty(N, dtype=torch.float32).pin_memory()

    def e2e_call(cp):
        L.check(L.lib().larql_cuda_matvec(be.ctx, wts[cp].handle, xh.data_ptr(), 1, yh.data_ptr()))

    for cp in range(copies):
        e2e_call(cp)
    t0 = time.perf_counter()
    for i in range(steps * copies):
        e2e_call(i % copies)
    e2e_s = (time.perf_counter() - t0) / (steps * copies)
    out = {"config": "BASELINE configs[0]: 11008 x 4096 Q4_K (W = numpy seed 0 ~ N(0, 0.02), quantized on the "
                     "device), x ~ N(0, 1), batch 1; a step = the matvec on each of 10 weight copies (261 MB > L2), "
                     "one CUDA graph",
           "value": round(per_launch * copies / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
           "us_per_matvec_in_step": round(ms * 1e3 / copies, 2), "gpu_launches_per_step": launches,
           "kernel": be.describe_matvec(wts[0], 1),
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(gbs / hbm, 4), "peak_kind": peak_kind, "algo_bytes_per_launch": per_launch,
                        "us_per_launch": round(us, 2),
                        "timing": "median of 10 cold-L2 launches (256 MB written, then 256 MB read before each)"},
           "e2e": {"value": round(per_launch / e2e_s / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * K,
                   "d2h_bytes_per_step": 4 * N, "us_per_call": round(e2e_s * 1e6, 2),
                   "api": "larql_cuda_matvec (pinned host x / y, synchronous)"}}
    if rank == 0 and world == 1 and not args.no_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        xn = xh.numpy().copy()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 6.0:
            O.q4k_matvec(w0_host, xn, N, K)
            n += 1
        per = (time.perf_counter() - t0) / n
        out["cpu_baseline"] = {"value": round(per_launch / per / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                               "ms_per_matvec": round(per * 1e3, 1), "host": host_cpu(),
                               "sample": f"{n} full configs[0] matvecs (copy 0, the same bytes) on one core; oracle "
                                         "restatement of q4k_matvec.rs:31-87 (sequential f32, as the reference)"}
    graph = None
    for w in wts:
        w.release()
    return out


PREFILL = dict(tokens=512, hidden=4096, inter=14336)


def run_prefill(args, world, rank, local, be, stream, dev):
    """512 tokens x 4096 f32 activations ~ N(0,1) through the Q4_K FFN (gate/up 14336 x 4096,
    down 4096 x 14336, from N(0, 0.02)): y = down . (silu(gate . x) * (up . x)), 180.4 GFLOP per call."""
    import torch
    import larql_cuda as Lc
    P = PREFILL
    T, H, I = P["tokens"], P["hidden"], P["inter"]
    gen = torch.Generator(device=dev).manual_seed(5151 + rank)

    w_host = {}

    def q4k(rows, cols, name):
        wf = torch.randn(rows * cols, generator=gen, device=dev) * 0.02
        q = torch.empty(rows * cols // 256 * 148, dtype=torch.uint8, device=dev)
        torch.cuda.synchronize()
        be.quantize_q4_k_dev(wf, q)
        be.sync()
        w_host[name] = q.cpu().numpy()
        return be.register_weight(q, Lc.FMT_Q4_K, rows, cols)

    wg, wu, wd = q4k(I, H, "g"), q4k(I, H, "u"), q4k(H, I, "d")
    x = torch.randn(T * H, generator=gen, device=dev)
    y = torch.empty(T * H, device=dev)
    for _ in range(3):
        be.prefill_ffn_dev(wg, wu, wd, x, T, y, stream=stream.cuda_stream)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    n0 = Lc.launch_count()
    with torch.cuda.graph(graph, stream=stream):
        be.prefill_ffn_dev(wg, wu, wd, x, T, y, stream=stream.cuda_stream)
    launches = Lc.launch_count() - n0
    steps = max(5, min(args.steps, 30))
    for _ in range(max(3, args.warmup)):
        with torch.cuda.stream(stream):
            graph.replay()
    stream.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        with torch.cuda.stream(stream):
            graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    flops = 2.0 * T * H * I * 3
    # the same graph replayed for ~0.1 s with the SM clock, power and clock-event reasons sampled: the timed
    # region above is too short for the sampler, and a long run shows whether the GEMMs settle under the power cap
    sus_n = max(50, int(100.0 / max(ms, 1e-3)))
    with ClockSampler(local) as clk:
        time.sleep(0.02)
        clk.mark_start()
        e0.record(stream)
        for _ in range(sus_n):
            with torch.cuda.stream(stream):
                graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        clk.mark_end()
    sus_ms = e0.elapsed_time(e1) / sus_n
    sustained = {"calls": sus_n, "ms_per_call": round(sus_ms, 4),
                 "TFLOPs": round(flops / (sus_ms * 1e-3) / 1e12, 1), "clocks": clk.summary()}
    peak = 1627.1
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        pass
    tf = flops / (ms * 1e-3) / 1e12
    out = {"config": "BASELINE configs[3]: 512 x 4096 f32 activations through Q4_K gate/up 14336 x 4096 and down "
                     "4096 x 14336 (SwiGLU); f16 dequantized tiles, f32 accumulate, one CUDA graph",
           "ms_per_call": round(ms, 4), "tokens_per_s": round(T / (ms * 1e-3), 1), "TFLOPs": round(tf, 1),
           "gpu_launches_per_call": launches,
           "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(tf / peak, 4), "peak_kind": "measured bf16 (dense f16 has the same rate)",
                        "algo_flops": flops},
           "sustained_0.1s": sustained}
    xh = x.cpu().pin_memory()
    yh = torch.empty(T * H, dtype=torch.float32).pin_memory()

    def e2e():
        with torch.cuda.stream(stream):
            x.copy_(xh, non_blocking=True)
            graph.replay()
            yh.copy_(y, non_blocking=True)
        stream.synchronize()

    e2e()
    t0 = time.perf_counter()
    for _ in range(steps):
        e2e()
    es = (time.perf_counter() - t0) / steps
    out["e2e"] = {"value": round(T / es, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * T * H,
                  "d2h_bytes_per_step": 4 * T * H, "api": "the captured graph with pinned host x / y copies"}
    # the prefill_q4 ownership form: host weights (placed once, found by pointer), host x in, host y out
    hw = [w_host[n] for n in ("g", "u", "d")]
    xn = xh.numpy()
    be.prefill_ffn(hw[0], hw[1], hw[2], xn, H, I)
    t0 = time.perf_counter()
    for _ in range(max(3, steps // 2)):
        be.prefill_ffn(hw[0], hw[1], hw[2], xn, H, I)
    es = (time.perf_counter() - t0) / max(3, steps // 2)
    out["e2e_host_entry"] = {"value": round(T / es, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * T * H,
                             "d2h_bytes_per_step": 4 * T * H,
                             "api": "larql_cuda_prefill_ffn (host weights / x / y, synchronous)"}
    del graph
    for w in (wg, wu, wd):
        w.release()
    return out


def run_prefill_only(args, world, rank, local):
    """--workload c4_prefill: the prefill FFN of configs[3] alone (1 GPU)."""
    import torch
    import larql_cuda as L
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    be = L.CudaBackend(local)
    stream = torch.cuda.Stream(device=dev)
    pf = run_prefill(args, world, rank, local, be, stream, dev)
    if rank == 0:
        line = {"metric": "prefill FFN TFLOP/s", "value": pf["TFLOPs"], "unit": "TFLOP/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": pf["ms_per_call"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f16 dequantized Q4_K x f16 activations, f32 accumulate", "data": "synthetic",
                "config": {"workload": "c4_prefill: " + pf["config"], "parallelism": "single GPU"},
                "roofline": pf["roofline"], "e2e": pf["e2e"], "prefill": pf,
                "gpu_launches": pf["gpu_launches_per_call"] * max(5, min(args.steps, 30))}
        print(json.dumps(line), flush=True)
    be.close()


def run_decode_partitions(args, world, rank, dev):
    """The collectives per decoded token of the two tensor-parallel partitions of the configs[2] layer (32 layers,
    hidden 4096, intermediate 14336), NCCL in one CUDA graph per token, max over ranks.  Both read 1/N of every
    weight per rank; they differ only in what crosses NVLink per layer.  "columns" (the library's decode): Q|K|V by
    heads and gate|up by rows, O and down by the matching input columns, their partial sums all-reduced: 2
    all-reduces of the 4096-float hidden vector.  "rows" (row shards with all-gathered outputs, the matvec's
    partition): O then needs the whole attention output and down the whole SwiGLU activation: all-gathers of the
    attention output (4096), the O output (4096), the activation (14336) and the down output (4096)."""
    import torch
    import torch.distributed as dist
    H, I, layers = DECODE["hidden"], DECODE["inter"], DECODE["layers"]
    stream = torch.cuda.Stream(device=dev)
    hid = torch.zeros(H, device=dev)
    shard_h, full_h = torch.zeros(H // world, device=dev), torch.zeros(H, device=dev)
    shard_i, full_i = torch.zeros(I // world, device=dev), torch.zeros(I, device=dev)

    def columns():
        for _ in range(layers):
            dist.all_reduce(hid)
            dist.all_reduce(hid)

    def rows():
        for _ in range(layers):
            dist.all_gather_into_tensor(full_h, shard_h)
            dist.all_gather_into_tensor(full_h, shard_h)
            dist.all_gather_into_tensor(full_i, shard_i)
            dist.all_gather_into_tensor(full_h, shard_h)

    out = {"what": "collectives per decoded token (NCCL, one CUDA graph, max over ranks); the weight bytes per rank "
                   "are the same in both partitions",
           "library_uses": "columns, over its peer-memory all-reduce (the decode section's timing)"}
    iters = max(10, min(args.steps, 50))
    for name, fn in (("columns_2_allreduce_per_layer", columns), ("rows_4_allgather_per_layer", rows)):
        with torch.cuda.stream(stream):
            fn()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            fn()
        for _ in range(3):
            with torch.cuda.stream(stream):
                graph.replay()
        stream.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(iters):
                graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph  # a graph holding NCCL calls goes before the process group
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
        out[name] = {"us_per_token": round(us, 1), "us_per_layer": round(us / layers, 2)}
    return out


def run_decode_only(args, world, rank, local):
    """--workload c3_decode: the decode token of configs[2] alone (heads and FFN rows sharded at N > 1)."""
    import torch
    import torch.distributed as dist
    import larql_cuda as L
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    be = L.CudaBackend(local)
    stream = torch.cuda.Stream(device=dev)
    dec = run_decode(args, world, rank, local, be, stream, dev)
    if rank == 0:
        line = {"metric": "decode tokens/s", "value": dec["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": dec["ms_per_token"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "q4k x f32 (int8 digit planes), f16 KV, f32 activations", "data": "synthetic",
                "config": {"workload": "c3_decode: " + dec["config"],
                           "parallelism": "single GPU" if world == 1 else f"tensor parallel x{world} (heads, FFN rows)"},
                "roofline": dec["roofline"], "e2e": dec["e2e"], "decode": dec,
                "gpu_launches": dec["gpu_launches_per_token"] * max(5, min(args.steps, 50))}
        print(json.dumps(line), flush=True)
    be.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_gate_only(args, world, rank, local):
    """--workload c5_gate (batches 1, 64, 1024) or gate:B: the gate walk alone, headline = queries/s of the
    largest batch."""
    import torch
    import torch.distributed as dist
    import larql_cuda as L
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    be = L.CudaBackend(local)
    stream = torch.cuda.Stream(device=dev)
    if args.workload.startswith("gate:"):
        GATE["batches"] = (int(args.workload[5:]),)
    n0 = L.launch_count()
    gate = run_gate_walk(args, world, rank, local, be, stream, dev)
    launches = L.launch_count() - n0
    if rank == 0:
        bmax = str(max(GATE["batches"]))
        ent = gate["batches"][bmax]
        line = {"metric": "gate-walk queries/s", "value": ent["queries_per_s"], "unit": "queries/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ent["ms_per_batch"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f16 gates x f32 queries (f16 hi/lo planes), f32 accumulate", "data": "synthetic",
                "config": {"workload": f"{args.workload}: {gate['config']}", "batch": int(bmax),
                           "parallelism": f"gate-row shard x{world}"},
                "roofline": ent["roofline"], "e2e": ent["e2e"], "gate_walk": gate,
                "gpu_launches": launches}
        if "cpu_baseline" in gate:
            line["cpu_baseline"] = gate["cpu_baseline"]
        print(json.dumps(line), flush=True)
    be.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_gate_q4_only(args, world, rank, local):
    """--workload gate_q4: the Q4_0 gate walk of gate_knn_q4 alone at the configs[4] shape (1 GPU)."""
    import torch
    import larql_cuda as L
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    be = L.CudaBackend(local)
    stream = torch.cuda.Stream(device=dev)
    g = run_gate_q4(args, world, rank, local, be, stream, dev)
    if rank == 0:
        line = {"metric": "gate-walk (Q4_0) queries/s", "value": g["queries_per_s"], "unit": "queries/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": g["ms_per_query"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "Q4_0 gates x Q8 queries, int32 / f32 accumulate", "data": "synthetic",
                "config": {"workload": "gate_q4: " + g["config"], "parallelism": "single GPU"},
                "roofline": g["roofline"], "e2e": g["e2e"], "gate_walk_q4": g,
                "gpu_launches": g["gpu_launches_per_query"] * max(10, min(args.steps, 50))}
        print(json.dumps(line), flush=True)
    be.close()


def run_ours(args, world, rank, local):
    import torch
    import torch.distributed as dist
    import larql_cuda as L

    if args.workload == "c5_gate" or args.workload.startswith("gate:"):
        return run_gate_only(args, world, rank, local)
    if args.workload == "gate_q4":
        return run_gate_q4_only(args, world, rank, local)
    if args.workload == "c3_decode":
        return run_decode_only(args, world, rank, local)
    if args.workload == "c4_prefill":
        return run_prefill_only(args, world, rank, local)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    be = L.CudaBackend(local)
    stream = torch.cuda.Stream(device=dev)

    wl_desc, wl_mats, BATCHES = workload_cells(args.workload)
    formats = ([f for f in args.formats.split(",") if f]
               if args.workload == "c2_q4k" or args.workload.startswith("cell:") else ["q4k"])
    if formats[0] != "q4k":
        raise SystemExit("the headline format (first in --formats) must be q4k")
    maxb = max(BATCHES)
    # ── weights: each rank owns a contiguous row shard of every matrix; quantized on the device ──
    xs = {}
    cells = {f: [] for f in formats}
    for fmt in formats:
        _, bpb, vpb, quantizer, _ = FORMATS[fmt]
        for (n, k, copies) in wl_mats:
            per = (n + world - 1) // world
            r0 = rank * per
            rs = max(0, min(per, n - r0))
            if k not in xs:
                gx = torch.Generator(device=dev).manual_seed(77 + k)
                xs[k] = torch.randn(maxb * k, generator=gx, device=dev, dtype=torch.float32)
            for cp in range(copies):
                g = torch.Generator(device=dev).manual_seed(1000 + n * 7 + k + rank + 100003 * cp)
                wf = torch.randn(max(rs, 1) * k, generator=g, device=dev, dtype=torch.float32) * 0.02
                q = torch.empty(max(rs, 1) * k // vpb * bpb, dtype=torch.uint8, device=dev)
                torch.cuda.synchronize()
                if quantizer is None:
                    q.view(-1, bpb).copy_(torch.randint(0, 256, (q.numel() // bpb, bpb), generator=g, device=dev,
                                                        dtype=torch.int64).to(torch.uint8))
                    q.view(-1, bpb)[:, 0:4] = torch.tensor([0x18, 0x1A, 0x18, 0x16], dtype=torch.uint8, device=dev)
                else:
                    getattr(be, quantizer)(wf, q)
                be.sync()
                del wf
                wt = be.register_weight(q, FORMATS[fmt][0], max(rs, 1), k)
                del q
                cells[fmt].append(dict(n=n, k=k, per=per, rs=rs, wt=wt, x=xs[k], copy=cp))
    # Every (cell, batch) of a format writes its own slice of one output buffer, so the row-shard outputs of a
    # whole step are all-gathered by ONE collective per step (N > 1).  Slices start on 16-byte boundaries.
    yslices, ybufs, yfull = {}, {}, {}
    for fmt in formats:
        off = 0
        for ci, c in enumerate(cells[fmt]):
            for b in BATCHES:
                yslices[(fmt, ci, b)] = off
                off += (b * c["per"] + 3) // 4 * 4
        ybufs[fmt] = torch.zeros(max(off, 4), device=dev, dtype=torch.float32)
        yfull[fmt] = torch.zeros(max(off, 4) * world, device=dev, dtype=torch.float32) if world > 1 else None
        for ci, c in enumerate(cells[fmt]):
            c["y"] = {b: ybufs[fmt][yslices[(fmt, ci, b)]:yslices[(fmt, ci, b)] + b * c["per"]] for b in BATCHES}
    torch.cuda.synchronize()

    def step(fmt, s):
        # batches outer, matrices inner: consecutive launches read different matrices, so no launch finds its
        # weights in L2 from the launch before (the lm-head's 304 MB sits between two reads of any matrix)
        for b in BATCHES:
            for c in cells[fmt]:
                if c["rs"] > 0:
                    be.matvec_dev(c["wt"], c["x"], c["y"][b], batch=b, stream=s.cuda_stream)

    def gather(fmt, s):
        if world > 1:
            with torch.cuda.stream(s):
                dist.all_gather_into_tensor(yfull[fmt], ybufs[fmt])

    # warm-up (also sets kernel attributes before capture); one CUDA graph per format
    graphs, launches = {}, {}
    for fmt in formats:
        for _ in range(2):
            step(fmt, stream)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        n0 = L.launch_count()
        with torch.cuda.graph(graph, stream=stream):
            step(fmt, stream)
        launches[fmt] = L.launch_count() - n0
        graphs[fmt] = graph
    torch.cuda.synchronize()

    def timed(n_iter, fn, clk=None):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        if clk:
            clk.mark_start()
        e0.record(stream)
        for _ in range(n_iter):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        if clk:
            clk.mark_end()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def one_step(fmt):
        with torch.cuda.stream(stream):
            graphs[fmt].replay()
        gather(fmt, stream)

    def step_bytes(fmt):
        return sum(fmt_algo_bytes(fmt, c["n"], c["k"], b) for c in cells[fmt] for b in BATCHES)

    with ClockSampler(local) as clk:
        time.sleep(0.05)
        for _ in range(args.warmup):
            one_step("q4k")
        total_ms = timed(args.steps, lambda: one_step("q4k"), clk)
    ms_step = total_ms / args.steps
    value = step_bytes("q4k") / (ms_step * 1e-3) / 1e9
    sharded = None
    if world > 1:
        # the same step split into its two parts, each timed on its own (max over ranks): the row-shard kernels
        # alone (aggregate HBM rate over all GPUs) and the one all-gather of the step's outputs alone
        def kern_step():
            with torch.cuda.stream(stream):
                graphs["q4k"].replay()

        ms_k = timed(args.steps, kern_step) / args.steps
        ms_g = timed(args.steps, lambda: gather("q4k", stream)) / args.steps
        sharded = {"kernels_only": {"value": round(step_bytes("q4k") / (ms_k * 1e-3) / 1e9, 2), "unit": "GB/s",
                                    "ms_per_step": round(ms_k, 4),
                                    "per_gpu_GBps": round(step_bytes("q4k") / world / (ms_k * 1e-3) / 1e9, 2)},
                   "gather_only": {"ms_per_step": round(ms_g, 4), "bytes_per_rank": int(ybufs["q4k"].numel() * 4),
                                   "collectives_per_step": 1},
                   "note": "value (end to end) = kernels + one NCCL all-gather of the step's 12 row-shard outputs"}

    other = {}
    for fmt in formats[1:]:
        for _ in range(args.warmup):
            one_step(fmt)
        ms = timed(args.steps, lambda: one_step(fmt)) / args.steps
        other[FORMATS[fmt][4]] = {"value": round(step_bytes(fmt) / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                                  "ms_per_step": round(ms, 4), "gpu_launches_per_step": launches[fmt]}

    # ── per-launch kernel timing (dominant kernel roofline) ──
    # Each launch is bracketed by CUDA events on the launching stream.  Before
    # it a 256 MB buffer is overwritten (no launch finds its weights in L2) and
    # a second 256 MB buffer is read, so the dirty lines of the first are
    # written back before the timed launch rather than during it.
    hbm, peak_kind = peaks()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    flush_rd = torch.ones(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    cell_stats = []
    dom = None
    for fmt in formats:
        seen = set()
        for c in cells[fmt]:
            key = (c["n"], c["k"])
            if key in seen or c["rs"] == 0:
                continue
            seen.add(key)
            for b in BATCHES:
                times = []
                for r in range(12):
                    with torch.cuda.stream(stream):
                        flush.fill_(float(r))
                        flush_rd.sum()
                    ev0 = torch.cuda.Event(enable_timing=True)
                    ev1 = torch.cuda.Event(enable_timing=True)
                    ev0.record(stream)
                    be.matvec_dev(c["wt"], c["x"], c["y"][b], batch=b, stream=stream.cuda_stream)
                    ev1.record(stream)
                    stream.synchronize()
                    if r >= 2:
                        times.append(ev0.elapsed_time(ev1) * 1e3)
                us = statistics.median(times)
                nb = fmt_algo_bytes(fmt, c["rs"], c["k"], b)
                gbs = nb / (us * 1e-6) / 1e9
                kern = be.describe_matvec(c["wt"], b)
                cell_stats.append({"format": FORMATS[fmt][4], "rows": c["rs"], "cols": c["k"], "batch": b,
                                   "us": round(us, 2), "GBps": round(gbs, 1), "frac": round(gbs / hbm, 3),
                                   "kernel": kern})
                if fmt == "q4k" and b == BATCHES[0] and (dom is None or nb > dom[0]):
                    dom = (nb, us, gbs, f"{c['rs']}x{c['k']} batch {b}", kern, c)
    del flush, flush_rd
    if dom is None:
        dom = (0, 0.0, 0.0, "none", "none", None)
    # The same kernel back to back: 10 launches on the largest Q4_K weight captured in one graph and replayed, the
    # average launch from CUDA events around the replays.  Where that weight is more than twice the 126 MB L2, each
    # launch streams it from HBM again (the previous launch leaves only its last ~126 MB in L2, which this one
    # evicts before it reaches them), so this is the steady state a token loop sees; it becomes `achieved`.
    # Smaller shards (N > 1) keep the cold single-launch figure.
    b2b = {}
    if dom[5] is not None and fmt_algo_bytes("q4k", dom[5]["rs"], dom[5]["k"], 1) > 2 * 126e6:
        c = dom[5]
        for b in BATCHES:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(10):
                    be.matvec_dev(c["wt"], c["x"], c["y"][b], batch=b, stream=stream.cuda_stream)
            for _ in range(2):
                with torch.cuda.stream(stream):
                    g.replay()
            stream.synchronize()
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    g.replay()
            ev1.record(stream)
            stream.synchronize()
            us = ev0.elapsed_time(ev1) * 1e3 / 30
            nb = fmt_algo_bytes("q4k", c["rs"], c["k"], b)
            b2b[str(b)] = {"us_per_launch": round(us, 2), "GBps": round(nb / (us * 1e-6) / 1e9, 1),
                           "frac": round(nb / (us * 1e-6) / 1e9 / hbm, 4), "kernel": be.describe_matvec(c["wt"], b)}
            g = None

    # ── e2e through the public API with host buffers (pinned), one call per Q4_K cell ──
    h2d = d2h = 0
    host_x = {}
    host_y = {}
    for c in cells["q4k"]:
        host_x[c["k"]] = c["x"].cpu().pin_memory()
        host_y[(c["n"], c["k"])] = torch.empty(maxb * max(c["rs"], 1), dtype=torch.float32).pin_memory()

    def e2e_step():
        for c in cells["q4k"]:
            for b in BATCHES:
                if c["rs"] == 0:
                    continue
                xh = host_x[c["k"]]
                yh = host_y[(c["n"], c["k"])]
                L.check(L.lib().larql_cuda_matvec(be.ctx, c["wt"].handle, xh.data_ptr(), b, yh.data_ptr()))

    for c in cells["q4k"]:
        for b in BATCHES:
            if c["rs"]:
                h2d += 4 * c["k"] * b
                d2h += 4 * c["rs"] * b
    for _ in range(2):
        e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    e2e_iters = max(3, args.steps // 2)
    for _ in range(e2e_iters):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / e2e_iters
    if world > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_val = step_bytes("q4k") / e2e_s / 1e9

    sb = step_bytes("q4k")
    n_step_cells = len(cells["q4k"])
    c1 = None
    if args.workload == "c2_q4k" and not args.no_c1 and world == 1:
        for fmt in formats:
            for c in cells[fmt]:
                c["wt"].release()
        cells = {f: [] for f in formats}
        graphs.clear()
        c1 = run_c1(args, world, rank, local, be, stream, dev)
    gate = None
    if args.workload == "c2_q4k" and not args.no_gate:
        for fmt in formats:
            for c in cells[fmt]:
                c["wt"].release()
        cells = {f: [] for f in formats}
        graphs.clear()
        gate = run_gate_walk(args, world, rank, local, be, stream, dev)
    gate_q4 = None
    if args.workload == "c2_q4k" and not args.no_gate and world == 1:
        gate_q4 = run_gate_q4(args, world, rank, local, be, stream, dev)
    lm_head = None
    if args.workload == "c2_q4k" and not args.no_lm_head:
        lm_head = (run_lm_head(args, world, rank, local, be, stream, dev) if world == 1 else
                   run_lm_head_sharded(args, world, rank, local, be, stream, dev))
    decode = None
    if args.workload == "c2_q4k" and not args.no_decode:
        decode = run_decode(args, world, rank, local, be, stream, dev)
        if world > 1 and decode is not None and DECODE["hidden"] % world == 0 and DECODE["inter"] % world == 0:
            decode["partitions_comm"] = run_decode_partitions(args, world, rank, dev)
    prefill = None
    if args.workload == "c2_q4k" and not args.no_prefill and world == 1:
        prefill = run_prefill(args, world, rank, local, be, stream, dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and args.workload == "c2_q4k":
        threads = 1
        gbs, reps, secs = cpu_q4k_baseline(threads, 64, 10.0)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port", "host": host_cpu(),
               "sample": f"{reps} pass(es) over every Q4_K sweep cell on 1/64 of its rows ({secs:.1f} s); "
                         "oracle restatement of q4k_matvec.rs:31-87 (the Rust crate cannot be built here)"}

    traffic = None
    tp = os.path.join(ROOT, "profiles", "q4k_matvec_traffic.json")
    if os.path.exists(tp):
        try:
            with open(tp) as f:
                tj = json.load(f)
            if tj.get("cell") == dom[3]:
                traffic = tj.get("dram_bytes_per_launch")
        except Exception:
            traffic = None

    # the batch-1 figure, or the smallest batch a single-cell workload runs
    ach = b2b[min(b2b, key=int)]["GBps"] if b2b else round(dom[2], 1)
    if rank == 0:
        line = {
            "metric": "Q4_K matvec HBM GB/s", "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "q4k x f32 (int8 digit planes, int32/f32 accumulate)",
            "data": "synthetic (W ~ N(0,0.02) quantized on device with the reference quantizers; x ~ N(0,1))",
            "config": {"workload": wl_desc, "matrices": [list(m) for m in wl_mats],
                       "batches": BATCHES, "step": f"{n_step_cells * len(BATCHES)} Q4_K matvecs, one CUDA graph",
                       "l2": f"inputs larger than L2 ({sb / 1e6:.0f} MB read per step vs 126 MB L2)"
                       if sb > 2 * 126e6 else "single cell (profiling): L2 may hold the weights",
                       "parallelism": f"row-shard x{world}"
                       + (" + NCCL all-gather of outputs" if world > 1 else "")},
            "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                         "frac": round(ach / hbm, 4), "traffic": traffic,
                         "timing": ("average of 30 back-to-back launches (10 per CUDA graph, the 304 MB weight > 2x L2, "
                                    "so every launch reads it from HBM), CUDA events on the launching stream"
                                    if b2b else
                                    "median of 10 cold-L2 launches (256 MB written, then 256 MB read before each), "
                                    "CUDA events on the launching stream"),
                         "kernel": f"{dom[4]} on {dom[3]} (largest batch-1 cell)",
                         "peak_kind": peak_kind, "algo_bytes_per_launch": dom[0],
                         "us_per_launch": b2b[min(b2b, key=int)]["us_per_launch"] if b2b else round(dom[1], 2),
                         "cold_single_launch": {"us": round(dom[1], 2), "GBps": round(dom[2], 1),
                                                "frac": round(dom[2] / hbm, 4)},
                         "back_to_back_by_batch": b2b or None},
            "formats": other,
            "sharded": sharded,
            "c1": c1,
            "cells": cell_stats,
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "api": "larql_cuda_matvec (host pinned x/y, synchronous per call)"},
            "gate_walk": gate,
            "gate_walk_q4": gate_q4,
            "lm_head_knn": lm_head,
            "decode": decode,
            "prefill": prefill,
            "gpu_launches": launches["q4k"] * args.steps,
            "clocks": clk.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    for fmt in formats:
        for c in cells[fmt]:
            c["wt"].release()
    graphs.clear()
    be.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2_q4k",
                    help="c2_q4k | c1_q4k | cell:NxKxB | c5_gate | gate:B | gate_q4 | c3_decode | c4_prefill")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-gate", action="store_true", help="skip the gate-walk (configs[4]) section")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode (configs[2]) section")
    ap.add_argument("--no-lm-head", action="store_true", help="skip the lm-head KNN section")
    ap.add_argument("--decode-layers", type=int, default=32,
                    help="layers of the decode token (32 = configs[2]; fewer only for small profiling captures)")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill (configs[3]) section")
    ap.add_argument("--no-c1", action="store_true", help="skip the configs[0] section")
    ap.add_argument("--formats", default="q4k,q4_0,q8_0,q6k,q4k_gguf,q4k_llama",
                    help="c2 formats: q4k (headline) then extra formats reported under 'formats'")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup()
    run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
