"""Benchmark of the quantization hot path on B200 (one JSON line on rank 0).

Headline workload (the second benchmark configuration, "C2"): quantize float32 weights
[11008, 4096] ~ N(0, 0.02^2) three ways per step, through the reference's op
API (torch.ops.quantized_ops):
  * NF4 per-group 64: quantize_mx(w, lut4 index table, [-1], 64, 1.0)
    (block absmax scale computed in the same pass),
  * posit8_1 per-tensor: quantize(w, amax/4096, qmap=posit8_1),
  * int8 per-output-channel: quantize(w, row_amax/127, qmap=int8).
metric = algorithmic GB/s over the three (8.0625 + 8 + 8 bytes per element),
whole job (all ranks).  Multi-GPU: every rank quantizes its own weight matrix
(weak scaling, no collective on the data path).

Secondary results in the same line ("secondary"): C1 NVFP4 round trip GB/s,
C3 MXFP8 quantized-linear TFLOP/s, the C4 W4A8 sweep on one GPU, the outlier
CSR side-stream (quantize_mx_outlier on C1's input, C3 with a 1 % activation
CSR), and the C5 4-layer decoder forward (tensor parallel over the ranks when
N > 1).

--impl reference times the reference algorithm's CPU restatement (the oracle
port under oracle/) on this host's cores, on whole steps of the same
workload (a window of rows that moves from step to step instead, should
--steps whole ones run past REF_BUDGET_SECONDS).
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "voyager-compiler_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

ROWS, COLS = 11008, 4096
# one metric string for both arms (the driver pairs the lines by it)
METRIC = ("C2 weight quantize throughput (NF4 g64 + posit8 per-tensor + int8 "
          "per-channel), algorithmic bytes")
DATA = "synthetic (seeded PCG64 N(0,0.02^2))"
WORKLOAD = ("C2 fp32 [11008,4096]: NF4 g64 quantize_mx / posit8_1 per-tensor / int8 "
            "per-channel quantize")
# per-launch DRAM bytes (read + write) of the C2 kernels, from one ncu capture
# of the current kernels: python bench.py --only c2 --steps 1 --warmup 1, under
# ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none
# -k regex:"k_qmx_last|k_rows" (mean of two launches each)
NCU_TRAFFIC = {"int8_channel": int(311.6e6), "nf4_g64": int(304.5e6),
               "posit8_tensor": int(309.8e6)}
L2_BYTES = 126e6  # B200 L2
BYTES_PER_ELEM = {"nf4_g64": 4 + 4 + 4.0 / 64, "posit8_tensor": 8.0, "int8_channel": 8.0}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", default=None,
                    choices=["c1", "c2", "c3", "c4", "c4m128", "c4m1024", "c5", "attn", "outlier",
                             "spmm", "dq", "nvf4", "observer"],
                    help="profiling aid: run only this workload's kernels, no JSON line")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port, threaded over row chunks
# ---------------------------------------------------------------------------
def cpu_step(w_rows, tables, threads):
    """One C2 step on a row sample with the oracle (all host threads)."""
    from concurrent.futures import ThreadPoolExecutor

    import oracle

    idx_tab, posit_tab, int8_tab = tables
    sp = np.array(np.abs(w_rows).max() / np.float32(4096.0), dtype=np.float32).reshape(())
    si = (np.abs(w_rows).max(axis=1, keepdims=True) / np.float32(127.0)).astype(np.float32)
    n = w_rows.shape[0]
    bounds = np.linspace(0, n, threads + 1).astype(int)

    def work(i):
        lo, hi = bounds[i], bounds[i + 1]
        oracle.quantize_mx(w_rows[lo:hi], idx_tab, [-1], 64, 1.0)
        oracle.quantize(w_rows[lo:hi], sp, qmap=posit_tab)
        oracle.quantize(w_rows[lo:hi], si[lo:hi], qmap=int8_tab)

    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(work, range(threads)))


def load_synth():
    """The seeded input generators, loaded by file path: the reference arm
    must not import the voyager_b200 package (that maps the CUDA library
    and registers its kernels)."""
    import importlib.util

    spec = importlib.util.spec_from_file_location(
        "vq_bench_synth", os.path.join(ROOT, "voyager-compiler_b200", "voyager_b200", "synth.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def cpu_tables():
    from oracle.numerics import index_table, quantization_map

    return index_table(quantization_map("lut4")), quantization_map("posit8_1"), quantization_map("int8")


def bytes_per_row():
    return COLS * sum(BYTES_PER_ELEM.values())


CPU_MIN_SECONDS = 10.0     # CPU work the cpu_baseline leg times at least
REF_BUDGET_SECONDS = 150.0  # the reference arm's timed steps, at most about


def cpu_baseline(min_seconds=CPU_MIN_SECONDS, min_reps=3):
    """The oracle port on whole C2 steps (all rows: the 180 MB weight does
    not stay in the host's caches, as a row sample would), all host
    threads, repeated for at least min_seconds."""
    synth = load_synth()

    threads = os.cpu_count() or 1
    w = synth.c2_weight()
    tabs = cpu_tables()
    cpu_step(w, tabs, threads)  # warm
    reps, t0 = 0, time.perf_counter()
    while reps < min_reps or time.perf_counter() - t0 < min_seconds:
        cpu_step(w, tabs, threads)
        reps += 1
    total = time.perf_counter() - t0
    return {"value": round(ROWS * bytes_per_row() / (total / reps) / 1e9, 3), "unit": "GB/s",
            "cores": threads, "kind": "port",
            "sample": f"whole steps: all {ROWS} rows of the C2 weight, 3 quantizations, "
                      f"mean of {reps} steps over {total:.1f} s"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    synth = load_synth()

    threads = os.cpu_count() or 1
    w_full = synth.c2_weight()
    tabs = cpu_tables()
    # the first warm-up step is a whole one and sizes the rest: whole steps
    # while --steps of them fit the time budget, else a window of rows that
    # moves through the weight from step to step
    t0 = time.perf_counter()
    cpu_step(w_full, tabs, threads)
    t_full = time.perf_counter() - t0
    sample_rows = ROWS
    if t_full * args.steps > REF_BUDGET_SECONDS:
        sample_rows = max(1024, int(ROWS * REF_BUDGET_SECONDS / (t_full * args.steps)))
    for i in range(max(0, args.warmup - 1)):
        cpu_step(w_full[:sample_rows], tabs, threads)
    times = []
    for i in range(args.steps):
        lo = (i * sample_rows) % (ROWS - sample_rows) if sample_rows < ROWS else 0
        t0 = time.perf_counter()
        cpu_step(w_full[lo:lo + sample_rows], tabs, threads)
        times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    val = sample_rows * bytes_per_row() / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": DATA,
        "config": {"workload": WORKLOAD, "sample_rows_per_step": sample_rows},
        "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port",
                         "sample": (f"whole steps ({ROWS} rows)" if sample_rows == ROWS else
                                    f"{sample_rows} of {ROWS} rows per step, a moving window")},
        "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            self.path = f"/tmp/vq_clocks_{os.getpid()}.csv"
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm,"
                 "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=self.f, stderr=subprocess.DEVNULL)
            t0 = time.time()
            while time.time() - t0 < 5 and os.path.getsize(self.path) == 0:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) < 7:
                continue
            try:
                sm.append(float(p[0]))
                mx = float(p[1])
            except ValueError:
                continue
            for n, v in zip(names, p[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        os.remove(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def run_ours(args):
    import torch

    rank, world, local = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py: needs a CUDA GPU (the CUDA path has no fallback)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        pg = dist
    import voyager_b200  # noqa: F401
    from voyager_b200 import synth
    from voyager_b200.tables import get_quantization_map, index_table

    Q = torch.ops.quantized_ops
    peaks = {}
    pth = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pth):
        peaks = json.load(open(pth))
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"

    w_host = synth.c2_weight()
    w = torch.from_numpy(w_host).to(dev)
    idx_tab = index_table(get_quantization_map("lut4")).to(dev)
    posit = get_quantization_map("posit8_1", dev)
    i8 = get_quantization_map("int8", dev)
    # the scales as calibration leaves them: the device amax observer
    sp, si = observed_scales(w)
    stream = torch.cuda.current_stream(dev)

    def step():
        Q.quantize_mx(w, idx_tab, [-1], 64, 1.0, False)
        Q.quantize(w, sp, qmap=posit)
        Q.quantize(w, si, qmap=i8)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    # per-kernel launch times (CUDA events on the launching stream)
    names = list(BYTES_PER_ELEM)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        # the stream first spins (about 40 us of GPU time per launch to come)
        # so the host queues the timed launches ahead of the device: the
        # events then time the kernels, not the host's first launch latency
        torch.cuda._sleep(int(3 * args.steps * 40e-6 * 2e9))
        t_start.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            Q.quantize_mx(w, idx_tab, [-1], 64, 1.0, False)
            ev[i][1].record(stream)
            Q.quantize(w, sp, qmap=posit)
            ev[i][2].record(stream)
            Q.quantize(w, si, qmap=i8)
            ev[i][3].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    if pg:
        pg.barrier()
    # no kernel of the library gave up a bounded wait (outside the timing)
    voyager_b200.check_errors(dev)
    ms = t_start.elapsed_time(t_end)
    per = {n: [ev[i][j].elapsed_time(ev[i][j + 1]) for i in range(args.steps)]
           for j, n in enumerate(names)}
    if pg:
        t = torch.tensor([ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    elems = ROWS * COLS
    total_bytes = elems * sum(BYTES_PER_ELEM.values()) * world * args.steps
    value = total_bytes / (ms / 1e3) / 1e9
    mean_ms = {n: sum(v) / len(v) for n, v in per.items()}
    dom = max(mean_ms, key=mean_ms.get)
    achieved = elems * BYTES_PER_ELEM[dom] / (mean_ms[dom] / 1e3) / 1e9
    kernels = {n: {"ms": round(mean_ms[n], 4),
                   "GB/s": round(elems * BYTES_PER_ELEM[n] / (mean_ms[n] / 1e3) / 1e9, 1)}
               for n in names}
    # the floor of one launch moving the dominant kernel's bytes (its input
    # read, its outputs written, nothing computed), timed the same way
    rd_bytes = elems * 4  # the fp32 input, whole (w holds exactly these bytes)
    wr_bytes = int(elems * (BYTES_PER_ELEM[dom] - 4)) // 16 * 16  # codes (+ scales)
    floor_dst = torch.empty(wr_bytes, dtype=torch.uint8, device=dev)
    floor_ms = _time_ms(lambda: stream_probe(w, rd_bytes, floor_dst, wr_bytes), stream, reps=20)
    floor_gbs = (rd_bytes + wr_bytes) / (floor_ms / 1e3) / 1e9
    del floor_dst

    # end-to-end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        pinned = torch.from_numpy(w_host).pin_memory()
        outs_host = [torch.empty((ROWS, COLS), dtype=torch.float32).pin_memory() for _ in range(3)]
        sc_host = torch.empty((ROWS, COLS // 64), dtype=torch.float32).pin_memory()
        wd = torch.empty_like(w)

        # rows in chunks: the host-to-device copies on a stream of their own,
        # each chunk's three quantizations and its device-to-host copies on
        # the main stream once the chunk has landed, so the two PCIe
        # directions overlap (rows are independent; the per-tensor scale is
        # the observer's)
        s_in = torch.cuda.Stream(dev)
        bounds = [int(b) for b in np.linspace(0, ROWS, 9)]

        def e2e_step():
            s_in.wait_stream(stream)  # the previous step is done with wd
            landed = []
            with torch.cuda.stream(s_in):
                for lo, hi in zip(bounds[:-1], bounds[1:]):
                    wd[lo:hi].copy_(pinned[lo:hi], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(s_in)
                    landed.append(ev)
            for (lo, hi), ev in zip(zip(bounds[:-1], bounds[1:]), landed):
                stream.wait_event(ev)
                x = wd[lo:hi]
                s, c = Q.quantize_mx(x, idx_tab, [-1], 64, 1.0, False)
                c1 = Q.quantize(x, sp, qmap=posit)
                c2 = Q.quantize(x, si[lo:hi], qmap=i8)
                sc_host[lo:hi].copy_(s, non_blocking=True)
                outs_host[0][lo:hi].copy_(c, non_blocking=True)
                outs_host[1][lo:hi].copy_(c1, non_blocking=True)
                outs_host[2][lo:hi].copy_(c2, non_blocking=True)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        k = max(2, min(args.steps, 5))
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(k):
            e2e_step()
        a1.record(stream)
        torch.cuda.synchronize()
        e_ms = a0.elapsed_time(a1) / k
        if pg:
            t = torch.tensor([e_ms], device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": round(elems * sum(BYTES_PER_ELEM.values()) * world / (e_ms / 1e3) / 1e9, 3),
               "unit": "GB/s", "ms_per_step": round(e_ms, 3),
               "h2d_bytes_per_step": elems * 4,
               "d2h_bytes_per_step": elems * 4 * 3 + ROWS * (COLS // 64) * 4}

    secondary = {}
    # one weight split by rows over the ranks (strong scaling; the shards
    # need no collective: rows are independent, the per-tensor scale is the
    # observer's)
    shard = run_c2_row_sharded(dev, pg, rank, world, w, si, idx_tab, posit, sp, i8, args)
    if not args.no_secondary and rank == 0:
        secondary = run_secondary(dev, hbm_peak, peaks)
    if rank == 0:
        secondary["c2_row_sharded"] = shard
    if not args.no_secondary and rank == 0:
        secondary["c2_amax_observer"] = run_observer(w, stream, hbm_peak)
    if not args.no_secondary and world > 1:
        tp = run_tp_linear(dev, pg, world)
        if rank == 0:
            secondary["c3_tp_linear"] = tp
        c4s = run_c4_sharded(dev, pg, rank, world)
        if rank == 0:
            secondary["c4_w4a8_n_sharded"] = c4s
    if not args.no_secondary:
        # C5 on all ranks: tensor parallel within NVLink pairs with the
        # sequences split across pairs (the split that keeps each GPU's
        # NVLink traffic below its compute), and, for N > 2, tensor parallel
        # over all N ranks
        bf16 = peaks.get("bf16_tflops", 1590.0)
        variants = [("c5_decoder", 2 if world % 2 == 0 else world)]
        if world > 2:
            variants.append((f"c5_decoder_tp{world}", world))
        for key, tp in variants:
            try:
                c5 = run_c5(dev, pg, world, bf16, tp=tp)
            except Exception as e:  # report, do not hide
                c5 = {"error": repr(e)[:200]}
            if rank == 0:
                secondary[key] = c5

    voyager_b200.check_errors(dev)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline()

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": DATA,
            "config": {"workload": WORKLOAD,
                       "per_gpu_bytes_per_step": int(elems * sum(BYTES_PER_ELEM.values())),
                       "l2": "inputs (180 MB) and outputs larger than the 126 MB L2",
                       "parallelism": f"replicas x{world} (row-sharded weak scaling)"},
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1),
                         "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "peak_source": peak_src,
                         "traffic": NCU_TRAFFIC.get(dom),
                         "stream_floor": round(floor_gbs, 1),
                         "frac_of_floor": round(achieved / floor_gbs, 4),
                         "floor_note": "one launch that only reads and writes the dominant "
                                       "kernel's bytes (vq_stream_probe), timed the same way",
                         "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum per "
                                         "launch from one ncu capture of this kernel; "
                                         "writes still draining from L2 at the kernel's "
                                         "end are not counted"},
            "kernels": kernels,
            "clocks": clk.summary(),
            "gpu_launches": 3 * args.steps,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


def run_c2_row_sharded(dev, pg, rank, world, w, si, idx_tab, posit, sp, i8, args):
    """The C2 step on this rank's rows of the one [11008, 4096] weight
    (rows r * 11008 / N ..): GB/s of the whole tensor over the slowest rank."""
    import torch

    Q = torch.ops.quantized_ops
    lo, hi = rank * ROWS // world, (rank + 1) * ROWS // world
    ws, sis = w[lo:hi], si[lo:hi]
    stream = torch.cuda.current_stream(dev)

    def step():
        Q.quantize_mx(ws, idx_tab, [-1], 64, 1.0, False)
        Q.quantize(ws, sp, qmap=posit)
        Q.quantize(ws, sis, qmap=i8)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    steps = max(args.steps, 10)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(int(3 * steps * 40e-6 * 2e9))
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    if pg:
        t = torch.tensor([ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    total = ROWS * COLS * sum(BYTES_PER_ELEM.values())
    return {"ms_per_step": round(ms, 4), "GBps": round(total / (ms / 1e3) / 1e9, 1),
            "gpus": world, "rows_per_gpu": hi - lo,
            "note": "one C2 weight split by rows over the GPUs (strong scaling), max over ranks"}


def observed_scales(w, hist=None):
    """C2's per-tensor (posit8_1, quant_max 4096) and per-output-channel
    (int8, quant_max 127) scales as the reference's calibration leaves them
    for a constant weight: two steps of the FusedAmaxObsFakeQuantize amax
    observer with a history of one (the first step only fills the history)."""
    import torch

    from voyager_b200.observer import update_amax_scale

    dev = w.device
    hp, sp = torch.zeros(1, device=dev), torch.ones((), device=dev)
    hi, si = torch.zeros(1, w.shape[0], 1, device=dev), torch.ones(w.shape[0], 1, device=dev)
    for _ in range(2):
        update_amax_scale(w, hp, sp, 4096.0, per_channel=False)
        update_amax_scale(w, hi, si, 127.0, per_channel=True, ch_axis=0)
    return sp, si


def run_observer(w, stream, hbm_peak):
    """One amax-observer step on the C2 weight (fp32 [11008, 4096], larger
    than L2), per output channel and per tensor: reads 180 MB each."""
    import torch

    from voyager_b200.observer import update_amax_scale

    dev = w.device
    hi, si = torch.zeros(2, w.shape[0], 1, device=dev), torch.ones(w.shape[0], 1, device=dev)
    hp, sp = torch.zeros(2, device=dev), torch.ones((), device=dev)
    tc = _time_ms(lambda: update_amax_scale(w, hi, si, 127.0, per_channel=True, ch_axis=0,
                                            power_of_two=True), stream, reps=20)
    tt = _time_ms(lambda: update_amax_scale(w, hp, sp, 4096.0, per_channel=False), stream, reps=20)
    nbytes = w.numel() * w.element_size()
    return {"per_channel_ms": round(tc, 4), "per_channel_GBps": round(nbytes / (tc / 1e3) / 1e9, 1),
            "per_tensor_ms": round(tt, 4), "per_tensor_GBps": round(nbytes / (tt / 1e3) / 1e9, 1),
            "frac_hbm_per_channel": round(nbytes / (tc / 1e3) / 1e9 / hbm_peak, 3),
            "note": "FusedAmaxObsFakeQuantize._update_amax_scale on the device: memset, amax "
                    "reduction, history / scale update (3 launches); bytes = the weight read once"}


def stream_probe(src, read_bytes, dst, write_bytes):
    """One launch that only moves these bytes (vq_stream_probe): the least
    time a launch doing the same traffic can take."""
    import torch

    from voyager_b200 import _lib

    dev = (src if src is not None else dst).device
    st = _lib.load().vq_stream_probe(src.data_ptr() if src is not None else None, int(read_bytes),
                                     dst.data_ptr() if dst is not None else None,
                                     int(write_bytes), torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(st, "stream probe")


def _time_ms(fn, stream, reps=10, warm=3):
    import torch

    for _ in range(warm):
        fn()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    torch.cuda._sleep(int(reps * 50e-6 * 2e9))  # the host queues ahead of the device
    a.record(stream)
    for _ in range(reps):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def run_tp_linear(dev, pg, world):
    """C3 MXFP8 linear, tensor parallel over N (weight shard per rank, NCCL
    all-gather of the output columns): strong scaling of one [8192, 11008]
    product.  All ranks take part; max time over ranks."""
    import torch

    from voyager_b200 import parallel, synth
    from voyager_b200.tables import get_quantization_map

    Q = torch.ops.quantized_ops
    a_np, w_np = synth.c3_operands()
    e4m3 = get_quantization_map("fp8_e4m3", dev)
    a = torch.from_numpy(a_np.view(np.int16)).view(torch.bfloat16).to(dev)
    w = torch.from_numpy(w_np.view(np.int16)).view(torch.bfloat16).to(dev)
    sa, ca = Q.quantize_mx(a, e4m3, [-1], 32, 448.0, True)
    sw, cw = Q.quantize_mx(w, e4m3, [-1], 32, 448.0, True)
    lin = parallel.NShardedLinear(cw, sw)
    stream = torch.cuda.current_stream(dev)
    for _ in range(3):
        lin(ca, sa)
    torch.cuda.synchronize()
    pg.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    e0.record(stream)
    for _ in range(reps):
        lin(ca, sa)
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms = float(t.item())
    mode = ("output columns copied into every rank through an NVLS multicast address"
            if lin.multicast else "output all-gathered (NCCL)")
    return {"ms": round(ms, 3), "TFLOPs": round(2 * 8192 * 4096 * 11008 / (ms / 1e3) / 1e12, 1),
            "gpus": world, "note": f"weight N-sharded, {mode}"}


def run_c5(dev, pg, world, bf16_peak, reps=8, warm=2, tp=None):
    """C5: the 4-layer LLaMA-style decoder forward (hidden 4096, 32 heads,
    ffn 11008, B=8, S=2048) through the MXFP8 quantized graph, strong
    scaling of one forward over the ranks: tensor parallel over groups of
    `tp` ranks (default: all of them), the 8 sequences split evenly across
    the world / tp groups.  Random-init weights N(0, 0.02) and N(0, 1)
    hidden states, made on the device from fixed seeds (every rank makes the
    same ones)."""
    import torch
    import torch.distributed as dist

    from voyager_b200.decoder import Decoder, DecoderConfig, init_weights

    cfg, B, S = DecoderConfig(), 8, 2048
    tp = world if tp is None else tp
    if world % tp or B % (world // tp):
        raise ValueError(f"tp {tp} does not split {world} ranks over {B} sequences")
    dp = world // tp
    group = None
    if world > 1:
        rank = dist.get_rank()
        # every rank creates every group, in the same order
        groups = [dist.new_group(list(range(d * tp, (d + 1) * tp))) for d in range(dp)] \
            if dp > 1 else [None]
        group = groups[rank // tp]
        d = rank // tp
    else:
        d = 0
    dec = Decoder(cfg, init_weights(cfg, 0, dev), group=group)
    columns = dec.columns
    torch.cuda.empty_cache()
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn((B * S, cfg.hidden), generator=g, device=dev).bfloat16()
    seqs = B // dp
    xs = dec.shard(x[d * seqs * S:(d + 1) * seqs * S])
    del x
    stream = torch.cuda.current_stream(dev)
    for _ in range(warm):
        dec.forward_shard(xs, seqs)
    torch.cuda.synchronize()
    # the forward captured once as a CUDA graph and replayed: the same
    # kernels, without the host's per-launch cost (about 150 launches per
    # forward and rank at tp2 x dp4, where a rank's share of the work is a
    # few ms); the barriers keep their epoch on the device, so replays stay
    # in step.  Every rank takes the same path (eager if any capture fails).
    graph, graph_note = None, "the NCCL form is not captured"
    if world == 1 or columns:
        try:
            cg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(cg):
                dec.forward_shard(xs, seqs)
            graph, graph_note = cg, None
        except Exception as e:  # report, and time the eager forward
            graph_note = repr(e)[:160]
    ok = torch.tensor([1 if graph is not None else 0], device=dev)
    if pg:
        pg.all_reduce(ok, op=pg.ReduceOp.MIN)
    if int(ok.item()) == 0:
        graph = None
    torch.cuda.synchronize()

    def forward():
        if graph is not None:
            graph.replay()
        else:
            dec.forward_shard(xs, seqs)

    forward()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        forward()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    if pg:
        t = torch.tensor([ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    tf = cfg.flops(B, S) / (ms / 1e3) / 1e12
    peak = 2 * bf16_peak * world  # the whole job's dense FP8 denominator
    dec.check_errors()
    del graph
    del dec, xs
    torch.cuda.empty_cache()
    if world == 1:
        par = "1 GPU"
    else:
        split = ("column-parallel linears, operands all-gathered by NVLS multicast stores"
                 if columns else "Megatron, sequence-parallel norms, NCCL")
        par = f"tp{tp} ({split})" + (f" x dp{dp} (sequences split across the groups)"
                                    if dp > 1 else "")
    return {"ms": round(ms, 2), "TFLOPs": round(tf, 1), "gpus": world,
            "launch": "CUDA graph replay" if int(ok.item()) else f"eager ({graph_note})",
            "frac_fp8_dense": round(tf / peak, 3),
            "fp8_dense_peak_TFLOPs": peak,
            "peak_note": "2 x measured cuBLAS bf16 burst per GPU, times the GPUs",
            "flop_per_forward": cfg.flops(B, S), "parallelism": par}


def _time_cold_ms(fn, stream, dev, reps=20, warm=3):
    """Mean device time of fn with the L2 flushed before each launch (a
    256 MB buffer written between launches, outside the timed events)."""
    import torch

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(warm):
        fn()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(reps)]
    for a, b in ev:
        flush.zero_()
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in ev) / reps
    del flush
    return ms


def _time_graph_cold_ms(fn, dev, reps=20, warm=3):
    """Device time of fn with the L2 cold and no host in the loop: a CUDA
    graph of (256 MB flush, fn) replayed, minus a graph of the flush alone."""
    import torch

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g0):
        flush.zero_()
    with torch.cuda.graph(g1):
        flush.zero_()
        fn()
    st = torch.cuda.current_stream()
    res = []
    for g in (g0, g1):
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        for _ in range(reps):
            g.replay()
        b.record(st)
        torch.cuda.synchronize()
        res.append(a.elapsed_time(b) / reps)
    del g0, g1, flush
    return max(res[1] - res[0], 1e-6)


def _time_graph_ms(fn, stream, reps=20, warm=3):
    """Device time of fn replayed from a CUDA graph (for µs-scale calls whose
    eager time is the host's launch cost, as in a graph-captured decode)."""
    import torch

    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st = torch.cuda.current_stream()
    a.record(st)
    for _ in range(reps):
        g.replay()
    b.record(st)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    del g
    return ms


def _time_rotating_ms(fns, stream, replays=3):
    """Device time per call of `fns` (calls on operands that together exceed
    L2, so that each call reads its own from HBM), captured in one CUDA graph
    and replayed with the host queued ahead of the device."""
    import torch

    for f in fns:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st = torch.cuda.current_stream()
    torch.cuda._sleep(int(replays * 20e-6 * 2e9))
    a.record(st)
    for _ in range(replays):
        g.replay()
    b.record(st)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / (replays * len(fns))
    del g
    return ms


def run_secondary(dev, hbm_peak, peaks):
    import torch

    from voyager_b200 import synth
    from voyager_b200.tables import get_quantization_map

    Q = torch.ops.quantized_ops
    stream = torch.cuda.current_stream(dev)
    out = {}
    # C1 NVFP4 round trip (bf16 [4096,4096], bs 16, e2m1 + e4m3 scale)
    x = torch.from_numpy(synth.c1_input().view(np.int16)).view(torch.bfloat16).to(dev)
    e2m1 = get_quantization_map("fp4_e2m1", dev)
    e4m3 = get_quantization_map("fp8_e4m3", dev)
    s, c = Q.quantize_mx(x, e2m1, [-1], 16, 6.0, False, e4m3)
    # a ~12 us launch: replayed from a CUDA graph, so launch gaps stay out
    tq = _time_graph_ms(lambda: Q.quantize_mx(x, e2m1, [-1], 16, 6.0, False, e4m3), stream,
                        reps=20)
    td = _time_graph_ms(lambda: Q.dequantize(c, s, None, [-1], 16), stream, reps=20)
    n = x.numel()
    out["c1_quantize_mx_GBps"] = round(n * 4.125 / (tq / 1e3) / 1e9, 1)
    out["c1_dequantize_GBps"] = round(n * 4.125 / (td / 1e3) / 1e9, 1)
    out["c1_quantize_mx_frac_hbm"] = round(out["c1_quantize_mx_GBps"] / hbm_peak, 3)
    out["c1_note"] = ("16.8M elems, 69 MB per launch (fits L2: warm-L2 figure, CUDA-graph "
                      "replay of 20 calls)")
    # device time with a cold L2: CUDA-graph replay of (flush, op) minus the
    # flush alone (the eager launch of a ~13 us kernel is host-bound)
    tqc = _time_graph_cold_ms(lambda: Q.quantize_mx(x, e2m1, [-1], 16, 6.0, False, e4m3), dev)
    tdc = _time_graph_cold_ms(lambda: Q.dequantize(c, s, None, [-1], 16), dev)
    tqe = _time_cold_ms(lambda: Q.quantize_mx(x, e2m1, [-1], 16, 6.0, False, e4m3), stream, dev)
    out["c1_cold"] = {"quantize_mx_GBps": round(n * 4.125 / (tqc / 1e3) / 1e9, 1),
                      "dequantize_GBps": round(n * 4.125 / (tdc / 1e3) / 1e9, 1),
                      "quantize_mx_frac_hbm": round(n * 4.125 / (tqc / 1e3) / 1e9 / hbm_peak, 3),
                      "dequantize_frac_hbm": round(n * 4.125 / (tdc / 1e3) / 1e9 / hbm_peak, 3),
                      "quantize_mx_eager_GBps": round(n * 4.125 / (tqe / 1e3) / 1e9, 1),
                      "note": "L2 flushed (256 MB written) before every call; CUDA-graph replay "
                              "of (flush, op) minus the flush alone; eager: one op call per "
                              "launch, host launch gaps included"}
    # the floor: one launch that only reads the input's bytes and writes the
    # outputs' (vq_stream_probe), timed the same way
    floor_out = torch.empty(n * 2 + n // 16 * 2 + 64, dtype=torch.uint8, device=dev)
    tfl = _time_graph_cold_ms(lambda: stream_probe(x, n * 2, floor_out, n * 2 + n // 16 * 2), dev)
    out["c1_cold"]["stream_floor_GBps"] = round(n * 4.125 / (tfl / 1e3) / 1e9, 1)
    out["c1_cold"]["quantize_mx_frac_of_floor"] = round(tfl / tqc, 3)
    out["c1_cold"]["dequantize_frac_of_floor"] = round(tfl / tdc, 3)
    # inputs larger than L2 instead of a flush: five copies of the input
    # (168 MB), one call on each in turn, from one CUDA graph
    xs = [x] + [x.clone() for _ in range(4)]
    cs = [c] + [c.clone() for _ in range(4)]
    tqr = _time_rotating_ms([(lambda xi=xi: Q.quantize_mx(xi, e2m1, [-1], 16, 6.0, False, e4m3))
                             for xi in xs], stream)
    tdr = _time_rotating_ms([(lambda ci=ci: Q.dequantize(ci, s, None, [-1], 16)) for ci in cs],
                            stream)
    tfr = _time_rotating_ms([(lambda xi=xi: stream_probe(xi, n * 2, floor_out, n * 2 + n // 16 * 2))
                             for xi in xs], stream)
    out["c1_rotating"] = {
        "quantize_mx_GBps": round(n * 4.125 / (tqr / 1e3) / 1e9, 1),
        "quantize_mx_frac_hbm": round(n * 4.125 / (tqr / 1e3) / 1e9 / hbm_peak, 3),
        "dequantize_GBps": round(n * 4.125 / (tdr / 1e3) / 1e9, 1),
        "dequantize_frac_hbm": round(n * 4.125 / (tdr / 1e3) / 1e9 / hbm_peak, 3),
        "stream_floor_GBps": round(n * 4.125 / (tfr / 1e3) / 1e9, 1),
        "quantize_mx_frac_of_floor": round(tfr / tqr, 3),
        "note": "five input copies (168 MB, larger than L2) used in turn, no flush; CUDA-graph "
                "replay; the floor moves the same bytes the same way"}
    del xs, cs
    # C3 MXFP8 linear
    try:
        a_np, w_np = synth.c3_operands()
        a = torch.from_numpy(a_np.view(np.int16)).view(torch.bfloat16).to(dev)
        wq = torch.from_numpy(w_np.view(np.int16)).view(torch.bfloat16).to(dev)
        sa, ca = Q.quantize_mx(a, e4m3, [-1], 32, 448.0, True)
        sw, cw = Q.quantize_mx(wq, e4m3, [-1], 32, 448.0, True)
        tl = _time_ms(lambda: Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw,
                                          block_size=32), stream, reps=10)
        fl = 2 * 8192 * 4096 * 11008
        out["c3_linear_mx_TFLOPs"] = round(fl / (tl / 1e3) / 1e12, 1)
        from voyager_b200 import mxgemm

        out["c3_path"] = "tcgen05 mxf8f6f4" if mxgemm.applies(
            ca, cw, sa, sw, 32, None, None, "kc", "linear") else "dequant + torch"
        # the same product with both operands NVFP4 (E2M1, E4M3 scales per 16)
        e2m1 = get_quantization_map("fp4_e2m1", dev)
        sa4, ca4 = Q.quantize_mx(a, e2m1, [-1], 16, 6.0, False, e4m3)
        sw4, cw4 = Q.quantize_mx(wq, e2m1, [-1], 16, 6.0, False, e4m3)
        t4 = _time_ms(lambda: Q.linear_mx(ca4, cw4, None, input_scale=sa4, weight_scale=sw4,
                                          block_size=16), stream, reps=10)
        tf4 = fl / (t4 / 1e3) / 1e12
        bf16 = peaks.get("bf16_tflops", 1590.0)
        out["c3_nvf4_linear_mx"] = {
            "ms": round(t4, 4), "TFLOPs": round(tf4, 1),
            "frac_fp4_dense": round(tf4 / (4 * bf16), 3),
            "path": "tcgen05 mxf4nvf4" if mxgemm.nvf4_applies(
                ca4, cw4, sa4, sw4, 16, None, None, "kc", "linear") else "other",
            "note": "M=8192 K=4096 N=11008, both operands NVFP4; time includes packing the "
                    "activations; denominator 4 x measured cuBLAS bf16 burst"}
    except Exception as e:  # report, do not hide
        out["c3_error"] = repr(e)[:200]
    try:
        out["c2_weight_linear"] = run_dq_linear(dev, peaks)
    except Exception as e:
        out["c2_weight_linear_error"] = repr(e)[:200]
    try:
        out["c4_w4a8_sweep"] = run_c4_sweep(dev, hbm_peak, peaks.get("bf16_tflops", 1590.0))
    except Exception as e:
        out["c4_error"] = repr(e)[:200]
    try:
        out["outlier"] = run_outlier(dev, hbm_peak)
    except Exception as e:
        out["outlier_error"] = repr(e)[:200]
    return out


def dq_weights(dev, w):
    """C2's three weight formats applied to a bf16 weight [N, K], as the
    reference's convert stores them: (name, codes, scale, codebook, block)."""
    import torch

    from voyager_b200.tables import get_quantization_map, index_table

    Q = torch.ops.quantized_ops
    lut = get_quantization_map("lut4")
    levels = torch.unique(lut.float()).bfloat16().to(dev)
    s_nf4, c_nf4 = Q.quantize_mx(w, index_table(lut).to(dev), [-1], 64, 1.0)
    K = w.shape[1]
    s_p8, c_p8 = Q.quantize_mx(w, get_quantization_map("posit8_1", dev), [-1], 32, 4096.0)
    s_i8, c_i8 = Q.quantize_mx(w, get_quantization_map("int8", dev), [-1], K, 127.0)
    return [("nf4_g64", c_nf4, s_nf4, levels, 64), ("posit8_bs32", c_p8, s_p8, None, 32),
            ("int8_per_row", c_i8, s_i8, None, K), ("bf16", w, None, None, None)]


def run_dq_linear(dev, peaks):
    """linear_mx with C2's weight formats (NF4 g64 + codebook, posit8_1 block
    32, int8 per row) and a plain bf16 weight at C3's shape: bf16 activations
    [8192, 4096] x weight [11008, 4096], the weight read back inside the
    tcgen05 bf16 GEMM.  TFLOP/s and the fraction of the measured bf16 peak."""
    import torch

    from voyager_b200 import dqgemm, synth

    Q = torch.ops.quantized_ops
    stream = torch.cuda.current_stream(dev)
    a_np, w_np = synth.c3_operands()
    a = torch.from_numpy(a_np.view(np.int16)).view(torch.bfloat16).to(dev)
    w = torch.from_numpy(w_np.view(np.int16)).view(torch.bfloat16).to(dev)
    peak = peaks.get("bf16_tflops", 1590.0)
    fl = 2.0 * 8192 * 4096 * 11008
    res = {}
    for name, c, sc, cb, bs in dq_weights(dev, w):
        fn = lambda: Q.linear_mx(a, c, None, weight_scale=sc, block_size=bs, weight_code=cb)
        fn()
        pw = dqgemm.packed_weight(c, sc, cb, bs, "kc")
        ms = _time_ms(fn, stream, reps=10)
        tf = fl / (ms / 1e3) / 1e12
        res[name] = {"ms": round(ms, 4), "TFLOPs": round(tf, 1), "frac_bf16": round(tf / peak, 3),
                     "path": dq_path(pw, 8192)}
    res["note"] = ("M=8192 K=4096 N=11008, bf16 activations; denominator: measured cuBLAS bf16 "
                   "burst")
    return res


def dq_path(pw, m):
    """Which kernels a linear_mx with a packed weight and m activation rows runs."""
    from voyager_b200 import dqgemm

    if pw is None:
        return "dequant + torch"
    if pw.mode == dqgemm.MODE_TMA:
        return "tcgen05 bf16 (weight by TMA)"
    bits = "4-bit" if pw.mode == dqgemm.MODE_LUT4 else "8-bit"
    if 0 < dqgemm.DECODE_ONCE_M <= m:
        return f"{bits} palette decoded once per call, tcgen05 bf16 (weight by TMA)"
    return f"tcgen05 bf16, {bits} palette decoded in smem"


def outlier_c3_operands(dev):
    """C3's operands with 1 % of the activations scaled by 50 (the C1
    recipe), quantized with their outliers above 4.0 split into a CSR."""
    import torch

    from voyager_b200 import synth
    from voyager_b200.tables import get_quantization_map

    Q = torch.ops.quantized_ops
    a_np, w_np = synth.c3_operands()
    a = torch.from_numpy(a_np.view(np.int16)).view(torch.bfloat16).to(dev)
    g = torch.Generator(device=dev).manual_seed(1)
    pos = torch.randperm(a.numel(), generator=g, device=dev)[: a.numel() // 100]
    a.view(-1)[pos] = (a.view(-1)[pos].float() * 50).bfloat16()
    wq = torch.from_numpy(w_np.view(np.int16)).view(torch.bfloat16).to(dev)
    e4m3 = get_quantization_map("fp8_e4m3", dev)
    d, i, p, sa, ca = Q.quantize_mx_outlier(a, e4m3, [-1], 32, 448.0, True, None, None, 4.0,
                                            0.02)
    sw, cw = Q.quantize_mx(wq, e4m3, [-1], 32, 448.0, True)
    return a, (d, i, p, sa, ca), (sw, cw)


def run_outlier(dev, hbm_peak):
    """The outlier CSR side-stream: quantize_mx_outlier / filter_outlier on
    C1's input (1 % outliers), and C3's linear_mx with a 1 % activation CSR
    (dense MXFP8 GEMM + spmm_csr in its epilogue)."""
    import torch

    from voyager_b200 import synth
    from voyager_b200.tables import get_quantization_map

    Q = torch.ops.quantized_ops
    stream = torch.cuda.current_stream(dev)
    res = {}
    x = torch.from_numpy(synth.c1_input().view(np.int16)).view(torch.bfloat16).to(dev)
    e2m1 = get_quantization_map("fp4_e2m1", dev)
    e4m3 = get_quantization_map("fp8_e4m3", dev)
    n, R = x.numel(), x.shape[0]
    cap = int(n * 0.02)
    csr_bytes = cap * 6 + (R + 1) * 4
    out = Q.quantize_mx_outlier(x, e2m1, [-1], 16, 6.0, False, e4m3, None, 6.0, 0.02)
    nse = int(out[2][-1])
    # µs-scale launch sequences: graph replay with the L2 flushed (the eager
    # time would include the host's launch gaps)
    tq = _time_graph_cold_ms(lambda: Q.quantize_mx_outlier(x, e2m1, [-1], 16, 6.0, False, e4m3,
                                                           None, 6.0, 0.02), dev)
    tf = _time_graph_cold_ms(lambda: Q.filter_outlier(x, 6.0, 0.02), dev)
    tqm = _time_graph_cold_ms(lambda: Q.quantize_mx(x, e2m1, [-1], 16, 6.0, False, e4m3), dev)
    qb = n * 4.125 + csr_bytes
    fb = n * 4.0 + csr_bytes
    res["c1_quantize_mx_outlier"] = {
        "ms": round(tq, 4), "GBps": round(qb / (tq / 1e3) / 1e9, 1),
        "frac_hbm": round(qb / (tq / 1e3) / 1e9 / hbm_peak, 3), "outliers": nse,
        "capacity": cap, "bytes": int(qb),
        "quantize_mx_alone_ms": round(tqm, 4),
        "note": "NVFP4 bs16 + e4m3 scales of the inliers, CSR of |x| > 6; CUDA-graph "
                "replay, L2 flushed before each call (flush time subtracted)"}
    res["c1_filter_outlier"] = {"ms": round(tf, 4), "GBps": round(fb / (tf / 1e3) / 1e9, 1),
                                "frac_hbm": round(fb / (tf / 1e3) / 1e9 / hbm_peak, 3)}
    del x, out
    a, (d, i, p, sa, ca), (sw, cw) = outlier_c3_operands(dev)
    nnz = int(p[-1])
    lin = lambda: Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32,
                              A_data=d, A_indices=i, A_indptr=p)
    dense = lambda: Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32)
    spmm = lambda: Q.spmm_csr(d, i, p, cw, sw, None, 32, "kc")
    tl = _time_ms(lin, stream, reps=10)
    td = _time_ms(dense, stream, reps=10)
    ts = _time_ms(spmm, stream, reps=10)
    M, K, N = 8192, 4096, 11008
    fl = 2.0 * M * N * K + 2.0 * nnz * N
    gather = nnz * N * 2  # B rows read (bf16), mostly from L2
    res["c3_linear_mx_outliers"] = {
        "ms": round(tl, 4), "dense_ms": round(td, 4), "spmm_ms": round(ts, 4),
        "TFLOPs": round(fl / (tl / 1e3) / 1e12, 1), "outliers": nnz,
        "spmm_gather_GBps": round(gather / (ts / 1e3) / 1e9, 1),
        "spmm_out_GBps": round((M * N * 2 + K * N * 2) / (ts / 1e3) / 1e9, 1),
        "note": "M=8192 K=4096 N=11008, 1% of activations x50, CSR of |x| > 4; spmm "
                "output added in the GEMM epilogue"}
    return res


def c4_operands(dev, m, k, n, seed, keep_input=False):
    """C4 inputs on the device: A ~ N(0,1) [M,K] MXFP8, W ~ N(0,0.02) [N,K] NVFP4
    (and the bf16 activations themselves with keep_input)."""
    import torch

    from voyager_b200.tables import get_quantization_map

    Q = torch.ops.quantized_ops
    g = torch.Generator(device=dev).manual_seed(seed)
    a = torch.randn((m, k), generator=g, device=dev, dtype=torch.float32).bfloat16()
    w = (torch.randn((n, k), generator=g, device=dev, dtype=torch.float32) * 0.02).bfloat16()
    e4m3 = get_quantization_map("fp8_e4m3", dev)
    sa, ca = Q.quantize_mx(a, e4m3, [-1], 32, 448.0, True)
    sw, cw = Q.quantize_mx(w, get_quantization_map("fp4_e2m1", dev), [-1], 16, 6.0, False, e4m3)
    del w
    if keep_input:
        return ca, sa, cw, sw, a
    return ca, sa, cw, sw


def run_c4_sharded(dev, pg, rank, world):
    """C4 N-sharded over the ranks: rank r multiplies the tokens by rows
    [r N/g, (r+1) N/g) of the NVFP4 weight (every rank makes the same weight
    from the same seed) and keeps its output columns (a column-parallel
    linear: no gather).  Whole-job TFLOP/s from the slowest rank's time per
    point.  Every rank runs the same points in the same order."""
    import torch

    from voyager_b200.tables import get_quantization_map
    from voyager_b200 import w4a8

    stream = torch.cuda.current_stream(dev)
    res = []
    for (k, n) in [(4096, 4096), (4096, 14336), (14336, 4096)]:
        ns = n // world
        lo = rank * ns
        ca0, sa0, cw, sw, a0 = c4_operands(dev, 16384, k, n, seed=k + n, keep_input=True)
        cw, sw = cw[lo:lo + ns].contiguous(), sw[lo:lo + ns].contiguous()
        e4m3 = get_quantization_map("fp8_e4m3", dev)
        wbytes = ns * k * (0.5 + 1 / 16)
        copies = [cw] + [cw.clone() for _ in range(int(np.ceil(2.5 * L2_BYTES / wbytes)) - 1)]
        for m in (1, 16, 128, 1024, 16384):
            sa, ca = torch.ops.quantized_ops.quantize_mx(a0[:m].contiguous(), e4m3, [-1], 32,
                                                         448.0, True)
            if m == 16384:
                ca, sa = ca0, sa0
            if m <= 16:
                ms = _time_rotating_ms([(lambda c=c: w4a8.linear(ca, sa, c, sw)) for c in copies],
                                       stream)
            else:
                ms = _time_graph_ms(lambda: w4a8.linear(ca, sa, cw, sw), stream,
                                    reps=20 if m <= 1024 else 5)
            t = torch.tensor([ms], device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms = float(t.item())
            res.append({"M": m, "K": k, "N": n, "ms": round(ms, 4),
                        "TFLOPs": round(2.0 * m * n * k / (ms / 1e3) / 1e12, 2)})
        del ca0, sa0, cw, sw, a0, copies
        torch.cuda.empty_cache()
    return {"gpus": world, "points": res,
            "note": "weight rows (N) split over the ranks, output columns kept sharded "
                    "(column-parallel, no gather); max over ranks"}


def run_c4_sweep(dev, hbm_peak, bf16_peak):
    """C4: W4A8 linear over M x (K, N); TFLOP/s per point, and packed-byte
    GB/s (fraction of HBM) for the weight-streaming points M <= 16."""
    import torch

    from voyager_b200 import dqgemm, w4a8
    from voyager_b200.tables import get_quantization_map

    stream = torch.cuda.current_stream(dev)
    res = []
    for (k, n) in [(4096, 4096), (4096, 14336), (14336, 4096)]:
        ca0, sa0, cw, sw, a0 = c4_operands(dev, 16384, k, n, seed=k + n, keep_input=True)
        e4m3 = get_quantization_map("fp8_e4m3", dev)
        wbytes = n * k * (0.5 + 1 / 16)
        copies = [cw] + [cw.clone() for _ in range(int(np.ceil(2.5 * L2_BYTES / wbytes)) - 1)]
        for m in (1, 16, 128, 1024, 16384):
            # the first m tokens quantized as a batch of m (the same codes as
            # the rows of the full batch: blocks run along K)
            sa, ca = torch.ops.quantized_ops.quantize_mx(a0[:m].contiguous(), e4m3, [-1], 32,
                                                         448.0, True)
            if m == 16384:
                ca, sa = ca0, sa0
            if m <= 16:
                # microsecond calls that stream the weights: one graph over
                # copies of the weights larger than L2 together, so that
                # every call reads its copy from HBM
                ms = _time_rotating_ms([(lambda c=c: w4a8.linear(ca, sa, c, sw))
                                        for c in copies], stream)
            else:
                ms = _time_graph_ms(lambda: w4a8.linear(ca, sa, cw, sw), stream,
                                    reps=20 if m <= 1024 else 5)
            fl = 2.0 * m * n * k
            pt = {"M": m, "K": k, "N": n, "ms": round(ms, 4),
                  "TFLOPs": round(fl / (ms / 1e3) / 1e12, 2),
                  "path": "packed-weight mma" if w4a8.applies_small(ca, cw)
                  else dq_path(dqgemm.packed_weight(cw, sw, None, 16, "kc"), m)}
            if m <= 16:
                byts = n * k * (0.5 + 1 / 16) + m * k * (1 + 1 / 32) + 2 * m * n
                pt["GBps"] = round(byts / (ms / 1e3) / 1e9, 1)
                pt["frac_hbm"] = round(pt["GBps"] / hbm_peak, 3)
                if m == 1:
                    # the floor of one launch reading the packed weight's bytes
                    wb = int(n * k * (0.5 + 1 / 16)) // 16 * 16
                    floor_ms = _time_rotating_ms([(lambda c=c: stream_probe(c, wb, None, 0))
                                                  for c in copies], stream)
                pt["stream_floor_ms"] = round(floor_ms, 4)
                pt["frac_of_floor"] = round(floor_ms / ms, 3)
            else:
                pt["frac_bf16"] = round(pt["TFLOPs"] / bf16_peak, 3)
            res.append(pt)
        del ca0, sa0, cw, sw, a0, copies
        torch.cuda.empty_cache()
    return res


def run_only(args):
    """Run one workload's kernels (for ncu captures of committed code)."""
    import torch

    import voyager_b200  # noqa: F401
    from voyager_b200 import synth
    from voyager_b200.tables import get_quantization_map, index_table

    Q = torch.ops.quantized_ops
    dev = torch.device("cuda", 0)
    if args.only == "c1":
        x = torch.from_numpy(synth.c1_input().view(np.int16)).view(torch.bfloat16).to(dev)
        e2m1, e4m3 = get_quantization_map("fp4_e2m1", dev), get_quantization_map("fp8_e4m3", dev)
        for _ in range(args.warmup + args.steps):
            s, c = Q.quantize_mx(x, e2m1, [-1], 16, 6.0, False, e4m3)
            Q.dequantize(c, s, None, [-1], 16)
    elif args.only == "c2":
        w_host = synth.c2_weight()
        w = torch.from_numpy(w_host).to(dev)
        idx_tab = index_table(get_quantization_map("lut4")).to(dev)
        posit, i8 = get_quantization_map("posit8_1", dev), get_quantization_map("int8", dev)
        sp, si = observed_scales(w)
        for _ in range(args.warmup + args.steps):
            Q.quantize_mx(w, idx_tab, [-1], 64, 1.0, False)
            Q.quantize(w, sp, qmap=posit)
            Q.quantize(w, si, qmap=i8)
    elif args.only == "c5":
        from voyager_b200.decoder import Decoder, DecoderConfig, init_weights

        cfg = DecoderConfig()
        dec = Decoder(cfg, init_weights(cfg, 0, dev))
        x = torch.randn((8 * 2048, cfg.hidden), device=dev).bfloat16()
        for _ in range(args.warmup + args.steps):
            dec.forward_shard(x, 8)
    elif args.only == "attn":
        # the C5 attention at batch 2: causal sdpa_mx, 32 heads, S 2048
        B, H, S = 2, 32, 2048
        e4m3 = get_quantization_map("fp8_e4m3", dev)
        q, k, v = (torch.randn((B, H, S, 128), device=dev).bfloat16() for _ in range(3))
        sq, cq = Q.quantize_mx(q, e4m3, [-1], 32, 448.0, True)
        sk, ck = Q.quantize_mx(k, e4m3, [-1], 32, 448.0, True)
        sv, cv = Q.quantize_mx(v.transpose(-1, -2).contiguous(), e4m3, [-1], 32, 448.0, True)
        for _ in range(args.warmup + args.steps):
            Q.sdpa_mx(cq, ck, cv.transpose(-1, -2), is_causal=True, query_scale=sq, key_scale=sk,
                      value_scale=sv.transpose(-1, -2), block_size=32, probs_qmap=e4m3,
                      probs_quant_max=448.0, force_scale_power_of_two=True)
    elif args.only == "outlier":
        x = torch.from_numpy(synth.c1_input().view(np.int16)).view(torch.bfloat16).to(dev)
        e2m1, e4m3 = get_quantization_map("fp4_e2m1", dev), get_quantization_map("fp8_e4m3", dev)
        a, (d, i, p, sa, ca), (sw, cw) = outlier_c3_operands(dev)
        for _ in range(args.warmup + args.steps):
            Q.quantize_mx_outlier(x, e2m1, [-1], 16, 6.0, False, e4m3, None, 6.0, 0.02)
            Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32, A_data=d,
                        A_indices=i, A_indptr=p)
    elif args.only == "spmm":
        # spmm_csr of the first 2048 rows of C3's outlier CSR (small enough
        # for a full counter capture of one launch)
        a, (d, i, p, sa, ca), (sw, cw) = outlier_c3_operands(dev)
        rows = 2048
        n = int(p[rows])
        d2, i2, p2 = d[:n].contiguous(), i[:n].contiguous(), p[:rows + 1].contiguous()
        for _ in range(args.warmup + args.steps):
            Q.spmm_csr(d2, i2, p2, cw, sw, None, 32, "kc")
    elif args.only == "dq":
        from voyager_b200 import synth as sy

        a_np, w_np = sy.c3_operands()
        a = torch.from_numpy(a_np.view(np.int16)).view(torch.bfloat16).to(dev)
        w = torch.from_numpy(w_np.view(np.int16)).view(torch.bfloat16).to(dev)
        fmts = dq_weights(dev, w)
        for _ in range(args.warmup + args.steps):
            for name, c, sc, cb, bs in fmts:
                Q.linear_mx(a, c, None, weight_scale=sc, block_size=bs, weight_code=cb)
    elif args.only == "nvf4":
        # C3's shape with both operands NVFP4
        a_np, w_np = synth.c3_operands()
        e2m1, e4m3 = get_quantization_map("fp4_e2m1", dev), get_quantization_map("fp8_e4m3", dev)
        a = torch.from_numpy(a_np.view(np.int16)).view(torch.bfloat16).to(dev)
        wq = torch.from_numpy(w_np.view(np.int16)).view(torch.bfloat16).to(dev)
        sa, ca = Q.quantize_mx(a, e2m1, [-1], 16, 6.0, False, e4m3)
        sw, cw = Q.quantize_mx(wq, e2m1, [-1], 16, 6.0, False, e4m3)
        for _ in range(args.warmup + args.steps):
            Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=16)
    elif args.only == "c4":
        from voyager_b200 import w4a8

        ca, sa, cw, sw = c4_operands(dev, 16, 4096, 14336, seed=1)
        for _ in range(args.warmup + args.steps):
            w4a8.linear(ca, sa, cw, sw)
    elif args.only in ("c4m128", "c4m1024"):
        # C4 at M = 128, K = 14336, N = 4096 (the split-K dequant GEMM) or at
        # M = 1024, K = N = 4096 (one wave of output tiles)
        from voyager_b200 import w4a8

        m, k, n = (128, 14336, 4096) if args.only == "c4m128" else (1024, 4096, 4096)
        ca, sa, cw, sw = c4_operands(dev, m, k, n, seed=1)
        for _ in range(args.warmup + args.steps):
            w4a8.linear(ca, sa, cw, sw)
    elif args.only == "observer":
        w = torch.from_numpy(synth.c2_weight()).to(dev)
        for _ in range(args.warmup + args.steps):
            observed_scales(w)
    else:
        a_np, w_np = synth.c3_operands()
        e4m3 = get_quantization_map("fp8_e4m3", dev)
        a = torch.from_numpy(a_np.view(np.int16)).view(torch.bfloat16).to(dev)
        wq = torch.from_numpy(w_np.view(np.int16)).view(torch.bfloat16).to(dev)
        sa, ca = Q.quantize_mx(a, e4m3, [-1], 32, 448.0, True)
        sw, cw = Q.quantize_mx(wq, e4m3, [-1], 32, 448.0, True)
        for _ in range(args.warmup + args.steps):
            Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32)
    torch.cuda.synchronize()


def main():
    args = parse()
    if args.only:
        run_only(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
