"""Benchmark of the B200 decode backend (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gemv_fp8]

Workload `gemv_fp8`: y = W x with W 4096x7168 e4m3 in
128x128 E8M0 blocks, x f32, batch 1. One step is one GEMV over a different
resident weight copy (8 copies, 235 MB, rotate so no step finds its weights in
the 126 MB L2). `value` is algorithmic HBM GB/s with inputs resident, timed
with CUDA events on the launching stream; `e2e` is the same metric through the
reference-facing C ABI (dsv4_cuda_mmq: host x in, host y out, copies inside
the timed region). Under torchrun every rank runs its own replica (the GEMV
does not shard at batch 1 without an exchange; weak scaling) and the slowest
rank's time is reported.

--impl reference times the reference's own CPU kernel (dsv4_matmul_fp8 from
oracle/_ref, or the oracle restatement where that was not built) on the host
cores, on the same config.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "deepseek-v4-in-c_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))

C1_ROWS, C1_COLS = 4096, 7168
# algorithmic bytes of one config-1 GEMV: W + S + x + y
C1_BYTES = C1_ROWS * C1_COLS + 32 * 56 + C1_COLS * 4 + C1_ROWS * 4
NCOPY = 8


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampled every 200 ms while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev):
        self.dev, self.rows, self.p = dev, [], None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), "--query-gpu=" + self.Q,
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.p = None
        return self

    def _read(self):
        for line in self.p.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            self.p.wait()
            self.t.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 4 + i and r[4 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


def dist_setup(n):
    if n <= 1 or "RANK" not in os.environ:
        return 0, 1, None
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    os.environ["DSV4_DEVICE"] = str(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    return rank, world, dist


def cpu_reference_gemv(seconds, threads=None):
    """The reference's CPU dsv4_matmul_fp8 on config 1, cycling weight copies
    larger than the LLC (reference bench/gemm_bw.c:11-26), best of the runs
    (bench/matmul_bw.c:96-99) over a bounded time budget."""
    import oracle as O
    import dsv4_quant as Q
    kind = "reference" if os.path.exists(O.REF_SO) else "port"
    chk = O.Checker(kind)
    W, S, x = Q.c1_gemv(seed=0)
    copies = [W] + [np.roll(W, i + 1, axis=0) for i in range(3)]   # 117 MB > LLC
    best, n, t_end = 1e9, 0, time.perf_counter() + seconds
    while time.perf_counter() < t_end or n < 3:
        t0 = time.perf_counter()
        chk.gemv_fp8(x, copies[n % len(copies)], S, C1_ROWS, C1_COLS)
        best = min(best, time.perf_counter() - t0)
        n += 1
    cores = threads or os.cpu_count()
    return {"value": C1_BYTES / best / 1e9, "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": "%d config-1 GEMVs over %d rotating weight copies (117 MB), best of runs, "
                      "OMP_NUM_THREADS=%s" % (n, len(copies), os.environ.get("OMP_NUM_THREADS", cores))}


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    secs = max(2.0, 20.0 / max(a.steps, 1))
    vals = []
    for _ in range(a.warmup):
        cpu_reference_gemv(0.5)
    base = None
    for _ in range(a.steps):
        base = cpu_reference_gemv(secs)
        vals.append(base["value"])
    v = float(np.median(vals))
    base["value"] = v
    print(json.dumps({
        "metric": "FP8 block-scaled GEMV HBM GB/s (config 1, 4096x7168 e4m3, batch 1)",
        "value": v, "unit": "GB/s", "impl": "reference", "n_gpus": a.gpus, "steps": a.steps,
        "warmup": a.warmup, "higher_is_better": True, "dtype": "e4m3 weights, f32 x, f64 accumulation",
        "data": "synthetic", "config": {"workload": "gemv_fp8 config 1", "rows": C1_ROWS, "cols": C1_COLS},
        "cpu_baseline": base,
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def run_ours(a):
    import torch
    import dsv4_b200 as B
    import dsv4_quant as Q
    rank, world, dist = dist_setup(a.gpus)
    L = B.init()
    W, S, x = Q.c1_gemv(seed=0)
    mats = []
    for i in range(NCOPY):                       # distinct bytes per copy
        Wi = W if i == 0 else np.roll(W, i, axis=1)
        m = B.Matrix(B.WFP8, Wi, S)
        B.check(m.upload(), "upload")
        mats.append(m)
    dev = torch.cuda.current_device()
    stream = torch.cuda.Stream()
    tx = torch.from_numpy(x).cuda()
    ty = torch.empty(C1_ROWS, dtype=torch.float32, device="cuda")
    ptrs = [m.device_ptrs() for m in mats]

    def step(i):
        dw, ds = ptrs[i % NCOPY]
        B.gemv(B.WFP8, ty, tx, dw, ds, C1_ROWS, C1_COLS, 128, 128, 1, stream)

    # Launch cost is not the kernel's: the K timed steps replay CUDA graphs of
    # up to 1000 captured GEMVs each (weights rotating over the 8 copies).
    with torch.cuda.stream(stream):
        for i in range(max(a.warmup, 3)):
            step(i)
    torch.cuda.synchronize()
    chunk = min(a.steps, 1000)
    plan = [(chunk, a.steps // chunk)] + ([(a.steps % chunk, 1)] if a.steps % chunk else [])
    graphs = []
    for n, reps in plan:
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for i in range(n):
                step(i)
        graphs.append((gr, reps))
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev) as clk:
        t_end = time.perf_counter() + 0.5          # load the GPU while sampling starts
        while time.perf_counter() < t_end:
            with torch.cuda.stream(stream):
                graphs[0][0].replay()
            torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            for gr, reps in graphs:
                for _ in range(reps):
                    gr.replay()
            e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / a.steps
    value = world * C1_BYTES / (ms_step * 1e-3) / 1e9

    # e2e: the reference-facing call, host buffers, copies inside the region
    for i in range(3):
        mats[i % NCOPY].mmq(x)
    ke = max(50, a.steps // 4)
    t0 = time.perf_counter()
    for i in range(ke):
        y = mats[i % NCOPY].mmq(x)
    e2e_s = (time.perf_counter() - t0) / ke
    e2e = {"value": C1_BYTES / e2e_s / 1e9, "unit": "GB/s", "ms_per_step": e2e_s * 1e3,
           "h2d_bytes_per_step": C1_COLS * 4, "d2h_bytes_per_step": C1_ROWS * 4,
           "api": "dsv4_cuda_mmq (host x -> host y), wall clock"}
    del y

    peak, src = peaks()
    ach = C1_BYTES / (ms_step * 1e-3) / 1e9
    out = {
        "metric": "FP8 block-scaled GEMV HBM GB/s (config 1, 4096x7168 e4m3, batch 1)",
        "value": value, "unit": "GB/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3 weights, f32 x, f64 accumulation", "data": "synthetic",
        "config": {"workload": "gemv_fp8 config 1", "rows": C1_ROWS, "cols": C1_COLS, "batch": 1,
                   "l2": "8 rotating resident weight copies (235 MB > 126 MB L2)",
                   "parallelism": "replica per GPU" if world > 1 else "single GPU"},
        "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                     "frac": ach / peak, "peak_source": src + " burst hbm_gbs",
                     "traffic": TRAFFIC_C1},
        "gpu_launches": a.steps,
        "clocks": clk.summary(),
        "e2e": e2e,
    }
    if rank == 0 and world == 1 and not a.no_cpu:
        out["cpu_baseline"] = cpu_reference_gemv(10.0)
    if rank == 0:
        print(json.dumps(out))
    L.dsv4_cuda_shutdown()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# dram bytes (read + write) of one k_gemv launch at config 1 from ncu, or None
# while no capture has been summarised (profiles/gemv_fp8_c1.md).
TRAFFIC_C1 = None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="gemv_fp8", choices=["gemv_fp8"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    a = ap.parse_args()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
