#!/usr/bin/env python3
"""Benchmark of the Veltrix B200 speculative-decoding hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload q4matvec]

Prints ONE JSON line on rank 0.  For N > 1 launch it with
torch.distributed.run (one rank per GPU, NCCL); ranks run independent
replicas and rank 0 reports the max-over-ranks time.

Workload `q4matvec`: Q4_0 verify matmuls 4096x4096 and
11008x4096 at M = 1, 2, 5, 8 activation rows, fp32 activations and
accumulation.  One step = one GEMV over every rotated weight copy for each of
the 8 (shape, M) cases; the copies of each shape exceed 2x the 126 MB L2, so
every step streams its weights from HBM.

--impl reference times the reference's own CPU kernel (oracle/_ref, compiled
from the reference sources with its shipped flags) on this host's cores.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "veltrix-engine_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

L2_BYTES = 126 * 1024 * 1024
SHAPES = [(4096, 4096), (11008, 4096)]
MS = [1, 2, 5, 8]


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# q4matvec
# ---------------------------------------------------------------------------
def q4_bytes(rows, cols, M):
    """Algorithmic bytes of one GEMV: Q4_0 weights + fp32 activations in + fp32 out."""
    return rows * (cols // 32) * 18 + M * cols * 4 + M * rows * 4


def run_q4matvec_gpu(args, ws, rank, local):
    import torch
    import vxb200
    from qgen import q4_0_blocks
    torch.cuda.set_device(local)
    vxb200.check(vxb200.lib().vxc_device_init(local), "vxc_device_init")
    dist = None
    if ws > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rng = np.random.default_rng(1234)
    mats = {}
    for (R, K) in SHAPES:
        blk = q4_0_blocks(R, K, rng)
        wbytes = R * (K // 32) * 18
        ncopy = max(2, (2 * L2_BYTES + wbytes - 1) // wbytes)
        mats[(R, K)] = [vxb200.QMat(2, blk, R, K) for _ in range(ncopy)]
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    xs = {M: torch.randn(M, 4096, device="cuda") for M in MS}
    ys = {(R, M): torch.empty(M, R, device="cuda") for (R, K) in SHAPES for M in MS}
    wsb = max(mats[s][0].workspace_bytes(M) for s in SHAPES for M in MS)
    wsp = torch.empty(max(wsb, 4) // 4 + 1, device="cuda")
    launches_per_call = {(s, M): (2 if mats[s][0].workspace_bytes(M) > 0 else 1) for s in SHAPES for M in MS}
    cases = [(s, M) for s in SHAPES for M in MS]

    def step(ev=None):
        for (s, M) in cases:
            for i, W in enumerate(mats[s]):
                if ev is not None:
                    ev[(s, M)][i][0].record(stream)
                W.gemv(xs[M].data_ptr(), M, ys[(s[0], M)].data_ptr(), wsp.data_ptr(), wsb, sp)
                if ev is not None:
                    ev[(s, M)][i][1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    # per-call events (one pair per GEMV) for the roofline of the kernel
    evs = [{c: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in mats[c[0]]] for c in cases} for _ in range(args.steps)]
    clk = ClockSampler(local)
    clk.start()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for k in range(args.steps):
        step(evs[k])
    t1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = clk.stop()
    ms_total = t0.elapsed_time(t1)
    per_case = {}
    kern_ms, kern_bytes = 0.0, 0
    for c in cases:
        (R, K), M = c
        tms = [evs[k][c][i][0].elapsed_time(evs[k][c][i][1]) for k in range(args.steps) for i in range(len(mats[c[0]]))]
        avg = sum(tms) / len(tms)
        b = q4_bytes(R, K, M)
        per_case[f"{R}x{K}_M{M}"] = round(b / (avg * 1e-3) / 1e9, 1)
        kern_ms += sum(tms)
        kern_bytes += b * len(tms)
    step_bytes = sum(q4_bytes(s[0], s[1], M) * len(mats[s]) for (s, M) in cases)
    # e2e through the C-ABI with host buffers: pinned x in, y out, each call
    hx = {M: torch.randn(M, 4096).pin_memory() for M in MS}
    hy = {(R, M): torch.empty(M, R).pin_memory() for (R, K) in SHAPES for M in MS}
    h2d = sum(hx[M].numel() * 4 * len(mats[s]) for (s, M) in cases)
    d2h = sum(hy[(s[0], M)].numel() * 4 * len(mats[s]) for (s, M) in cases)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(args.steps):
        for (s, M) in cases:
            for W in mats[s]:
                xs[M].copy_(hx[M], non_blocking=True)
                W.gemv(xs[M].data_ptr(), M, ys[(s[0], M)].data_ptr(), wsp.data_ptr(), wsb, sp)
                hy[(s[0], M)].copy_(ys[(s[0], M)], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    code = ctypes.c_uint(0)
    vxb200.check(vxb200.lib().vxc_check_device_error(ctypes.byref(code)), "device error check")
    t = torch.tensor([ms_total, e2e_ms, kern_ms], device="cuda", dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, e2e_ms, kern_ms_max = t.tolist()
    n_launch = args.steps * sum(launches_per_call[c] * len(mats[c[0]]) for c in cases)
    res = dict(step_bytes=step_bytes, ms_total=ms_total, e2e_ms=e2e_ms, per_case=per_case,
               kern_ms=kern_ms, kern_bytes=kern_bytes, clocks=clocks, launches=n_launch,
               h2d=h2d // args.steps, d2h=d2h // args.steps)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    for lst in mats.values():
        for W in lst:
            W.close()
    return res


def cpu_q4matvec(budget_s, threads, ship=True):
    """Reference CPU kernel on this host: the shipped AVX2 Q4_0 GEMV
    (src/simd/avx2.c:311-370) when oracle/_ref holds the reference build, else
    the oracle's scalar restatement.  M rows = M sequential calls (the
    reference has no batched GEMV).  Returns (GB/s, kind, sample text)."""
    from qgen import q4_0_blocks
    kind = "reference"
    try:
        from _paths import ref
        R_ = ref(ship=True)
        R_.vx_set_n_threads(threads)
        fn = lambda blk, x, y, r, c: R_.vx_gemv_q4_0_avx2(blk.ctypes.data, x.ctypes.data, y.ctypes.data, r, c)
    except Exception:
        from _paths import oracle
        O = oracle()
        kind = "port"
        fn = lambda blk, x, y, r, c: O.vxo_qgemv(2, blk.ctypes.data, x.ctypes.data, y.ctypes.data, 1, r, c)
    rng = np.random.default_rng(7)
    tot_b, tot_t = 0, 0.0
    per = budget_s / (len(SHAPES) * len(MS))
    for (R, K) in SHAPES:
        blks = [q4_0_blocks(R, K, rng) for _ in range(4)]   # 4 copies > LLC-resident reuse
        x = rng.standard_normal(K).astype(np.float32)
        y = np.zeros(R, np.float32)
        for M in MS:
            n = 0
            t0 = time.perf_counter()
            while time.perf_counter() - t0 < per or n == 0:
                for _ in range(M):
                    fn(blks[n % 4], x, y, R, K)
                n += 1
            dt = time.perf_counter() - t0
            tot_b += q4_bytes(R, K, M) * n
            tot_t += dt
    return tot_b / tot_t / 1e9, kind, f"8 (shape, M) cases x ~{per:.1f}s each, 4 weight copies per shape"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="q4matvec", choices=["q4matvec"])
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    args = ap.parse_args()
    ws, rank, local = dist_setup(args)
    metric = "Q4 matvec HBM GB/s (verify-matmul microbench)"
    config = {"workload": "q4matvec: Q4_0 4096x4096 + 11008x4096, M=1,2,5,8 fp32 rows",
              "l2": "weights rotated over copies > 2x L2 per shape (no flush needed)",
              "parallelism": f"replicas x{ws}"}
    threads = host_threads()

    if args.impl == "reference":
        if rank != 0:
            return
        gbs, kind, sample = cpu_q4matvec(max(args.steps, 1) * args.cpu_budget / 5, threads)
        print(json.dumps({"impl": "reference", "metric": metric, "value": round(gbs, 3), "unit": "GB/s",
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "higher_is_better": True, "dtype": "f32", "data": "synthetic", "config": config,
                          "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                                           "kind": kind, "sample": sample},
                          "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return

    r = run_q4matvec_gpu(args, ws, rank, local)
    if rank != 0:
        return
    value = ws * r["step_bytes"] * args.steps / (r["ms_total"] * 1e-3) / 1e9
    e2e = ws * r["step_bytes"] * args.steps / (r["e2e_ms"] * 1e-3) / 1e9
    peak, peak_kind = peaks()
    achieved = r["kern_bytes"] / (r["kern_ms"] * 1e-3) / 1e9
    cpu = None
    if ws == 1:
        gbs, kind, sample = cpu_q4matvec(args.cpu_budget, threads)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample}
    out = {"metric": metric, "value": round(value, 1), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(r["ms_total"] / args.steps, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic", "config": config,
           "per_case_gbs": r["per_case"],
           "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(achieved / peak, 4), "traffic": None,
                        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                        "kernel": "vxc_qgemv (k_qgemv_tc + split-K reduce), per-call CUDA events"},
           "cpu_baseline": cpu,
           "e2e": {"value": round(e2e, 1), "unit": "GB/s", "h2d_bytes_per_step": r["h2d"],
                   "d2h_bytes_per_step": r["d2h"]},
           "gpu_launches": r["launches"], "clocks": r["clocks"]}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
