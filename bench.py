#!/usr/bin/env python3
"""Benchmark of the Veltrix B200 speculative-decoding hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload spec7b|spec2l|spec70b|spec_tiny|q4matvec|accept]

Prints ONE JSON line on rank 0.  For N > 1 launch it with
torch.distributed.run (one rank per GPU, NCCL for the barrier and the
max-over-ranks timing only).

Workload `spec7b` (default; benchmark configuration 4, the headline metric
"accepted tok/s"): a Llama-2-7B-shaped Q4_0 target and a 1.1B-shaped Q8_0
draft (random N(0,0.02) weights written by the library's own GGUF writer),
8 independent sequences per GPU with 512-id uniform random prompts, k = 4,
greedy, 256 new tokens each.  Sequences are sharded across GPUs with no
communication (weak scaling: 8 per GPU).  One step = one
vx_speculative_generate_batch call (prompt pass + round loop) through the
reference's C API with host buffers.  `value` = emitted tokens of all ranks /
max-over-ranks device time of the round loops (prompt pass excluded, as the
metric defines); `e2e` = the same tokens / wall time of the whole API calls
(prompt pass, H2D and D2H included).  The KV cache of every step is far
larger than L2 (>= 4 GB per verify), so no flush is needed.

Workload `spec70b` (benchmark configuration 5): a Llama-3-70B-shaped Q4_0 target
(80 layers, 64/8 heads of 128, FFN 28672, vocabulary 128256, RoPE theta 5e5)
split over the N GPUs by tensor parallelism (NCCL all-reduce after the
output and down projections, all-gather of the vocabulary-split logits) and
a 1B-shaped Q8_0 draft on every GPU; 32 sequences of 4096-id prompts, k = 6,
T = 0.8 with seeded Philox sampling, 128 new tokens.  Every GPU runs every
sequence on its shard (strong scaling); tokens are counted once.

Workload `q4matvec` (benchmark configuration 2): Q4_0 verify matmuls 4096x4096 and
11008x4096 at M = 1, 2, 5, 8 activation rows, fp32 activations and
accumulation.  One step = one GEMV over every rotated weight copy for each of
the 8 (shape, M) cases; the copies of each shape exceed 2x the 126 MB L2, so
every step streams its weights from HBM.  The device-side numbers replay a
CUDA graph of the public vxc_qgemv calls (the host's per-call launch cost is
not GPU time); `e2e` calls vxc_qgemv one by one with host buffers.

Workload `spec_tiny` (benchmark configuration 1): the tiny Q8_0 target and
draft of the parity tests, batch 1, k = 4, greedy, 32-id prompt, 128 new
tokens (launch-bound: reported, not judged).  Its CPU baseline is the
oracle's corrected speculative loop over the whole workload.

Workload `accept` (benchmark configuration 3): the fused acceptance kernel
for 64 sequences, k = 5, V = 32000, T = 0.8 (target logits N(0, 2^2), draft
logits = target + N(0, 0.5^2)); 90.1 MB of logits per launch, rotated over
copies larger than 2x L2.  Its CPU baseline is the oracle's acceptance.

--impl reference times the reference's own CPU implementation (oracle/_ref,
compiled from the reference sources with its shipped flags) on this host's
cores, on a bounded sample of the same workload.
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


def verify_mma_flops(rows, weights):
    """Tensor-pipe work of one forward of `rows` rows under the exact scheme.
    Below 64 rows the GEMV pads the rows to N = 16 * ceil(rows / 16) and per
    K16 step multiplies A = w_hi by the 2N-row stacked [x_hi; x_lo] and
    A = w_lo by the N rows of x_hi: 6 N flop per weight.  From 64 rows the
    GEMM takes slabs of 256 rows, each padded to N = 16 * ceil(rows / 16), with
    three N-row MMAs per K16 step (w_hi x_hi, w_hi x_lo, w_lo x_hi): again
    6 N flop per weight."""
    step = 64 if rows < 64 else 256
    n = 0
    for c0 in range(0, rows, step):
        c = min(step, rows - c0)
        n += 16 * ((c + 15) // 16)
    return 6 * n * weights


def target_weights(cfg):
    """Weights one target forward multiplies (all layer matrices + LM head)."""
    E, L_, H, KH, F, V = cfg[:6]
    hd = E // H
    return L_ * ((E + 2 * KH * hd) * E + E * E + 3 * F * E) + V * E


def tensor_peak():
    """Sustained dense bf16 TFLOP/s (a kernel timed inside a long step)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), "measured, sustained"
    return 1400.0, "fallback, sustained"


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


def matvec_records(torch, reps=3):
    """Configuration 2 on this GPU, both weight types: per (type, shape, M),
    GB/s of back-to-back vxc_qgemv calls (activation image, GEMV and split-K
    reduction, launched as the public entry point does) over weight copies
    larger than 2x L2, timed by CUDA events around the whole loop.  Bytes
    follow the configuration's formula: weights + fp32 activations in + fp32
    results out."""
    import vxb200
    from qgen import q4_0_blocks, q8_0_blocks
    rng = np.random.default_rng(1234)
    peak, _ = peaks()
    out = {}
    stream = torch.cuda.current_stream()
    for qt, gen, bpb in ((2, q4_0_blocks, 18), (8, q8_0_blocks, 34)):
        for (R, K) in SHAPES:
            blk = gen(R, K, rng)
            wbytes = R * (K // 32) * bpb
            ncopy = max(2, (2 * L2_BYTES + wbytes - 1) // wbytes)
            mats = [vxb200.QMat(qt, blk, R, K) for _ in range(ncopy)]
            for M in MS:
                x = torch.randn(M, K, device="cuda")
                y = torch.empty(M, R, device="cuda")
                wsb = max(mats[0].workspace_bytes(M), 16)
                wsp = torch.empty(wsb // 4 + 4, device="cuda")
                calls = lambda n: [mats[i % ncopy].gemv(x.data_ptr(), M, y.data_ptr(), wsp.data_ptr(), wsb,
                                                         stream.cuda_stream) for i in range(n)]
                calls(2 * ncopy)
                n = reps * ncopy
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                calls(n)
                e1.record(stream)
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / n
                gbs = (wbytes + M * K * 4 + M * R * 4) / (us * 1e-6) / 1e9
                out[f"{'q4_0' if qt == 2 else 'q8_0'} {R}x{K} M={M}"] = {"us": round(us, 2), "gbs": round(gbs, 1),
                                                                         "frac": round(gbs / peak, 4)}
            for W in mats:
                W.close()
    return out


# The GEMM (64+ rows): the 7B target's Q4_0 matrices at prompt-pass row counts.
GEMM_SHAPES = [(12288, 4096), (4096, 4096), (22016, 4096), (4096, 11008)]
GEMM_ROWS = 4096


def gemm_records(torch, cases=None, reps=3):
    """The tensor-core GEMM through the public vxc_qgemv (activation image,
    GEMM, and the ordered sum of its K-slices, as the entry point launches
    them), per (shape, rows): microseconds per call from CUDA events around
    `reps` back-to-back calls after two warm-up calls; algorithmic TFLOP/s
    (2 M R K) and the exact scheme's tensor work (6 x padded rows x weights,
    three fp16 products per weight x activation) against the measured dense
    bf16 peak.  Every call writes K-slice partials and an output far larger
    than L2."""
    import vxb200
    from qgen import q4_0_blocks
    rng = np.random.default_rng(4321)
    tpk, tkind = tensor_peak()
    out = {}
    stream = torch.cuda.current_stream()
    for (R, K, M) in (cases or [(r, k, GEMM_ROWS) for (r, k) in GEMM_SHAPES]):
        W = vxb200.QMat(2, q4_0_blocks(R, K, rng), R, K)
        x = torch.randn(M, K, device="cuda")
        y = torch.empty(M, R, device="cuda")
        wsb = max(W.workspace_bytes(M), 16)
        wsp = torch.empty(wsb // 4 + 4, device="cuda")
        for _ in range(2):
            W.gemv(x.data_ptr(), M, y.data_ptr(), wsp.data_ptr(), wsb, stream.cuda_stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            W.gemv(x.data_ptr(), M, y.data_ptr(), wsp.data_ptr(), wsb, stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        alg = 2.0 * M * R * K / (us * 1e-6) / 1e12
        mma = verify_mma_flops(M, R * K) / (us * 1e-6) / 1e12
        out[f"q4_0 {R}x{K} M={M}"] = {"us": round(us, 1), "tflops": round(alg, 1), "mma_tflops": round(mma, 1),
                                      "mma_frac": round(mma / tpk, 4)}
        W.close()
        del x, y, wsp
    code = ctypes.c_uint(0)
    vxb200.check(vxb200.lib().vxc_check_device_error(ctypes.byref(code)), "device error check")
    out["peak"] = {"tflops": tpk, "source": tkind + " (MEASURED_PEAKS.json bf16; fallback if absent)"}
    return out


def main_q4gemm(args, ws, rank, threads):
    """The tensor-core GEMM alone (the prompt pass's and wide verifies' kernel):
    one line, value = algorithmic TFLOP/s over GEMM_SHAPES at --gemm-rows rows
    (or the single case --gemm-case R,K,M)."""
    import torch
    import vxb200
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    vxb200.check(vxb200.lib().vxc_device_init(local), "vxc_device_init")
    if args.gemm_case:
        R, K, M = (int(v) for v in args.gemm_case.split(","))
        cases = [(R, K, M)]
    else:
        cases = [(r, k, args.gemm_rows) for (r, k) in GEMM_SHAPES]
    clk = ClockSampler(local)
    clk.start()
    rec = gemm_records(torch, cases, reps=max(args.steps, 1))
    clocks = clk.stop()
    tot_us = sum(v["us"] for k, v in rec.items() if k != "peak")
    flop = sum(2.0 * M * R * K for (R, K, M) in cases)
    mma = sum(verify_mma_flops(M, R * K) for (R, K, M) in cases)
    tpk, tkind = tensor_peak()
    if rank == 0:
        print(json.dumps({"metric": "Q4_0 GEMM TFLOP/s (7B target matrices, prompt-pass rows)",
                          "value": round(flop / (tot_us * 1e-6) / 1e12, 1), "unit": "TFLOP/s", "n_gpus": 1,
                          "steps": args.steps, "warmup": 2, "ms_per_step": round(tot_us / 1e3, 3),
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "f32 (exact fp16 hi/lo products, fp32 accumulation)", "data": "synthetic",
                          "config": {"workload": "q4gemm: " + ", ".join(f"{R}x{K} M={M}" for (R, K, M) in cases),
                                     "l2": "no flush: each call writes K-slice partials and outputs far above L2"},
                          "roofline": {"bound": "tensor", "achieved": round(mma / (tot_us * 1e-6) / 1e12, 1),
                                       "peak": tpk, "unit": "TFLOP/s",
                                       "frac": round(mma / (tot_us * 1e-6) / 1e12 / tpk, 4), "traffic": None,
                                       "peak_source": tkind,
                                       "note": "achieved = the exact scheme's tensor work (3 fp16 products per "
                                               "weight x activation) over whole vxc_qgemv calls"},
                          "cases": rec, "clocks": clocks, "cpu_baseline": None, "e2e": None}))


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
    cases = [(s, M) for s in SHAPES for M in MS]
    # The device-side numbers replay CUDA graphs of the public vxc_qgemv calls, so the
    # host's per-call launch cost (ctypes) does not hide the GPU time; e2e below keeps it.
    gs = torch.cuda.Stream()

    def calls(case_list, st):
        for (s, M) in case_list:
            for W in mats[s]:
                W.gemv(xs[M].data_ptr(), M, ys[(s[0], M)].data_ptr(), wsp.data_ptr(), wsb, st)

    def capture(case_list):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=gs):
            calls(case_list, gs.cuda_stream)
        return g

    with torch.cuda.stream(gs):
        for _ in range(max(args.warmup, 1)):
            calls(cases, gs.cuda_stream)
    torch.cuda.synchronize()
    l0 = vxb200.lib().vxc_launch_count()
    g_step = capture(cases)
    launches_per_step = vxb200.lib().vxc_launch_count() - l0
    g_case = {c: capture([c]) for c in cases}
    with torch.cuda.stream(gs):
        for _ in range(max(args.warmup, 3)):
            g_step.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = ClockSampler(local)
    clk.start()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(gs):
        t0.record()
        for k in range(args.steps):
            g_step.replay()
        t1.record()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    n_launch = launches_per_step * args.steps
    clocks = clk.stop()
    ms_total = t0.elapsed_time(t1)
    # per case: its calls alone, replayed 3 times (one GEMV and, for split-K shapes, its reduction per call)
    per_case = {}
    kern_ms, kern_bytes, kern_wbytes, kern_launches = 0.0, 0, 0, 0
    for c in cases:
        (R, K), M = c
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(gs):
            g_case[c].replay()
            e0.record()
            for _ in range(3):
                g_case[c].replay()
            e1.record()
        torch.cuda.synchronize()
        n = 3 * len(mats[c[0]])
        avg = e0.elapsed_time(e1) / n
        b = q4_bytes(R, K, M)
        per_case[f"{R}x{K}_M{M}"] = round(b / (avg * 1e-3) / 1e9, 1)
        kern_ms += avg * n
        kern_bytes += b * n
        kern_wbytes += R * (K // 32) * 18 * n
        kern_launches += n
    del g_step, g_case
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
    res = dict(step_bytes=step_bytes, ms_total=ms_total, e2e_ms=e2e_ms, per_case=per_case,
               kern_ms=kern_ms, kern_bytes=kern_bytes, kern_wbytes=kern_wbytes, kern_launches=kern_launches,
               clocks=clocks, launches=n_launch,
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


# ---------------------------------------------------------------------------
# spec7b
# ---------------------------------------------------------------------------
# (n_embd, n_layers, n_heads, n_kv_heads, n_ff, n_vocab, wtype, seed): benchmark configuration 4
SPEC_TARGET = (4096, 32, 32, 32, 11008, 32000, 2, 11)   # Llama-2-7B shape, Q4_0
SPEC_DRAFT = (2048, 22, 32, 4, 5632, 32000, 8, 12)      # 1.1B shape (GQA 32/4), Q8_0
SPEC = {"seqs_per_gpu": 8, "k": 4, "prompt": 512, "new": 256, "temp": 0.0, "seed": 1}
# 2-layer versions of the same widths: the small case for ncu captures (well under 2 GB on the device)
# configuration 5: Llama-3-70B-shape Q4_0 target split over the GPUs (tensor parallel,
# NCCL all-reduce after the output and down projections), 1B-shape Q8_0 draft on every GPU
SPEC70_TARGET = (8192, 80, 64, 8, 28672, 128256, 2, 21)
SPEC70_DRAFT = (2048, 16, 32, 8, 8192, 128256, 8, 22)
SPEC70 = {"seqs_per_gpu": 32, "k": 6, "prompt": 4096, "new": 128, "temp": 0.8, "seed": 1}
ROPE_THETA = {False: 10000.0, True: 500000.0}
TP = False   # set by --workload spec70b
# configuration 1: tiny Llama target / draft, Q8_0, batch 1, k=4, greedy, 32-id prompt, 128 new tokens
SPEC_TINY_TARGET = (256, 4, 8, 8, 768, 4096, 8, 1)
SPEC_TINY_DRAFT = (128, 2, 4, 4, 384, 4096, 8, 2)
SPEC_TINY = {"seqs_per_gpu": 1, "k": 4, "prompt": 32, "new": 128, "temp": 0.0, "seed": 1}
TINY = False   # set by --workload spec_tiny
SPEC_TARGET_2L = (4096, 2, 32, 32, 11008, 32000, 2, 13)
SPEC_DRAFT_2L = (2048, 2, 32, 4, 5632, 32000, 8, 14)


GOLDEN_SEQ0 = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tests", "golden", "spec7b_seq0.npz")


def first_tokens_vs_golden(first):
    """Sequence 0's first emitted tokens against the committed CPU greedy stream
    of the same target and prompt (tests/golden/spec7b_seq0.npz, written by
    tests/golden/make_spec7b_golden.py from the oracle's scalar forward).  At
    temperature 0 speculative decoding emits the target's greedy stream, so the
    benchmark's rule applies: identical up to the first step whose CPU top-2
    logit margin is at most 1e-3.  Only the full spec7b workload has a golden;
    None elsewhere, when the file is absent or when it was made for another
    model or prompt."""
    try:
        if TP or TINY or SPEC_TARGET != (4096, 32, 32, 32, 11008, 32000, 2, 11) or SPEC["temp"] != 0.0:
            return None
        if not os.path.exists(GOLDEN_SEQ0):
            return None
        g = np.load(GOLDEN_SEQ0)
        if not np.array_equal(g["prompt"], spec_prompts(0, 1)[0]):
            return None
        want, marg = g["greedy"], g["margins"]
        n = min(len(first), len(want))
        same, ok = 0, True
        for i in range(n):
            if int(first[i]) != int(want[i]):
                ok = bool(marg[i] <= 1e-3)
                break
            same += 1
        return {"match": ok, "identical_prefix": same, "compared": n,
                "golden": "tests/golden/spec7b_seq0.npz (CPU oracle greedy stream of sequence 0)",
                "rule": "identical until the first step whose CPU top-2 margin is <= 1e-3"}
    except Exception as e:   # a report field only: never fail the benchmark over it
        return {"match": None, "error": repr(e)[:200]}


def q_bytes(rows, cols, wtype):
    return rows * (cols // 32) * (18 if wtype == 2 else 34)


def model_bytes(cfg):
    """Quantised weight bytes one forward reads: every layer matrix plus the LM
    head (the token-embedding table is gathered by row, not streamed)."""
    E, L, H, KH, F, V, wt, _ = cfg
    hd = E // H
    per_layer = (q_bytes(E + 2 * KH * hd, E, wt) + q_bytes(E, E, wt) + q_bytes(2 * F, E, wt) + q_bytes(E, F, wt))
    return L * per_layer + q_bytes(V, E, wt)


def fixture_dir(need=8 << 30):
    d = os.environ.get("VX_BENCH_DIR")
    if d:
        return d
    import shutil
    if os.path.isdir("/dev/shm") and (os.path.isdir("/dev/shm/vx_bench") or
                                      shutil.disk_usage("/dev/shm").free > need + (4 << 30)):
        return "/dev/shm/vx_bench"
    import tempfile
    return os.path.join(tempfile.gettempdir(), "vx_bench")


def spec_fixtures(write):
    """Paths of the two synthetic GGUFs; written once by the caller that passes write=True."""
    import vxb200
    d = fixture_dir(model_bytes(SPEC_TARGET) + model_bytes(SPEC_DRAFT) + 2 * q_bytes(SPEC_TARGET[5], 8192, 2))
    os.makedirs(d, exist_ok=True)
    paths = []
    if TP:
        names = ("target70b_q4_0", "draft1b70_q8_0")
    elif TINY:
        names = ("tiny_target_q8_0", "tiny_draft_q8_0")
    elif SPEC_TARGET[1] == 32:
        names = ("target7b_q4_0", "draft1b_q8_0")
    else:
        names = ("target7b2l_q4_0", "draft1b2l_q8_0")
    for name, c in zip(names, (SPEC_TARGET, SPEC_DRAFT)):
        p = os.path.join(d, name + ".gguf")
        if write and not os.path.exists(p):
            E, L, H, KH, F, V, wt, seed = c
            tmp = p + ".tmp%d" % os.getpid()
            vxb200.write_synth(tmp, E, L, H, KH, F, V, wt, seed, ROPE_THETA[TP])
            os.replace(tmp, p)
        paths.append(p)
    return paths


def shard(rank, world, per_rank):
    """Global sequence ids of this rank: weak scaling, `per_rank` sequences per GPU."""
    return rank * per_rank, per_rank


def reduce_over_ranks(dist, maxes, sums, device):
    """Max-over-ranks of the timings, sum-over-ranks of the counters (no-op on one rank)."""
    import torch
    t = torch.tensor(maxes, device=device, dtype=torch.float64)
    n = torch.tensor(sums, device=device, dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(n, op=dist.ReduceOp.SUM)
    return t.tolist(), n.tolist()


def spec_prompts(first_seq, n):
    """512 uniform random ids per sequence, seeded by the global sequence index."""
    V = SPEC_TARGET[5]
    return [np.random.default_rng(1000 + first_seq + i).integers(0, V, SPEC["prompt"], dtype=np.int32)
            for i in range(n)]


def run_spec7b_gpu(args, ws, rank, local):
    import torch
    import vxb200
    torch.cuda.set_device(local)
    vxb200.check(vxb200.lib().vxc_device_init(local), "vxc_device_init")
    dist = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                device_id=torch.device("cuda", local))
    t_start = time.time()

    def progress(what):
        if rank == 0:
            print(f"[bench] {time.time() - t_start:7.1f} s  {what}", file=sys.stderr, flush=True)

    if TP:
        # one tensor-parallel group over all GPUs: rank 0's NCCL id reaches the others.  The
        # weights are generated on each GPU (its shard only): the writer's numbers, no 41 GB file
        ids = [vxb200.tp_unique_id() if rank == 0 else None]
        if dist:
            dist.broadcast_object_list(ids, src=0)
        synth = lambda c: c[:7] + (c[7], ROPE_THETA[True])
        target = vxb200.Model(None, tp=(rank, ws, ids[0]), synth=synth(SPEC_TARGET))
        draft = vxb200.Model(None, synth=synth(SPEC_DRAFT))
        first, S = 0, SPEC["seqs_per_gpu"]          # every GPU runs every sequence, on its shard
    else:
        if local == 0:
            spec_fixtures(write=True)
        if dist:
            dist.barrier()
        tpath, dpath = spec_fixtures(write=False)
        target = vxb200.Model(tpath)
        draft = vxb200.Model(dpath)
        first, S = shard(rank, ws, SPEC["seqs_per_gpu"])
    progress("models loaded")
    k = SPEC["k"]
    # generation stops at the target's n_ctx (the reference's rule); configuration 5's
    # 4096-id prompts need a context above the loader's default of 4096
    need = SPEC["prompt"] + SPEC["new"] + k + 8
    for m in (target, draft):
        if m.head.config.n_ctx < need:
            m.head.config.n_ctx = need
    sp = vxb200.Speculative(draft, target, k, temp=SPEC["temp"], seed=SPEC["seed"], seq_id_base=first)
    prompts = spec_prompts(first, S)
    new = SPEC["new"]

    def step():
        t0 = time.perf_counter()
        outs = sp.generate_batch(prompts, new)
        wall = time.perf_counter() - t0
        st = sp.stats()
        return outs, wall, st

    for _ in range(args.warmup):
        step()
        progress("warm-up step done")
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = ClockSampler(local)
    clk.start()
    l0 = vxb200.lib().vxc_launch_count()
    emitted = accepted = drafted = rounds = 0
    dec_ms = pre_ms = wall_s = 0.0
    outs = None
    for _ in range(args.steps):
        outs, wall, st = step()
        emitted += st.emitted
        accepted += st.accepted
        drafted += st.drafted
        rounds += st.rounds
        dec_ms += st.decode_ms
        pre_ms += st.prefill_ms
        wall_s += wall
    torch.cuda.synchronize()
    launches = vxb200.lib().vxc_launch_count() - l0
    if dist:
        dist.barrier()
    clocks = clk.stop()
    progress("timed steps done")
    # per-piece device time of the last round (verify forward, draft step, acceptance)
    v_ms, v_kv = sp.probe(0, 10)
    d_ms, d_kv = sp.probe(1, 10)
    a_ms, _ = sp.probe(2, 10)
    # stage breakdown of one verify / draft forward (events between kernels: slightly slower than v_ms)
    stages = {}
    names = ["embed", "attn_norm", "qkv_gemv", "rope_kv", "attention", "attn_merge", "o_gemv", "ffn_norm",
             "gate_up_gemv", "swiglu", "down_gemv", "lm_head"]
    for which, key in ((0, "verify"), (1, "draft_step")):
        vxb200.lib().vxc_profile_enable(1)
        sp.probe(which, 5)
        buf = (ctypes.c_double * 12)()
        vxb200.lib().vxc_profile_read(buf, 12)
        vxb200.lib().vxc_profile_enable(0)
        stages[key] = {nm: round(buf[i] / 6, 4) for i, nm in enumerate(names)}
    extra = {}
    if ws == 1 and not TP and not TINY:
        # batch 1: one sequence's verify (5 rows), the cleanest weight-dominated roofline case
        one = vxb200.Speculative(draft, target, k, temp=SPEC["temp"], seed=SPEC["seed"], seq_id_base=first)
        one.generate_batch(prompts[:1], 8)
        extra["v1_ms"], extra["v1_kv"] = one.probe(0, 10)
        one.close()
        # the same engine with a draft that agrees with the target (the target drafts for
        # itself): greedy acceptance is then complete and a round emits k + 1 tokens
        agree = vxb200.Speculative(target, target, k, temp=0.0, seed=SPEC["seed"], seq_id_base=first)
        agree.generate_batch(prompts, 16)
        torch.cuda.synchronize()
        agree.generate_batch(prompts, 32)
        st = agree.stats()
        extra["agree"] = {"emitted": st.emitted, "accepted": st.accepted, "drafted": st.drafted,
                          "rounds": st.rounds, "decode_ms": st.decode_ms}
        agree.close()
        progress("batch-1 verify and full-acceptance runs done")
    if TP and dist:
        # the verify's exchanges at the engine's message sizes (every rank, same order)
        rows = S * (k + 1)
        extra["collectives"] = measure_collectives(torch, dist, ws, rows * SPEC_TARGET[0],
                                                   rows * (SPEC_TARGET[5] // ws))
        progress("collective timing done")
    t, n = reduce_over_ranks(dist, [dec_ms, pre_ms, wall_s, v_ms, d_ms, a_ms],
                             [emitted, accepted, drafted, rounds, launches], "cuda")
    dec_ms, pre_ms, wall_s, v_ms_max, d_ms_max, a_ms_max = t
    emitted, accepted, drafted, rounds, launches = [int(x) for x in n]
    if TP:   # every rank emitted the same tokens: count them once
        emitted, accepted, drafted, rounds = [x // ws for x in (emitted, accepted, drafted, rounds)]
    h2d = S * SPEC["prompt"] * 4
    d2h = S * new * 4
    res = dict(emitted=emitted, accepted=accepted, drafted=drafted, rounds=rounds, dec_ms=dec_ms, pre_ms=pre_ms,
               wall_s=wall_s, v_ms=v_ms_max, v_kv=v_kv, d_ms=d_ms_max, d_kv=d_kv, a_ms=a_ms_max, clocks=clocks,
               launches=launches, h2d=h2d, d2h=d2h, first=[int(x) for x in outs[0][:8]], stages=stages,
               extra=extra)
    sp.close()
    draft.close()
    target.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return res


def measure_collectives(torch, dist, ws, n_sum, n_gather_per_rank, reps=20):
    """Device time of the tensor-parallel verify's two exchanges, through
    torch.distributed's NCCL (the library the engine's vxc_tp.cu calls too) at
    the engine's message sizes: the fp32 all-reduce of one row-split
    projection's output (two per layer) and the all-gather of the
    vocabulary-split logits (one per forward).  CUDA events over `reps`
    back-to-back calls after 3 warm-ups; max over ranks."""
    a = torch.ones(n_sum, device="cuda")
    g_in = torch.ones(n_gather_per_rank, device="cuda")
    g_out = torch.empty(n_gather_per_rank * ws, device="cuda")
    for _ in range(3):
        dist.all_reduce(a)
        dist.all_gather_into_tensor(g_out, g_in)
    torch.cuda.synchronize()
    dist.barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    for _ in range(reps):
        dist.all_reduce(a)
    ev[1].record()
    for _ in range(reps):
        dist.all_gather_into_tensor(g_out, g_in)
    ev[2].record()
    torch.cuda.synchronize()
    t = torch.tensor([ev[0].elapsed_time(ev[1]) * 1e3 / reps, ev[1].elapsed_time(ev[2]) * 1e3 / reps],
                     device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ar_us, ag_us = float(t[0]), float(t[1])
    ar_b, ag_b = n_sum * 4, n_gather_per_rank * ws * 4
    return {"allreduce_bytes": ar_b, "allreduce_us": round(ar_us, 2),
            "allreduce_busbw_gbs": round(2 * (ws - 1) / ws * ar_b / (ar_us * 1e-6) / 1e9, 1),
            "gather_bytes": ag_b, "gather_us": round(ag_us, 2),
            "gather_busbw_gbs": round((ws - 1) / ws * ag_b / (ag_us * 1e-6) / 1e9, 1),
            "note": "torch.distributed NCCL at the engine's sizes: one row-split projection's fp32 output "
                    "(all-reduced twice per layer) and the vocabulary-split logits (gathered once per forward); "
                    "CUDA events, max over ranks"}


def cpu_spec7b_reference(threads, reps=2):
    """The reference's own CPU forward (oracle/_ref/libvxref_ship.so: its
    sources built with the shipped AVX2 flags) on the same two GGUFs, all host
    threads.  A full 7B speculative run on the CPU takes hours, so the sample
    is: one 1-token target forward and one 1-token draft forward at context
    512 (cache_len set directly, as the reference's own callers do,
    src/speculative.c:101,153), `reps` times each.  A round of a correct loop
    with the ~0 greedy acceptance of independent random models costs k draft
    forwards + 1 target forward and emits one token per sequence; sequences
    run one after another on the CPU (one vx_model per sequence).  The
    reference's own loop is slower still: it re-runs the draft over the whole
    context every round (src/speculative.c:148-176).  Returns
    (tok/s, kind, sample, detail)."""
    import ctypes as C
    from _paths import ref
    R_ = ref(ship=True)
    R_.vx_set_n_threads(threads)
    tpath, dpath = spec_fixtures(write=True)
    times = {}
    for name, p in (("target", tpath), ("draft", dpath)):
        h = C.c_void_p()
        t0 = time.perf_counter()
        rc = R_.vx_model_create(p.encode(), C.byref(h))
        load_s = time.perf_counter() - t0
        if rc != 0:
            raise RuntimeError(f"reference vx_model_create({p}) = {rc}")
        cfg = (C.c_int * 8)()
        R_.vxref_config(h, cfg)
        logits = np.zeros(cfg[6], np.float32)
        tok = np.array([17], np.int32)
        ts = []
        for _ in range(reps):
            R_.vxref_set_cache_len(h, SPEC["prompt"])
            t0 = time.perf_counter()
            R_.vx_model_forward(h, tok.ctypes.data, 1, logits.ctypes.data)
            ts.append(time.perf_counter() - t0)
        R_.vx_model_destroy(h)
        times[name] = (min(ts), load_s)
    k = SPEC["k"]
    t_round = k * times["draft"][0] + times["target"][0]
    sample = (f"reference AVX2 build, {threads} threads: 1-token forward at context {SPEC['prompt']}, best of {reps}: "
              f"target {times['target'][0] * 1e3:.1f} ms, draft {times['draft'][0] * 1e3:.1f} ms; "
              f"round = {k} draft + 1 target forward -> 1 token")
    return 1.0 / t_round, "reference", sample, {"target_ms": times["target"][0] * 1e3,
                                                 "draft_ms": times["draft"][0] * 1e3}


def main_q4matvec(args, ws, rank, threads):
    metric = "Q4 matvec HBM GB/s (verify-matmul microbench)"
    config = {"workload": "q4matvec: Q4_0 4096x4096 + 11008x4096, M=1,2,5,8 fp32 rows",
              "l2": "weights rotated over copies > 2x L2 per shape (no flush needed)",
              "parallelism": f"replicas x{ws}"}
    if args.impl == "reference":
        gbs, kind, sample = cpu_q4matvec(max(args.steps, 1) * args.cpu_budget / 5, threads)
        print(json.dumps({"impl": "reference", "metric": metric, "value": round(gbs, 3), "unit": "GB/s",
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "higher_is_better": True, "dtype": "f32", "data": "synthetic", "config": config,
                          "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                                           "kind": kind, "sample": sample},
                          "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return
    r = run_q4matvec_gpu(args, ws, rank, int(os.environ.get("LOCAL_RANK", "0")))
    if rank != 0:
        return
    value = ws * r["step_bytes"] * args.steps / (r["ms_total"] * 1e-3) / 1e9
    e2e = ws * r["step_bytes"] * args.steps / (r["e2e_ms"] * 1e-3) / 1e9
    peak, peak_kind = peaks()
    achieved = r["kern_bytes"] / (r["kern_ms"] * 1e-3) / 1e9
    cpu = None
    if ws == 1 and not args.no_cpu:
        gbs, kind, sample = cpu_q4matvec(args.cpu_budget, threads)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample}
    out = {"metric": metric, "value": round(value, 1), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(r["ms_total"] / args.steps, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic", "config": config,
           "per_case_gbs": r["per_case"],
           "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(achieved / peak, 4),
                        "traffic": int(0.5 * (TRAFFIC_Q4_PER_WEIGHT_BYTE + TRAFFIC_Q4_SKINNY_PER_WEIGHT_BYTE)
                                       * r["kern_wbytes"] / r["kern_launches"]),
                        "traffic_note": "per GEMV call: mean weight bytes x the ncu-measured DRAM ratio, averaged "
                                        "over the cases' two kernels (CUDA-core M <= 2: 1.004; tensor-core M >= 5: "
                                        "1.033)",
                        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                        "kernel": "vxc_qgemv calls (GEMV + split-K reduction where the shape has one), "
                                  "CUDA-graph replay per case"},
           "cpu_baseline": cpu,
           "e2e": {"value": round(e2e, 1), "unit": "GB/s", "h2d_bytes_per_step": r["h2d"],
                   "d2h_bytes_per_step": r["d2h"]},
           "gpu_launches": r["launches"], "clocks": r["clocks"]}
    print(json.dumps(out))


SPEC_METRIC = "accepted tok/s (7B-shape Q4_0 spec decode)"

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) from ncu captures of the current
# kernels on B200.  One verify forward of the 2-layer profiling case
#   VX_SPEC_EAGER=1 ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum \
#       --clock-control none -s 2808 -c 24 python bench.py --workload spec2l --steps 1 --warmup 0 --no-cpu --new 8
# gave 170.3 MB per layer outside attention (1.52x its 111.9 MB of Q4_0 weights: image and
# split-K partial traffic), attention at 0.99x its K/V bytes, and 111 MB for the embedding,
# final norm and LM head.  Scaled to 32 layers: traffic = 32 * 170.3 MB + 0.99 * KV bytes + 111 MB.
TRAFFIC_LAYER_NONATTN = 170.3e6
TRAFFIC_HEAD = 111.0e6
TRAFFIC_ATTN_PER_KV_BYTE = 0.99
# A 4096x4096 Q4_0 GEMV launch read 9.745 MB (9,437,184 weight bytes + activations): 1.033x.
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum --clock-control none \
#       -k regex:k_qgemv_mma -s 0 -c 4 python bench.py --workload q4matvec --steps 1 --warmup 0 --no-cpu
TRAFFIC_Q4_PER_WEIGHT_BYTE = 9.745e6 / 9437184
# The CUDA-core GEMV (M <= 2), 4096x4096 Q4_0 M = 1: 9,471,488 DRAM bytes read, 0 written per launch (1.004x):
#   ncu --set full --clock-control none -k regex:k_qgemv_skinny -s 2 -c 1 python bench.py --workload q4matvec \
#       --steps 1 --warmup 0 --no-cpu
TRAFFIC_Q4_SKINNY_PER_WEIGHT_BYTE = 9471488 / 9437184


SPEC70_METRIC = "accepted tok/s (70B-shape Q4_0 tensor-parallel spec decode)"


def spec_config(ws):
    if TP:
        small = "" if (SPEC_TARGET[1], SPEC["prompt"]) == (80, 4096) else " (reduced: functional/profiling case)"
        return {"workload": f"spec70b: Llama-3-70B-shape Q4_0 target ({SPEC_TARGET[1]} layers) split over the "
                            f"GPUs, 1B-shape Q8_0 draft on each, k={SPEC['k']}, T={SPEC['temp']} Philox sampling, "
                            f"{SPEC['seqs_per_gpu']} sequences of {SPEC['prompt']}-id prompts, "
                            f"{SPEC['new']} new tokens, weights generated on the device" + small,
                "global_seqs": SPEC["seqs_per_gpu"], "k": SPEC["k"], "prompt": SPEC["prompt"],
                "new_tokens": SPEC["new"], "temp": SPEC["temp"],
                "l2": "no flush: >= 20 GB of weights and KV per GPU per verify step, far above L2",
                "parallelism": f"tp{ws}: heads, FFN columns and vocabulary split over {ws} GPU(s), "
                               "NCCL all-reduce after the output and down projections, all-gather of the logits"}
    if TINY:
        return {"workload": "spec_tiny: tiny Llama Q8_0 target (dim 256, 4 layers) + draft (dim 128, 2 layers), "
                            f"k={SPEC['k']}, greedy, {SPEC['prompt']}-id prompt, {SPEC['new']} new tokens, batch 1",
                "seqs_per_gpu": SPEC["seqs_per_gpu"], "global_seqs": SPEC["seqs_per_gpu"] * ws, "k": SPEC["k"],
                "prompt": SPEC["prompt"], "new_tokens": SPEC["new"], "temp": SPEC["temp"],
                "l2": "none needed: launch-bound (4.7 MB of weights, L2-resident); reported, not judged",
                "parallelism": f"replicas x{ws}"}
    layers = "" if SPEC_TARGET[1] == 32 else f" ({SPEC_TARGET[1]}+{SPEC_DRAFT[1]} layers: profiling case)"
    return {"workload": "spec7b: Llama-2-7B-shape Q4_0 target + 1.1B-shape Q8_0 draft, k=4, greedy, "
                        f"512-id prompts, {SPEC['new']} new tokens" + layers,
            "seqs_per_gpu": SPEC["seqs_per_gpu"], "global_seqs": SPEC["seqs_per_gpu"] * ws, "k": SPEC["k"],
            "prompt": SPEC["prompt"], "new_tokens": SPEC["new"], "temp": SPEC["temp"],
            "l2": "no flush: >= 4 GB of KV + 3.7 GB of weights per verify step, far above L2",
            "parallelism": f"sequences sharded over {ws} GPU(s), no collective on the data path"}


def main_spec7b(args, ws, rank, threads):
    if args.impl == "reference" and TP:
        print(json.dumps({"impl": "reference", "unavailable": "spec70b: the reference's CPU forward streams 39 GB "
                          "of weights per token; only the configuration 4 sample is timed"}))
        return
    if args.impl == "reference":
        toks, kind, sample, det = cpu_spec_tiny_port(threads) if TINY else cpu_spec7b_reference(threads)
        toks *= 1.0
        print(json.dumps({"impl": "reference", "metric": SPEC_TINY_METRIC if TINY else SPEC_METRIC,
                          "value": round(toks, 4), "unit": "tok/s",
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "higher_is_better": True, "scaling": "weak", "dtype": "f32", "data": "synthetic",
                          "config": spec_config(ws),
                          "cpu_baseline": {"value": round(toks, 4), "unit": "tok/s", "cores": threads,
                                           "kind": kind, "sample": sample},
                          "e2e": {"value": round(toks, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}, "detail": det}))
        return
    r = run_spec7b_gpu(args, ws, rank, int(os.environ.get("LOCAL_RANK", "0")))
    if rank != 0:
        return
    subs = {}
    if ws == 1 and not TP and not TINY:
        # configurations 2 and 3 on the same GPU, so the driver's run records them too
        import torch
        subs["q4matvec"] = matvec_records(torch)
        subs["q4gemm"] = gemm_records(torch)
        a = argparse.Namespace(**vars(args))
        a.steps, a.warmup = 3, 3
        ra = run_accept_gpu(a, 1, 0, int(os.environ.get("LOCAL_RANK", "0")))
        pk, _ = peaks()
        nb = accept_bytes()
        subs["accept"] = {"workload": f"{ACC['seqs']} sequences, k={ACC['k']}, V={ACC['V']}, T={ACC['temp']}",
                          "kernel_us": round(ra["kern_ms"] * 1e3, 2),
                          "gbs": round(nb / (ra["kern_ms"] * 1e-3) / 1e9, 1),
                          "frac": round(nb / (ra["kern_ms"] * 1e-3) / 1e9 / pk, 4), "algorithmic_bytes": nb}
    value = r["emitted"] / (r["dec_ms"] * 1e-3)
    e2e = r["emitted"] / r["wall_s"]
    peak, peak_kind = peaks()
    tw, dw = model_bytes(SPEC_TARGET), model_bytes(SPEC_DRAFT)
    # bytes one GPU must move: its shard of the target (weights and KV) under tensor parallelism
    v_bytes = (tw + r["v_kv"]) / (ws if TP else 1)
    achieved = v_bytes / (r["v_ms"] * 1e-3) / 1e9
    rounds_per_step = r["rounds"] / max(1, (1 if TP else ws) * args.steps)
    round_ms = r["dec_ms"] / args.steps / rounds_per_step
    round_bytes = v_bytes + SPEC["k"] * (dw + r["d_kv"])
    cpu = None
    if TP or TINY:
        traffic, traffic_note = None, "not captured for this workload"
    else:
        traffic = int(SPEC_TARGET[1] * TRAFFIC_LAYER_NONATTN + TRAFFIC_ATTN_PER_KV_BYTE * r["v_kv"] + TRAFFIC_HEAD)
        traffic_note = "ncu DRAM bytes of the 2-layer case's verify, scaled per layer"
    if ws == 1 and not args.no_cpu and not TP:
        try:
            toks, kind, sample, _ = cpu_spec_tiny_port(threads) if TINY else cpu_spec7b_reference(threads)
            cpu = {"value": round(toks, 4), "unit": "tok/s", "cores": threads, "kind": kind, "sample": sample}
        except Exception as ex:   # the reference build is absent: say so, never substitute
            cpu = {"value": None, "unit": "tok/s", "cores": threads, "kind": "reference",
                   "sample": f"not run: {ex}"}
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": traffic, "traffic_note": traffic_note,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
            "kernel": "one (k+1)-row target verify forward (all its kernels), CUDA events on the "
                      "engine stream, 10 re-runs" + (", per GPU (max over GPUs)" if TP else ""),
            "algorithmic_bytes": int(v_bytes), "weight_bytes": tw // (ws if TP else 1),
            "kv_bytes": int(r["v_kv"] / (ws if TP else 1)),
            "verify_ms": round(r["v_ms"], 4)}
    # the same verify seen from the tensor pipe: the exact scheme's MMA work (3 fp16 products per
    # weight x activation product, padded rows included) over the sustained bf16 peak
    rows = SPEC["seqs_per_gpu"] * (SPEC["k"] + 1)
    flops = verify_mma_flops(rows, target_weights(SPEC_TARGET)) / (ws if TP else 1)
    tpk, tpk_kind = tensor_peak()
    ach = flops / (r["v_ms"] * 1e-3) / 1e12
    tview = {"achieved": round(ach, 1), "peak": tpk, "unit": "TFLOP/s", "frac": round(ach / tpk, 4),
             "mma_flops": int(flops), "peak_source": f"{tpk_kind} (MEASURED_PEAKS.json bf16_tflops_sustained)",
             "note": "6 x padded rows x weights of this GPU per verify: the exact hi/lo scheme's MMA work (3 fp16 products per weight x activation)"}
    if TP:
        # 224 rows: the tensor work takes several times the weight streaming (HBM view kept)
        roof = {"bound": "tensor", "achieved": tview["achieved"], "peak": tpk, "unit": "TFLOP/s",
                "frac": tview["frac"], "traffic": None, "traffic_note": traffic_note,
                "peak_source": tview["peak_source"], "kernel": roof["kernel"], "algorithmic_flops": int(flops),
                "flops_note": tview["note"],
                "hbm_view": {"achieved_gbs": round(achieved, 1), "algorithmic_bytes": int(v_bytes)},
                "verify_ms": round(r["v_ms"], 4)}
    else:
        roof["tensor_view"] = tview
    ex = r.get("extra") or {}
    if "v1_ms" in ex:
        b1 = tw + ex["v1_kv"]
        a1 = b1 / (ex["v1_ms"] * 1e-3) / 1e9
        roof["batch1"] = {"verify_ms": round(ex["v1_ms"], 4), "achieved": round(a1, 1), "frac": round(a1 / peak, 4),
                          "algorithmic_bytes": int(b1), "rows": SPEC["k"] + 1,
                          "note": "one sequence's (k+1)-row verify forward: weight-dominated"}
    out = {"metric": SPEC70_METRIC if TP else SPEC_TINY_METRIC if TINY else SPEC_METRIC,
           "value": round(value, 2), "unit": "tok/s",
           "n_gpus": ws, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round((r["dec_ms"] + r["pre_ms"]) / args.steps, 3),
           "higher_is_better": True, "scaling": "strong" if TP else "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic (random N(0,0.02) weights, uniform random prompt ids)", "config": spec_config(ws),
           "roofline": roof,
           "round": {"ms": round(round_ms, 3), "roofline_ms": round(round_bytes / (peak * 1e9) * 1e3, 3),
                     "frac": round(round_bytes / (peak * 1e9) * 1e3 / round_ms, 4),
                     "draft_step_ms": round(r["d_ms"], 4), "accept_ms": round(r["a_ms"], 4)},
           "acceptance": {"rounds": r["rounds"], "drafted": r["drafted"], "accepted": r["accepted"],
                          "emitted": r["emitted"], "rate": round(r["accepted"] / max(1, r["drafted"]), 4),
                          "note": "value counts emitted tokens (accepted drafts + the correction or bonus token); "
                                  "independent random draft and target agree on almost no draft, so a round "
                                  "emits about one token per sequence"},
           "prefill_ms_per_step": round(r["pre_ms"] / args.steps, 2),
           "stage_ms": r["stages"],
           "cpu_baseline": cpu,
           "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": r["h2d"] * ws,
                   "d2h_bytes_per_step": r["d2h"] * ws,
                   "note": "wall time of the vx_speculative_generate_batch calls, prompt pass included"},
           "gpu_launches": r["launches"], "clocks": r["clocks"], "first_tokens_seq0": r["first"]}
    chk = first_tokens_vs_golden(r["first"])
    if chk is not None:
        out["first_tokens_vs_oracle"] = chk
    if "agree" in ex:
        g = ex["agree"]
        out["acceptance"]["full_acceptance"] = {
            "tok_s": round(g["emitted"] / (g["decode_ms"] * 1e-3), 2), "rounds": g["rounds"],
            "drafted": g["drafted"], "accepted": g["accepted"], "emitted": g["emitted"],
            "rate": round(g["accepted"] / max(1, g["drafted"]), 4),
            "note": "the same engine and sequences, 32 new tokens, greedy, with the target drafting for itself "
                    "(every draft accepted: k + 1 tokens per round; each draft step is a 7B forward)"}
    if "collectives" in ex:
        c = dict(ex["collectives"])
        per_verify = 2 * SPEC_TARGET[1] * c["allreduce_us"] + c["gather_us"]
        c["per_verify_us"] = round(per_verify, 1)
        c["share_of_verify"] = round(per_verify * 1e-3 / r["v_ms"], 4)
        out["collectives"] = c
    out.update(subs)
    if not TP and not TINY:
        out["dtype"] = "f32 (tensor-core GEMV: exact weights, fp32 activations split into fp16 hi + lo, 22 bits)"
    print(json.dumps(out))


SPEC_TINY_METRIC = "accepted tok/s (tiny spec decode, configuration 1)"


def cpu_spec_tiny_port(threads):
    """Configuration 1 on the host, timed in full: the oracle's corrected
    speculative loop (oracle/vxo_spec.c: the reference's scalar forward with
    standard rejection sampling; the reference's own loop corrupts its heap
    and samples other distributions) on the same two GGUFs and prompt.
    Returns (tok/s, kind, sample, detail)."""
    import ctypes as C
    from _paths import oracle
    O = oracle()
    tpath, dpath = spec_fixtures(write=True)
    ot = O.vxo_model_load(tpath.encode(), 0)
    od = O.vxo_model_load(dpath.encode(), 0)
    prompt = spec_prompts(0, 1)[0]
    n = SPEC["new"]
    out = np.zeros(n, np.int32)
    rounds = C.c_int()
    t0 = time.perf_counter()
    got = O.vxo_spec_generate(ot, od, prompt.ctypes.data, len(prompt), SPEC["k"], SPEC["temp"], SPEC["seed"], 0,
                              out.ctypes.data, n, C.byref(rounds))
    dt = time.perf_counter() - t0
    O.vxo_model_free(ot)
    O.vxo_model_free(od)
    got = got if got > 0 else n
    sample = (f"oracle speculative loop (scalar reference forward, OpenMP over rows, {threads} threads): "
              f"the whole workload, {got} tokens in {dt:.2f} s, {rounds.value} rounds")
    return got / dt, "port", sample, {"seconds": dt, "rounds": rounds.value}


# ---------------------------------------------------------------------------
# accept: configuration 3, the fused acceptance kernel
# ---------------------------------------------------------------------------
ACC = {"seqs": 64, "k": 5, "V": 32000, "temp": 0.8, "seed": 77}
ACC_METRIC = "acceptance kernel HBM GB/s (configuration 3)"
DRAFT_PURPOSE = 1


def accept_inputs():
    """Target logits [S][k+1][V] ~ N(0, 2^2) (the last row for the bonus
    token), draft logits = target rows + N(0, 0.5^2), positions and ids."""
    S, k, V = ACC["seqs"], ACC["k"], ACC["V"]
    rng = np.random.default_rng(1)
    P = (rng.standard_normal((S, k + 1, V)) * 2.0).astype(np.float32)
    Q = (P[:, :k] + rng.standard_normal((S, k, V)) * 0.5).astype(np.float32)
    pos0 = (100 + np.arange(S)).astype(np.int32)
    ids = np.arange(S, dtype=np.int32)
    return P, Q, pos0, ids


def accept_bytes():
    """Algorithmic bytes of one launch: every logit of P and Q read once."""
    S, k, V = ACC["seqs"], ACC["k"], ACC["V"]
    return S * (2 * k + 1) * V * 4


def run_accept_gpu(args, ws, rank, local):
    import torch
    import vxb200
    torch.cuda.set_device(local)
    L = vxb200.lib()
    vxb200.check(L.vxc_device_init(local), "vxc_device_init")
    dist = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    S, k, V, T, seed = ACC["seqs"], ACC["k"], ACC["V"], ACC["temp"], ACC["seed"]
    P, Q, pos0, ids = accept_inputs()
    nb = accept_bytes()
    ncopy = max(2, (2 * L2_BYTES + nb - 1) // nb)       # rotated copies: more than 2x L2 in total
    Pd = [torch.from_numpy(P).cuda() for _ in range(ncopy)]
    Qd = [torch.from_numpy(Q).cuda() for _ in range(ncopy)]
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    # draft tokens drawn from q by the library's own sampler (Philox purpose DRAFT), as the engine does
    rpos = torch.from_numpy((pos0[:, None] + np.arange(k)[None, :]).astype(np.int32).ravel()).cuda()
    rseq = torch.from_numpy(np.repeat(ids, k).astype(np.int32)).cuda()
    d = torch.zeros(S * k, dtype=torch.int32, device="cuda")
    vxb200.check(L.vxc_sample_rows(Qd[0].data_ptr(), S * k, V, T, seed, rpos.data_ptr(), rseq.data_ptr(),
                                   DRAFT_PURPOSE, d.data_ptr(), ctypes.c_void_p(sp)), "vxc_sample_rows")
    posd, idd = torch.from_numpy(pos0).cuda(), torch.from_numpy(ids).cuda()
    na = torch.zeros(S, dtype=torch.int32, device="cuda")
    nx = torch.zeros(S, dtype=torch.int32, device="cuda")
    wsb = L.vxc_accept_workspace_bytes(S, k)
    wsp = torch.zeros(wsb // 4 + 1, dtype=torch.int32, device="cuda")

    def launch(i):
        vxb200.check(L.vxc_accept(Pd[i].data_ptr(), (k + 1) * V, V, Qd[i].data_ptr(), k * V, V, d.data_ptr(), S, k,
                                  V, T, seed, idd.data_ptr(), posd.data_ptr(), na.data_ptr(), nx.data_ptr(),
                                  wsp.data_ptr(), wsb, ctypes.c_void_p(sp)), "vxc_accept")

    for _ in range(max(args.warmup, 3)):
        for i in range(ncopy):
            launch(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps * ncopy)]
    clk = ClockSampler(local)
    clk.start()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = L.vxc_launch_count()
    t0.record(stream)
    for j in range(args.steps * ncopy):
        evs[j][0].record(stream)
        launch(j % ncopy)
        evs[j][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    launches = L.vxc_launch_count() - l0
    clocks = clk.stop()
    ms_total = t0.elapsed_time(t1)
    kern = [a.elapsed_time(b) for a, b in evs]
    # e2e: logits from pinned host memory each step, accepted lengths and tokens back
    hP, hQ = torch.from_numpy(P).pin_memory(), torch.from_numpy(Q).pin_memory()
    hna, hnx = torch.zeros(S, dtype=torch.int32).pin_memory(), torch.zeros(S, dtype=torch.int32).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        Pd[0].copy_(hP, non_blocking=True)
        Qd[0].copy_(hQ, non_blocking=True)
        launch(0)
        hna.copy_(na, non_blocking=True)
        hnx.copy_(nx, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    code = ctypes.c_uint(0)
    vxb200.check(L.vxc_check_device_error(ctypes.byref(code)), "device error check")
    t = torch.tensor([ms_total, e2e_ms, max(kern)], device="cuda", dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, e2e_ms, _ = t.tolist()
    res = dict(ms_total=ms_total, e2e_ms=e2e_ms, kern_ms=sum(kern) / len(kern), n=len(kern), ncopy=ncopy,
               clocks=clocks, launches=launches, d=d.cpu().numpy(), na=na.cpu().numpy(),
               h2d=P.nbytes + Q.nbytes, d2h=2 * S * 4)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return res


def cpu_accept_port(threads, d=None, budget_s=10.0):
    """The acceptance of all 64 sequences on the host: the oracle's restatement
    (oracle/vxo_spec.c vxo_accept: standard rejection sampling with Philox
    uniforms; the reference's verify_draft, src/speculative.c:178-236, is a
    static part of its broken loop and samples other distributions), one
    thread, repeated for about budget_s.  d = the draft tokens (drawn with
    the oracle's sampler when not given).  Returns (GB/s, kind, sample)."""
    import ctypes as C
    from _paths import oracle
    O = oracle()
    S, k, V, T, seed = ACC["seqs"], ACC["k"], ACC["V"], ACC["temp"], ACC["seed"]
    P, Q, pos0, ids = accept_inputs()
    if d is None:
        d = np.zeros(S * k, np.int32)
        for s in range(S):
            for i in range(k):
                d[s * k + i] = O.vxo_sample(Q[s, i].ctypes.data, V, T,
                                            O.vxo_philox_u32(seed, int(pos0[s]) + i, int(ids[s]), DRAFT_PURPOSE))
    d = np.ascontiguousarray(d, np.int32).reshape(S, k)
    nxt = C.c_int()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s or n == 0:
        for s in range(S):
            O.vxo_accept(P[s].ctypes.data, Q[s].ctypes.data, d[s].ctypes.data, k, V, T, seed, int(ids[s]),
                         int(pos0[s]), C.byref(nxt))
        n += 1
    dt = time.perf_counter() - t0
    return accept_bytes() * n / dt / 1e9, "port", f"oracle acceptance, 1 thread, all {S} sequences x {n} repetitions"


def main_accept(args, ws, rank, threads):
    config = {"workload": f"accept: fused acceptance of {ACC['seqs']} sequences, k={ACC['k']}, V={ACC['V']}, "
                          f"T={ACC['temp']}; target logits N(0,2^2), draft = target + N(0,0.5^2)",
              "l2": "inputs rotated over copies > 2x L2 (no flush needed)", "parallelism": f"replicas x{ws}"}
    if args.impl == "reference":
        gbs, kind, sample = cpu_accept_port(threads, budget_s=max(1, args.steps) * 2.0)
        print(json.dumps({"impl": "reference", "metric": ACC_METRIC, "value": round(gbs, 4), "unit": "GB/s",
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "higher_is_better": True, "dtype": "f32", "data": "synthetic", "config": config,
                          "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": kind,
                                           "sample": sample},
                          "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return
    r = run_accept_gpu(args, ws, rank, int(os.environ.get("LOCAL_RANK", "0")))
    if rank != 0:
        return
    nb = accept_bytes()
    value = ws * nb * r["n"] / (r["ms_total"] * 1e-3) / 1e9
    e2e = ws * nb * args.steps / (r["e2e_ms"] * 1e-3) / 1e9
    peak, peak_kind = peaks()
    achieved = nb / (r["kern_ms"] * 1e-3) / 1e9
    cpu = None
    if ws == 1 and not args.no_cpu:
        gbs, kind, sample = cpu_accept_port(threads, d=r["d"])
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": kind, "sample": sample}
    out = {"metric": ACC_METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(r["ms_total"] / args.steps, 4), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
           "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(achieved / peak, 4), "traffic": None,
                        "traffic_note": "not captured for this workload",
                        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                        "kernel": "vxc_accept, per-launch CUDA events", "algorithmic_bytes": nb,
                        "kernel_us": round(r["kern_ms"] * 1e3, 2)},
           "accepted_mean": round(float(np.mean(r["na"])), 3),
           "cpu_baseline": cpu,
           "e2e": {"value": round(e2e, 1), "unit": "GB/s", "h2d_bytes_per_step": r["h2d"],
                   "d2h_bytes_per_step": r["d2h"]},
           "gpu_launches": r["launches"], "clocks": r["clocks"]}
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="spec7b",
                    choices=["spec7b", "spec2l", "spec70b", "spec_tiny", "q4matvec", "q4gemm", "accept"],
                    help="spec2l: spec7b with 2-layer models, the small case for profilers; "
                         "spec70b: configuration 5, the 70B-shape target tensor-parallel over --gpus")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--new", type=int, default=None, help="new tokens per sequence (spec workloads)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg (profiling runs)")
    ap.add_argument("--layers", type=int, default=None,
                    help="spec70b: target layers (fewer than 80 = a small functional/profiling case)")
    ap.add_argument("--prompt", type=int, default=None, help="spec70b: prompt ids per sequence")
    ap.add_argument("--gemm-rows", type=int, default=GEMM_ROWS, help="q4gemm: activation rows")
    ap.add_argument("--gemm-case", default=None, help="q4gemm: one case R,K,M (a small case for profilers)")
    args = ap.parse_args()
    global SPEC_TARGET, SPEC_DRAFT, TP, TINY
    if args.workload == "spec_tiny":
        TINY = True
        SPEC_TARGET, SPEC_DRAFT = SPEC_TINY_TARGET, SPEC_TINY_DRAFT
        SPEC.update(SPEC_TINY)
    if args.workload == "spec70b":
        TP = True
        SPEC_TARGET, SPEC_DRAFT = SPEC70_TARGET, SPEC70_DRAFT
        SPEC.update(SPEC70)
        if args.layers is not None:
            SPEC_TARGET = SPEC_TARGET[:1] + (args.layers,) + SPEC_TARGET[2:]
        if args.prompt is not None:
            SPEC["prompt"] = args.prompt
    if args.new is not None:
        SPEC["new"] = args.new
    ws, rank, _ = dist_setup(args)
    threads = host_threads()
    if args.impl == "reference" and rank != 0:
        return   # the CPU reference runs on rank 0 only
    if args.workload == "spec2l":
        SPEC_TARGET, SPEC_DRAFT = SPEC_TARGET_2L, SPEC_DRAFT_2L
    if args.workload in ("spec7b", "spec2l", "spec70b", "spec_tiny"):
        main_spec7b(args, ws, rank, threads)
    elif args.workload == "accept":
        main_accept(args, ws, rank, threads)
    elif args.workload == "q4gemm":
        main_q4gemm(args, ws, rank, threads)
    else:
        main_q4matvec(args, ws, rank, threads)


if __name__ == "__main__":
    main()
