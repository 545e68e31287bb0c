#!/usr/bin/env python3
"""Throughput of the fused checksum-protected GEMM on B200.

Workload (one step = one protected GEMM):
  C[M, N_r] = A[M, K] B_r[N_r, K]^T, bf16 in, fp32 accumulate, bf16 out,
  M = N_r = K = 8192 per GPU (--size), with per-tile weighted row checksums,
  detect + locate + correct in the kernel. A is replicated; B[N, K] with
  N = 8192 * n_gpus is split by columns across the ranks (weak scaling: at 8
  GPUs this is the sharded A[8192 x 8192] . B[8192 x 65536] configuration).
  Each step ends with one all-gather of the ranks' fault reports (NCCL).

Printed: one JSON line (rank 0). value = whole-job TFLOP/s (2 M N K / step
time, max over ranks); roofline from CUDA-event timing of the fused kernel
alone; e2e through the public API with A and B_r copied from pinned host
memory every step and the gathered fault reports read back.

``--impl reference`` times the reference's CPU path (torch.matmul + the
python-backend corner check, restated in oracle/ref_port.py) on a row sample
of the same workload with all host threads.

``--model qwen2-7b`` times a Qwen2-7B-shaped prefill of 512 tokens (batch 1,
random init N(0, 0.02), every nn.Linear protected through AbftInjector's
fused path) against plain torch and against the same kernel with checks off.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_BF16_TFLOPS = 1590.0
NOMINAL_BF16_TFLOPS = 2250.0
REF_SAMPLE_ROWS = 512


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--size", type=int, default=8192, help="M = K = per-GPU N")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true",
                    help="one JSON line per shape of the square sweep, the 512x4096x4096 case and the "
                         "Qwen2-7B layer GEMMs: checked / unchecked TFLOP/s and 1- and 4-fault outcomes")
    ap.add_argument("--bmm-sweep", action="store_true",
                    help="batched products (torch.bmm, attention-shaped): cuBLAS vs the fused kernel vs the "
                         "reference's per-batch check loop")
    ap.add_argument("--tile-grid", action="store_true",
                    help="every allowed tile shape (128x128, 128x256, CTA pairs 256x128 and 256x256) per GEMM shape, "
                         "checks off and on, "
                         "against the library's own pick")
    ap.add_argument("--profile-bmm", default=None, metavar="SHAPE",
                    help="two rounds (checks off, then on) of one --bmm-sweep shape: an ncu capture target")
    ap.add_argument("--profile-shape", default=None, metavar="SHAPE",
                    help="two rounds (checks off, then on) of one --sweep shape with the library's tile "
                         "pick: an ncu capture target")
    ap.add_argument("--model", choices=["qwen2-7b", "cogact"], default=None,
                    help="qwen2-7b: prefill-512 tokens/s and decode of a random-init Qwen2-7B-shaped decoder; "
                         "cogact: one CogACT-style VLA forward (ViT-L + SigLIP + Llama-2-7B + DiT-B, 10 "
                         "denoising steps); every linear ABFT-protected (one JSON line)")
    ap.add_argument("--profile-case", choices=["off", "check", "both"], default=None,
                    help="only run two rounds of the fused GEMM (unchecked then checked for 'both') "
                         "on randn inputs, for an ncu capture")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return float(pk["bf16_tflops"]), float(pk.get("bf16_tflops_sustained", pk["bf16_tflops"])), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def load_traffic(workload: str):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload)
    except (OSError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled in the background."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids, period_ms=25):
        self.uuids = {u.lower() for u in uuids}
        self.period_ms = period_ms
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          f"-lms={self.period_ms}"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            self.samples.append((time.time(), parts))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0, t1):
        def pick(lo, hi):
            out = []
            for t, p in self.samples:
                if lo <= t <= hi and (not self.uuids or p[0].lower().replace("gpu-", "") in self.uuids
                                      or p[0].lower() in self.uuids):
                    out.append(p)
            return out

        window = "timed"
        rows = pick(t0, t1)
        if len(rows) < 3:  # timed region shorter than the sampling period: widen to the whole run
            rows, window = pick(-math.inf, math.inf), "run"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "window": window}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        smax = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons, "samples": len(rows),
                "window": window, "power_w_max": max((num(r[3]) or 0.0) for r in rows)}


def init_dist(n_gpus):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def cpu_reference(size, seconds):
    """The reference CPU path on a REF_SAMPLE_ROWS x size x size sample."""
    import torch

    from oracle.ref_port import time_reference_sample

    torch.set_num_threads(os.cpu_count() or 1)
    per, reps, tflops = time_reference_sample(REF_SAMPLE_ROWS, size, size, min_seconds=seconds, max_reps=1)
    return {"value": tflops, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"A[{REF_SAMPLE_ROWS}x{size}] @ B[{size}x{size}] bf16 torch.matmul + corner check "
                      f"(oracle/ref_port.py), {reps} reps, {per * 1e3:.1f} ms each"}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    from oracle.ref_port import reference_protected_matmul

    torch.set_num_threads(os.cpu_count() or 1)
    s = args.size
    g = torch.Generator().manual_seed(0)
    a = (torch.randn(REF_SAMPLE_ROWS, s, generator=g) * s ** -0.5).bfloat16()
    b = (torch.randn(s, s, generator=g) * s ** -0.5).bfloat16()
    for _ in range(args.warmup):
        reference_protected_matmul(a, b)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        reference_protected_matmul(a, b)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    value = 2.0 * REF_SAMPLE_ROWS * s * s / dt / 1e12
    sample = (f"each step: A[{REF_SAMPLE_ROWS}x{s}] @ B[{s}x{s}] bf16 on CPU + python-backend corner check "
              f"(oracle/ref_port.py); a {REF_SAMPLE_ROWS}-row sample of the {s}x{s * world}x{s} job")
    line = {
        "impl": "reference", "metric": "ABFT GEMM TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"square ABFT GEMM {s}x{s}x{s} per GPU, B split by columns",
                   "M": s, "K": s, "N_per_gpu": s, "parallelism": f"dp{world} (column shards)"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    from vla_abft_estimate_b200 import _native as N
    from vla_abft_estimate_b200 import ops
    from vla_abft_estimate_b200.sharded import ShardedAbftGemm, gather_reports, shard_bounds

    world, rank, local = init_dist(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    s = args.size
    n_total = s * world
    c0, c1 = shard_bounds(n_total, world, rank)
    n_r = c1 - c0
    flops_rank = 2.0 * s * n_r * s

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[dev.index])

    # inputs: A replicated (same seed), B shard per rank; both exceed L2 (126 MB) together
    ga = torch.Generator(device=dev).manual_seed(1234)
    gb = torch.Generator(device=dev).manual_seed(5678 + rank)
    a = (torch.randn(s, s, device=dev, generator=ga) * s ** -0.5).bfloat16()
    w = (torch.randn(n_r, s, device=dev, generator=gb) * s ** -0.5).bfloat16()
    out = torch.empty(s, n_r, device=dev, dtype=torch.bfloat16)
    gemm = ShardedAbftGemm(w, c0, mode=N.MODE_DETECT | N.MODE_CORRECT)
    off = ShardedAbftGemm(w, c0, mode=N.MODE_OFF)
    tile_n, _ = gemm._checksums_for(s)
    tile_m = ops.pick_tile_m(s, n_r, s, tile_n, dev)

    # fault-detection sanity outside the timed region: one seeded fault per rank
    from vla_abft_estimate_b200.faults import seeded_fault_positions

    ref_out = gemm(a, out=out)
    delta = 256.0 * out.float().abs().max().item()
    (fr, fc), = seeded_fault_positions(s, n_r, 1, 100 + rank)
    gemm(a, out=torch.empty_like(out), inject=[(fr, fc, delta)])
    grep = gemm.global_report()
    expected = sorted((r_fr, r_fc + shard_bounds(n_total, world, r)[0])
                      for r, (r_fr, r_fc) in ((r, seeded_fault_positions(s, shard_bounds(n_total, world, r)[1]
                                                                              - shard_bounds(n_total, world, r)[0],
                                                                              1, 100 + r)[0]) for r in range(world)))
    detect_ok = grep.coords() == expected and grep.n_corrected == world
    del ref_out

    # encode cost of B_r's checksums (a fresh weight pays it once)
    e_enc0, e_enc1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_enc0.record()
    for _ in range(5):
        ops.encode_weight(w, tile_n)
    e_enc1.record()

    sampler = None
    if local == 0:
        uuids = []
        for i in range(torch.cuda.device_count()):
            try:
                uuids.append(str(torch.cuda.get_device_properties(i).uuid))
            except Exception:  # noqa: BLE001
                pass
        sampler = ClockSampler(uuids)
        sampler.start()
        time.sleep(0.3)

    for _ in range(max(args.warmup, 3)):
        gemm(a, out=out)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_begin, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # untimed GPU spin: the host queues the first steps ahead of the GPU
    torch.cuda._sleep(50_000_000)
    wall0 = time.time()
    t_begin.record()
    for i in range(args.steps):
        starts[i].record()
        gemm(a, out=out, gather=False)
        kends[i].record()
        gather_reports(gemm.report.tensor, gemm.gathered, None)
    t_end.record()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    wall1 = time.time()
    step_ms = t_begin.elapsed_time(t_end) / args.steps
    kernel_ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, kends)) / args.steps
    clean = gemm.global_report()

    # overhead: the same kernel with checksums compiled out, launches
    # interleaved with checked ones so that both see the same clocks
    for _ in range(3):
        off(a, out=out)
    torch.cuda.synchronize()
    n_pair = min(args.steps, 100)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n_pair)]
    torch.cuda._sleep(50_000_000)
    for e in ev:
        e[0].record()
        off(a, out=out, gather=False)
        e[1].record()
        gemm(a, out=out, gather=False)
        e[2].record()
    torch.cuda.synchronize()
    off_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / n_pair
    chk_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / n_pair

    # End to end through the public API with host buffers: every step copies
    # its A and B_r from pinned host memory and reads its gathered fault
    # reports back. Two device buffer sets: step i+1's copies run on a copy
    # stream while step i's GEMM runs (each copy waits until the GEMM that
    # last read its buffers has finished).
    a_h = a.cpu().pin_memory()
    w_h = w.cpu().pin_memory()
    bufs = [(torch.empty_like(a), torch.empty_like(w)) for _ in range(2)]
    e2e_gemms = [ShardedAbftGemm(wd, c0, mode=N.MODE_DETECT | N.MODE_CORRECT) for _, wd in bufs]
    rep_h = [torch.empty(gemm.gathered.shape, dtype=torch.uint8).pin_memory() for _ in range(2)]
    main_stream = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(dev)
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def e2e_copy(j, after=None):
        with torch.cuda.stream(copy_stream):
            if after is not None:
                copy_stream.wait_event(after)
            copy_stream.wait_event(consumed[j])
            bufs[j][0].copy_(a_h, non_blocking=True)
            bufs[j][1].copy_(w_h, non_blocking=True)
            copied[j].record(copy_stream)

    def e2e_compute(j):
        main_stream.wait_event(copied[j])
        g = e2e_gemms[j]
        # the weight copy changed B_r: its checksums are part of this step
        g.checksums = None
        g(bufs[j][0], out=out)
        consumed[j].record(main_stream)
        rep_h[j].copy_(g.gathered, non_blocking=True)

    def e2e_run(steps, start=None):
        e2e_copy(0, start)
        for i in range(steps):
            if i + 1 < steps:
                e2e_copy((i + 1) % 2)
            e2e_compute(i % 2)

    e2e_run(2)
    torch.cuda.synchronize()
    barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = min(args.steps, 50)
    x0.record(main_stream)
    e2e_run(e2e_steps, start=x0)
    x1.record(main_stream)
    torch.cuda.synchronize()
    e2e_ms = x0.elapsed_time(x1) / e2e_steps
    enc_ms = e_enc0.elapsed_time(e_enc1) / 5

    if sampler is not None:
        sampler.stop()

    # max over ranks
    vals = torch.tensor([step_ms, kernel_ms, off_ms, e2e_ms, chk_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        ok_t = torch.tensor([1 if detect_ok else 0, 1 if clean.n_faults == 0 else 0], device=dev)
        dist.all_reduce(ok_t, op=dist.ReduceOp.MIN)
        detect_ok, clean_ok = bool(ok_t[0].item()), bool(ok_t[1].item())
    else:
        clean_ok = clean.n_faults == 0
    step_ms, kernel_ms, off_ms, e2e_ms, chk_ms = [float(x) for x in vals.cpu()]

    if rank == 0:
        flops_job = 2.0 * s * n_total * s
        peak_burst, peak_sus, peak_src = load_peaks()
        # a timed region long enough to reach the power cap is compared with
        # the sustained cuBLAS figure, a short one with the burst figure
        timed_s = step_ms * args.steps * 1e-3
        sustained = timed_s >= 0.1 and peak_sus is not None
        peak = peak_sus if sustained else peak_burst
        achieved = flops_rank / (kernel_ms * 1e-3) / 1e12
        workload = f"abft_gemm_{s}"
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_reference(s, seconds=8.0)
        line = {
            "metric": "ABFT GEMM TFLOP/s",
            "value": flops_job / (step_ms * 1e-3) / 1e12,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": step_ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded randn * K^-1/2)",
            "config": {"workload": f"square ABFT GEMM {s}x{s}x{s} per GPU; B[{n_total}x{s}] split by columns",
                       "M": s, "K": s, "N": n_total, "N_per_gpu": n_r, "tile": [tile_m, tile_n],
                       "cta_pairs": tile_m == 256,
                       "mode": "detect+locate+correct, weight checksums cached", "parallelism": f"dp{world} (column shards)",
                       "l2": "inputs exceed L2 (A+B_r = %d MB > 126 MB)" % ((s * s + n_r * s) * 2 // 2 ** 20)},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": load_traffic(workload),
                         "peak_source": f"{peak_src} ({'sustained' if sustained else 'burst'} cuBLAS bf16, "
                                        f"timed region {timed_s:.3f} s)",
                         "frac_of_burst": achieved / peak_burst,
                         "frac_of_nominal_2250": achieved / NOMINAL_BF16_TFLOPS},
            "cpu_baseline": cpu,
            "e2e": {"value": flops_job / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": (s * s + n_r * s) * 2 * world,
                    "d2h_bytes_per_step": int(gemm.gathered.numel()) * world,
                    "note": "per step: A and B_r from pinned host memory + checksum encode + fused GEMM + report "
                            "gather + D2H; the next step's copies overlap this step's GEMM (two buffer sets)"},
            "gpu_launches": args.steps,
            "clocks": sampler.summary(wall0, wall1) if sampler is not None else None,
            "unchecked_tflops": flops_job / (off_ms * 1e-3) / 1e12,
            "overhead_pct": 100.0 * (chk_ms / off_ms - 1.0),
            "overhead_method": f"{n_pair} checked and {n_pair} unchecked launches interleaved",
            "encode_ms": enc_ms,
            "fault_check": {"injected_located_corrected": detect_ok, "clean_no_false_positive": clean_ok},
        }
        print(json.dumps(line), flush=True)

    if world > 1:
        dist.destroy_process_group()


def profile_case(args):
    """Two rounds of the fused GEMM at --size: the capture target of ncu."""
    import torch

    from vla_abft_estimate_b200 import _native as N
    from vla_abft_estimate_b200 import ops

    dev = torch.device("cuda", 0)
    s = args.size
    a = (torch.randn(s, s, device=dev) * s ** -0.5).bfloat16()
    w = (torch.randn(s, s, device=dev) * s ** -0.5).bfloat16()
    out = torch.empty(s, s, device=dev, dtype=torch.bfloat16)
    tile_n = ops.pick_tile_n(s, s, s, dev, N.MODE_DETECT | N.MODE_CORRECT)
    cks = ops.encode_weight(w, tile_n)
    rep = ops.ReportBuffer(64, dev)
    for _ in range(2):
        if args.profile_case in ("off", "both"):
            ops.abft_gemm(a, w, mode=N.MODE_OFF, out=out, tile_n=ops.pick_tile_n(s, s, s, dev, N.MODE_OFF))
        if args.profile_case in ("check", "both"):
            ops.abft_gemm(a, w, mode=N.MODE_DETECT | N.MODE_CORRECT, out=out, tile_n=tile_n, checksums=cks,
                          report=rep)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": args.profile_case, "size": s, "faults": rep.read().n_faults}))


SWEEP_SHAPES = [
    # (name, M, N, K)
    ("square_1024", 1024, 1024, 1024), ("square_2048", 2048, 2048, 2048), ("square_4096", 4096, 4096, 4096),
    ("square_8192", 8192, 8192, 8192), ("square_16384", 16384, 16384, 16384),
    ("single_512x4096x4096", 512, 4096, 4096),
    ("qwen7b_qkv", 512, 4608, 3584), ("qwen7b_o", 512, 3584, 3584), ("qwen7b_gate_up", 512, 37888, 3584),
    ("qwen7b_down", 512, 3584, 18944), ("qwen7b_lm_head", 512, 152064, 3584),
    # decode: few token rows, HBM-bound on the weight (operands swapped)
    ("decode_m1_qkv", 1, 4608, 3584), ("decode_m1_gate_up", 1, 37888, 3584), ("decode_m1_down", 1, 3584, 18944),
    ("decode_m32_gate_up", 32, 37888, 3584), ("decode_m32_down", 32, 3584, 18944),
    ("decode_m1_o", 1, 3584, 3584),
    # DiT-B action head of the VLA: 16 action tokens through its MLP
    ("dit_m16_fc1", 16, 3072, 768), ("dit_m16_fc2", 16, 768, 3072),
]


def sweep(args):
    """Kernel times with an L2 flush before every timed launch."""
    import torch

    from vla_abft_estimate_b200 import _native as N
    from vla_abft_estimate_b200 import ops
    from vla_abft_estimate_b200.faults import seeded_fault_positions

    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    iters = max(args.steps, 5)
    for name, m, n, k in SWEEP_SHAPES:
        torch.manual_seed(m + n + k)
        a = (torch.randn(m, k, device=dev) * k ** -0.5).bfloat16()
        w = (torch.randn(n, k, device=dev) * k ** -0.5).bfloat16()
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        chk_mode = N.MODE_DETECT | N.MODE_CORRECT
        tn_chk = ops.pick_tile_n(m, n, k, dev, chk_mode)
        tn_off = ops.pick_tile_n(m, n, k, dev, N.MODE_OFF)
        cks = ops.encode_weight(w, tn_chk)
        rep = ops.ReportBuffer(64, dev)

        def timed(fn):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            # a GPU-side spin first, so the host queues every launch ahead of
            # the GPU and no event interval contains host launch latency
            torch.cuda._sleep(200_000_000)
            pairs = []
            for _ in range(iters):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                pairs.append((e0, e1))
            torch.cuda.synchronize()
            ms = sorted(e0.elapsed_time(e1) for e0, e1 in pairs)
            return ms[len(ms) // 2]

        t_cublas = timed(lambda: torch.matmul(a, w.t(), out=out))
        t_off = timed(lambda: ops.abft_gemm(a, w, mode=N.MODE_OFF, out=out, tile_n=tn_off))
        t_chk = timed(lambda: ops.abft_gemm(a, w, mode=chk_mode, out=out, tile_n=tn_chk, checksums=cks, report=rep))
        clean = rep.read()
        outcomes = {"clean_records": clean.n_faults}
        ref = out.clone()
        delta = 256.0 * ref.float().abs().max().item()
        for count in (1, 4):
            faults = seeded_fault_positions(m, n, min(count, m), count)
            c, r = ops.abft_gemm(a, w, mode=chk_mode, tile_n=tn_chk, checksums=cks,
                                 inject=[(i, j, delta) for i, j in faults])
            r = r.read()
            err = (c.float() - ref.float()).abs().max().item() / max(ref.float().abs().max().item(), 1e-30)
            outcomes[f"{count}_fault"] = {"located_exact": r.coords() == sorted(faults),
                                          "corrected": r.n_corrected, "max_rel_err_vs_clean": err}
            if r.coords() != sorted(faults):  # keep the evidence of a mismatch
                outcomes[f"{count}_fault"]["report"] = {
                    "injected": sorted(faults), "n_faults": r.n_faults, "status": r.status,
                    "records": [(x.row, x.col, x.flags, x.residual, x.residual_w, x.threshold) for x in r.records]}
        fl = 2.0 * m * n * k
        wbytes = 2.0 * n * k  # the weight streams once: the HBM-bound term at few rows
        print(json.dumps({"shape": name, "M": m, "N": n, "K": k, "tile_n": [tn_off, tn_chk],
                          "weight_gbs": {"cublas": wbytes / t_cublas / 1e6, "unchecked": wbytes / t_off / 1e6,
                                         "checked": wbytes / t_chk / 1e6},
                          "cublas_tflops": fl / t_cublas / 1e9,
                          "unchecked_tflops": fl / t_off / 1e9, "checked_tflops": fl / t_chk / 1e9,
                          "overhead_pct": 100.0 * (t_chk / t_off - 1.0), "unchecked_ms": t_off, "checked_ms": t_chk,
                          **outcomes}), flush=True)
        del a, w, out, ref, cks


BMM_SHAPES = [
    # (name, batch, M, N, K, mat2 layout): "view" = the transpose of a K-major
    # [B, N, K] tensor (q @ k^T), "rowmajor" = a row-major [B, K, N] (p @ v)
    ("qwen7b_prefill512_scores", 28, 512, 512, 128, "view"),
    ("qwen7b_prefill512_pv", 28, 512, 128, 512, "rowmajor"),
    ("s4096_scores_h32", 32, 4096, 4096, 128, "view"),
    ("s4096_pv_h32", 32, 4096, 128, 4096, "rowmajor"),
    ("decode_scores_kv4096", 28, 1, 4096, 128, "view"),
    ("decode_pv_kv4096", 28, 1, 128, 4096, "rowmajor"),
    ("batched_2048_b8", 8, 2048, 2048, 2048, "rowmajor"),
]


TILE_GRID_SHAPES = [
    ("qwen7b_o", 512, 3584, 3584), ("qwen7b_qkv", 512, 4608, 3584), ("qwen7b_gate_up", 512, 37888, 3584),
    ("qwen7b_down", 512, 3584, 18944), ("qwen7b_lm_head", 512, 152064, 3584), ("single_512x4096x4096", 512, 4096, 4096),
    ("square_2048", 2048, 2048, 2048), ("square_4096", 4096, 4096, 4096), ("vit_l_mlp_up", 256, 4096, 1024),
    ("vit_l_qkv", 256, 3072, 1024), ("llama7b_288_gate_up", 288, 22016, 4096), ("llama7b_288_down", 288, 4096, 11008),
    ("m1024_4096", 1024, 4096, 4096), ("square_8192", 8192, 8192, 8192),
]


def tile_grid(args):
    """Kernel time (L2 flushed, median) of every allowed tile shape per GEMM
    shape, checks off and on, next to the tile shape the library picks."""
    import torch

    from vla_abft_estimate_b200 import _native as N
    from vla_abft_estimate_b200 import ops

    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    iters = max(min(args.steps, 50), 5)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        torch.cuda._sleep(100_000_000)
        ev = []
        for _ in range(iters):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            ev.append((e0, e1))
        torch.cuda.synchronize()
        return sorted(a.elapsed_time(b) for a, b in ev)[iters // 2] * 1e3

    for name, m, n, k in TILE_GRID_SHAPES:
        a = (torch.randn(m, k, device=dev) * k ** -0.5).bfloat16()
        w = (torch.randn(n, k, device=dev) * k ** -0.5).bfloat16()
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        rep = ops.ReportBuffer(64, dev)
        row = {"shape": name, "M": m, "N": n, "K": k}
        for mode, tag in ((N.MODE_OFF, "off"), (N.MODE_DETECT | N.MODE_CORRECT, "checked")):
            tn = ops.pick_tile_n(m, n, k, dev, mode)
            tm = ops.pick_tile_m(m, n, k, tn, dev, mode)
            us = {}
            for ctn, ctm in ((128, 128), (256, 128), (128, 256), (256, 256)):
                cks = ops.encode_weight(w, ctn) if mode else None
                us[f"{ctm}x{ctn}"] = round(timed(lambda: ops.abft_gemm(
                    a, w, mode=mode, out=out, tile_n=ctn, tile_m=ctm, swap_ab=1, checksums=cks,
                    report=rep if mode else None)), 2)
            best = min(us, key=us.get)
            pick = f"{tm}x{tn}"  # tile rows x columns
            row[tag] = {"us": us, "pick": pick, "best": best, "pick_loss_pct": round(100 * (us[pick] / us[best] - 1), 1)}
        print(json.dumps(row), flush=True)
        del a, w, out


def profile_shape(args):
    """Two rounds of one --sweep GEMM shape, checks off then on: the ncu target."""
    import torch

    from vla_abft_estimate_b200 import _native as N
    from vla_abft_estimate_b200 import ops

    _, m, n, k = {s[0]: s for s in SWEEP_SHAPES}[args.profile_shape]
    dev = torch.device("cuda", 0)
    a = (torch.randn(m, k, device=dev) * k ** -0.5).bfloat16()
    w = (torch.randn(n, k, device=dev) * k ** -0.5).bfloat16()
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    rep = ops.ReportBuffer(64, dev)
    for _ in range(2):
        ops.abft_gemm(a, w, mode=N.MODE_OFF, out=out)
        ops.abft_gemm(a, w, mode=N.MODE_DETECT | N.MODE_CORRECT, out=out, report=rep)
    torch.cuda.synchronize()
    print(json.dumps({"profile_shape": args.profile_shape, "faults": rep.read().n_faults}))


def profile_bmm(args):
    """Two rounds of one batched shape, checks off then on: the ncu target."""
    import torch

    from vla_abft_estimate_b200 import _native as N
    from vla_abft_estimate_b200 import ops

    shape = {s[0]: s for s in BMM_SHAPES}[args.profile_bmm]
    _, bsz, m, n, k, lay = shape
    dev = torch.device("cuda", 0)
    a = (torch.randn(bsz, m, k, device=dev) * k ** -0.5).bfloat16()
    w = (torch.randn(bsz, n, k, device=dev) * k ** -0.5).bfloat16()
    b = w.transpose(1, 2) if lay == "view" else w.transpose(1, 2).contiguous()
    out = torch.empty(bsz, m, n, device=dev, dtype=torch.bfloat16)
    rep = ops.ReportBuffer(64, dev, batch=bsz)
    for _ in range(2):
        ops.abft_bmm(a, b, mode=N.MODE_OFF, out=out)
        ops.abft_bmm(a, b, mode=N.MODE_DETECT | N.MODE_CORRECT, out=out, report=rep)
    torch.cuda.synchronize()
    print(json.dumps({"profile_bmm": args.profile_bmm, "faults": rep.read().n_faults}))


def reference_bmm_flow(a, b):
    """What the reference's bmm hook runs on the GPU: torch.bmm, then per
    batch the python-backend corner check (pytorch/abft/checkers.py:112-126)
    ending in a host read (:103), inside the loop of injector.py:180-186."""
    import torch

    out = torch.bmm(a, b)
    ok = True
    for bi in range(a.shape[0]):
        s_a = a[bi].sum(dim=0)
        s_b = b[bi].sum(dim=1)
        corner = torch.dot(s_a, s_b)
        sum_c = out[bi].sum()
        diff = torch.abs(corner - sum_c)
        rel = diff / torch.clamp(torch.abs(sum_c), min=1.0)
        ok &= bool((diff <= 1e-2) or (rel <= 1e-2))
    return out, ok


def bmm_sweep(args):
    """Batched products: device times (L2 flushed) of cuBLAS bmm, the fused
    kernel with checks off and on; wall times of the reference's hook flow
    (bmm + per-batch checks with a host read each) and of AbftInjector's
    fused bmm (deferred reports), both per call."""
    import torch

    from vla_abft_estimate_b200 import _native as N
    from vla_abft_estimate_b200 import ops
    from vla_abft_estimate_b200.abft import AbftConfig, AbftInjector, AbftStatsCollector, CheapSumChecker

    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    iters = max(args.steps, 5)
    chk = N.MODE_DETECT | N.MODE_CORRECT

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        torch.cuda._sleep(200_000_000)
        pairs = []
        for _ in range(iters):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            pairs.append((e0, e1))
        torch.cuda.synchronize()
        ms = sorted(e0.elapsed_time(e1) for e0, e1 in pairs)
        return ms[len(ms) // 2]

    def wall(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) * 1e3 / reps

    for name, bsz, m, n, k, lay in BMM_SHAPES:
        torch.manual_seed(bsz + m + n + k)
        a = (torch.randn(bsz, m, k, device=dev) * k ** -0.5).bfloat16()
        w = (torch.randn(bsz, n, k, device=dev) * k ** -0.5).bfloat16()
        b = w.transpose(1, 2) if lay == "view" else w.transpose(1, 2).contiguous()
        out = torch.empty(bsz, m, n, device=dev, dtype=torch.bfloat16)
        rep = ops.ReportBuffer(64, dev, batch=bsz)
        t_cublas = timed(lambda: torch.bmm(a, b, out=out))
        t_off = timed(lambda: ops.abft_bmm(a, b, mode=N.MODE_OFF, out=out))
        t_chk = timed(lambda: ops.abft_bmm(a, b, mode=chk, out=out, report=rep))
        clean = rep.read().n_faults
        ref = out.clone()
        delta = 256.0 * ref.float().abs().max().item()
        bf = bsz // 2
        _, r1 = ops.abft_bmm(a, b, mode=chk, inject=[(bf * m + m // 2, n // 3, delta)])
        r1 = r1.read()
        reps = max(5, min(50, iters // 4))
        t_ref = wall(lambda: reference_bmm_flow(a, b), reps)
        cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=False)
        stats = AbftStatsCollector()
        inj = AbftInjector(cfg, CheapSumChecker(cfg), stats, defer_reports=True)
        with torch.inference_mode(), inj:
            t_inj = wall(lambda: torch.bmm(a, b), reps)
        s = stats.export_summary()["abft"]
        fl = 2.0 * bsz * m * n * k
        print(json.dumps({
            "shape": name, "batch": bsz, "M": m, "N": n, "K": k, "mat2": lay,
            "cublas_tflops": fl / t_cublas / 1e9, "unchecked_tflops": fl / t_off / 1e9,
            "checked_tflops": fl / t_chk / 1e9, "cublas_ms": t_cublas, "unchecked_ms": t_off, "checked_ms": t_chk,
            "overhead_vs_cublas_pct": 100.0 * (t_chk / t_cublas - 1.0),
            "reference_flow_ms": t_ref, "injector_fused_ms": t_inj, "speedup_vs_reference_flow": t_ref / t_inj,
            "injector_checks": s["checks_total"], "injector_fails": s["fail_total"],
            "clean_records": clean, "fault_located_exact": r1.coords() == [(bf * m + m // 2, n // 3)],
            "fault_batch_counts": r1.batch_counts[bf] if r1.batch_counts else None}), flush=True)
        del a, w, b, out, ref


# ------------------------------------------------------------------ model path
QWEN2_7B = dict(hidden=3584, inter=18944, layers=28, heads=28, kv_heads=4, head_dim=128, vocab=152064,
                rope_theta=1000000.0, eps=1e-6)


def build_qwen2(cfg, device, seed=0):
    """Qwen2-style decoder: RMSNorm, fused QKV (with bias) + RoPE + GQA
    attention (SDPA), SwiGLU MLP with fused gate+up, tied-free lm_head.
    Every projection is an nn.Linear, so F.linear hooks see all of them."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F

    class RMSNorm(nn.Module):
        def __init__(self, h):
            super().__init__()
            self.weight = nn.Parameter(torch.ones(h))

        def forward(self, x):
            xf = x.float()
            return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + cfg["eps"])).to(x.dtype) * self.weight

    def rope(x, cos, sin):  # x [T, H, D]
        x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
        return x * cos + torch.cat((-x2, x1), dim=-1) * sin

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            h, nh, nkv, hd, it = cfg["hidden"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["inter"]
            self.ln1, self.ln2 = RMSNorm(h), RMSNorm(h)
            self.qkv = nn.Linear(h, (nh + 2 * nkv) * hd, bias=True)
            self.o = nn.Linear(nh * hd, h, bias=False)
            self.gate_up = nn.Linear(h, 2 * it, bias=False)
            self.down = nn.Linear(it, h, bias=False)

        def forward(self, x, cos, sin, cache=None, pos=0):
            nh, nkv, hd = cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
            t = x.shape[0]
            q, k, v = self.qkv(self.ln1(x)).split([nh * hd, nkv * hd, nkv * hd], dim=-1)
            q = rope(q.view(t, nh, hd), cos, sin).transpose(0, 1)
            k = rope(k.view(t, nkv, hd), cos, sin).transpose(0, 1)
            v = v.view(t, nkv, hd).transpose(0, 1)
            if cache is not None:  # [2, nkv, T_max, hd]: keys and values of positions < pos + t
                cache[0, :, pos:pos + t] = k
                cache[1, :, pos:pos + t] = v
                k, v = cache[0, :, :pos + t], cache[1, :, :pos + t]
            a = F.scaled_dot_product_attention(q, k, v, is_causal=(t > 1), enable_gqa=True)
            x = x + self.o(a.transpose(0, 1).reshape(t, nh * hd))
            g, u = self.gate_up(self.ln2(x)).chunk(2, dim=-1)
            return x + self.down(F.silu(g) * u)

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = nn.Embedding(cfg["vocab"], cfg["hidden"])
            self.layers = nn.ModuleList([Layer() for _ in range(cfg["layers"])])
            self.norm = RMSNorm(cfg["hidden"])
            self.lm_head = nn.Linear(cfg["hidden"], cfg["vocab"], bias=False)

        def forward(self, ids, caches=None, pos=0):
            t = ids.shape[0]
            hd = cfg["head_dim"]
            inv = 1.0 / (cfg["rope_theta"] ** (torch.arange(0, hd, 2, device=ids.device).float() / hd))
            ang = torch.outer(torch.arange(pos, pos + t, device=ids.device).float(), inv)
            ang = torch.cat((ang, ang), dim=-1)[:, None, :]
            cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
            x = self.embed(ids)
            for i, layer in enumerate(self.layers):
                x = layer(x, cos, sin, None if caches is None else caches[i], pos)
            return self.lm_head(self.norm(x))

        def new_caches(self, t_max):
            return [torch.zeros(2, cfg["kv_heads"], t_max, cfg["head_dim"], dtype=torch.bfloat16,
                                device=self.embed.weight.device) for _ in range(cfg["layers"])]

    torch.manual_seed(seed)
    with torch.device(device):
        model = Model().to(torch.bfloat16)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, (nn.Linear, nn.Embedding)):
                mod.weight.normal_(0.0, 0.02)
                if getattr(mod, "bias", None) is not None:
                    mod.bias.zero_()
    return model.eval()


def cpu_model_baseline(cfg, tokens, seconds):
    """Reference flow on the host CPU for one decoder layer's four linears
    (torch.matmul + corner check, oracle/ref_port.py), scaled to a full
    prefill: layers x (that time) + the lm_head sample's time."""
    import torch

    from oracle.ref_port import time_reference_sample

    torch.set_num_threads(os.cpu_count() or 1)
    h, it, nh, nkv, hd, V = (cfg["hidden"], cfg["inter"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"],
                             cfg["vocab"])
    shapes = [(h, (nh + 2 * nkv) * hd), (nh * hd, h), (h, 2 * it), (it, h)]
    per_layer = 0.0
    t_end = time.perf_counter() + seconds
    for k, n in shapes:
        per, _, _ = time_reference_sample(tokens, k, n, max_reps=1)
        per_layer += per
    # lm_head: time a 1/16 column slice, scale by 16
    per_head, _, _ = time_reference_sample(tokens, h, V // 16, max_reps=1)
    total = per_layer * cfg["layers"] + per_head * 16
    del t_end
    return {"value": tokens / total, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"one decoder layer's 4 linears + 1/16 of lm_head at M={tokens} through the reference "
                      f"flow (torch.matmul + corner check, oracle/ref_port.py), scaled to "
                      f"{cfg['layers']} layers + lm_head; attention and norms excluded"}


def run_model(args):
    import torch

    from vla_abft_estimate_b200.abft import AbftConfig, AbftInjector, AbftStatsCollector, CheapSumChecker

    cfg = QWEN2_7B
    tokens = 512
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    model = build_qwen2(cfg, dev)
    ids = torch.randint(0, cfg["vocab"], (tokens,), device=dev, generator=torch.Generator(device=dev).manual_seed(7))
    reps = max(args.steps, 3) if args.steps < 300 else 10

    def timed_forward(ctx_factory):
        """Median forward time (host work included: launches, report
        reads), and the median device time of the forward's kernels alone
        (host queued ahead behind a device sleep)."""
        times, gpu_times = [], []
        out = None
        with torch.inference_mode():
            for i in range(max(args.warmup, 2) + reps):
                ctx = ctx_factory()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                e0.record()
                with ctx:
                    out = model(ids)
                e1.record()
                torch.cuda.synchronize()
                g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda._sleep(100_000_000)
                g0.record()
                with ctx:
                    out = model(ids)
                    g1.record()
                torch.cuda.synchronize()
                if i >= max(args.warmup, 2):
                    times.append(e0.elapsed_time(e1))
                    gpu_times.append(g0.elapsed_time(g1))
        return statistics.median(times), out, statistics.median(gpu_times)

    import contextlib

    # one injector per leg, reused across repetitions (its weight checksum
    # cache is what a serving process keeps); flush() at exit reads the
    # deferred reports once per forward
    stats_chk = AbftStatsCollector()
    cfg_chk = AbftConfig(enable=True, checker_backend="b200", detect_only=False)
    inj_chk = AbftInjector(cfg_chk, CheapSumChecker(cfg_chk), stats_chk, defer_reports=True)
    stats_off = AbftStatsCollector()
    cfg_off = AbftConfig(enable=True, check_enable=False, checker_backend="b200")
    inj_off = AbftInjector(cfg_off, CheapSumChecker(cfg_off), stats_off, defer_reports=True)

    t_torch, ref_logits, g_torch = timed_forward(contextlib.nullcontext)
    t_off, off_logits, g_off = timed_forward(lambda: inj_off)
    t_chk, chk_logits, g_chk = timed_forward(lambda: inj_chk)
    summ = stats_chk.export_summary()
    n_checks = summ["abft"]["checks_total"] // 2  # two forwards per repetition

    # fault leg: every linear of one forward may be hit (probability 0.05),
    # each fault +1.0 on the fp32 accumulator; detect + locate + correct
    stats_f = AbftStatsCollector()
    cfg_f = AbftConfig(enable=True, checker_backend="b200", detect_only=False, inject_fault=True,
                       inject_probability=0.05, inject_magnitude=1.0, seed=11)
    inj_f = AbftInjector(cfg_f, CheapSumChecker(cfg_f), stats_f, defer_reports=True)
    with torch.inference_mode(), inj_f:
        f_logits = model(ids)
    torch.cuda.synchronize()
    fs = stats_f.export_summary()
    flt = {k: v for k, v in fs["abft"]["faults"].items() if k != "located"}
    max_diff = (f_logits.float() - chk_logits.float()).abs().max().item()
    logits_scale = chk_logits.float().abs().max().item()

    # decode: prefill 512 tokens into a KV cache, then time single-token steps
    def timed_decode(ctx_factory, steps=32):
        caches = model.new_caches(tokens + steps + 8)
        with torch.inference_mode():
            with ctx_factory():
                model(ids, caches, 0)
            nxt = ids[-1:].clone()
            for i in range(4):  # warm-up steps
                with ctx_factory():
                    model(nxt, caches, tokens + i)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(steps):
                with ctx_factory():
                    model(nxt, caches, tokens + 4 + i)
            e1.record()
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    d_torch = timed_decode(contextlib.nullcontext)
    d_off = timed_decode(lambda: inj_off)
    d_chk = timed_decode(lambda: inj_chk)

    linear_flops = 0.0
    h, it, nh, nkv, hd, V = (cfg["hidden"], cfg["inter"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"],
                             cfg["vocab"])
    for k, n in [(h, (nh + 2 * nkv) * hd), (nh * hd, h), (h, 2 * it), (it, h)]:
        linear_flops += 2.0 * tokens * k * n * cfg["layers"]
    linear_flops += 2.0 * tokens * h * V
    cpu = None if args.no_cpu_baseline else cpu_model_baseline(cfg, tokens, 20.0)
    line = {
        "metric": "Qwen2-7B prefill-512 tokens/s (every linear ABFT-protected)",
        "value": tokens / (t_chk * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": reps,
        "warmup": max(args.warmup, 2), "ms_per_step": t_chk, "higher_is_better": True, "scaling": "none",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random init N(0,0.02), random token ids)",
        "config": {"workload": "Qwen2-7B-shaped decoder prefill, batch 1, 512 tokens", **cfg,
                   "fused_shapes": "qkv 3584->4608 (bias), o 3584->3584, gate_up 3584->37888, down 18944->3584, "
                                   "lm_head 3584->152064",
                   "abft": "b200 backend: one fused GEMM + row-checksum check + correct per linear, "
                           "reports deferred to one read per forward"},
        "torch_tokens_per_s": tokens / (t_torch * 1e-3),
        "unchecked_kernel_tokens_per_s": tokens / (t_off * 1e-3),
        "ms": {"torch": t_torch, "b200_unchecked": t_off, "b200_abft": t_chk},
        "device_ms": {"torch": g_torch, "b200_unchecked": g_off, "b200_abft": g_chk,
                      "note": "kernels only: the host queued the forward behind a device sleep"},
        "decode_ms_per_token": {"torch": d_torch, "b200_unchecked": d_off, "b200_abft": d_chk,
                                "abft_overhead_vs_torch_pct": 100.0 * (d_chk / d_torch - 1.0),
                                "note": "after a 512-token prefill into a KV cache; every linear at M = 1 "
                                        "(operands swapped: weight on the MMA's 128-row side)"},
        "overhead_vs_torch_pct": 100.0 * (t_chk / t_torch - 1.0),
        "overhead_vs_unchecked_pct": 100.0 * (t_chk / t_off - 1.0),
        "linear_tflops_abft": linear_flops / (t_chk * 1e-3) / 1e12,
        "checked_linears_per_forward": n_checks // (reps + max(args.warmup, 2)),
        "clean_false_positives": summ["abft"]["faults"]["detected_total"],
        "fault_leg": {"injected": fs["fault_injection"]["injections_total"],
                      "detected_injections": fs["fault_injection"]["detected_injections_total"],
                      "faults": flt,
                      "max_abs_logit_diff_vs_clean": max_diff, "max_abs_logit": logits_scale},
        "logits_max_abs_diff_torch_vs_abft": (ref_logits.float() - chk_logits.float()).abs().max().item(),
        "cpu_baseline": cpu,
        "reference_published": {"tokens_per_s_no_abft": 7217, "tokens_per_s_abft_python": 5909,
                                "decode_ms_no_abft": 29.90, "decode_ms_abft_python": 73.97,
                                "source": "pytorch/baseline_7b_prefill512.json:44, "
                                          "pytorch/abft_7b_prefill512_nsys.json:44 (GPU unrecorded)"},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------- VLA (CogACT-style)
COGACT = dict(
    vit=dict(hidden=1024, mlp=4096, layers=24, heads=16),        # ViT-L/14 at 224^2
    siglip=dict(hidden=1152, mlp=4304, layers=27, heads=16),     # SigLIP-So400m/14 at 224^2
    llm=dict(hidden=4096, mlp=11008, layers=32, heads=32),       # Llama-2-7B
    dit=dict(hidden=768, mlp=3072, layers=12, heads=12),         # DiT-B action head
    patches=256, text_tokens=32, action_tokens=16, action_dim=7, denoise_steps=10, vocab=32000)


def build_cogact(cfg, device, seed=0):
    """Random-init CogACT-style VLA: two ViT encoders (patch conv, pre-norm
    blocks with fused QKV + GELU MLP), an MLP projector, a Llama-style
    decoder (RMSNorm, RoPE, fused QKV, SwiGLU with fused gate+up) and a
    DiT-B action head (adaLN-zero blocks conditioned on the decoder's last
    hidden state and the denoising step). Every projection is an nn.Linear."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F

    class RMSNorm(nn.Module):
        def __init__(self, h):
            super().__init__()
            self.weight = nn.Parameter(torch.ones(h))

        def forward(self, x):
            xf = x.float()
            return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype) * self.weight

    def attend(qkv, heads, causal, cos=None, sin=None):
        t, three_h = qkv.shape
        hd = three_h // 3 // heads
        q, k, v = qkv.view(t, 3, heads, hd).unbind(1)
        if cos is not None:
            def rope(x):
                x1, x2 = x[..., : hd // 2], x[..., hd // 2:]
                return x * cos + torch.cat((-x2, x1), dim=-1) * sin
            q, k = rope(q), rope(k)
        o = F.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1), is_causal=causal)
        return o.transpose(0, 1).reshape(t, heads * hd)

    class VitBlock(nn.Module):
        def __init__(self, c):
            super().__init__()
            h = c["hidden"]
            self.heads = c["heads"]
            self.n1, self.n2 = nn.LayerNorm(h), nn.LayerNorm(h)
            self.qkv, self.o = nn.Linear(h, 3 * h), nn.Linear(h, h)
            self.fc1, self.fc2 = nn.Linear(h, c["mlp"]), nn.Linear(c["mlp"], h)

        def forward(self, x):
            x = x + self.o(attend(self.qkv(self.n1(x)), self.heads, False))
            return x + self.fc2(F.gelu(self.fc1(self.n2(x)), approximate="tanh"))

    class Vit(nn.Module):
        def __init__(self, c):
            super().__init__()
            self.patch = nn.Conv2d(3, c["hidden"], kernel_size=14, stride=14)
            self.pos = nn.Parameter(torch.zeros(cfg["patches"], c["hidden"]))
            self.blocks = nn.ModuleList([VitBlock(c) for _ in range(c["layers"])])
            self.norm = nn.LayerNorm(c["hidden"])

        def forward(self, img):
            x = self.patch(img).flatten(2).transpose(1, 2)[0] + self.pos
            for b in self.blocks:
                x = b(x)
            return self.norm(x)

    class LlamaBlock(nn.Module):
        def __init__(self, c):
            super().__init__()
            h = c["hidden"]
            self.heads = c["heads"]
            self.n1, self.n2 = RMSNorm(h), RMSNorm(h)
            self.qkv, self.o = nn.Linear(h, 3 * h, bias=False), nn.Linear(h, h, bias=False)
            self.gate_up, self.down = nn.Linear(h, 2 * c["mlp"], bias=False), nn.Linear(c["mlp"], h, bias=False)

        def forward(self, x, cos, sin):
            x = x + self.o(attend(self.qkv(self.n1(x)), self.heads, True, cos, sin))
            g, u = self.gate_up(self.n2(x)).chunk(2, dim=-1)
            return x + self.down(F.silu(g) * u)

    class DitBlock(nn.Module):
        def __init__(self, c):
            super().__init__()
            h = c["hidden"]
            self.heads = c["heads"]
            self.n1 = nn.LayerNorm(h, elementwise_affine=False)
            self.n2 = nn.LayerNorm(h, elementwise_affine=False)
            self.qkv, self.o = nn.Linear(h, 3 * h), nn.Linear(h, h)
            self.fc1, self.fc2 = nn.Linear(h, c["mlp"]), nn.Linear(c["mlp"], h)
            self.ada = nn.Linear(h, 6 * h)

        def forward(self, x, c):
            s1, b1, g1, s2, b2, g2 = self.ada(F.silu(c)).chunk(6, dim=-1)
            x = x + g1 * self.o(attend(self.qkv(self.n1(x) * (1 + s1) + b1), self.heads, False))
            return x + g2 * self.fc2(F.gelu(self.fc1(self.n2(x) * (1 + s2) + b2), approximate="tanh"))

    class Vla(nn.Module):
        def __init__(self):
            super().__init__()
            v, s, l, d = cfg["vit"], cfg["siglip"], cfg["llm"], cfg["dit"]
            self.vit, self.siglip = Vit(v), Vit(s)
            self.proj1 = nn.Linear(v["hidden"] + s["hidden"], l["hidden"])
            self.proj2 = nn.Linear(l["hidden"], l["hidden"])
            self.embed = nn.Embedding(cfg["vocab"], l["hidden"])
            self.llm = nn.ModuleList([LlamaBlock(l) for _ in range(l["layers"])])
            self.llm_norm = RMSNorm(l["hidden"])
            self.cond = nn.Linear(l["hidden"], d["hidden"])
            self.t_embed = nn.Linear(256, d["hidden"])
            self.act_in = nn.Linear(cfg["action_dim"], d["hidden"])
            self.dit = nn.ModuleList([DitBlock(d) for _ in range(d["layers"])])
            self.act_out = nn.Linear(d["hidden"], cfg["action_dim"])

        def forward(self, img, text_ids, noise):
            vis = torch.cat((self.vit(img), self.siglip(img)), dim=-1)
            vis = self.proj2(F.gelu(self.proj1(vis), approximate="tanh"))
            x = torch.cat((vis, self.embed(text_ids)), dim=0)
            t, hd = x.shape[0], cfg["llm"]["hidden"] // cfg["llm"]["heads"]
            inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, device=x.device).float() / hd))
            ang = torch.outer(torch.arange(t, device=x.device).float(), inv)
            ang = torch.cat((ang, ang), dim=-1)[:, None, :]
            cos, sin = ang.cos().to(x.dtype), ang.sin().to(x.dtype)
            for b in self.llm:
                x = b(x, cos, sin)
            cog = self.cond(self.llm_norm(x)[-1:])  # cognition feature of the last token
            a = noise
            for step in range(cfg["denoise_steps"]):
                freq = torch.exp(-torch.arange(128, device=x.device).float() * (9.21 / 128)) * (1000.0 * step)
                temb = torch.cat((freq.sin(), freq.cos()))[None].to(x.dtype)
                c = cog + self.t_embed(temb)
                h = self.act_in(a)
                for b in self.dit:
                    h = b(h, c)
                a = a - 0.1 * self.act_out(h)
            return a

    torch.manual_seed(seed)
    with torch.device(device):
        model = Vla().to(torch.bfloat16)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, (nn.Linear, nn.Embedding, nn.Conv2d)):
                mod.weight.normal_(0.0, 0.02)
                if getattr(mod, "bias", None) is not None:
                    mod.bias.zero_()
    return model.eval()


def run_cogact(args):
    import contextlib

    import torch

    from vla_abft_estimate_b200.abft import AbftConfig, AbftInjector, AbftStatsCollector, CheapSumChecker

    cfg = COGACT
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    model = build_cogact(cfg, dev)
    g = torch.Generator(device=dev).manual_seed(3)
    img = torch.randn(1, 3, 224, 224, device=dev, generator=g).bfloat16()
    text = torch.randint(0, cfg["vocab"], (cfg["text_tokens"],), device=dev, generator=g)
    noise = torch.randn(cfg["action_tokens"], cfg["action_dim"], device=dev, generator=g).bfloat16()
    reps = max(min(args.steps, 10), 3)

    def timed(ctx_factory):
        times = []
        out = None
        with torch.inference_mode():
            for i in range(2 + reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                e0.record()
                with ctx_factory():
                    out = model(img, text, noise)
                e1.record()
                torch.cuda.synchronize()
                if i >= 2:
                    times.append(e0.elapsed_time(e1))
        return statistics.median(times), out

    stats_chk = AbftStatsCollector()
    cfg_chk = AbftConfig(enable=True, checker_backend="b200", detect_only=False)
    inj_chk = AbftInjector(cfg_chk, CheapSumChecker(cfg_chk), stats_chk, defer_reports=True)
    stats_off = AbftStatsCollector()
    cfg_off = AbftConfig(enable=True, check_enable=False, checker_backend="b200")
    inj_off = AbftInjector(cfg_off, CheapSumChecker(cfg_off), stats_off, defer_reports=True)
    t_torch, a_torch = timed(contextlib.nullcontext)
    t_off, _ = timed(lambda: inj_off)
    t_chk, a_chk = timed(lambda: inj_chk)
    summ = stats_chk.export_summary()

    stats_f = AbftStatsCollector()
    cfg_f = AbftConfig(enable=True, checker_backend="b200", detect_only=False, inject_fault=True,
                       inject_probability=0.02, inject_magnitude=4.0, seed=5)
    inj_f = AbftInjector(cfg_f, CheapSumChecker(cfg_f), stats_f, defer_reports=True)
    with torch.inference_mode(), inj_f:
        a_f = model(img, text, noise)
    torch.cuda.synchronize()
    fs = stats_f.export_summary()
    per_fwd = summ["abft"]["checks_total"] // (2 + reps)
    line = {
        "metric": "CogACT-style VLA forward latency (every linear ABFT-protected)",
        "value": t_chk, "unit": "ms", "n_gpus": 1, "steps": reps, "warmup": 2, "ms_per_step": t_chk,
        "higher_is_better": False, "scaling": "none", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random init N(0,0.02), random image, text ids and action noise)",
        "config": {"workload": "ViT-L/14 + SigLIP-So400m/14 (256 patches) -> MLP projector -> Llama-2-7B-shaped "
                               "decoder over 256 + 32 tokens -> DiT-B action head, 16 action tokens x 7, "
                               f"{cfg['denoise_steps']} denoising steps, batch 1", **{k: v for k, v in cfg.items()}},
        "ms": {"torch": t_torch, "b200_unchecked": t_off, "b200_abft": t_chk},
        "overhead_vs_torch_pct": 100.0 * (t_chk / t_torch - 1.0),
        "overhead_vs_unchecked_pct": 100.0 * (t_chk / t_off - 1.0),
        "checked_linears_per_forward": per_fwd,
        "skipped_unsupported_per_forward": summ["abft"]["faults"]["skipped_unsupported"] // (2 + reps),
        "clean_detections": summ["abft"]["faults"]["detected_total"],
        "fault_leg": {"injected": fs["fault_injection"]["injections_total"],
                      "detected_injections": fs["fault_injection"]["detected_injections_total"],
                      "faults": {k: v for k, v in fs["abft"]["faults"].items() if k != "located"},
                      "max_abs_action_diff_vs_clean": (a_f.float() - a_chk.float()).abs().max().item()},
        "actions_max_abs_diff_torch_vs_abft": (a_torch.float() - a_chk.float()).abs().max().item(),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.model == "cogact":
        run_cogact(args)
        return
    if args.model:
        run_model(args)
        return
    if args.sweep:
        sweep(args)
        return
    if args.bmm_sweep:
        bmm_sweep(args)
        return
    if args.profile_bmm:
        profile_bmm(args)
        return
    if args.profile_shape:
        profile_shape(args)
        return
    if args.tile_grid:
        tile_grid(args)
        return
    if args.profile_case:
        profile_case(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
