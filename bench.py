#!/usr/bin/env python3
"""Throughput of the fused checksum-protected GEMM on B200.

Workload (one step = one protected GEMM):
  C[M, N_r] = A[M, K] B_r[N_r, K]^T, bf16 in, fp32 accumulate, bf16 out,
  M = N_r = K = 8192 per GPU (--size), with per-tile weighted row checksums,
  detect + locate + correct in the kernel. A is replicated; B[N, K] with
  N = 8192 * n_gpus is split by columns across the ranks (weak scaling: at 8
  GPUs this is the sharded A[8192 x 8192] . B[8192 x 65536] configuration).
  The fault reports of every 16 consecutive steps are exchanged in one
  all-gather (NCCL); detection and correction need no exchange.

Printed: one JSON line (rank 0). value = whole-job TFLOP/s (2 M N K / step
time, max over ranks); roofline from CUDA-event timing of the fused kernel
alone; e2e through the public API with A and B_r copied from pinned host
memory every step and the gathered fault reports read back. On one GPU the
line also carries the other BASELINE metrics, measured in the same process:
config 1 (one 512x4096x4096 protected GEMM) and 16384^3, each against
cuBLAS and the unchecked kernel, and the Qwen2-7B prefill-512 tokens/s with
every linear protected (--no-extras skips them).

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
import functools
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
    ap.add_argument("--nvtx-enable", action="store_true",
                    help="--model qwen2-7b: NVTX ranges prefill_len_<n> / decode_len_<n> around the timed work, as "
                         "the reference driver marks them, and abft.<op> MxNxK around every hooked call")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the config-1, 16384^3 and Qwen2-7B prefill points of the default 1-GPU line")
    ap.add_argument("--sweep", action="store_true",
                    help="one JSON line per shape of the square sweep, the 512x4096x4096 case and the "
                         "Qwen2-7B layer GEMMs: checked / unchecked TFLOP/s and 1- and 4-fault outcomes")
    ap.add_argument("--dtype", choices=["bf16", "f16"], default="bf16",
                    help="operand type of --model qwen2-7b (the reference driver's --dtype) and --profile-case")
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
    """SM clock, power and clock-event reasons of this process's GPUs,
    polled about every millisecond by a background thread through NVML
    (read-only queries), with a time stamp per sample so that a summary can
    cover exactly a timed region. Falls back to ``nvidia-smi -lms`` when NVML
    is unavailable."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))
    SMI_FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids, period_ms=1.0):
        self.uuids = [u if u.lower().startswith("gpu-") else f"GPU-{u}" for u in uuids]
        self.period = period_ms * 1e-3
        self.samples = []  # (time.time(), sm_mhz, max_mhz, power_w, reasons bitmask or -1)
        self.source = None
        self.errors = 0
        self.first_error = None
        self._stop = threading.Event()
        self.thread = None
        self.proc = None

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            handles = [pynvml.nvmlDeviceGetHandleByUUID(u) for u in self.uuids]
            if not handles:
                raise RuntimeError("no device")
            self._nvml = pynvml
            self._handles = handles
            self._max = [pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM) for h in handles]
            self.source = f"nvml, {self.period * 1e3:.0f} ms"
            self.thread = threading.Thread(target=self._poll_nvml, daemon=True)
            self.thread.start()
            return
        except Exception:  # noqa: BLE001 - fall back to nvidia-smi
            pass
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms=25"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        self.source = "nvidia-smi, 25 ms"
        self.thread = threading.Thread(target=self._read_smi, daemon=True)
        self.thread.start()

    def _reasons(self, h):
        """Clock-event reason bits (newer drivers' name first), or None."""
        nv = self._nvml
        for fn in ("nvmlDeviceGetCurrentClocksEventReasons", "nvmlDeviceGetCurrentClocksThrottleReasons"):
            f = getattr(nv, fn, None)
            if f is None:
                continue
            try:
                return int(f(h))
            except Exception as e:  # noqa: BLE001
                self._note_error(f"{fn}: {e}")
        return None

    def _note_error(self, msg):
        self.errors += 1
        if self.first_error is None:
            self.first_error = msg

    def _poll_nvml(self):
        nv = self._nvml
        while not self._stop.is_set():
            t = time.time()
            for h, mx in zip(self._handles, self._max):
                try:
                    sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                except Exception as e:  # noqa: BLE001
                    self._note_error(f"clock: {e}")
                    continue
                try:
                    pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                except Exception:  # noqa: BLE001
                    pw = float("nan")
                rs = self._reasons(h)
                self.samples.append((t, sm, float(mx), pw, -1 if rs is None else rs))
            time.sleep(self.period)

    def _read_smi(self):
        wanted = {u.lower().replace("gpu-", "") for u in self.uuids}
        for line in self.proc.stdout:
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9 or (wanted and p[0].lower().replace("gpu-", "") not in wanted):
                continue
            try:
                bits = sum(m for (_, m), v in zip(self.REASONS[:4], p[5:9]) if v.lower() == "active")
                self.samples.append((time.time(), float(p[1]), float(p[2]), float(p[3]), bits))
            except ValueError:
                continue

    def stop(self):
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0, t1):
        """Median SM clock and the union of slowdown reasons over the samples
        taken in [t0, t1] (wall-clock seconds)."""
        rows = [s for s in self.samples if t0 <= s[0] <= t1]
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": len(rows), "window": "timed",
               "source": self.source, "window_s": round(t1 - t0, 4)}
        if self.errors:
            out["query_errors"] = self.errors
            out["first_error"] = self.first_error
        if not rows:
            out["samples_in_run"] = len(self.samples)
            return out
        out["sm_mhz"] = statistics.median(r[1] for r in rows)
        out["sm_max_mhz"] = max(r[2] for r in rows)
        known = [r for r in rows if r[4] >= 0]
        out["reasons"] = [name for name, bit in self.REASONS if any(r[4] & bit for r in known)]
        if len(known) < len(rows):
            out["reasons_unavailable_samples"] = len(rows) - len(known)
        out["power_w_max"] = max(r[3] for r in rows)
        return out


def timed_median(fn, iters, flush=None, sleep_cycles=100_000_000):
    """Median CUDA-event time (ms) of ``fn`` over ``iters`` launches after 3
    warm-up calls; ``flush`` (a tensor larger than L2) is overwritten before
    every launch, outside the timed interval. A device-side sleep first lets
    the host queue every launch ahead of the GPU, so no interval contains
    host launch latency."""
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    torch.cuda._sleep(sleep_cycles)
    pairs = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        pairs.append((e0, e1))
    torch.cuda.synchronize()
    ms = sorted(e0.elapsed_time(e1) for e0, e1 in pairs)
    return ms[len(ms) // 2]


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


def timed_interleaved(fns, iters, flush, sleep_cycles=100_000_000):
    """CUDA-event times (ms) of each of ``fns``, launched in rounds (fn 0,
    fn 1, ... then again) so that every variant sees the same clocks and
    power state; ``flush`` is overwritten before every launch. Returns one
    list per fn, in round order."""
    import torch

    for fn in fns:
        for _ in range(3):
            fn()
    torch.cuda.synchronize()
    torch.cuda._sleep(sleep_cycles)
    ev = [[] for _ in fns]
    for _ in range(iters):
        for i, fn in enumerate(fns):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            ev[i].append((e0, e1))
    torch.cuda.synchronize()
    return [[e0.elapsed_time(e1) for e0, e1 in pairs] for pairs in ev]


def timed_medians_interleaved(fns, iters, flush, sleep_cycles=100_000_000):
    """Median of each fn's times from ``timed_interleaved``."""
    return [statistics.median(ms) for ms in timed_interleaved(fns, iters, flush, sleep_cycles)]


def paired_overhead_pct(chk_ms, off_ms):
    """Median over rounds of checked / unchecked - 1, in percent: each ratio
    compares two launches of one round, so clock drift under the power cap
    between rounds cancels."""
    return 100.0 * (statistics.median(c / o for c, o in zip(chk_ms, off_ms)) - 1.0)


def gemm_point(m, n, k, iters, flush, seed=0, dtype="bf16"):
    """One BASELINE GEMM configuration on cuda:0: median kernel times (L2
    flushed before each launch, the variants interleaved) of cuBLAS, the
    fused kernel with checks off and on (weight checksums cached), and of
    the checked call that encodes the checksums itself (a fresh weight);
    then the BASELINE fault runs:
    clean, 1 and 4 faults of 2^8 max|C| at seeded distinct rows and columns
    (exact coordinates and corrections required). ``dtype`` "f16" runs the
    same on fp16 operands (cuBLAS fp16 beside it)."""
    import torch

    from vla_abft_estimate_b200 import _native as N
    from vla_abft_estimate_b200 import ops
    from vla_abft_estimate_b200.faults import seeded_fault_positions

    dev = torch.device("cuda", 0)
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(seed)
    a = (torch.randn(m, k, device=dev, generator=g) * k ** -0.5).to(tdt)
    w = (torch.randn(n, k, device=dev, generator=g) * k ** -0.5).to(tdt)
    out = torch.empty(m, n, device=dev, dtype=tdt)
    chk = N.MODE_DETECT | N.MODE_CORRECT
    tn_chk = ops.pick_tile_n(m, n, k, dev, chk)
    tn_off = ops.pick_tile_n(m, n, k, dev, N.MODE_OFF)
    cks = ops.encode_weight(w, tn_chk)
    rep = ops.ReportBuffer(64, dev)
    samples = timed_interleaved([
        lambda: torch.matmul(a, w.t(), out=out),
        lambda: ops.abft_gemm(a, w, mode=N.MODE_OFF, out=out, tile_n=tn_off),
        lambda: ops.abft_gemm(a, w, mode=chk, out=out, tile_n=tn_chk, checksums=cks, report=rep),
        lambda: ops.abft_gemm(a, w, mode=chk, out=out, tile_n=tn_chk, report=rep),
    ], iters, flush)
    t_cublas, t_off, t_chk, t_enc = (statistics.median(ms) for ms in samples)
    c0, r0 = ops.abft_gemm(a, w, mode=chk, tile_n=tn_chk, checksums=cks)
    r0 = r0.read()
    delta = 256.0 * c0.float().abs().max().item()
    faults_ok = {"clean_no_record": r0.n_faults == 0 and r0.status == 0}
    for count in (1, 4):
        pos = seeded_fault_positions(m, n, count, seed + count)
        c, r = ops.abft_gemm(a, w, mode=chk, tile_n=tn_chk, checksums=cks, inject=[(i, j, delta) for i, j in pos])
        r = r.read()
        err = (c.float() - c0.float()).abs().max().item() / max(c0.float().abs().max().item(), 1e-30)
        faults_ok[f"{count}_fault_located_corrected"] = (r.coords() == sorted(pos) and r.n_corrected == count
                                                          and err <= 1e-2)
    fl = 2.0 * m * n * k
    res = {"M": m, "N": n, "K": k, "dtype": dtype, "tile_n": {"unchecked": tn_off, "checked": tn_chk},
           "cublas_tflops": fl / t_cublas / 1e9, "unchecked_tflops": fl / t_off / 1e9,
           "checked_tflops": fl / t_chk / 1e9, "overhead_pct": paired_overhead_pct(samples[2], samples[1]),
           "overhead_of_medians_pct": 100.0 * (t_chk / t_off - 1.0),
           "overhead_method": f"median over {iters} rounds of checked / unchecked, each round's launches back to back",
           "checked_vs_cublas": t_cublas / t_chk,
           "checked_encode_included_tflops": fl / t_enc / 1e9,
           "overhead_encode_included_pct": paired_overhead_pct(samples[3], samples[1]),
           "us": {"cublas": t_cublas * 1e3, "unchecked": t_off * 1e3, "checked": t_chk * 1e3,
                  "checked_encode_included": t_enc * 1e3},
           "fault_check": faults_ok}
    del a, w, out, cks, c0
    return res


def _nvtx_range(enabled, name):
    """An NVTX range when ``enabled`` (the reference driver's --nvtx-enable,
    pytorch/qwen_abft_benchmark.py:120-127), else nothing."""
    import contextlib

    import torch

    if not enabled:
        return contextlib.nullcontext()

    @contextlib.contextmanager
    def rng():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()

    return rng()


def qwen_prefill_point(reps, warmup, decode_steps=0, cpu_seconds=0.0, dtype="bf16", nvtx=False):
    """a Qwen2-7B-shaped decoder prefill of 512 tokens
    (batch 1, random init N(0, 0.02), random token ids) with every nn.Linear
    through AbftInjector's fused path (reports deferred to one read per
    forward), against plain torch (cuBLAS) and the same kernel with checks
    off. Times are medians over ``reps`` forwards: wall time around the
    forward (host work included), and device time with the host queued
    ahead behind a device sleep. Then one forward with the injector's
    random faults (probability 0.05 per linear, +1.0 on the fp32
    accumulator) and, with ``decode_steps``, single-token decode steps after
    the prefill. ``dtype`` "f16" builds the model in fp16 (the reference
    driver's --dtype float16)."""
    import contextlib

    import torch

    from vla_abft_estimate_b200.abft import AbftConfig, AbftInjector, AbftStatsCollector, CheapSumChecker

    cfg = QWEN2_7B
    tokens = 512
    dev = torch.device("cuda", 0)
    model = build_qwen2(cfg, dev, dtype=torch.float16 if dtype == "f16" else torch.bfloat16)
    ids = torch.randint(0, cfg["vocab"], (tokens,), device=dev, generator=torch.Generator(device=dev).manual_seed(7))

    def timed_forward(ctx_factory):
        times, gpu_times = [], []
        out = None
        with torch.inference_mode():
            for i in range(warmup + reps):
                ctx = ctx_factory()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                e0.record()
                with ctx, _nvtx_range(nvtx, f"prefill_len_{tokens}"):
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
                if i >= warmup:
                    times.append(e0.elapsed_time(e1))
                    gpu_times.append(g0.elapsed_time(g1))
        return statistics.median(times), out, statistics.median(gpu_times)

    # one injector per leg, reused across repetitions (its weight checksum
    # cache is what a serving process keeps)
    stats_chk = AbftStatsCollector()
    cfg_chk = AbftConfig(enable=True, checker_backend="b200", detect_only=False, nvtx=nvtx)
    inj_chk = AbftInjector(cfg_chk, CheapSumChecker(cfg_chk), stats_chk, defer_reports=True)
    stats_off = AbftStatsCollector()
    cfg_off = AbftConfig(enable=True, check_enable=False, checker_backend="b200", nvtx=nvtx)
    inj_off = AbftInjector(cfg_off, CheapSumChecker(cfg_off), stats_off, defer_reports=True)

    t_torch, ref_logits, g_torch = timed_forward(contextlib.nullcontext)
    t_off, _, g_off = timed_forward(lambda: inj_off)
    t_chk, chk_logits, g_chk = timed_forward(lambda: inj_chk)
    summ = stats_chk.export_summary()
    forwards = 2 * (warmup + reps)

    stats_f = AbftStatsCollector()
    cfg_f = AbftConfig(enable=True, checker_backend="b200", detect_only=False, inject_fault=True,
                       inject_probability=0.05, inject_magnitude=1.0, seed=11)
    inj_f = AbftInjector(cfg_f, CheapSumChecker(cfg_f), stats_f, defer_reports=True)
    with torch.inference_mode(), inj_f:
        f_logits = model(ids)
    torch.cuda.synchronize()
    fs = stats_f.export_summary()

    res = {
        "tokens_per_s": {"torch": tokens / (t_torch * 1e-3), "unchecked": tokens / (t_off * 1e-3),
                         "abft": tokens / (t_chk * 1e-3)},
        "ms": {"torch": t_torch, "unchecked": t_off, "abft": t_chk},
        "device_ms": {"torch": g_torch, "unchecked": g_off, "abft": g_chk},
        "overhead_vs_torch_pct": 100.0 * (t_chk / t_torch - 1.0),
        "overhead_vs_unchecked_pct": 100.0 * (t_chk / t_off - 1.0),
        "checked_linears_per_forward": summ["abft"]["checks_total"] // forwards,
        "clean_detections": summ["abft"]["faults"]["detected_total"],
        "fault_leg": {"injected": fs["fault_injection"]["injections_total"],
                      "detected_injections": fs["fault_injection"]["detected_injections_total"],
                      "faults": {k: v for k, v in fs["abft"]["faults"].items() if k != "located"},
                      "max_abs_logit_diff_vs_clean": (f_logits.float() - chk_logits.float()).abs().max().item(),
                      "max_abs_logit": chk_logits.float().abs().max().item(),
                      "note": "+1.0 on the fp32 accumulator; a fault below the bound tau*sqrt(K)*max|C_row| "
                              "of its row is by design not flagged"},
        "logits_max_abs_diff_torch_vs_abft": (ref_logits.float() - chk_logits.float()).abs().max().item(),
        "reps": reps, "warmup": warmup,
        "reference_published": {"tokens_per_s_no_abft": 7217, "tokens_per_s_abft_python": 5909,
                                "source": "pytorch/baseline_7b_prefill512.json:44, "
                                          "pytorch/abft_7b_prefill512_nsys.json:44 (GPU unrecorded)"},
    }

    if decode_steps:
        def timed_decode(ctx_factory):
            caches = model.new_caches(tokens + decode_steps + 8)
            with torch.inference_mode():
                with ctx_factory():
                    model(ids, caches, 0)
                nxt = ids[-1:].clone()
                for i in range(4):
                    with ctx_factory():
                        model(nxt, caches, tokens + i)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                with _nvtx_range(nvtx, f"decode_len_{decode_steps}"):
                    for i in range(decode_steps):
                        with ctx_factory():
                            model(nxt, caches, tokens + 4 + i)
                e1.record()
                torch.cuda.synchronize()
            return e0.elapsed_time(e1) / decode_steps

        d_torch = timed_decode(contextlib.nullcontext)
        d_off = timed_decode(lambda: inj_off)
        d_chk = timed_decode(lambda: inj_chk)
        res["decode_ms_per_token"] = {"torch": d_torch, "unchecked": d_off, "abft": d_chk,
                                      "abft_overhead_vs_torch_pct": 100.0 * (d_chk / d_torch - 1.0),
                                      "note": "after a 512-token prefill into a KV cache; every linear at M = 1 "
                                              "(operands swapped: weight on the MMA's 128-row side)"}

        def graph_decode(inj, record="sync"):
            """One decode step captured as a CUDA graph (position on the
            device, attention over the whole cache, masked), replayed
            ``decode_steps`` times. With an injector, ``record`` says when
            each replay's reports are read and recorded: "sync" before the
            next replay, "overlap" one replay late from pinned copies (the
            host work runs under the next replay), "end" only the last
            replay's, after the timed loop (device cost alone)."""
            t_max = tokens + decode_steps + 8
            caches = model.new_caches(t_max)
            pos = torch.full((), tokens, dtype=torch.long, device=dev)
            nxt = ids[-1:].clone()
            ctx = inj if inj is not None else contextlib.nullcontext()
            with torch.inference_mode(), ctx:
                model(ids, caches, 0)
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s):
                    for _ in range(3):
                        model(nxt, caches, pos)
                torch.cuda.current_stream().wait_stream(s)
                g = torch.cuda.CUDAGraph()
                cap = inj.capture(g) if inj is not None else torch.cuda.graph(g)
                with cap as checks:
                    model(nxt, caches, pos)
                    pos.add_(1)
                pos.fill_(tokens)
                per_step = inj is not None and record != "end"
                for _ in range(3):
                    g.replay()
                    if per_step:
                        checks.record(overlap=record == "overlap")
                if per_step:
                    checks.finish()
                pos.fill_(tokens)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(decode_steps):
                    g.replay()
                    if per_step:
                        checks.record(overlap=record == "overlap")
                e1.record()
                if per_step:
                    checks.finish()
                elif inj is not None:
                    checks.record()
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / decode_steps
                n_checked = len(checks) if inj is not None else 0
            del g
            return ms, n_checked

        gd_torch, _ = graph_decode(None)
        gd_off, _ = graph_decode(inj_off)
        before = stats_chk.export_summary()["abft"]["faults"]["detected_total"]
        gd_chk, n_checked = graph_decode(inj_chk)
        gd_ovl, _ = graph_decode(inj_chk, "overlap")
        gd_end, _ = graph_decode(inj_chk, "end")
        res["decode_graph_ms_per_token"] = {
            "torch": gd_torch, "unchecked": gd_off, "abft": gd_chk, "abft_overlapped_reports": gd_ovl,
            "abft_reports_after_last_step": gd_end,
            "abft_overhead_vs_torch_pct": 100.0 * (gd_chk / gd_torch - 1.0),
            "abft_overlapped_overhead_vs_torch_pct": 100.0 * (gd_ovl / gd_torch - 1.0),
            "checked_linears_per_step": n_checked,
            "clean_detections": stats_chk.export_summary()["abft"]["faults"]["detected_total"] - before,
            "note": "one decode step per CUDA graph replay (fixed shapes: position on the device, attention over "
                    f"the {tokens + decode_steps + 8}-slot cache, masked), the same for all three legs; "
                    "abft: every step's reports read and recorded before the next replay; abft_overlapped_reports: "
                    "recorded one step late from pinned copies queued behind each replay (record(overlap=True)), "
                    "the host work under the next replay; abft_reports_after_last_step: device cost alone"}
    if cpu_seconds > 0:
        res["cpu_baseline"] = cpu_model_baseline(cfg, tokens, cpu_seconds)
    linear_flops = 0.0
    h, it, nh, nkv, hd, V = (cfg["hidden"], cfg["inter"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"],
                             cfg["vocab"])
    for k, n in [(h, (nh + 2 * nkv) * hd), (nh * hd, h), (h, 2 * it), (it, h)]:
        linear_flops += 2.0 * tokens * k * n * cfg["layers"]
    linear_flops += 2.0 * tokens * h * V
    res["linear_tflops_abft"] = linear_flops / (t_chk * 1e-3) / 1e12
    del model
    torch.cuda.empty_cache()
    return res


EXCHANGE_EVERY = 16  # GEMMs whose fault reports one all-gather exchanges


def run_ours(args):
    import torch
    import torch.distributed as dist

    from vla_abft_estimate_b200 import _native as N
    from vla_abft_estimate_b200 import ops
    from vla_abft_estimate_b200.faults import seeded_fault_positions
    from vla_abft_estimate_b200.sharded import ShardedAbftGemm, shard_bounds

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
    gemm = ShardedAbftGemm(w, c0, mode=N.MODE_DETECT | N.MODE_CORRECT, exchange_every=EXCHANGE_EVERY)
    off = ShardedAbftGemm(w, c0, mode=N.MODE_OFF)
    tile_n, _ = gemm._checksums_for(s)
    tile_m = ops.pick_tile_m(s, n_r, s, tile_n, dev)

    # fault detection outside the timed region: clean, then 1 and 4 seeded
    # faults of 2^8 max|C| per rank (distinct rows and columns); every
    # rank's faults must come back located, corrected, in global columns
    gemm(a, out=out, gather=True)
    clean_ok = gemm.global_report().n_faults == 0
    delta = 256.0 * out.float().abs().max().item()
    faulty = torch.empty_like(out)
    detect = {}
    for count in (1, 4):
        mine = seeded_fault_positions(s, n_r, count, 100 * count + rank)
        gemm(a, out=faulty, inject=[(i, j, delta) for i, j in mine], gather=True)
        grep = gemm.global_report()
        want = []
        for r in range(world):
            r0, r1 = shard_bounds(n_total, world, r)
            want += [(i, j + r0) for i, j in seeded_fault_positions(s, r1 - r0, count, 100 * count + r)]
        err = (faulty.float() - out.float()).abs().max().item() / max(out.float().abs().max().item(), 1e-30)
        detect[count] = grep.coords() == sorted(want) and grep.n_corrected == world * count and err <= 1e-2
    del faulty

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

    # Timed steps: one fused GEMM each; the reports of EXCHANGE_EVERY
    # consecutive GEMMs are all-gathered in one collective (the ring's last,
    # partial batch inside the timed region too).
    for _ in range(max(args.warmup, 3)):
        gemm(a, out=out)
    gemm.exchange()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_begin, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # untimed GPU spin: the host queues the first steps ahead of the GPU
    torch.cuda._sleep(50_000_000)
    t_begin.record()
    for i in range(args.steps):
        starts[i].record()
        gemm(a, out=out, gather=False)
        kends[i].record()
        if (i + 1) % EXCHANGE_EVERY == 0 or i + 1 == args.steps:
            gemm.exchange()
    t_end.record()
    # poll with sleeps (not a blocking synchronize) so that the clock
    # sampler's thread gets the interpreter while the device works
    while not t_end.query():
        time.sleep(2e-4)
    wall1 = time.time()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    step_ms = t_begin.elapsed_time(t_end) / args.steps
    kernel_ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, kends)) / args.steps
    clean_timed = all(r.n_faults == 0 for r in gemm.global_reports())
    wall0 = wall1 - step_ms * args.steps * 1e-3  # the device-timed region, on the wall clock

    # overhead: the same kernel with checksums compiled out, launches
    # interleaved with checked ones so that both see the same clocks
    for _ in range(3):
        off(a, out=out, gather=False)
    torch.cuda.synchronize()
    n_pair = min(args.steps, 100)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n_pair)]
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
    # its A and B_r from pinned host memory, encodes B_r's checksums, runs
    # the GEMM, exchanges the step's fault reports and reads them back. Two
    # device buffer sets: step i+1's copies run on a copy stream while step
    # i's GEMM runs (each copy waits until the GEMM that last read its
    # buffers has finished).
    a_h = a.cpu().pin_memory()
    w_h = w.cpu().pin_memory()
    bufs = [(torch.empty_like(a), torch.empty_like(w)) for _ in range(2)]
    e2e_gemms = [ShardedAbftGemm(wd, c0, mode=N.MODE_DETECT | N.MODE_CORRECT) for _, wd in bufs]
    rep_h = [torch.empty(e2e_gemms[0].gathered.shape, dtype=torch.uint8).pin_memory() for _ in range(2)]
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
    del bufs, e2e_gemms

    if sampler is not None:
        sampler.stop()

    # max over ranks
    vals = torch.tensor([step_ms, kernel_ms, off_ms, e2e_ms, chk_ms], device=dev, dtype=torch.float64)
    oks = torch.tensor([int(detect[1]), int(detect[4]), int(clean_ok and clean_timed)], device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        dist.all_reduce(oks, op=dist.ReduceOp.MIN)
    step_ms, kernel_ms, off_ms, e2e_ms, chk_ms = [float(x) for x in vals.cpu()]
    one_ok, four_ok, clean_all = (bool(x) for x in oks.cpu())

    extras = {}
    if world == 1 and rank == 0 and not args.no_extras:
        # The other BASELINE metrics, measured in the same process: config 1
        # (one 512x4096x4096 protected GEMM), the largest square shape, and
        # the Qwen2-7B prefill-512 tokens/s with every linear protected (and
        # its decode steps, eager and as one CUDA graph per step); plus the
        # headline shape on fp16 operands.
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        it = max(args.steps, 10)
        extras["config1_512x4096x4096"] = gemm_point(512, 4096, 4096, it, flush)
        extras["square_16384"] = gemm_point(16384, 16384, 16384, min(it, 16), flush)
        extras["fp16_8192"] = gemm_point(8192, 8192, 8192, it, flush, dtype="f16")
        del flush
        torch.cuda.empty_cache()
        extras["qwen2_7b_prefill512"] = qwen_prefill_point(reps=5, warmup=2, decode_steps=16)

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
            "fault_check": {"clean_no_false_positive": clean_all, "injected_1_located_corrected": one_ok,
                            "injected_4_located_corrected": four_ok,
                            "per_rank_faults": "1 and 4 of 2^8 max|C|, distinct rows and columns, every rank"},
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
                       "mode": "detect+locate+correct, weight checksums cached",
                       "parallelism": f"dp{world} (column shards)",
                       "report_exchange": f"one all-gather per {EXCHANGE_EVERY} GEMMs",
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
                    "d2h_bytes_per_step": int(rep_h[0].numel()) * world,
                    "note": "per step: A and B_r from pinned host memory + checksum encode + fused GEMM + report "
                            "gather + D2H; the next step's copies overlap this step's GEMM (two buffer sets)"},
            "gpu_launches": args.steps,
            "clocks": sampler.summary(wall0, wall1) if sampler is not None else None,
            "unchecked_tflops": flops_job / (off_ms * 1e-3) / 1e12,
            "overhead_pct": 100.0 * (chk_ms / off_ms - 1.0),
            "overhead_method": f"{n_pair} checked and {n_pair} unchecked launches interleaved",
            "encode_ms": enc_ms,
            "checked_encode_included_tflops": flops_job / ((chk_ms + enc_ms) * 1e-3) / 1e12,
            "overhead_encode_included_pct": 100.0 * ((chk_ms + enc_ms) / off_ms - 1.0),
            "step_minus_kernel_us": (step_ms - kernel_ms) * 1e3,
            **extras,
        }
        print(json.dumps(line), flush=True)

    if world > 1:
        dist.destroy_process_group()


def profile_case(args):
    """Two rounds of the fused GEMM at --size (operands of --dtype): the
    capture target of ncu."""
    import torch

    from vla_abft_estimate_b200 import _native as N
    from vla_abft_estimate_b200 import ops

    dev = torch.device("cuda", 0)
    s = args.size
    tdt = torch.float16 if args.dtype == "f16" else torch.bfloat16
    a = (torch.randn(s, s, device=dev) * s ** -0.5).to(tdt)
    w = (torch.randn(s, s, device=dev) * s ** -0.5).to(tdt)
    out = torch.empty(s, s, device=dev, dtype=tdt)
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
    print(json.dumps({"profile_case": args.profile_case, "size": s, "dtype": args.dtype,
                      "faults": rep.read().n_faults}))


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
            return timed_median(fn, iters, flush, 200_000_000)

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
    shapes = ((128, 128), (256, 128), (128, 256), (256, 256))  # (tile_n, tile_m)

    for name, m, n, k in TILE_GRID_SHAPES:
        a = (torch.randn(m, k, device=dev) * k ** -0.5).bfloat16()
        w = (torch.randn(n, k, device=dev) * k ** -0.5).bfloat16()
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        rep = ops.ReportBuffer(64, dev)
        row = {"shape": name, "M": m, "N": n, "K": k}
        for mode, tag in ((N.MODE_OFF, "off"), (N.MODE_DETECT | N.MODE_CORRECT, "checked")):
            tn = ops.pick_tile_n(m, n, k, dev, mode)
            tm = ops.pick_tile_m(m, n, k, tn, dev, mode)
            # the tile shapes interleaved round by round: each sees the same clocks
            cks = {ctn: (ops.encode_weight(w, ctn) if mode else None) for ctn in (128, 256)}
            fns = [functools.partial(ops.abft_gemm, a, w, mode=mode, out=out, tile_n=ctn, tile_m=ctm, swap_ab=1,
                                     checksums=cks[ctn], report=rep if mode else None) for ctn, ctm in shapes]
            ts = timed_medians_interleaved(fns, iters, flush)
            us = {f"{ctm}x{ctn}": round(t * 1e3, 2) for (ctn, ctm), t in zip(shapes, ts)}
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
        return timed_median(fn, iters, flush, 200_000_000)

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
from vla_abft_estimate_b200.workloads import COGACT, QWEN2_7B, build_cogact, build_qwen2  # noqa: E402
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
    """``--model qwen2-7b``: the prefill point of the default line, with
    decode steps and the CPU reference flow, as its own JSON line."""
    import torch

    torch.cuda.set_device(0)
    reps = max(args.steps, 3) if args.steps < 300 else 10
    warmup = max(args.warmup, 2)
    res = qwen_prefill_point(reps, warmup, decode_steps=32, cpu_seconds=0.0 if args.no_cpu_baseline else 20.0,
                             dtype=args.dtype, nvtx=args.nvtx_enable)
    cfg = QWEN2_7B
    line = {
        "metric": "Qwen2-7B prefill-512 tokens/s (every linear ABFT-protected)",
        "value": res["tokens_per_s"]["abft"], "unit": "tokens/s", "n_gpus": 1, "steps": reps,
        "warmup": warmup, "ms_per_step": res["ms"]["abft"], "higher_is_better": True, "scaling": "none",
        "vs_baseline": None, "dtype": args.dtype, "data": "synthetic (random init N(0,0.02), random token ids)",
        "config": {"workload": "Qwen2-7B-shaped decoder prefill, batch 1, 512 tokens", **cfg,
                   "fused_shapes": "qkv 3584->4608 (bias), o 3584->3584, gate_up 3584->37888, down 18944->3584, "
                                   "lm_head 3584->152064",
                   "abft": "b200 backend: one fused GEMM + row-checksum check + correct per linear, "
                           "reports deferred to one read per forward"},
        **res,
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------- VLA (CogACT-style)
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

    def graph_timed(inj):
        """The whole forward captured as one CUDA graph (through the
        injector's capture() when given) and replayed; with an injector the
        replay's reports are read and recorded inside the timed region, as
        the eager leg's flush is."""
        ctx = inj if inj is not None else contextlib.nullcontext()
        times = []
        with torch.inference_mode(), ctx:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for _ in range(2):
                    model(img, text, noise)
            torch.cuda.current_stream().wait_stream(s)
            graph = torch.cuda.CUDAGraph()
            cap = inj.capture(graph) if inj is not None else torch.cuda.graph(graph)
            with cap as checks:
                out = model(img, text, noise)
            for i in range(2 + reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                e0.record()
                graph.replay()
                if inj is not None:
                    checks.record()
                e1.record()
                torch.cuda.synchronize()
                if i >= 2:
                    times.append(e0.elapsed_time(e1))
            n_checked = len(checks) if inj is not None else 0
            out = out.clone()
        del graph
        return statistics.median(times), out, n_checked

    before = summ["abft"]["faults"]["detected_total"]
    gt_torch, ga_torch, _ = graph_timed(None)
    gt_off, _, _ = graph_timed(inj_off)
    gt_chk, ga_chk, g_checked = graph_timed(inj_chk)
    graph_leg = {
        "ms": {"torch": gt_torch, "b200_unchecked": gt_off, "b200_abft": gt_chk},
        "overhead_vs_torch_pct": 100.0 * (gt_chk / gt_torch - 1.0),
        "overhead_vs_unchecked_pct": 100.0 * (gt_chk / gt_off - 1.0),
        "checked_calls_per_forward": g_checked,
        "clean_detections": stats_chk.export_summary()["abft"]["faults"]["detected_total"] - before,
        "actions_max_abs_diff_graph_vs_eager_abft": (ga_chk.float() - a_chk.float()).abs().max().item(),
        "actions_max_abs_diff_graph_torch_vs_graph_abft": (ga_torch.float() - ga_chk.float()).abs().max().item(),
        "note": "the whole forward (10 denoising steps included) as one CUDA graph per leg; the ABFT leg reads "
                "and records the replay's reports inside the timed region"}

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
        "cuda_graph": graph_leg,
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
