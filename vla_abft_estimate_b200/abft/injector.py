"""AbftInjector: the operator hook of pytorch/abft/injector.py on libabft_b200.

Inside ``with AbftInjector(cfg, checker, stats):`` the module attributes
``F.linear``, ``torch.matmul`` and ``torch.bmm`` are replaced by wrappers, as
in the reference (injector.py:31-51), and restored on exit.

* ``F.linear`` with ``checker_backend="b200"`` and ``fused_linear`` replaces
  "torch GEMM, then check" by one call of the fused kernel
  (``abft_gemm``, bf16 or fp16 operands): the GEMM, its per-tile weighted
  row checksums and the compare run in one launch, a drawn fault is added
  to the fp32 accumulator before the compare, and with
  ``detect_only=False`` located faults are corrected before the store.
* ``torch.bmm`` and ``torch.matmul`` with a 2-D right operand, with
  ``fused_matmul``, run the same way as one batched launch; a bmm records
  one check per batch, as the reference's per-batch loop does
  (injector.py:176-187). ``torch.matmul`` with a batched right operand is
  unchecked in the reference (its ``b_2d`` is None, checkers.py:145-149);
  ``check_batched_matmul`` checks it per batch.
* A linear with K or N not a multiple of 8 (the library reads rows in
  16-byte pieces; e.g. a VLA's 7-wide action projections) runs the same
  fused kernel on zero-padded copies of its operands.
* Other backends, operands the library cannot take (CPU, fp32, mixed
  types) and
  calls that need autograd follow the reference flow: run the op, maybe
  perturb one output element, then ``checker.check`` on the flattened
  operands (injector.py:152-187).

The random stream is the reference's: one ``random.Random(cfg.seed)`` per
injector, consumed in the same order -- the injection coin and index after
the op (:58-75), then the sampling coin inside the check gate (:53-56,
:77-99) -- so a seed selects the same faults on both implementations.

Reports of fused calls can be deferred (``defer_reports=True``): the fault
report stays on the device and is read at ``flush()`` (called on exit)
instead of forcing a device->host sync per GEMM like the reference (:103).

``capture(graph)`` captures a forward's calls, checks included, in a CUDA
graph; the returned ``CapturedChecks`` records each replay's reports.
"""
from __future__ import annotations

import random
import warnings
import weakref
from contextlib import AbstractContextManager
from typing import Any, Callable, List, Optional, Tuple

import numpy as np
import torch
import torch.nn.functional as F

from .. import _native as N
from .. import ops
from .checkers import AbftChecker, OpMeta, UnsupportedOperand, flatten_to_2d_for_mm
from .config import AbftConfig
from .stats import AbftStatsCollector, CheckResult, CleanChecks


def _shape_key(a2: torch.Tensor, b2: torch.Tensor, c2: torch.Tensor) -> str:
    return f"A{tuple(a2.shape)}_B{tuple(b2.shape)}_C{tuple(c2.shape)}"


# What result_from_report gives for any report with n_faults == 0.
_CLEAN_RESULT = CheckResult(ok=True, abs_err=0.0, rel_err=0.0, abft_corner=0.0, sum_c=0.0)


def result_from_report(rep: N.FaultReport) -> CheckResult:
    """CheckResult of a fused-linear report.

    ok: no checksum mismatch. abs_err: the largest |row-sum residual| of the
    recorded faults; rel_err: the largest residual / bound ratio (> 1 for a
    detected fault). abft_corner / sum_c stay 0: the fused check compares
    per-tile row checksums, not the scalar corner.
    """
    abs_err = max((abs(r.residual) for r in rep.records), default=0.0)
    rel_err = max((abs(r.residual) / r.threshold if r.threshold > 0 else float("inf") for r in rep.records),
                  default=0.0)
    located = tuple((r.row, r.col) for r in rep.records if r.located)
    return CheckResult(ok=rep.n_faults == 0, abs_err=float(abs_err), rel_err=float(rel_err), abft_corner=0.0,
                       sum_c=0.0, n_faults=int(rep.n_faults), n_located=int(rep.n_located),
                       n_corrected=int(rep.n_corrected), located=located)


class WeightChecksumCache:
    """Per-weight checksum blocks (``ops.encode_weight``), reused across calls.

    The reference recomputes ``b_2d.sum(dim=1)`` on every call
    (pytorch/abft/checkers.py:119); this cache encodes a weight once. An
    entry is found by (address, shape, strides, tile width, device) and is
    used only while it still describes the same memory and contents:

    * it holds a weak reference to the weight's storage (torch keeps one
      storage object per allocation, shared by every view of it). When the
      weight is freed the entry is dropped, so a new tensor that the
      allocator places at the same address is encoded afresh instead of
      inheriting another tensor's checksums;
    * it records the tensor's version counter (shared with its views),
      which every in-place op through them bumps (``copy_`` under
      ``no_grad``, optimizer steps), so such an update re-encodes.

    Writes that bypass the version counter (``weight.data.copy_(...)``,
    in-place writes to a weight created under ``inference_mode``, which has
    no counter, writes through another framework or a raw pointer) cannot
    be seen here;
    call ``invalidate(weight)`` (or ``clear()``) after them. If that is
    forgotten, the kernel still does not corrupt the output: the stale
    checksums make most rows of a slab mismatch, which the kernel reports
    as ``STATUS_SUSPECT`` without correcting anything, and the injector
    then clears this cache.
    """

    def __init__(self, max_entries: int = 4096):
        self.max_entries = max_entries
        self._d: dict = {}

    @staticmethod
    def _key(weight: torch.Tensor, tile_n: int) -> tuple:
        return (weight.data_ptr(), tuple(weight.shape), weight.stride(), tile_n, weight.get_device(), weight.dtype)

    @staticmethod
    def _version(weight: torch.Tensor) -> int:
        # tensors made under inference_mode carry no version counter
        return -1 if weight.is_inference() else weight._version

    def get(self, weight: torch.Tensor, tile_n: int) -> torch.Tensor:
        key = self._key(weight, tile_n)
        storage = weight.untyped_storage()
        version = self._version(weight)
        e = self._d.get(key)
        if e is not None and e[0]() is storage and e[1] == version:
            return e[2]
        if e is None and len(self._d) >= self.max_entries:
            self._d.pop(next(iter(self._d)))
        v = ops.encode_weight(weight, tile_n)
        d = self._d

        def _drop(ref, key=key, d=d):
            # the storage is gone: forget its checksums (unless a newer
            # entry for a new tensor at that address replaced this one)
            cur = d.get(key)
            if cur is not None and cur[0] is ref:
                d.pop(key, None)

        self._d[key] = (weakref.ref(storage, _drop), version, v)
        return v

    def invalidate(self, weight: torch.Tensor) -> None:
        """Forget every entry of ``weight``'s address and shape (after a
        write the version counter does not see, e.g. ``.data.copy_``)."""
        ptr, shape, dev = weight.data_ptr(), tuple(weight.shape), weight.get_device()
        for key in [k for k in list(self._d) if k[0] == ptr and k[1] == shape and k[4] == dev]:
            self._d.pop(key, None)

    def __len__(self) -> int:
        return len(self._d)

    def clear(self) -> None:
        self._d.clear()


class _Slot:
    """A report slot of an arena chunk: what the fused call needs of a
    ReportBuffer (its capacity and device address), without a tensor view."""

    __slots__ = ("capacity", "ptr")

    def __init__(self, capacity: int, ptr: int):
        self.capacity = capacity
        self.ptr = ptr

    def data_ptr(self) -> int:
        return self.ptr


class _ReportArena:
    """Device slots for the reports of deferred fused linears.

    Each fused call writes its report into the next slot (the kernel resets
    the header on the call's stream); ``drain()`` copies every used slot of a
    chunk to the host in one transfer. Chunks are added when one fills.
    """

    def __init__(self, capacity: int, device: torch.device, slots: int = 256):
        self.capacity = capacity
        self.device = device
        self.slot_bytes = (int(N.lib().abft_report_bytes(capacity)) + 255) // 256 * 256
        self.slots = slots
        self.chunks: List[torch.Tensor] = []
        self.used = 0  # slots taken in the last chunk
        self.suspect = False  # a drained report had STATUS_SUSPECT (stale checksums?)

    def take(self) -> "_Slot":
        if not self.chunks or self.used == self.slots:
            self.chunks.append(torch.empty(self.slots * self.slot_bytes, dtype=torch.uint8, device=self.device))
            self.base = self.chunks[-1].data_ptr()
            self.used = 0
        ptr = self.base + self.used * self.slot_bytes
        self.used += 1
        return _Slot(self.capacity, ptr)

    def drain(self) -> List[CheckResult]:
        """``read()``, then the slots are free for the next forward."""
        results = self.read()
        # keep the first chunk for the next forward
        self.chunks = self.chunks[:1]
        self.base = self.chunks[0].data_ptr() if self.chunks else 0
        self.used = 0
        return results

    def used_views(self) -> List[torch.Tensor]:
        """The used bytes of each chunk (device tensors), in order."""
        return [chunk[: (self.slots if i < len(self.chunks) - 1 else self.used) * self.slot_bytes]
                for i, chunk in enumerate(self.chunks)]

    def read(self, host_chunks: Optional[List[np.ndarray]] = None) -> List[CheckResult]:
        """The CheckResult of every used slot, in order (from ``host_chunks``,
        host copies of ``used_views()``, when given). A report without
        faults always gives the same clean result, so only the slots whose
        fault count (header word 1) is non-zero are parsed."""
        results: List[CheckResult] = []
        for i, view in enumerate(self.used_views()):
            n = view.numel() // self.slot_bytes
            host = (view.cpu().numpy() if host_chunks is None else host_chunks[i]).reshape(n, self.slot_bytes)
            n_faults = host[:, 4:8].copy().view(np.uint32)[:, 0]
            for j in range(n):
                if n_faults[j] == 0:
                    results.append(_CLEAN_RESULT)
                    continue
                rep = N.FaultReport.from_bytes(host[j].tobytes())
                self.suspect |= rep.suspect
                results.append(result_from_report(rep))
        return results


class _DeferredCheck:
    """A checker call queued on the device (report buffer + the checker that
    turns the read report into a CheckResult), recorded at flush."""

    __slots__ = ("report", "checker")

    def __init__(self, report, checker):
        self.report = report
        self.checker = checker


class AbftInjector(AbstractContextManager):
    def __init__(self, cfg: AbftConfig, checker: AbftChecker, stats: AbftStatsCollector,
                 defer_reports: bool = False):
        self.cfg = cfg
        self.checker = checker
        self.stats = stats
        self.rng = random.Random(cfg.seed)
        self.defer_reports = defer_reports
        self.checksums = WeightChecksumCache()

        self._orig_linear: Optional[Callable[..., torch.Tensor]] = None
        self._orig_matmul: Optional[Callable[..., torch.Tensor]] = None
        self._orig_bmm: Optional[Callable[..., torch.Tensor]] = None
        self._dump_done: bool = False
        # deferred records: (device, op, phase, shape key, injected, batched)
        # with batched = None (next report of the device's arena),
        # (report buffer, batches, rows per batch, gates), or a _DeferredCheck
        # (a checker call whose report is read at flush)
        self._pending: List[Tuple[int, str, str, Any, bool, Any]] = []
        self._arenas: dict = {}
        self._tile_n: dict = {}
        # checksum blocks read by the calls of a CUDA-graph capture in
        # progress (None outside one): the graph keeps their addresses
        self._graph_keep: Optional[list] = None

    # ------------------------------------------------------------------ context
    def __enter__(self) -> "AbftInjector":
        self._orig_linear = F.linear
        self._orig_matmul = torch.matmul
        self._orig_bmm = torch.bmm
        if self.cfg.enable_linear:
            F.linear = self._wrap_linear(self._orig_linear)
        if self.cfg.enable_matmul:
            torch.matmul = self._wrap_matmul(self._orig_matmul)
        if self.cfg.enable_bmm:
            torch.bmm = self._wrap_bmm(self._orig_bmm)
        return self

    def __exit__(self, exc_type, exc, tb) -> None:
        if self._orig_linear is not None:
            F.linear = self._orig_linear
        if self._orig_matmul is not None:
            torch.matmul = self._orig_matmul
        if self._orig_bmm is not None:
            torch.bmm = self._orig_bmm
        if exc_type is None:
            self.flush()
        return None

    def flush(self) -> None:
        """Record every deferred fused-call report, in call order (one copy
        per device for the fused linears, one per batched call)."""
        pending, self._pending = self._pending, []
        if not pending:
            return
        reports = {dev: iter(arena.drain()) for dev, arena in self._arenas.items()}
        if any(arena.suspect for arena in self._arenas.values()):
            # a slab mismatched in most rows: cached checksums may be stale
            # (a weight written behind the version counter); re-encode all
            self.checksums.clear()
            for arena in self._arenas.values():
                arena.suspect = False
        self._record_pending(pending, reports)

    def _record_pending(self, pending: list, reports: dict, reads: Optional[dict] = None) -> None:
        """Record deferred calls in order; ``reports`` maps a device to an
        iterator over its arena's results, ``reads`` (optional) the id of a
        batched or post-hoc report buffer to its host copy."""

        def read(rb):
            return rb.read() if reads is None else reads[id(rb)]

        keys: dict = {}
        saved = self.stats.current_phase
        try:
            for dev, op_name, phase, shape_key, injected, batched in pending:
                if isinstance(shape_key, tuple):  # (m, k, n) of a fused call
                    key = keys.get(shape_key)
                    if key is None:
                        m, k, n = shape_key
                        key = keys[shape_key] = f"A{(m, k)}_B{(k, n)}_C{(m, n)}"
                    shape_key = key
                self.stats.current_phase = phase
                if batched is None:
                    self.stats.record_check(op_name=op_name, shape_key=shape_key, result=next(reports[dev]),
                                            injected=injected)
                elif isinstance(batched, _DeferredCheck):
                    self.stats.record_check(op_name=op_name, shape_key=shape_key,
                                            result=batched.checker.result(read(batched.report)), injected=injected)
                else:
                    rb, nb, rows, gates = batched
                    self._record_batches(op_name, shape_key, read(rb), nb, rows, gates, injected)
        finally:
            self.stats.current_phase = saved

    def _record_batches(self, op_name: str, shape_key: str, rep: N.FaultReport, nb: int, rows: int,
                        gates: List[bool], injected: bool) -> None:
        for bi in range(nb):
            if gates[bi]:
                self.stats.record_check(op_name=op_name, shape_key=shape_key,
                                        result=result_from_report(rep.batch_view(bi, rows)), injected=injected)

    # ------------------------------------------------------------ CUDA graphs
    def capture(self, graph: "torch.cuda.CUDAGraph", **graph_kwargs: Any) -> "_GraphCapture":
        """Context manager capturing the calls made inside it into ``graph``
        (``torch.cuda.graph(graph, **graph_kwargs)``), checks included. It
        yields a ``CapturedChecks``; after each ``graph.replay()`` its
        ``record()`` reads that replay's reports into the stats::

            with injector:
                model(x)                    # eager first: encodes the checksums
                g = torch.cuda.CUDAGraph()
                with injector.capture(g) as checks:
                    y = model(x)
                for _ in range(steps):
                    g.replay()
                    checks.record()

        A replay repeats the captured decisions, so configurations that
        draw from the random stream per call are refused: fault injection
        and ``sample_rate`` < 1 (the reference's per-call coins,
        injector.py:53-75), and ``dump_file``, which copies operands to the
        host. Reports are deferred during the capture whatever
        ``defer_reports`` says. The weights' checksum blocks are captured as
        they are: after a weight update, capture again (a replay that finds
        them stale reports it, and ``record()`` warns)."""
        return _GraphCapture(self, graph, graph_kwargs)

    # -------------------------------------------------------- reference gates
    def _sample(self) -> bool:
        if self.cfg.sample_rate >= 1.0:
            return True
        return self.rng.random() < self.cfg.sample_rate

    def _draw_fault(self, numel: int) -> Optional[int]:
        """The injection decision of injector.py:58-75 without the tensor op."""
        if not self.cfg.inject_fault:
            return None
        if not self.cfg.inject_phase_enabled(self.stats.current_phase):
            return None
        if self.cfg.inject_probability <= 0.0:
            return None
        if self.rng.random() >= self.cfg.inject_probability:
            return None
        if numel == 0:
            return None
        idx = self.rng.randrange(numel)
        self.stats.record_injection()
        return idx

    def _maybe_inject_fault(self, out: torch.Tensor) -> Tuple[torch.Tensor, bool]:
        idx = self._draw_fault(out.numel())
        if idx is None:
            return out, False
        perturbed = out.clone()
        perturbed.reshape(-1)[idx] += self.cfg.inject_magnitude
        return perturbed, True

    def _check_gate(self, a_2d, b_2d, c_2d) -> bool:
        """Gates of injector.py:86-99, in order (the sample coin is drawn third)."""
        if not self.cfg.enable:
            return False
        if not self.cfg.check_enable:
            return False
        if not self.cfg.phase_enabled(self.stats.current_phase):
            return False
        if not self._sample():
            return False
        if a_2d is None or b_2d is None or c_2d is None:
            return False
        if a_2d.numel() == 0 or b_2d.numel() == 0 or c_2d.numel() == 0:
            return False
        if a_2d.shape[1] != b_2d.shape[0]:
            return False
        return True

    def _check_gate_dims(self, m: int, k: int, n: int) -> bool:
        """_check_gate for a fused linear (A [m, k], B [k, n], C [m, n]):
        the same gates in the same order, without materialising C."""
        if not self.cfg.enable or not self.cfg.check_enable:
            return False
        if not self.cfg.phase_enabled(self.stats.current_phase):
            return False
        if not self._sample():
            return False
        return m * k > 0 and k * n > 0 and m * n > 0

    def _maybe_check(self, op_name: str, a_2d, b_2d, c_2d, injected: bool,
                     bias_1d: Optional[torch.Tensor] = None) -> None:
        if not self._check_gate(a_2d, b_2d, c_2d):
            return
        shape_key = _shape_key(a_2d, b_2d, c_2d)
        if self.defer_reports and self.cfg.record_enable and hasattr(self.checker, "launch"):
            # Same check, report read at flush: no host sync per call.
            try:
                rb = self.checker.launch(a_2d, b_2d, c_2d, bias_1d)
            except UnsupportedOperand:
                self.stats.record_skip_unsupported()
                return
            self._pending.append((a_2d.device.index, op_name, self.stats.current_phase, shape_key, injected,
                                  _DeferredCheck(rb, self.checker)))
            self._maybe_dump_tensors(op_name, shape_key, a_2d, b_2d, c_2d, bias_1d)
            return
        try:
            result = self.checker.check(
                a_2d, b_2d, c_2d, OpMeta(op_name=op_name, phase=self.stats.current_phase, shape_key=shape_key),
                bias_1d=bias_1d)
        except UnsupportedOperand:
            self.stats.record_skip_unsupported()
            return
        if self.cfg.record_enable:
            self.stats.record_check(op_name=op_name, shape_key=shape_key, result=result, injected=injected)
        self._maybe_dump_tensors(op_name, shape_key, a_2d, b_2d, c_2d, bias_1d)

    def _maybe_dump_tensors(self, op_name, shape_key, a_2d, b_2d, c_2d, bias_1d) -> None:
        if self._dump_done or not self.cfg.dump_file or not self.cfg.dump_shape_key:
            return
        if not self.cfg.dump_phase_enabled(self.stats.current_phase):
            return
        if shape_key != self.cfg.dump_shape_key:
            return
        payload = {
            "meta": {"phase": self.stats.current_phase, "op_name": op_name, "shape_key": shape_key},
            "a": a_2d.detach().cpu(),
            "b": b_2d.detach().cpu(),
            "c": c_2d.detach().cpu(),
            "bias": None if bias_1d is None else bias_1d.detach().cpu(),
        }
        torch.save(payload, self.cfg.dump_file)
        self._dump_done = True

    # ---------------------------------------------------------- fused linear
    @staticmethod
    def _needs_grad(*ts: Optional[torch.Tensor]) -> bool:
        """The fused kernels have no backward: calls that autograd records
        take the reference flow."""
        return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ts)

    def _fused_linear_ok(self, x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor]) -> bool:
        if self.cfg.checker_backend != "b200" or not self.cfg.fused_linear:
            return False
        if self._needs_grad(x, weight, bias):
            return False
        if not (x.is_cuda and weight.is_cuda) or x.dtype not in ops.GEMM_DTYPES or weight.dtype != x.dtype:
            return False
        if weight.dim() != 2 or x.dim() < 1 or x.shape[-1] != weight.shape[1]:
            return False
        n, k = weight.shape
        if k == 0 or n == 0 or x.numel() == 0:
            return False
        if bias is not None and (not bias.is_cuda or bias.dtype != x.dtype or bias.dim() != 1):
            return False
        if k % 8 or n % 8:
            return True  # run on zero-padded copies (_fused_linear_padded)
        if weight.stride(1) != 1 or weight.stride(0) % 8 or weight.data_ptr() % 16:
            return False
        return True

    def _fused_linear_padded(self, x: torch.Tensor, weight: torch.Tensor,
                             bias: Optional[torch.Tensor]) -> torch.Tensor:
        """A linear whose K or N is not a multiple of 8 (the library reads
        rows in 16-byte pieces), e.g. a VLA's 7-wide action projections:
        the fused kernel runs on copies zero-padded to multiples of 8 and the
        output is the first N columns. Zero rows and columns change no
        product and no checksum, so the padded call detects, locates and
        corrects exactly the faults of the original one (the reference can
        only run its scalar check on such a linear). The copies are made
        per call: a cached padded weight could go stale behind a write the
        version counter does not see, and these weights are small."""
        n, k = weight.shape
        pk, pn = -k % 8, -n % 8
        xp = F.pad(x, (0, pk)) if pk else x
        wp = F.pad(weight, (0, pk, 0, pn))
        bp = None if bias is None else (F.pad(bias, (0, pn)) if pn else bias)
        out = self._fused_linear(xp, wp, bp, real=(k, n))
        return out[..., :n] if pn else out

    def _fused_linear(self, x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                      real: Optional[Tuple[int, int]] = None) -> torch.Tensor:
        """``real``: (K, N) of the caller's linear when ``x`` and ``weight``
        are zero-padded copies (the fault draw and the shape key use the
        caller's shape; the kernel encodes the copy's checksums itself)."""
        n, k = weight.shape
        k_key, n_key = real if real is not None else (k, n)
        # A contiguous input is read in place as m rows of k (no reshape
        # dispatch per call); anything else as a 2-D view with its own row
        # stride, or a copy when that view cannot be read in place.
        if x.is_contiguous() and x.data_ptr() % 16 == 0:
            x2, lda = x, k
        else:
            x2 = x.reshape(-1, k)
            if x2.stride(1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
                x2 = x2.contiguous()
            lda = x2.stride(0)
        m = x2.numel() // k
        dix = x2.get_device()
        # injection first, then the check gate: the reference's rng order
        idx = self._draw_fault(m * n_key)
        injected = idx is not None
        check = self._check_gate_dims(m, k_key, n_key)
        mode = N.MODE_OFF
        if check:
            mode = N.MODE_DETECT | (0 if self.cfg.detect_only else N.MODE_CORRECT)
        tkey = (m, n, k, mode, dix)
        tile_n = self._tile_n.get(tkey)
        if tile_n is None:
            tile_n = self._tile_n[tkey] = ops.pick_tile_n(m, n, k, x2.device, mode)
        # few rows: the library swaps the operands and checksums the tokens
        # itself, so the weight's checksum block is not needed
        swapped = m <= 64 and n >= 2 * m
        cks = self.checksums.get(weight, tile_n) if check and not swapped and real is None else None
        if cks is not None and self._graph_keep is not None:
            self._graph_keep.append(cks)
        inject = [(idx // n_key, idx % n_key, float(self.cfg.inject_magnitude))] if injected else None
        rep = None
        if check:
            if self.defer_reports and self.cfg.record_enable:
                # one arena per device: reports of one device are drained in call order
                arena = self._arenas.get(dix)
                if arena is None:
                    arena = self._arenas[dix] = _ReportArena(self.cfg.report_capacity, x2.device)
                rep = arena.take()
            else:
                rep = ops.ReportBuffer(self.cfg.report_capacity, x2.device)
        if bias is not None and not bias.is_contiguous():
            bias = bias.contiguous()
        # the output in its final shape: m contiguous rows of n
        out = torch.empty(x.shape[:-1] + (n,), dtype=x2.dtype, device=x2.device)
        # operands checked by _fused_linear_ok: straight to the launch
        ops._gemm_launch(x2, weight, bias, out, m, n, k, mode, 0 if swapped else tile_n, 0, 0, self.cfg.thr_scale,
                         self.cfg.thr_abs, 1e-2, 1e-2, cks, inject, rep, 0, lda=lda, ldc=n)
        if check:
            if self.cfg.record_enable:
                if self.defer_reports:
                    self._pending.append((dix, "linear", self.stats.current_phase, (m, k_key, n_key), injected,
                                          None))
                else:
                    host_rep = rep.read()
                    if host_rep.suspect:
                        self.checksums.clear()
                    self.stats.record_check(op_name="linear",
                                            shape_key=f"A{(m, k_key)}_B{(k_key, n_key)}_C{(m, n_key)}",
                                            result=result_from_report(host_rep), injected=injected)
            if self.cfg.dump_file:
                self._maybe_dump_tensors("linear", f"A{(m, k_key)}_B{(k_key, n_key)}_C{(m, n_key)}",
                                         x.reshape(m, k)[:, :k_key], weight.t()[:k_key, :n_key],
                                         out.reshape(m, n)[:, :n_key], None if bias is None else bias[:n_key])
        return out

    # -------------------------------------------------- fused bmm / matmul
    def _fused_mm_ok(self, a: torch.Tensor, b: torch.Tensor) -> bool:
        """[..., M, K] x [..., K, N] operands the batched fused kernel takes."""
        if self.cfg.checker_backend != "b200" or not self.cfg.fused_matmul:
            return False
        if not isinstance(a, torch.Tensor) or not isinstance(b, torch.Tensor) or a.dim() < 2 or b.dim() < 2:
            return False
        if not (a.is_cuda and b.is_cuda) or a.device != b.device:
            return False
        if a.dtype not in ops.GEMM_DTYPES or b.dtype != a.dtype or self._needs_grad(a, b):
            return False
        k, n = b.shape[-2], b.shape[-1]
        return a.shape[-1] == k and k % 8 == 0 and n % 8 == 0 and k > 0 and n > 0 and a.numel() > 0

    def _run_batched(self, op_name: str, a3: torch.Tensor, b3: torch.Tensor, idx: Optional[int],
                     gates: List[bool]) -> torch.Tensor:
        """out[i] = a3[i] @ b3[i] through the fused kernel: the drawn fault
        (flat index into out) goes into the accumulator, batches whose gate
        passed are checked and recorded one check each. Gates that differ
        across batches (sample_rate < 1) take one launch per batch, so that
        only sampled batches are checked or corrected."""
        bsz, m, _ = a3.shape
        n = b3.shape[2]
        injected = idx is not None
        mag = float(self.cfg.inject_magnitude)
        if bsz > 1 and any(gates) and not all(gates):
            outs = []
            for bi in range(bsz):
                inj = None
                if injected and idx // (m * n) == bi:
                    inj = [(idx // n - bi * m, idx % n, mag)]
                outs.append(self._launch_batched(op_name, a3[bi:bi + 1], b3[bi:bi + 1], inj, [gates[bi]], injected))
            return torch.cat(outs)
        inj = [(idx // n, idx % n, mag)] if injected else None
        return self._launch_batched(op_name, a3, b3, inj, gates, injected)

    def _launch_batched(self, op_name: str, a3: torch.Tensor, b3: torch.Tensor, inject, gates: List[bool],
                        injected: bool) -> torch.Tensor:
        bsz, m, k = a3.shape
        n = b3.shape[2]
        check = bool(gates[0])
        mode = N.MODE_OFF
        rep = None
        if check:
            mode = N.MODE_DETECT | (0 if self.cfg.detect_only else N.MODE_CORRECT)
            rep = ops.ReportBuffer(self.cfg.report_capacity, a3.device, batch=bsz)
        out, rep = ops.abft_bmm(a3, b3, mode=mode, thr_scale=self.cfg.thr_scale, thr_abs=self.cfg.thr_abs,
                                inject=inject, report=rep)
        if check:
            key = f"A{(m, k)}_B{(k, n)}_C{(m, n)}"
            if self.cfg.record_enable:
                if self.defer_reports:
                    self._pending.append((a3.device.index, op_name, self.stats.current_phase, key, injected,
                                          (rep, bsz, m, list(gates))))
                else:
                    self._record_batches(op_name, key, rep.read(), bsz, m, gates, injected)
            if self.cfg.dump_file:
                for bi in range(bsz):
                    self._maybe_dump_tensors(op_name, key, a3[bi], b3[bi], out[bi], None)
        return out

    def _fused_bmm(self, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        bsz, m, k = a.shape
        n = b.shape[2]
        # the reference's rng order: the injection draw over out, then one
        # check gate (sample coin) per batch (injector.py:176-187)
        idx = self._draw_fault(bsz * m * n)
        gates = [self._check_gate_dims(m, k, n) for _ in range(bsz)]
        return self._run_batched("bmm", a, b, idx, gates)

    def _fused_matmul(self, a: torch.Tensor, b: torch.Tensor) -> Optional[torch.Tensor]:
        """torch.matmul through the fused kernel, or None for the reference
        flow (nothing drawn from the rng yet)."""
        k, n = b.shape[-2], b.shape[-1]
        if b.dim() == 2:
            # checked by the reference as one 2-D product [M*, K] x [K, N]
            a2 = a.reshape(-1, k)
            m = a2.shape[0]
            idx = self._draw_fault(m * n)
            gate = self._check_gate_dims(m, k, n)
            out = self._run_batched("matmul", a2.unsqueeze(0), b.unsqueeze(0), idx, [gate])
            return out.reshape(*a.shape[:-1], n)
        if not self.cfg.check_batched_matmul or a.dim() != b.dim() or a.shape[:-2] != b.shape[:-2]:
            return None
        # batched right operand: one sample coin for the call, as in the
        # reference (whose check then stops at b_2d None); every batch checked
        a3 = a.reshape(-1, a.shape[-2], k)
        b3 = b.reshape(-1, k, n)
        bsz, m = a3.shape[0], a3.shape[1]
        if bsz > 65535:
            return None
        idx = self._draw_fault(bsz * m * n)
        gate = self._check_gate_dims(m, k, n)
        out = self._run_batched("matmul", a3, b3, idx, [gate] * bsz)
        return out.reshape(*a.shape[:-1], n)

    # ------------------------------------------------------------- wrappers
    @staticmethod
    def _nvtx_name(op: str, a: Any, b: Any, linear: bool = False) -> str:
        """"abft.<op> MxNxK" of a hooked call (rows of the flattened left
        operand; N from the weight's rows for a linear)."""
        try:
            k = a.shape[-1]
            m = a.numel() // k if k else 0
            n = b.shape[0] if linear else b.shape[-1]
            return f"abft.{op} {m}x{n}x{k}"
        except (AttributeError, IndexError, TypeError):
            return f"abft.{op}"

    def _in_nvtx_range(self, name: str, fn: Callable[..., torch.Tensor], *args: Any, **kwargs: Any) -> Any:
        torch.cuda.nvtx.range_push(name)
        try:
            return fn(*args, **kwargs)
        finally:
            torch.cuda.nvtx.range_pop()

    def _wrap_linear(self, fn: Callable[..., torch.Tensor]) -> Callable[..., torch.Tensor]:
        def wrapped(input: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
            return self._in_nvtx_range(self._nvtx_name("linear", input, weight, linear=True), body, input, weight,
                                       bias)

        def body(input: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
            if self._fused_linear_ok(input, weight, bias):
                if weight.shape[0] % 8 or weight.shape[1] % 8:
                    return self._fused_linear_padded(input, weight, bias)
                return self._fused_linear(input, weight, bias)
            out = fn(input, weight, bias)
            out2, injected = self._maybe_inject_fault(out)
            a2 = flatten_to_2d_for_mm(input, right_operand=False)
            b2 = flatten_to_2d_for_mm(weight.t(), right_operand=True)  # [k, n]
            c2 = flatten_to_2d_for_mm(out2, right_operand=False)
            self._maybe_check("linear", a2, b2, c2, injected, bias_1d=bias)
            return out2

        # cfg.nvtx is read when the injector is entered
        return wrapped if self.cfg.nvtx else body

    def _wrap_matmul(self, fn: Callable[..., torch.Tensor]) -> Callable[..., torch.Tensor]:
        def wrapped(input: torch.Tensor, other: torch.Tensor, *args: Any, **kwargs: Any) -> torch.Tensor:
            return self._in_nvtx_range(self._nvtx_name("matmul", input, other), body, input, other, *args, **kwargs)

        def body(input: torch.Tensor, other: torch.Tensor, *args: Any, **kwargs: Any) -> torch.Tensor:
            if not args and not kwargs and self._fused_mm_ok(input, other):
                out = self._fused_matmul(input, other)
                if out is not None:
                    return out
            out = fn(input, other, *args, **kwargs)
            out2, injected = self._maybe_inject_fault(out)
            a2 = flatten_to_2d_for_mm(input, right_operand=False)
            b2 = flatten_to_2d_for_mm(other, right_operand=True)
            c2 = flatten_to_2d_for_mm(out2, right_operand=False)
            self._maybe_check("matmul", a2, b2, c2, injected)
            return out2

        # cfg.nvtx is read when the injector is entered
        return wrapped if self.cfg.nvtx else body

    def _wrap_bmm(self, fn: Callable[..., torch.Tensor]) -> Callable[..., torch.Tensor]:
        def wrapped(input: torch.Tensor, mat2: torch.Tensor, *args: Any, **kwargs: Any) -> torch.Tensor:
            return self._in_nvtx_range(self._nvtx_name("bmm", input, mat2), body, input, mat2, *args, **kwargs)

        def body(input: torch.Tensor, mat2: torch.Tensor, *args: Any, **kwargs: Any) -> torch.Tensor:
            if (not args and not kwargs and self._fused_mm_ok(input, mat2) and input.dim() == 3 and mat2.dim() == 3
                    and input.shape[0] == mat2.shape[0] and 0 < input.shape[0] <= 65535):
                return self._fused_bmm(input, mat2)
            out = fn(input, mat2, *args, **kwargs)
            out2, injected = self._maybe_inject_fault(out)
            # per-batch 2-D checks, as the reference (injector.py:180-186)
            for bi in range(input.shape[0]):
                self._maybe_check("bmm", input[bi], mat2[bi], out2[bi], injected)
            return out2

        # cfg.nvtx is read when the injector is entered
        return wrapped if self.cfg.nvtx else body


class CapturedChecks:
    """The checks of one captured graph (``AbftInjector.capture``).

    ``record()`` after a replay copies the reports that replay wrote to the
    host (one copy per arena chunk and per batched call) and records them in
    the injector's stats in call order, as ``flush()`` does for an eager
    forward. The object keeps the report slots and checksum blocks the graph
    addresses alive."""

    def __init__(self, injector: AbftInjector):
        self._inj = injector
        self._pending: list = []
        self._arenas: dict = {}
        self._keep: list = []
        self.replays_recorded = 0
        self.stale_checksums = False
        # overlapped recording: two sets of pinned host copies of every
        # report the graph writes, the set in flight and its event
        self._host_sets: List[Optional[tuple]] = [None, None]
        self._next_set = 0
        self._in_flight: Optional[Tuple[tuple, Any]] = None
        # the graph's checks as one bulk record for clean replays (built at
        # the first record; None when some call is not a fused linear)
        self._clean: Optional[CleanChecks] = None
        self._clean_ready = False

    def _adopt(self, pending: list, arenas: dict, keep: Optional[list]) -> None:
        self._pending, self._arenas, self._keep = pending, arenas, keep or []

    def __len__(self) -> int:
        """Checked calls in the graph."""
        return len(self._pending)

    def record(self, overlap: bool = False) -> None:
        """Record the reports of the latest replay.

        By default this waits for the replay. With ``overlap=True`` it
        queues a copy of the reports into pinned host memory on the current
        stream (behind the replay) and records the copy that the previous
        call queued instead, so the host work runs while the GPU runs the
        next replay; ``finish()`` records the last copy. Replays and these
        calls must then alternate on one stream."""
        if not self._pending:
            return
        if not overlap:
            self.finish()
            self._record({dev: iter(arena.read()) for dev, arena in self._arenas.items()}, None)
            return
        host = self._host_set()
        stream = torch.cuda.current_stream()
        for (dst, src) in zip(host[0], [v for a in self._arenas.values() for v in a.used_views()]):
            dst.copy_(src, non_blocking=True)
        for rb, dst in host[1].items():
            dst.copy_(rb.tensor, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        prev, self._in_flight = self._in_flight, (host, ev)
        if prev is not None:
            self._record_copy(*prev)

    def finish(self) -> None:
        """Record the copy the last overlapped ``record()`` queued, if any."""
        prev, self._in_flight = self._in_flight, None
        if prev is not None:
            self._record_copy(*prev)

    def _host_set(self) -> tuple:
        """The next of two sets of pinned buffers: one per arena chunk view
        (in ``_arenas`` order) and one per batched or post-hoc report."""
        i = self._next_set
        self._next_set ^= 1
        if self._host_sets[i] is None:
            chunks = [torch.empty(v.numel(), dtype=torch.uint8, pin_memory=True)
                      for a in self._arenas.values() for v in a.used_views()]
            rbs = {}
            for entry in self._pending:
                batched = entry[5]
                rb = batched.report if isinstance(batched, _DeferredCheck) else (
                    batched[0] if isinstance(batched, tuple) else None)
                if rb is not None:
                    rbs[rb] = torch.empty(rb.tensor.numel(), dtype=torch.uint8, pin_memory=True)
            self._host_sets[i] = (chunks, rbs)
        return self._host_sets[i]

    def _record_copy(self, host: tuple, ev: Any) -> None:
        ev.synchronize()
        chunks, rbs = host
        arrays = [c.numpy() for c in chunks]
        reports, at = {}, 0
        for dev, arena in self._arenas.items():
            n = len(arena.chunks)
            reports[dev] = iter(arena.read(arrays[at:at + n]))
            at += n
        reads = {id(rb): N.FaultReport.from_bytes(t.numpy().tobytes()) for rb, t in rbs.items()}
        self._record(reports, reads)

    def _clean_checks(self) -> Optional[CleanChecks]:
        if not self._clean_ready:
            self._clean_ready = True
            if all(e[5] is None for e in self._pending):
                calls = []
                for _, op_name, phase, (m, k, n), _, _ in self._pending:
                    calls.append((phase, op_name, f"A{(m, k)}_B{(k, n)}_C{(m, n)}"))
                self._clean = CleanChecks(calls)
        return self._clean

    def _record(self, reports: dict, reads: Optional[dict]) -> None:
        clean = self._clean_checks()
        if clean is not None and self._inj.cfg.record_enable:
            results = {dev: list(it) for dev, it in reports.items()}
            if all(r is _CLEAN_RESULT for rs in results.values() for r in rs):
                # the common replay: every fused linear clean, one bulk record
                self._inj.stats.record_clean(clean)
                self.replays_recorded += 1
                return
            reports = {dev: iter(rs) for dev, rs in results.items()}
        if any(arena.suspect for arena in self._arenas.values()):
            self.stale_checksums = True
            for arena in self._arenas.values():
                arena.suspect = False
            warnings.warn("a replay found checksum blocks that no longer match their weights (a weight was "
                          "written after the capture): capture the graph again", RuntimeWarning, stacklevel=2)
        self._inj._record_pending(self._pending, reports, reads)
        self.replays_recorded += 1


class _GraphCapture:
    """``AbftInjector.capture``: swaps in empty deferred-report state for the
    capture, and hands what the captured calls queued to a CapturedChecks."""

    def __init__(self, injector: AbftInjector, graph: "torch.cuda.CUDAGraph", graph_kwargs: dict):
        self._inj = injector
        self._graph = graph
        self._kwargs = graph_kwargs
        self._ctx = None
        self._saved = None
        self.checks = CapturedChecks(injector)

    def __enter__(self) -> CapturedChecks:
        inj, cfg = self._inj, self._inj.cfg
        if cfg.inject_fault and cfg.inject_probability > 0.0:
            raise RuntimeError("fault injection draws per call from the random stream, which a graph replay "
                               "cannot repeat: capture with inject_fault off")
        if cfg.sample_rate < 1.0:
            raise RuntimeError("sample_rate < 1 draws a coin per call, which a graph replay cannot repeat")
        if cfg.dump_file:
            raise RuntimeError("dump_file copies operands to the host, which a graph cannot capture")
        inj.flush()  # eager calls' reports first
        self._saved = (inj._pending, inj._arenas, inj.defer_reports)
        inj._pending, inj._arenas, inj.defer_reports = [], {}, True
        inj._graph_keep = []
        self._ctx = torch.cuda.graph(self._graph, **self._kwargs)
        try:
            self._ctx.__enter__()
        except BaseException:
            self._restore()
            raise
        return self.checks

    def _restore(self) -> None:
        inj = self._inj
        inj._pending, inj._arenas, inj.defer_reports = self._saved
        inj._graph_keep = None

    def __exit__(self, exc_type, exc, tb) -> bool:
        try:
            self._ctx.__exit__(exc_type, exc, tb)
        finally:
            inj = self._inj
            self.checks._adopt(inj._pending, inj._arenas, inj._graph_keep)
            self._restore()
        return False
