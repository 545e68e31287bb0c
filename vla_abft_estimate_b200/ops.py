"""Torch-facing wrappers of the C ABI.

PyTorch supplies device memory, the current stream and the caching allocator
for workspaces; every computation runs in libabft_b200.so. Inputs must be CUDA
bf16 or fp16 tensors (the post-hoc check also fp32) on an sm_100 device;
anything else raises (no CPU fallback).

Functions
  encode_weight(weight, tile_n)          per-tile checksums of a [N, K] weight
  abft_gemm(a, weight, bias, ...)        fused checksum-protected GEMM
  abft_linear(x, weight, bias, ...)      the same with F.linear's shapes:
                                         any leading dimensions, any K, N
  abft_bmm(a, b, ...)                    the same for a batch of products
                                         (torch.bmm), one launch
  check_only(a, b, c, bias, ...)         post-hoc check of an existing output
  wait_selftest()                        the bounded device waits giving up
                                         (failure detection, no fault)

abft_gemm, abft_linear, abft_bmm and check_only may be captured in a CUDA
graph (``torch.cuda.graph``): under capture the library clears its
stream-K flags and the report's launch tag in the graph (one small kernel
ahead of the GEMM), so every
replay writes a fresh report, and the workspace a capture used is kept for
the graph's replays.
"""
from __future__ import annotations

import collections
import ctypes
import functools
import math
from typing import Optional, Sequence, Tuple

import torch

from . import _native as N
from ._native import FaultReport

DEFAULT_THR_SCALE = 1e-3
DEFAULT_CAPACITY = 64


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


# Element types of the fused GEMM (the post-hoc check adds fp32).
GEMM_DTYPES = {torch.bfloat16: N.DTYPE_BF16, torch.float16: N.DTYPE_F16}


def _require_cuda(name: str, t: torch.Tensor, dim: int, dtype: torch.dtype = torch.bfloat16) -> None:
    """``t`` is a CUDA tensor of ``dtype`` with ``dim`` dimensions and unit
    stride in its last one."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the library has no CPU path)")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {str(dtype).replace('torch.', '')}, got {t.dtype}")
    if t.dim() != dim:
        raise ValueError(f"{name} must be {dim}-D, got shape {tuple(t.shape)}")
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must have unit stride in its last dimension")


class ReportBuffer:
    """Device buffer holding one ``abft_report`` with ``capacity`` records
    (and, for a batched call, the per-batch counters of ``batch`` products)."""

    def __init__(self, capacity: int = DEFAULT_CAPACITY, device: Optional[torch.device] = None,
                 tensor: Optional[torch.Tensor] = None, batch: int = 1):
        self.capacity = int(capacity)
        self.batch = max(int(batch), 1)
        nbytes = int(N.lib().abft_report_bytes_batched(self.capacity, self.batch))
        if tensor is None:
            tensor = torch.zeros(nbytes, dtype=torch.uint8, device=device or torch.device("cuda"))
        elif tensor.dtype != torch.uint8 or tensor.numel() < nbytes or tensor.data_ptr() % 16:
            raise ValueError(f"a report of capacity {capacity} needs {nbytes} 16-byte aligned bytes")
        self.tensor = tensor

    def data_ptr(self) -> int:
        return self.tensor.data_ptr()

    def read(self) -> FaultReport:
        """Copy the report to the host (synchronises with the producing stream)."""
        return FaultReport.from_bytes(self.tensor.cpu().numpy().tobytes())

    def read_header_async(self, pinned: torch.Tensor) -> None:
        """Start a device->host copy of the 64-byte header into ``pinned``."""
        pinned.copy_(self.tensor[: N.REPORT_HEADER_BYTES], non_blocking=True)


@functools.lru_cache(maxsize=None)
def _sm_count(index: int) -> int:
    return torch.cuda.get_device_properties(index).multi_processor_count


def _device_index(device: Optional[torch.device]) -> int:
    if device is None or device.index is None:
        return torch.cuda.current_device()
    return device.index


_WORKSPACES: "collections.OrderedDict[tuple, torch.Tensor]" = collections.OrderedDict()
_MAX_WORKSPACES = 64
# Workspaces used while a CUDA graph was being captured, by address. A
# graph's kernel nodes hold their addresses for every replay, so they are
# never freed, even once the per-stream cache above replaces or evicts them.
# (Replays must not overlap on the GPU with other fused calls on the capture
# stream's workspace: like those calls, they share it.)
_GRAPH_HELD: dict = {}


def _workspace(device: torch.device, nbytes: int, stream: Optional[int] = None) -> torch.Tensor:
    """Scratch for the current stream of ``device``, grown on demand.

    One buffer per (device, raw stream handle), allocated while that stream
    is current. Calls on one stream run in order, so reusing the buffer is
    safe, and a buffer that is replaced or evicted is freed in that stream's
    order by the caching allocator.

    Keying on the raw handle is safe when a handle is recycled: torch's own
    streams come from a fixed pool and are never destroyed (two Stream
    objects with one handle share one in-order queue), and the driver only
    hands out a destroyed stream's handle again once the work queued on it
    has completed. The dictionary is bounded (least recently used first out)
    so that callers cycling through many external streams do not keep one
    buffer each alive.
    """
    if stream is None:
        stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index, stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
        if len(_WORKSPACES) > _MAX_WORKSPACES:
            _WORKSPACES.popitem(last=False)
    _WORKSPACES.move_to_end(key)
    return ws


# abft_gemm_workspace_bytes depends on the shape, mode, tile requests and
# layout only: remembered per key so a repeated call makes one library call.
_WS_BYTES: dict = {}


def _run_gemm(args: N.GemmArgs, dev: torch.device, key: tuple) -> None:
    """Workspace, current stream and device guard around abft_gemm. (The
    operands are CUDA tensors, so CUDA is initialised: the raw device query
    skips torch.cuda.current_device()'s lazy-init checks, a few hundred ns of
    a decode step's every linear.)"""
    cur = torch._C._cuda_getDevice()
    idx = dev.index if dev.index is not None else cur
    stream = torch._C._cuda_getCurrentRawStream(idx)
    L = N.lib()
    if cur != idx:
        with torch.cuda.device(idx):
            return _run_gemm(args, dev, key)
    key = (idx,) + key
    ws_bytes = _WS_BYTES.get(key)
    if ws_bytes is None:
        ws_bytes = _WS_BYTES[key] = int(L.abft_gemm_workspace_bytes(ctypes.byref(args)))
    if ws_bytes:
        ws = _workspace(dev, ws_bytes, stream)
        args.workspace = ws.data_ptr()
        args.workspace_bytes = ws.numel()
        if torch._C._cuda_isCurrentStreamCapturing():
            # the captured kernel nodes keep this address for every replay
            _GRAPH_HELD[ws.data_ptr()] = ws
    N.check("abft_gemm", L.abft_gemm(ctypes.byref(args), ctypes.c_void_p(stream)))


def pick_tile_n(m: int, n: int, k: int, device: Optional[torch.device] = None,
                mode: int = N.MODE_DETECT | N.MODE_CORRECT) -> int:
    """Tile width the library would pick for an m x n x k GEMM in ``mode``."""
    sms = _sm_count(_device_index(device))
    return int(N.lib().abft_pick_tile_n(int(m), int(n), int(k), int(sms), int(mode)))


def pick_tile_m(m: int, n: int, k: int, tile_n: int, device: Optional[torch.device] = None,
                mode: int = N.MODE_DETECT | N.MODE_CORRECT) -> int:
    """Tile height (128, or 256 = one 2-CTA pair per tile) the library would pick."""
    sms = _sm_count(_device_index(device))
    return int(N.lib().abft_pick_tile_m(int(m), int(n), int(k), int(sms), int(mode), int(tile_n)))


def gemm_plan(m: int, n: int, k: int, *, dtype: torch.dtype = torch.bfloat16,
              mode: int = N.MODE_DETECT | N.MODE_CORRECT, tile_n: int = 0, tile_m: int = 0, swap_ab: int = 0,
              num_sms: int = 0, batch: int = 1, cached_checksums: bool = True,
              device: Optional[torch.device] = None) -> dict:
    """What ``abft_gemm`` would launch for an m x n x k product (x ``batch``)
    of contiguous ``dtype`` operands on ``device``: tile shape, tile columns,
    the last column's width, schedule and workspace (abft_gemm_plan). No
    device work: the call sees only placeholder addresses."""
    code = GEMM_DTYPES.get(dtype)
    if code is None:
        raise ValueError(f"the fused GEMM takes bfloat16 or float16 operands, got {dtype}")
    fake = 1 << 20  # an aligned placeholder address; nothing is read or written
    args = N.GemmArgs()
    args.A = args.B = args.C = fake
    args.M, args.N, args.K = int(m), int(n), int(k)
    args.lda = args.ldb = int(k)
    args.ldc = int(n)
    args.mode = int(mode)
    args.tile_n, args.tile_m, args.swap_ab = int(tile_n), int(tile_m), int(swap_ab)
    args.thr_scale = DEFAULT_THR_SCALE
    args.checksums = fake if (cached_checksums and mode != N.MODE_OFF) else None
    args.report = fake if mode != N.MODE_OFF else None
    args.report_capacity = DEFAULT_CAPACITY
    args.num_sms = int(num_sms)
    args.batch = int(batch)
    if batch > 1:
        args.stride_a, args.stride_b, args.stride_c = int(m) * int(k), int(n) * int(k), int(m) * int(n)
    args.dtype = code
    info = N.PlanInfo()
    with torch.cuda.device(_device_index(device)):
        N.check("abft_gemm_plan", N.lib().abft_gemm_plan(ctypes.byref(args), ctypes.byref(info)))
    return info.as_dict()


def _gemm_dtype(t: torch.Tensor) -> int:
    code = GEMM_DTYPES.get(t.dtype) if isinstance(t, torch.Tensor) else None
    if code is None:
        got = t.dtype if isinstance(t, torch.Tensor) else type(t)
        raise ValueError(f"the fused GEMM takes bfloat16 or float16 operands, got {got}")
    return code


def checksum_bytes(n: int, k: int, tile_n: int, dtype: torch.dtype = torch.bfloat16) -> int:
    """Bytes of the checksum block of an [n, k] weight of ``dtype``."""
    return int(N.lib().abft_checksum_bytes_typed(int(n), int(k), int(tile_n), GEMM_DTYPES.get(dtype, -1)))


def encode_weight(weight: torch.Tensor, tile_n: int) -> torch.Tensor:
    """Per-tile checksum block of ``weight`` [N, K] for tile width ``tile_n``.

    bf16 weights: returns bf16 [ceil(N / (tile_n - 8)) * 8, K]: for each
    tile, the plain and the column-index-weighted row checksums, each as
    three bf16 terms, and the Thue-Morse signed checksum as two bf16 terms
    (the 8 extra B-operand rows of the fused kernel's tile).
    fp16 weights: returns the block as flat uint8 bytes: the same rows in
    fp16 terms, each checksum of a tile scaled by a power of two that keeps
    it inside fp16's range, followed by the table of those factors.
    """
    dt = _gemm_dtype(weight)
    _require_cuda("weight", weight, 2, weight.dtype)
    n, k = weight.shape
    nbytes = checksum_bytes(n, k, tile_n, weight.dtype)
    if nbytes == 0:
        raise ValueError(f"tile_n must be 128 or 256, got {tile_n}")
    if weight.dtype == torch.bfloat16:
        out = torch.empty((nbytes // (2 * k), k), dtype=torch.bfloat16, device=weight.device)
    else:
        out = torch.empty((nbytes,), dtype=torch.uint8, device=weight.device)
    with torch.cuda.device(weight.device):
        rc = N.lib().abft_encode_weight_typed(_ptr(weight), n, k, weight.stride(0), 0, 1, int(tile_n), dt, _ptr(out),
                                              _stream(weight.device))
    N.check("abft_encode_weight_typed", rc)
    return out


class DeviceFaults:
    """Device copy of a debug fault list [(row, col, delta), ...] for the
    ``inject`` argument of the fused calls. A plain list is copied to the
    device on every call; build this once instead to reuse the copy, or
    before a CUDA graph capture, whose replays then inject the same faults
    (the copy is made here, outside the capture)."""

    def __init__(self, faults: Sequence[Tuple[int, int, float]], device: torch.device):
        if len(faults) > N.MAX_INJECT:
            raise ValueError(f"at most {N.MAX_INJECT} injected faults per call")
        rows = [int(f[0]) for f in faults]
        cols = [int(f[1]) for f in faults]
        deltas = [float(f[2]) for f in faults]
        self.n = len(faults)
        self.rows = torch.tensor(rows or [0], dtype=torch.int32, device=device)
        self.cols = torch.tensor(cols or [0], dtype=torch.int32, device=device)
        self.deltas = torch.tensor(deltas or [0.0], dtype=torch.float32, device=device)


def abft_gemm(
    a: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    *,
    mode: int = N.MODE_DETECT | N.MODE_CORRECT,
    tile_n: int = 0,
    tile_m: int = 0,
    swap_ab: int = 0,
    thr_scale: float = DEFAULT_THR_SCALE,
    thr_abs: float = 0.0,
    tol_abs: float = 1e-2,
    tol_rel: float = 1e-2,
    checksums: Optional[torch.Tensor] = None,
    inject: Optional[Sequence[Tuple[int, int, float]]] = None,
    report: Optional[ReportBuffer] = None,
    out: Optional[torch.Tensor] = None,
    num_sms: int = 0,
) -> Tuple[torch.Tensor, Optional[ReportBuffer]]:
    """``out = a @ weight.T (+ bias)`` with the fused checksum epilogue.

    ``a`` is [M, K], ``weight`` [N, K] (nn.Linear layout), ``bias`` [N], all
    bfloat16 or all float16 (``out`` too).
    ``checksums`` is ``encode_weight(weight, tile_n)`` (cache it for a fixed
    weight); when omitted and checks are on, the call encodes into its
    workspace. ``tile_m`` 256 runs each 256-row tile on a 2-CTA pair (either
    tile_n); 0 lets the library choose. ``swap_ab`` (0 choose, 1 never,
    2 always) computes out^T = weight a^T instead, for few rows of ``a``:
    the weight then streams through the MMA's 128-row side, the checksums
    come from ``a`` per call and fault records keep ``out``'s coordinates.
    ``inject`` adds debug faults to the fp32 accumulator (a list of
    (row, col, delta), or a ``DeviceFaults`` built ahead).
    Returns the output and the report buffer (None when mode == MODE_OFF).
    """
    _gemm_dtype(a)
    dtype = a.dtype
    _require_cuda("a", a, 2, dtype)
    _require_cuda("weight", weight, 2, dtype)
    m, k = a.shape
    n, k2 = weight.shape
    if k != k2:
        raise ValueError(f"inner dimensions differ: a {tuple(a.shape)} vs weight {tuple(weight.shape)}")
    if weight.device != a.device:
        raise ValueError("a and weight must be on the same device")
    if bias is not None:
        _require_cuda("bias", bias, 1, dtype)
        if bias.shape[0] != n:
            raise ValueError(f"bias has {bias.shape[0]} entries, expected {n}")
    dev = a.device
    if out is None:
        out = torch.empty((m, n), dtype=dtype, device=dev)
    else:
        _require_cuda("out", out, 2, dtype)
        if tuple(out.shape) != (m, n):
            raise ValueError(f"out must be [{m}, {n}]")
    if mode != N.MODE_OFF and report is None:
        report = ReportBuffer(DEFAULT_CAPACITY, dev)
    if checksums is not None:
        block = torch.bfloat16 if dtype == torch.bfloat16 else torch.uint8
        if checksums.dtype != block or not checksums.is_cuda:
            raise ValueError(f"checksums must be the CUDA {block} tensor encode_weight() returns for a {dtype} weight")
        if tile_n == 0:
            raise ValueError("pass the tile_n the checksums were encoded for")
        need = checksum_bytes(n, k, tile_n, dtype)
        if checksums.numel() * checksums.element_size() < need:
            raise ValueError("checksums were encoded for a different weight shape or tile width")
    _gemm_launch(a, weight, bias, out, m, n, k, mode, tile_n, tile_m, swap_ab, thr_scale, thr_abs, tol_abs, tol_rel,
                 checksums, inject, report, num_sms)
    return out, report


def _gemm_launch(a, weight, bias, out, m, n, k, mode, tile_n, tile_m, swap_ab, thr_scale, thr_abs, tol_abs, tol_rel,
                 checksums, inject, report, num_sms, lda=None, ldc=None) -> None:
    """abft_gemm after argument validation (callers that have checked the
    operands themselves call this directly). ``lda`` / ``ldc`` override the
    leading dimensions read from 2-D ``a`` / ``out``, for callers that pass
    contiguous tensors of any rank holding m rows."""
    dev = a.device
    inj = inject if isinstance(inject, DeviceFaults) else (DeviceFaults(inject, dev) if inject else None)
    args = N.GemmArgs()
    args.A, args.B, args.C, args.bias = _ptr(a), _ptr(weight), _ptr(out), _ptr(bias)
    args.M, args.N, args.K = m, n, k
    args.lda = a.stride(0) if lda is None else lda
    args.ldb = weight.stride(0)
    args.ldc = out.stride(0) if ldc is None else ldc
    args.mode = int(mode)
    args.tile_n = int(tile_n)
    args.tile_m = int(tile_m)
    args.swap_ab = int(swap_ab)
    args.thr_scale, args.thr_abs = float(thr_scale), float(thr_abs)
    args.tol_abs, args.tol_rel = float(tol_abs), float(tol_rel)
    args.checksums = _ptr(checksums)
    args.report = report.data_ptr() if report is not None else None
    args.report_capacity = report.capacity if report is not None else 0
    args.num_sms = int(num_sms)
    args.dtype = GEMM_DTYPES[a.dtype]
    if inj is not None:
        args.inject_rows, args.inject_cols, args.inject_deltas = _ptr(inj.rows), _ptr(inj.cols), _ptr(inj.deltas)
        args.n_inject = inj.n
    _run_gemm(args, dev, (m, n, k, int(mode), int(tile_n), int(tile_m), int(swap_ab), checksums is None,
                          int(num_sms), 1, 0, args.dtype))


def abft_linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    *,
    cfg=None,
    mode: Optional[int] = None,
    checksums: Optional[torch.Tensor] = None,
    tile_n: int = 0,
    thr_scale: Optional[float] = None,
    thr_abs: Optional[float] = None,
    inject: Optional[Sequence[Tuple[int, int, float]]] = None,
    report: Optional[ReportBuffer] = None,
) -> Tuple[torch.Tensor, Optional[ReportBuffer]]:
    """``F.linear(x, weight, bias)`` with the fused checksum check: the op
    the reference's linear hook runs followed by its check
    (pytorch/abft/injector.py:152-161), in one launch.

    ``x`` is [..., K] and the output [..., N], bfloat16 or float16 like
    ``weight`` [N, K] and ``bias`` [N]. Fault coordinates (``inject`` and the
    report's records) index the output flattened to [rows, N]. ``cfg`` (an
    ``AbftConfig``) supplies the mode (``detect_only``), thresholds and
    report capacity unless they are given here; by default faults are
    detected, located and corrected. K or N not a multiple of 8 (the
    library reads rows in 16-byte pieces) runs on zero-padded copies, which
    change no product and no checksum; ``checksums`` must then be None.
    Returns the output and the report (None when mode is MODE_OFF).
    """
    _gemm_dtype(x)
    if weight.dim() != 2 or x.shape[-1] != weight.shape[1]:
        raise ValueError(f"x {tuple(x.shape)} and weight {tuple(weight.shape)} do not match as F.linear operands")
    n, k = weight.shape
    if mode is None:
        mode = N.MODE_DETECT | (0 if (cfg is not None and cfg.detect_only) else N.MODE_CORRECT)
    if thr_scale is None:
        thr_scale = cfg.thr_scale if cfg is not None else DEFAULT_THR_SCALE
    if thr_abs is None:
        thr_abs = cfg.thr_abs if cfg is not None else 0.0
    if report is None and mode != N.MODE_OFF:
        report = ReportBuffer(cfg.report_capacity if cfg is not None else DEFAULT_CAPACITY, x.device)
    x2 = x.reshape(-1, k)
    pk, pn = -k % 8, -n % 8
    if pk or pn:
        if checksums is not None:
            raise ValueError("checksums cannot be used when K or N needs padding to a multiple of 8")
        x2 = torch.nn.functional.pad(x2, (0, pk))
        weight = torch.nn.functional.pad(weight, (0, pk, 0, pn))
        bias = None if bias is None else (torch.nn.functional.pad(bias, (0, pn)) if pn else bias)
    elif x2.stride(1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    if bias is not None and not bias.is_contiguous():
        bias = bias.contiguous()
    out, rep = abft_gemm(x2, weight, bias, mode=mode, tile_n=tile_n, thr_scale=thr_scale, thr_abs=thr_abs,
                         checksums=checksums, inject=inject, report=report)
    if pn:
        out = out[:, :n]
    return out.reshape(*x.shape[:-1], n), rep


def _mat_layout(t: torch.Tensor) -> Optional[Tuple[int, int]]:
    """(leading dimension, batch stride) in elements under which the library
    can read the [batch, rows, cols] tensor ``t`` in place (unit stride in
    cols, both strides multiples of 8, 16-byte aligned), else None. Strides
    of size-1 dimensions are not used and get a valid stand-in."""
    bsz, rows, cols = t.shape
    if t.stride(2) != 1 and cols > 1:
        return None
    ld = t.stride(1) if rows > 1 else (cols + 7) // 8 * 8
    bs = t.stride(0) if bsz > 1 else rows * ld
    if ld < cols or ld % 8 or bs % 8 or bs < 0 or t.data_ptr() % 16:
        return None
    return ld, bs


def abft_bmm(
    a: torch.Tensor,
    b: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    *,
    b_layout: str = "kn",
    mode: int = N.MODE_DETECT | N.MODE_CORRECT,
    tile_n: int = 0,
    tile_m: int = 0,
    swap_ab: int = 0,
    thr_scale: float = DEFAULT_THR_SCALE,
    thr_abs: float = 0.0,
    inject: Optional[Sequence[Tuple[int, int, float]]] = None,
    report: Optional[ReportBuffer] = None,
    out: Optional[torch.Tensor] = None,
    num_sms: int = 0,
) -> Tuple[torch.Tensor, Optional[ReportBuffer]]:
    """Batched ``out[i] = a[i] @ b[i] (+ bias)`` with the fused checksum
    epilogue: every product of the batch in one launch.

    ``a`` is [B, M, K]. ``b_layout="kn"``: ``b`` is [B, K, N], torch.bmm's
    ``mat2``; a ``b`` whose K dimension has unit stride (the transpose of a
    [B, N, K] tensor, e.g. ``k.transpose(1, 2)``) is read in place, a
    row-major one is copied K-major by the call (with its checksums formed
    on the way). ``b_layout="nk"``: ``b`` is [B, N, K] (weight layout).
    Operands (and ``bias``, ``out``) are all bfloat16 or all float16.
    ``inject`` rows and the report's record rows are flattened over the
    batch (row ``i`` of batch ``j`` is ``j * M + i``); ``report.read()
    .batch_view(j, M)`` gives batch ``j`` alone. Returns ``out`` [B, M, N]
    and the report (None when mode == MODE_OFF).
    """
    if a.dim() != 3 or b.dim() != 3:
        raise ValueError(f"abft_bmm takes 3-D operands, got {tuple(a.shape)} and {tuple(b.shape)}")
    _gemm_dtype(a)
    dtype = a.dtype
    for name, t in (("a", a), ("b", b)):
        if not t.is_cuda or t.dtype != dtype:
            raise ValueError(f"{name} must be a CUDA {dtype} tensor (the library has no CPU path)")
    bsz, m, k = a.shape
    n_dim = 2 if b_layout == "kn" else 1
    if k % 8 or b.shape[n_dim] % 8:
        raise ValueError(f"K and N must be multiples of 8 (K={k}, N={b.shape[n_dim]})")
    if b_layout == "kn":
        if b.shape[0] != bsz or b.shape[1] != k:
            raise ValueError(f"b {tuple(b.shape)} does not match a {tuple(a.shape)} as [B, K, N]")
        n = b.shape[2]
        bt = b.transpose(1, 2)  # [B, N, K]
        if _mat_layout(bt) is not None:
            bmat, b_kn = bt, 0
        else:
            bmat, b_kn = (b if _mat_layout(b) is not None else b.contiguous()), 1
    elif b_layout == "nk":
        if b.shape[0] != bsz or b.shape[2] != k:
            raise ValueError(f"b {tuple(b.shape)} does not match a {tuple(a.shape)} as [B, N, K]")
        n = b.shape[1]
        bmat, b_kn = (b if _mat_layout(b) is not None else b.contiguous()), 0
    else:
        raise ValueError("b_layout must be 'kn' or 'nk'")
    if b.device != a.device:
        raise ValueError("a and b must be on the same device")
    if _mat_layout(a) is None:
        a = a.contiguous()
    if bias is not None:
        _require_cuda("bias", bias, 1, dtype)
        if bias.shape[0] != n:
            raise ValueError(f"bias has {bias.shape[0]} entries, expected {n}")
    dev = a.device
    if out is None:
        out = torch.empty((bsz, m, n), dtype=dtype, device=dev)
    elif (out.dtype != dtype or tuple(out.shape) != (bsz, m, n) or not out.is_contiguous()):
        raise ValueError(f"out must be a contiguous {dtype} [{bsz}, {m}, {n}] tensor")
    if mode != N.MODE_OFF:
        if report is None:
            report = ReportBuffer(DEFAULT_CAPACITY, dev, batch=bsz)
        elif report.batch < bsz:
            raise ValueError(f"the report holds counters for {report.batch} batches, the call has {bsz}")

    try:
        return _bmm_call(a, bmat, b_kn, bias, out, bsz, m, n, k, mode, tile_n, tile_m, swap_ab, thr_scale, thr_abs,
                         inject, report, num_sms)
    except N.AbftError as e:
        # Strides the tensor-map encoder rejects (e.g. heads interleaved
        # along rows): the call queued no device work; run on packed copies.
        if e.code != -2 or (a.is_contiguous() and bmat.is_contiguous()):
            raise
        return _bmm_call(a.contiguous(), bmat.contiguous(), b_kn, bias, out, bsz, m, n, k, mode, tile_n, tile_m,
                         swap_ab, thr_scale, thr_abs, inject, report, num_sms)


def _bmm_call(a, bmat, b_kn, bias, out, bsz, m, n, k, mode, tile_n, tile_m, swap_ab, thr_scale, thr_abs, inject,
              report, num_sms):
    dev = a.device
    inj = inject if isinstance(inject, DeviceFaults) else (DeviceFaults(inject, dev) if inject else None)
    lda, sa = _mat_layout(a)
    ldb, sb = _mat_layout(bmat)
    args = N.GemmArgs()
    args.A, args.B, args.C, args.bias = _ptr(a), _ptr(bmat), _ptr(out), _ptr(bias)
    args.M, args.N, args.K = m, n, k
    args.lda, args.ldb, args.ldc = lda, ldb, max(n, 1)
    args.batch, args.b_kn = bsz, b_kn
    args.stride_a, args.stride_b, args.stride_c = sa, sb, m * max(n, 1)
    args.mode = int(mode)
    args.tile_n, args.tile_m, args.swap_ab = int(tile_n), int(tile_m), int(swap_ab)
    args.thr_scale, args.thr_abs = float(thr_scale), float(thr_abs)
    args.tol_abs, args.tol_rel = 1e-2, 1e-2
    args.report = report.data_ptr() if report is not None and mode != N.MODE_OFF else None
    args.report_capacity = report.capacity if report is not None and mode != N.MODE_OFF else 0
    args.num_sms = int(num_sms)
    args.dtype = GEMM_DTYPES[a.dtype]
    if inj is not None:
        args.inject_rows, args.inject_cols, args.inject_deltas = _ptr(inj.rows), _ptr(inj.cols), _ptr(inj.deltas)
        args.n_inject = inj.n
    _run_gemm(args, dev, (m, n, k, int(mode), int(tile_n), int(tile_m), int(swap_ab), True, int(num_sms), bsz,
                          b_kn, args.dtype))
    return out, (report if mode != N.MODE_OFF else None)


CHECK_DTYPES = {torch.bfloat16: N.DTYPE_BF16, torch.float16: N.DTYPE_F16, torch.float32: N.DTYPE_F32}


def check_only(
    a: torch.Tensor,
    b: torch.Tensor,
    c: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    *,
    b_layout: str = "kn",
    tol_abs: float = 1e-2,
    tol_rel: float = 1e-2,
    locate: bool = False,
    bf16_sums: bool = False,
    thr_scale: float = DEFAULT_THR_SCALE,
    report: Optional[ReportBuffer] = None,
) -> ReportBuffer:
    """Check an existing ``c`` against ``a`` and ``b`` (no GEMM).

    Operands are CUDA tensors of one type: bfloat16, float16 or float32 (the
    types the reference's native checker dispatches on).
    ``b_layout="kn"``: b is [K, N] (the reference checker's b_2d);
    ``b_layout="nk"``: b is an nn.Linear weight [N, K] (no transpose copy).
    Fills report.corner / sum_c / abs_err / rel_err / ref_ok; ``bf16_sums``
    rounds the intermediates to the operands' type (bf16 or fp16) like the
    reference's python backend on tensors of that type; ``locate`` also
    records mismatching rows and columns.
    """
    dtype = a.dtype
    if dtype not in CHECK_DTYPES:
        raise ValueError(f"check_only takes bfloat16, float16 or float32 operands, got {dtype}")
    for name, t in (("a", a), ("c", c)):
        if not t.is_cuda or t.dtype != dtype or t.dim() != 2 or t.stride(-1) != 1:
            raise ValueError(f"{name} must be a 2-D CUDA {dtype} tensor with unit stride in its last dimension")
    if b.dim() != 2 or not b.is_cuda or b.dtype != dtype:
        raise ValueError(f"b must be a 2-D CUDA {dtype} tensor")
    m, k = a.shape
    if b_layout == "kn":
        kn = 1
        if b.shape[0] != k:
            raise ValueError("b [K, N] does not match a")
        n = b.shape[1]
    elif b_layout == "nk":
        kn = 0
        if b.shape[1] != k:
            raise ValueError("b [N, K] does not match a")
        n = b.shape[0]
    else:
        raise ValueError("b_layout must be 'kn' or 'nk'")
    if b.stride(1) != 1:
        b = b.contiguous()
    if tuple(c.shape) != (m, n):
        raise ValueError(f"c must be [{m}, {n}]")
    if bias is not None and (not bias.is_cuda or bias.dtype != dtype or bias.dim() != 1 or bias.stride(0) != 1):
        raise ValueError(f"bias must be a contiguous 1-D CUDA {dtype} tensor")
    dev = a.device
    if report is None:
        report = ReportBuffer(DEFAULT_CAPACITY, dev)
    args = N.CheckArgs()
    args.dtype = CHECK_DTYPES[dtype]
    args.A, args.B, args.C, args.bias = _ptr(a), _ptr(b), _ptr(c), _ptr(bias)
    args.M, args.N, args.K = m, n, k
    args.lda, args.ldb, args.ldc = a.stride(0), b.stride(0), c.stride(0)
    args.b_kn = kn
    args.flags = (N.CHECK_LOCATE if locate else 0) | (N.CHECK_BF16_SUMS if bf16_sums else 0)
    args.tol_abs, args.tol_rel, args.thr_scale = float(tol_abs), float(tol_rel), float(thr_scale)
    args.report, args.report_capacity = report.data_ptr(), report.capacity
    L = N.lib()
    with torch.cuda.device(dev):
        ws_bytes = int(L.abft_check_workspace_bytes(ctypes.byref(args)))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        args.workspace, args.workspace_bytes = _ptr(ws), ws_bytes
        rc = L.abft_check_only(ctypes.byref(args), _stream(dev))
    N.check("abft_check_only", rc)
    ws.record_stream(torch.cuda.current_stream(dev))
    return report


def wait_selftest(device: Optional[torch.device] = None) -> FaultReport:
    """Run the library's bounded-wait self-test on ``device`` (default: the
    current one) and return its report: ``device_timeout`` set and
    ``n_faults`` 2 when both test waits gave up after their limit, as they
    must. Takes about 4 s; synchronises the device."""
    dev = torch.device("cuda", _device_index(device))
    rep = ReportBuffer(0, dev)
    with torch.cuda.device(dev):
        N.check("abft_wait_selftest", N.lib().abft_wait_selftest(ctypes.c_void_p(rep.data_ptr()), _stream(dev)))
    return rep.read()


def flops(m: int, n: int, k: int) -> float:
    return 2.0 * m * n * k


def thr_k(thr_scale: float, k: int) -> float:
    return float(thr_scale) * math.sqrt(k)
