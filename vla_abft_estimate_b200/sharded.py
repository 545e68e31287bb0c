"""N-sharded checksum-protected GEMM over torch.distributed (NCCL on NVLink).

The reference has no distributed code; this is the multi-GPU mode of the
fused GEMM. With P ranks, A[M, K] is replicated and B[N, K] (nn.Linear
layout, i.e. the columns of C) is split into P contiguous shards; rank r
computes C[:, cols_r] = A B_r^T with the fused kernel and its own per-tile
checksums, so the data path has no collective. The one exchange per call is
an ``all_gather`` of every rank's fixed-size fault reports (64-byte header +
records per call, batched over a ring of calls), after which each rank
holds the job-wide fault list with global column indices.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _native as N
from . import ops


def shard_bounds(n: int, world: int, rank: int, align: int = 8) -> Tuple[int, int]:
    """[start, end) of rank's column shard: near-equal, multiples of ``align``."""
    if n % align:
        raise ValueError(f"N={n} must be a multiple of {align}")
    units = n // align
    base, extra = divmod(units, world)
    start = (rank * base + min(rank, extra)) * align
    size = (base + (1 if rank < extra else 0)) * align
    return start, start + size


@dataclass
class GlobalFaultReport:
    """Job-wide view merged from every rank's report."""

    status: int = 0
    n_faults: int = 0
    n_located: int = 0
    n_corrected: int = 0
    overflow: int = 0
    per_rank: List[N.FaultReport] = field(default_factory=list)
    records: List[N.FaultRecord] = field(default_factory=list)  # columns made global

    def coords(self) -> List[tuple]:
        return sorted((r.row, r.col) for r in self.records)


def merge_reports(buffers: Sequence[bytes], col_offsets: Sequence[int]) -> GlobalFaultReport:
    """Merge per-rank report bytes; local columns become global (col + offset)."""
    out = GlobalFaultReport()
    for buf, off in zip(buffers, col_offsets):
        rep = N.FaultReport.from_bytes(bytes(buf))
        out.per_rank.append(rep)
        out.status |= rep.status
        out.n_faults += rep.n_faults
        out.n_located += rep.n_located
        out.n_corrected += rep.n_corrected
        out.overflow += rep.overflow
        for r in rep.records:
            out.records.append(N.FaultRecord(r.row, r.col + off if r.col >= 0 else -1, r.residual, r.residual_w,
                                             r.threshold, r.flags))
    return out


def gather_reports(report: torch.Tensor, out: torch.Tensor, group=None) -> None:
    """All-gather one uint8 report buffer per rank into ``out`` [world, nbytes].

    NCCL gathers into the flat buffer in one call; other backends (gloo on
    CPU) gather into per-rank views.
    """
    world = out.shape[0]
    if world == 1 or not dist.is_initialized():
        out[0].copy_(report)
        return
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out.view(-1), report, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), report, group=group)


class ShardedAbftGemm:
    """One rank's part of C = A B^T with B split by columns across the group.

    ``weight_shard`` is this rank's rows of B ([N_r, K], bf16, on this rank's
    GPU); ``col_offset`` the global index of its first column. Checksums of
    the shard are encoded once. ``__call__(a)`` runs the fused kernel, which
    detects, locates and corrects faults on its own; its fault report goes
    to the next slot of a ring of ``exchange_every`` reports, and the ring
    is all-gathered in one collective when it is full (or when the call
    passes ``gather=True``; ``exchange()`` forces it). With the default
    ``exchange_every=1`` every call ends with the exchange. A larger ring
    amortises the collective's latency over several GEMMs, e.g. the linears
    of one forward. Every rank must make the same calls in the same order.
    """

    def __init__(self, weight_shard: torch.Tensor, col_offset: int, *, group=None,
                 mode: int = N.MODE_DETECT | N.MODE_CORRECT, tile_n: int = 0, capacity: int = 64,
                 thr_scale: float = ops.DEFAULT_THR_SCALE, exchange_every: int = 1):
        if exchange_every < 1:
            raise ValueError("exchange_every must be at least 1")
        self.weight = weight_shard
        self.col_offset = int(col_offset)
        self.group = group
        self.mode = mode
        self.thr_scale = thr_scale
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.device = weight_shard.device
        self.tile_n = tile_n
        self.checksums = None
        self.capacity = capacity
        self.slots = int(exchange_every)
        self._next = 0   # ring slot of the next call
        self._used = 0   # slots holding reports at the last exchange
        checked = mode != N.MODE_OFF
        nbytes = int(N.lib().abft_report_bytes(capacity)) if checked else 0
        nbytes = (nbytes + 15) // 16 * 16  # every slot 16-byte aligned
        self.ring = torch.zeros((self.slots, nbytes), dtype=torch.uint8, device=self.device)
        self._reports = [ops.ReportBuffer(capacity, self.device, tensor=self.ring[i]) for i in range(self.slots)] \
            if checked else []
        self.gathered = torch.zeros((self.world, self.slots, nbytes), dtype=torch.uint8, device=self.device)
        offs = torch.tensor([self.col_offset], dtype=torch.int64, device=self.device)
        self.col_offsets = [self.col_offset]
        if self.world > 1:
            all_offs = torch.zeros(self.world, dtype=torch.int64, device=self.device)
            dist.all_gather_into_tensor(all_offs, offs, group=group)
            self.col_offsets = [int(x) for x in all_offs.cpu()]

    @property
    def report(self) -> Optional[ops.ReportBuffer]:
        """The report slot the last call wrote (None with checks off)."""
        if not self._reports:
            return None
        return self._reports[(self._next - 1) % self.slots]

    def _checksums_for(self, m: int) -> Tuple[int, Optional[torch.Tensor]]:
        tile_n = self.tile_n or ops.pick_tile_n(m, self.weight.shape[0], self.weight.shape[1], self.device, self.mode)
        if self.mode & (N.MODE_DETECT | N.MODE_CORRECT):
            if self.checksums is None or self.checksums[0] != tile_n:
                self.checksums = (tile_n, ops.encode_weight(self.weight, tile_n))
            return tile_n, self.checksums[1]
        return tile_n, None

    def __call__(self, a: torch.Tensor, *, out: Optional[torch.Tensor] = None,
                 inject: Optional[Sequence[Tuple[int, int, float]]] = None,
                 gather: Optional[bool] = None) -> torch.Tensor:
        """``gather``: True exchanges after this call, False never (the slot
        is kept for a later exchange; a full ring then wraps), None when the
        ring is full."""
        tile_n, cks = self._checksums_for(a.shape[0])
        rep = None
        if self._reports:
            if self._next == self.slots:  # a full ring that was not exchanged: start over
                self._next = 0
            rep = self._reports[self._next]
            self._next += 1
        out, _ = ops.abft_gemm(a, self.weight, mode=self.mode, tile_n=tile_n, checksums=cks, inject=inject,
                               report=rep, out=out, thr_scale=self.thr_scale)
        if rep is not None and (gather or (gather is None and self._next == self.slots)):
            self.exchange()
        return out

    def exchange(self) -> None:
        """All-gather the ring (one collective, fixed size) and start a new one."""
        if not self._reports:
            return
        gather_reports(self.ring.view(-1), self.gathered.view(self.world, -1), self.group)
        self._used = self._next
        self._next = 0

    def global_reports(self) -> List[GlobalFaultReport]:
        """Host view of the last exchange: one job-wide report per call, in
        call order (one device->host copy)."""
        rows = self.gathered.cpu().numpy()
        return [merge_reports([rows[r, s].tobytes() for r in range(self.world)], self.col_offsets)
                for s in range(self._used)]

    def global_report(self) -> GlobalFaultReport:
        """The job-wide report of the last call before the last exchange."""
        reps = self.global_reports()
        return reps[-1] if reps else GlobalFaultReport()
