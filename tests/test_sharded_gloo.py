"""N-sharded mode's host logic on CPU ranks (gloo, world size 2).

Covers the column split, the all-gather of fixed-size fault reports and the
merge into global coordinates, and failure detection: a rank that leaves
before the exchange makes the other rank's collective fail within the
process group's timeout instead of hanging.
"""
import datetime
import os
import socket
import struct

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vla_abft_estimate_b200 import _native as N
from vla_abft_estimate_b200.sharded import gather_reports, merge_reports, shard_bounds


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def fake_report(records, capacity=4, status=None):
    n = len(records)
    st = N.STATUS_FAULT if n else 0
    if status is not None:
        st = status
    hdr = struct.pack("<8I4fi3I", st, n, sum(1 for r in records if r[1] >= 0), 0, max(n - capacity, 0), capacity,
                      128, 248, 0.0, 0.0, 0.0, 0.0, -1, 0, 0, 0)
    body = b"".join(struct.pack("<iifffI", r[0], r[1], 1.0, 2.0, 0.1, N.REC_DETECTED | (N.REC_LOCATED if r[1] >= 0
                                                                                           else 0))
                    for r in records[:capacity])
    body += bytes(N.RECORD_BYTES * (capacity - min(n, capacity)))
    return torch.frombuffer(bytearray(hdr + body), dtype=torch.uint8).clone()


def test_shard_bounds_cover_columns():
    for n, world in ((65536, 8), (8192, 3), (1000, 4), (8, 2)):
        spans = [shard_bounds(n, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert all((e - s) % 8 == 0 for s, e in spans)
    with pytest.raises(ValueError):
        shard_bounds(1001, 2, 0)


def test_merge_reports_globalizes_columns():
    reps = [fake_report([(3, 10), (7, -1)]).numpy().tobytes(), fake_report([(5, 2)]).numpy().tobytes()]
    g = merge_reports(reps, [0, 4096])
    assert g.coords() == [(3, 10), (5, 4098), (7, -1)]
    assert g.n_faults == 3 and g.n_located == 2 and g.status == N.STATUS_FAULT


def _worker(rank, world, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        n = 8192
        start, end = shard_bounds(n, world, rank)
        if mode == "leave" and rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()
            os._exit(0)  # leaves between steps, with no collective in flight
        rep = fake_report([(rank * 11, 5 + rank)] if rank == 1 else [])
        out = torch.zeros((world, rep.numel()), dtype=torch.uint8)
        offs = [shard_bounds(n, world, r)[0] for r in range(world)]
        gather_reports(rep, out, None)
        g = merge_reports([r.numpy().tobytes() for r in out], offs)
        q.put((rank, g.coords()))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, f"error:{type(e).__name__}"))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
    out = {}
    while not q.empty():
        r, v = q.get()
        out[r] = v
    return out


def test_two_rank_report_exchange():
    out = _run("ok")
    assert out == {0: [(11, 4102)], 1: [(11, 4102)]}


def test_rank_leaving_is_detected_by_timeout():
    out = _run("leave")
    assert out[1] == "left"
    assert isinstance(out.get(0), str) and out[0].startswith("error:")


def _ring_worker(rank, world, port, q):
    """ShardedAbftGemm's report ring and batched exchange, with the GEMM
    replaced by a stand-in that writes a known report (no GPU here)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        from vla_abft_estimate_b200 import sharded

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        calls = []

        def fake_gemm(a, w, *, report=None, out=None, **kw):
            step = len(calls)
            calls.append(step)
            buf = fake_report([(100 * step + rank, rank)], capacity=report.capacity)
            report.tensor[: buf.numel()].copy_(buf)
            return out, report

        sharded.ops.abft_gemm = fake_gemm
        sharded.ops.pick_tile_n = lambda *a, **k: 256
        n = 16
        c0, c1 = shard_bounds(n, world, rank)
        g = sharded.ShardedAbftGemm(torch.zeros(c1 - c0, 8, dtype=torch.bfloat16), c0, mode=N.MODE_DETECT,
                                    capacity=4, exchange_every=2)
        g.checksums = (256, None)  # no encode on the CPU
        a = torch.zeros(4, 8, dtype=torch.bfloat16)
        seen = []
        for _ in range(5):  # exchanges after calls 2 and 4 (ring full), then one forced for call 5
            g(a)
            seen.append(len(g.global_reports()))
        g.exchange()
        last = [r.coords() for r in g.global_reports()]
        q.put((rank, (seen, last)))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, f"error:{type(e).__name__}:{e}"))


def test_two_rank_report_ring_exchanged_in_batches():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ring_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
    out = {}
    while not q.empty():
        r, v = q.get()
        out[r] = v
    # after call 1 nothing is exchanged yet; calls 2 and 4 fill the ring
    want_seen = [0, 2, 2, 2, 2]
    # the forced exchange holds call 5 (step 4): rank 0 at column 0, rank 1 at column 8 + 1
    want_last = [[(400, 0), (401, 9)]]
    assert out == {0: (want_seen, want_last), 1: (want_seen, want_last)}
