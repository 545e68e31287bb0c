"""N-sharded mode on two GPUs over NCCL (skipped with fewer than two).

Each rank holds a column shard of B and runs the fused kernel on it; the
fault reports of a ring of two calls are all-gathered in one collective.
Bars: every rank's output shard within 1e-2 of an fp32 product, the first
call clean, the second call's fault (planted in rank 1's shard) located
at its global column and corrected, and both ranks holding the same
job-wide reports -- for bf16 and for fp16 operands.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, dtype_name, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        from vla_abft_estimate_b200.sharded import ShardedAbftGemm, shard_bounds

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        dtype = getattr(torch, dtype_name)
        m, n, k = 512, 4096, 2048
        g = torch.Generator().manual_seed(7)  # same inputs on every rank
        a = (torch.randn(m, k, generator=g) * k ** -0.5).to(dtype).to(dev)
        w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dtype)
        c0, c1 = shard_bounds(n, world, rank)
        shard = ShardedAbftGemm(w[c0:c1].contiguous().to(dev), c0, exchange_every=2)
        ref = a.float() @ w[c0:c1].to(dev).float().T
        delta = 256.0 * ref.abs().max().item()
        out1 = shard(a)
        inject = [(100, 37, delta)] if rank == 1 else None
        out2 = shard(a, inject=inject)  # fills the ring: one all-gather of both calls' reports
        torch.cuda.synchronize()
        errs = [((o.float() - ref).abs().max() / ref.abs().max()).item() for o in (out1, out2)]
        reps = shard.global_reports()
        res = {"errs": errs, "coords": [r.coords() for r in reps], "corrected": [r.n_corrected for r in reps],
               "offset_rank1": shard_bounds(n, world, 1)[0]}
        del shard
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, f"error:{type(e).__name__}:{e}"))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("dtype_name", ["bfloat16", "float16"])
def test_two_gpu_shards_and_report_ring(dtype_name):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, dtype_name, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        if p.is_alive():
            p.kill()
    out = {}
    while not q.empty():
        r, v = q.get()
        out[r] = v
    assert set(out) == {0, 1}, out
    for r in (0, 1):
        assert not isinstance(out[r], str), out[r]
        assert max(out[r]["errs"]) <= 1e-2
    off = out[0]["offset_rank1"]
    want = [[], [(100, off + 37)]]
    assert out[0]["coords"] == want and out[1]["coords"] == want
    assert out[0]["corrected"] == [0, 1] and out[1]["corrected"] == [0, 1]
