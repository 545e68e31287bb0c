"""Fused calls captured in CUDA graphs (``torch.cuda.graph``).

A captured launch replays with the launch nonce frozen in its kernel node.
These tests replay graphs over changing inputs. Each replay must match an
eager call on the same inputs bit for bit, report included:
- stream-K shapes, where a finisher folds partials that other CTAs publish
  under the nonce;
- few-row (swapped) and batched products;
- injected faults, which must be reported once per replay and corrected;
- the post-hoc check;
- the injector's ``capture()`` over a small decoder, for a prefill forward
  and a fixed-shape decode step. Each replay's reports are recorded, and a
  weight written after the capture is flagged as stale, not corrected.
- the VLA forward as one graph, and overlapped report recording.
The last test covers the programmatic dependent launch of the fused GEMM:
a host->device copy queued right before it must still finish first.
"""
import warnings

import pytest
import torch

from vla_abft_estimate_b200 import ops
from vla_abft_estimate_b200.abft import AbftConfig, AbftInjector, AbftStatsCollector, CheapSumChecker
from vla_abft_estimate_b200.workloads import build_qwen2

pytestmark = pytest.mark.gpu

OUT_TOL = 1e-2


def _capture(fn):
    """Eager warm-up on a side stream (torch's recipe), then one capture."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out


def _records(r):
    return sorted((x.row, x.col, x.flags) for x in r.records)


def _randn(shape, seed, dev, dtype=torch.bfloat16, scale=1.0):
    g = torch.Generator(device=dev).manual_seed(seed)
    return (torch.randn(*shape, device=dev, generator=g) * scale).to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(512, 4096, 4096), (512, 4608, 3584), (1, 4608, 3584), (8, 1024, 2048)])
def test_graph_replays_match_eager(cuda_device, dtype, m, n, k):
    w = _randn((n, k), m + n + k, cuda_device, dtype, k ** -0.5)
    b = _randn((n,), 1, cuda_device, dtype, 0.02)
    if (m, n, k) == (512, 4096, 4096):
        assert ops.gemm_plan(m, n, k, dtype=dtype)["sk_units"] > 0  # a stream-K schedule
    x_static = torch.zeros(m, k, device=cuda_device, dtype=dtype)
    rep = ops.ReportBuffer(16, cuda_device)
    graph, (y, _) = _capture(lambda: ops.abft_linear(x_static, w, b, report=rep))
    for seed in range(3):
        x = _randn((m, k), seed, cuda_device, dtype)
        x_static.copy_(x)
        graph.replay()
        torch.cuda.synchronize()
        ref, ref_rep = ops.abft_linear(x, w, b)
        assert torch.equal(y, ref), f"replay {seed} differs from the eager call"
        r, rr = rep.read(), ref_rep.read()
        assert r.status == 0 and r.n_faults == 0
        assert (r.tile_m, r.tile_n) == (rr.tile_m, rr.tile_n)
    del graph


@pytest.mark.parametrize("m,n,k", [(512, 4096, 4096), (1, 4608, 3584)])
def test_graph_replays_report_and_correct_injected_faults(cuda_device, m, n, k):
    w = _randn((n, k), 5, cuda_device, scale=k ** -0.5)
    coords = [(0, 17), (m - 1, n - 3), (m // 2, n // 2), (m // 3, 1000)] if m > 1 else [(0, 17), (0, n - 3)]
    faults = ops.DeviceFaults([(r, c, 4.0) for r, c in coords], cuda_device)
    x_static = torch.zeros(m, k, device=cuda_device, dtype=torch.bfloat16)
    rep = ops.ReportBuffer(16, cuda_device)
    graph, (y, _) = _capture(lambda: ops.abft_gemm(x_static, w, inject=faults, report=rep))
    for seed in range(3):
        x = _randn((m, k), seed, cuda_device)
        x_static.copy_(x)
        graph.replay()
        torch.cuda.synchronize()
        r = rep.read()
        ref, ref_rep = ops.abft_gemm(x, w, inject=[(r_, c_, 4.0) for r_, c_ in coords])
        rr = ref_rep.read()
        assert torch.equal(y, ref)
        # every fault reported once per replay: none lost to, or kept from, another replay
        assert (r.n_faults, r.n_located, r.n_corrected, r.overflow) == (rr.n_faults, rr.n_located,
                                                                        rr.n_corrected, 0)
        assert _records(r) == _records(rr)
        assert r.coords() == sorted(coords) and r.n_corrected == len(coords)
        clean = (x.float() @ w.float().t())
        assert (y.float() - clean).abs().max().item() <= OUT_TOL * clean.abs().max().item()
    del graph


def test_graph_replays_batched_products(cuda_device):
    bsz, m, n, k = 6, 256, 1024, 128
    bmat = _randn((bsz, k, n), 9, cuda_device, scale=k ** -0.5)
    a_static = torch.zeros(bsz, m, k, device=cuda_device, dtype=torch.bfloat16)
    rep = ops.ReportBuffer(16, cuda_device, batch=bsz)
    faults = ops.DeviceFaults([(m + 3, 40, 4.0)], cuda_device)  # batch 1, row 3
    graph, (y, _) = _capture(lambda: ops.abft_bmm(a_static, bmat, inject=faults, report=rep))
    for seed in range(3):
        a = _randn((bsz, m, k), seed, cuda_device)
        a_static.copy_(a)
        graph.replay()
        torch.cuda.synchronize()
        ref, ref_rep = ops.abft_bmm(a, bmat, inject=[(m + 3, 40, 4.0)],
                                    report=ops.ReportBuffer(16, cuda_device, batch=bsz))
        r, rr = rep.read(), ref_rep.read()
        assert torch.equal(y, ref)
        assert r.coords() == rr.coords() == [(m + 3, 40)] and r.batch_counts == rr.batch_counts
    del graph


def test_graph_replays_post_hoc_check(cuda_device):
    m, n, k = 256, 512, 384
    a_static = torch.zeros(m, k, device=cuda_device, dtype=torch.bfloat16)
    b = _randn((k, n), 3, cuda_device, scale=k ** -0.5)
    c_static = torch.zeros(m, n, device=cuda_device, dtype=torch.bfloat16)
    rep = ops.ReportBuffer(16, cuda_device)
    graph, _ = _capture(lambda: ops.check_only(a_static, b, c_static, report=rep, locate=True))
    for seed in range(2):
        a = _randn((m, k), seed, cuda_device)
        c = (a.float() @ b.float()).bfloat16()
        if seed == 1:
            c[7, 11] += 50.0
        a_static.copy_(a)
        c_static.copy_(c)
        graph.replay()
        torch.cuda.synchronize()
        r = rep.read()
        rr = ops.check_only(a, b, c, locate=True).read()
        assert (r.ref_ok, r.n_faults, r.coords()) == (rr.ref_ok, rr.n_faults, rr.coords())
        assert r.corner == rr.corner and r.sum_c == rr.sum_c
        assert (r.ref_ok == 0) == (seed == 1)
    del graph


SMALL_QWEN = dict(hidden=512, inter=1536, layers=2, heads=4, kv_heads=2, head_dim=128, vocab=4096,
                  rope_theta=1000000.0, eps=1e-6)
LINEARS = 4 * SMALL_QWEN["layers"] + 1


def _injector(**kw):
    cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=False, **kw)
    stats = AbftStatsCollector()
    return AbftInjector(cfg, CheapSumChecker(cfg), stats, defer_reports=True), stats


def _ids(n, seed, dev):
    return torch.randint(0, SMALL_QWEN["vocab"], (n,), device=dev,
                         generator=torch.Generator(device=dev).manual_seed(seed))


def test_injector_capture_prefill(cuda_device):
    model = build_qwen2(SMALL_QWEN, cuda_device, seed=1)
    ids_static = _ids(128, 2, cuda_device)
    inj, stats = _injector()
    with torch.inference_mode(), inj:
        model(ids_static)  # eager: encodes the checksum blocks
        g = torch.cuda.CUDAGraph()
        with inj.capture(g) as checks:
            logits = model(ids_static)
        assert len(checks) == LINEARS
        before = stats.export_summary()["abft"]["checks_total"]
        for seed in range(2):
            ids = _ids(128, 10 + seed, cuda_device)
            ids_static.copy_(ids)
            g.replay()
            checks.record()
            eager = model(ids)
            inj.flush()
            assert torch.equal(logits, eager)
        summ = stats.export_summary()["abft"]
        assert summ["checks_total"] - before == 2 * 2 * LINEARS  # two replays, two eager forwards
        assert summ["faults"]["detected_total"] == 0 and not checks.stale_checksums
        assert checks.replays_recorded == 2
    del g


def test_injector_capture_decode_step(cuda_device):
    model = build_qwen2(SMALL_QWEN, cuda_device, seed=1)
    tokens = 128
    ids = _ids(tokens, 2, cuda_device)
    inj, stats = _injector()
    with torch.inference_mode(), inj:
        caches = model.new_caches(tokens + 16)
        model(ids, caches, 0)
        caches_eager = [c.clone() for c in caches]
        pos = torch.full((), tokens, dtype=torch.long, device=cuda_device)
        nxt = ids[-1:].clone()

        def step():
            out = model(nxt, caches, pos)
            pos.add_(1)
            return out

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()  # warm-up: writes position `tokens`, which the first replay rewrites
        torch.cuda.current_stream().wait_stream(s)
        gd = torch.cuda.CUDAGraph()
        with inj.capture(gd) as checks:
            dlogits = step()
        assert len(checks) == LINEARS
        pos.fill_(tokens)
        pos_e = torch.full((), tokens, dtype=torch.long, device=cuda_device)
        for i in range(4):
            gd.replay()
            checks.record()
            eager = model(nxt, caches_eager, pos_e)
            pos_e.add_(1)
            inj.flush()
            assert torch.equal(dlogits, eager), f"decode step {i}"
        assert int(pos.item()) == tokens + 4
        assert stats.export_summary()["abft"]["faults"]["detected_total"] == 0
    del gd


def test_injector_capture_flags_a_weight_written_after_capture(cuda_device):
    model = build_qwen2(SMALL_QWEN, cuda_device, seed=3)
    ids = _ids(128, 4, cuda_device)
    inj, stats = _injector()
    with torch.inference_mode(), inj:
        model(ids)
        g = torch.cuda.CUDAGraph()
        with inj.capture(g) as checks:
            logits = model(ids)
        g.replay()
        checks.record()
        assert not checks.stale_checksums
        good = logits.clone()
        model.layers[0].gate_up.weight.mul_(2.0)
        g.replay()
        with warnings.catch_warnings(record=True) as caught:
            warnings.simplefilter("always")
            checks.record()
        assert checks.stale_checksums
        assert any("capture the graph again" in str(w.message) for w in caught)
        # nothing was "corrected" towards the stale checksums: the replay's
        # output is the written weight's product, as an eager forward (whose
        # cache re-encodes the weight) gives it
        eager = model(ids)
        inj.flush()
        assert torch.equal(logits, eager) and not torch.equal(logits, good)
    del g


def test_injector_capture_overlapped_recording(cuda_device):
    """record(overlap=True) records each replay one call late, from pinned
    copies queued behind it; the counts match synchronous recording, and a
    stale checksum block is still reported (a non-clean report parsed from
    the host copy)."""
    import torch.nn.functional as F

    w = _randn((1024, 512), 21, cuda_device, scale=512 ** -0.5)
    bm = _randn((4, 256, 384), 22, cuda_device, scale=256 ** -0.5)
    x_static = torch.zeros(192, 512, device=cuda_device, dtype=torch.bfloat16)
    a_static = torch.zeros(4, 128, 256, device=cuda_device, dtype=torch.bfloat16)

    def fwd():
        return F.linear(x_static, w), torch.bmm(a_static, bm)

    inj, stats = _injector()
    with torch.inference_mode(), inj:
        fwd()
        g = torch.cuda.CUDAGraph()
        with inj.capture(g) as checks:
            y, z = fwd()
        assert len(checks) == 2  # the linear, and the bmm's one launch
        for seed in range(5):
            x = _randn((192, 512), 30 + seed, cuda_device)
            a = _randn((4, 128, 256), 40 + seed, cuda_device)
            x_static.copy_(x)
            a_static.copy_(a)
            g.replay()
            checks.record(overlap=True)
            assert checks.replays_recorded == seed  # one replay behind
            assert torch.equal(y, F.linear(x, w)) and torch.equal(z, torch.bmm(a, bm))
            inj.flush()
        checks.finish()
        assert checks.replays_recorded == 5
        summ = stats.export_summary()["abft"]
        # eager forward + 5 replays + 5 eager checks inside the loop, 1 linear + 4 batches each
        assert summ["checks_total"] == 11 * 5 and summ["faults"]["detected_total"] == 0
        w.mul_(2.0)
        g.replay()
        with warnings.catch_warnings(record=True) as caught:
            warnings.simplefilter("always")
            checks.record(overlap=True)
            checks.finish()
        assert checks.stale_checksums and any("capture the graph again" in str(m.message) for m in caught)
    del g


def test_injector_capture_vla_forward(cuda_device):
    """The CogACT-style VLA (2 ViT / SigLIP layers, 2 decoder layers, the
    full DiT-B head over 10 denoising steps, its 7-wide action projections
    on zero-padded copies) captured as one graph through the injector:
    every replay equals the eager checked forward and records as many
    checks."""
    from vla_abft_estimate_b200 import workloads as W

    cfg = {k: (dict(v) if isinstance(v, dict) else v) for k, v in W.COGACT.items()}
    cfg["vit"]["layers"] = cfg["siglip"]["layers"] = 2
    cfg["llm"]["layers"] = 2
    model = W.build_cogact(cfg, cuda_device)
    gen = torch.Generator(device=cuda_device).manual_seed(6)
    img = torch.randn(1, 3, 224, 224, device=cuda_device, generator=gen).bfloat16()
    text = torch.randint(0, cfg["vocab"], (cfg["text_tokens"],), device=cuda_device, generator=gen)
    noise = torch.randn(cfg["action_tokens"], cfg["action_dim"], device=cuda_device, generator=gen).bfloat16()
    inj, stats = _injector()
    with torch.inference_mode(), inj:
        eager = model(img, text, noise)
        inj.flush()
        per_forward = stats.export_summary()["abft"]["checks_total"]
        g = torch.cuda.CUDAGraph()
        with inj.capture(g) as checks:
            out = model(img, text, noise)
        for _ in range(2):
            g.replay()
            checks.record()
            assert torch.equal(out, eager)
        summ = stats.export_summary()["abft"]
        assert summ["checks_total"] == 3 * per_forward and summ["faults"]["detected_total"] == 0
    del g


def test_fused_call_right_after_host_copies_sees_the_copied_data(cuda_device):
    """The fused GEMM launches with programmatic stream serialization; a
    host->device copy queued just before it (no kernel in between) must
    still complete before the kernel reads its operand."""
    m, n, k = 512, 4096, 4096
    w = _randn((n, k), 7, cuda_device, scale=k ** -0.5)
    tile_n = ops.pick_tile_n(m, n, k, cuda_device)
    cks = ops.encode_weight(w, tile_n)
    hosts = [_randn((m, k), 50 + i, cuda_device).cpu().pin_memory() for i in range(4)]
    refs = [ops.abft_gemm(h.to(cuda_device), w, checksums=cks, tile_n=tile_n)[0] for h in hosts]
    x = torch.empty(m, k, device=cuda_device, dtype=torch.bfloat16)
    outs = []
    for rnd in range(3):
        for h in hosts:
            x.copy_(h, non_blocking=True)
            y, rep = ops.abft_gemm(x, w, checksums=cks, tile_n=tile_n)
            outs.append((y, rep))
    torch.cuda.synchronize()
    for i, (y, rep) in enumerate(outs):
        assert torch.equal(y, refs[i % len(hosts)]), f"call {i} read a stale operand"
        assert rep.read().n_faults == 0
