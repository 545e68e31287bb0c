"""libabft_b200.so on the host: it loads, exports every declared entry point,
its structs match ctypes, and it validates arguments without a GPU."""
import ctypes
import re
import shutil
import subprocess

import pytest

from vla_abft_estimate_b200 import _build
from vla_abft_estimate_b200 import _native as N

HEADER = _build.INCLUDE_DIR / "abft_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*[\w\s\*]+?\b(abft_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_binding_symbols():
    assert declared_functions() == sorted(N.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    L = N.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    assert L.abft_version() == N.LIB_VERSION == 5


def test_status_strings():
    assert N.status_string(0) == "ok"
    assert "alignment" in N.status_string(-2)
    assert N.status_string(12345) == "unknown status"


def test_host_only_helpers():
    L = N.lib()
    assert L.abft_report_bytes(0) == 64
    assert L.abft_report_bytes(10) == 64 + 10 * 24
    assert L.abft_report_bytes_batched(10, 1) == 64 + 10 * 24
    assert L.abft_report_bytes_batched(10, 32) == 64 + 10 * 24 + 32 * 16  # counters after the records
    # 34 pair tiles with stream-K beat 140 narrow tiles in one wave (bench.py --tile-grid: 34.9 vs 38.9 us)
    assert L.abft_pick_tile_n(512, 4096, 4096, 148, 3) == 256
    assert L.abft_pick_tile_m(512, 4096, 4096, 148, 3, 256) == 256
    assert L.abft_pick_tile_n(256, 4096, 1024, 148, 3) == 128  # ViT-L MLP: narrow tiles stay faster
    assert L.abft_pick_tile_m(512, 4608, 3584, 148, 3, 256) == 256  # 38 pair tiles beat 39 x 4 narrow ones
    assert L.abft_pick_tile_m(8192, 8192, 8192, 148, 3, 256) == 256
    assert L.abft_pick_tile_m(1024, 1024, 1024, 148, 3, 128) == 128  # 128-wide pairs run only on request
    assert L.abft_pick_tile_n(8192, 8192, 8192, 148, 3) == 256
    assert L.abft_pick_tile_n(4096, 4096, 4096, 148, 0) == 256  # 4 waves of 256 beat 7 waves of 128
    assert L.abft_pick_tile_n(512, 37888, 3584, 148, 0) == 256  # 592 tiles: exactly 4 waves
    assert L.abft_pick_tile_n(512, 37888, 3584, 148, 3) == 256  # 4 waves + a stream-K tail
    assert L.abft_pick_tile_n(1024, 1024, 64, 148, 0) == 128  # one k-block: nothing to stream
    assert L.abft_checksum_bytes(4096, 4096, 256) == 17 * 8 * 4096 * 2  # ceil(4096/248) tiles
    assert L.abft_checksum_bytes(4096, 4096, 128) == 35 * 8 * 4096 * 2  # ceil(4096/120) tiles
    assert L.abft_checksum_bytes(4096, 4096, 64) == 0
    assert L.abft_gemm_plan(None, None) == -1


def test_gemm_argument_validation_without_gpu():
    L = N.lib()
    assert L.abft_gemm_bf16(None, None) == -1
    a = N.GemmArgs()
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -1  # null operands
    a.A, a.B, a.C = 0x10000, 0x20000, 0x30000
    a.M, a.N, a.K, a.lda, a.ldb, a.ldc = 128, 256, 72, 72, 72, 256
    a.K = 70
    a.lda = a.ldb = 70
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -2  # K % 8
    a.K = a.lda = a.ldb = 72
    a.A = 0x10008
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -2  # misaligned base
    a.A = 0x10000
    a.mode = 64
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -1  # unknown mode bit
    a.mode = N.MODE_DETECT
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -1  # checks need a report
    a.report, a.report_capacity = 0x40000, 8
    a.tile_n = 192
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -3  # tile width not built
    a.tile_n = 0
    a.n_inject = N.MAX_INJECT + 1
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -1
    a.n_inject = 0
    # batched products
    a.batch = -1
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -1
    a.batch = 4
    a.stride_a, a.stride_b, a.stride_c = 128 * 72, 256 * 72, 128 * 256
    a.stride_b += 4
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -2  # stride not a multiple of 8
    a.stride_b -= 4
    a.stride_c = 127 * 256
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -1  # C batches would overlap
    a.stride_c = 128 * 256 + 8
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -1  # not whole rows of ldc
    a.stride_c = 128 * 256
    a.mode = N.MODE_REF
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -3  # scalar check is per product only
    a.mode = N.MODE_DETECT
    a.batch = 70000
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -3
    a.batch = 4
    a.b_kn = 2
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -1
    a.b_kn = 1
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -1  # [K, ldb] needs ldb >= N (72 < 256)
    a.ldb = 256
    a.checksums = 0x50000
    assert L.abft_gemm_bf16(ctypes.byref(a), None) == -1  # an N-major B gets its checksums from the copy
    a.checksums = None
    assert L.abft_encode_weight_batched(ctypes.c_void_p(0x10000), 8, 8, 8, 12, 2, 256, ctypes.c_void_p(0x20000),
                                        None) == -2
    # valid arguments: the next step is the device query, which fails cleanly here
    import torch

    if not torch.cuda.is_available():
        assert L.abft_gemm_bf16(ctypes.byref(a), None) == -6


def test_fp16_gemm_and_typed_encode_validation_without_gpu():
    L = N.lib()
    k, n, tiles = 4096, 4096, 17
    assert L.abft_checksum_bytes_typed(n, k, 256, N.DTYPE_BF16) == L.abft_checksum_bytes(n, k, 256)
    # fp16: the same rows, then 8 float32 scale entries per tile
    assert L.abft_checksum_bytes_typed(n, k, 256, N.DTYPE_F16) == tiles * 8 * k * 2 + tiles * 8 * 4
    assert L.abft_checksum_bytes_typed(n, k, 256, N.DTYPE_F32) == 0
    assert L.abft_checksum_bytes_typed(n, k, 64, N.DTYPE_F16) == 0
    B, out = ctypes.c_void_p(0x10000), ctypes.c_void_p(0x20000)
    assert L.abft_encode_weight_typed(B, 8, 8, 8, 0, 1, 256, N.DTYPE_F32, out, None) == -3
    assert L.abft_encode_weight_typed(B, 8, 8, 8, 0, 1, 256, 7, out, None) == -1
    assert L.abft_encode_weight_typed(B, 8, 12, 16, 0, 1, 256, N.DTYPE_F16, out, None) == -2  # K % 8
    assert L.abft_encode_weight_typed(B, 8, 8, 8, 0, 1, 100, N.DTYPE_F16, out, None) == -3
    a = N.GemmArgs()
    a.A, a.B, a.C = 0x10000, 0x20000, 0x30000
    a.M, a.N, a.K, a.lda, a.ldb, a.ldc = 128, 256, 72, 72, 72, 256
    a.dtype = N.DTYPE_F32
    assert L.abft_gemm(ctypes.byref(a), None) == -3  # fp32 operands: post-hoc check only
    a.dtype = 5
    assert L.abft_gemm(ctypes.byref(a), None) == -1
    a.dtype = N.DTYPE_F16
    import torch

    if not torch.cuda.is_available():
        assert L.abft_gemm(ctypes.byref(a), None) == -6
        assert L.abft_encode_weight_typed(B, 8, 8, 8, 0, 1, 256, N.DTYPE_F16, out, None) == -6


def test_wait_selftest_validation_without_gpu():
    L = N.lib()
    assert L.abft_wait_selftest(None, None) == -1
    assert L.abft_wait_selftest(ctypes.c_void_p(0x10008), None) == -2
    import torch

    if not torch.cuda.is_available():
        assert L.abft_wait_selftest(ctypes.c_void_p(0x10000), None) == -6


def test_check_argument_validation_without_gpu():
    L = N.lib()
    c = N.CheckArgs()
    assert L.abft_check_only(ctypes.byref(c), None) == -1
    c.A, c.B, c.C, c.report = 0x10000, 0x20000, 0x30000, 0x40000
    c.M, c.N, c.K, c.lda, c.ldb, c.ldc, c.b_kn = 64, 64, 64, 64, 64, 64, 0
    c.flags = 8
    assert L.abft_check_only(ctypes.byref(c), None) == -1
    c.flags = N.CHECK_LOCATE
    c.b_kn = 2
    assert L.abft_check_only(ctypes.byref(c), None) == -1
    c.b_kn = 1
    c.ldb = 60
    assert L.abft_check_only(ctypes.byref(c), None) == -1  # ldb < N for [K, N]
    assert L.abft_encode_weight(None, 8, 8, 8, 256, None, None) == -1
    assert L.abft_encode_weight(ctypes.c_void_p(0x10000), 8, 8, 8, 100, ctypes.c_void_p(0x20000), None) == -3


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_struct_layouts_match_c(tmp_path):
    src = tmp_path / "sz.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "abft_b200.h"\n'
        "int main(void){printf(\"%zu %zu %zu %zu %zu %zu %zu %zu\\n\", sizeof(abft_gemm_args), "
        "offsetof(abft_gemm_args, report), offsetof(abft_gemm_args, batch), offsetof(abft_gemm_args, stride_c), "
        "sizeof(abft_check_args), offsetof(abft_check_args, workspace), "
        "sizeof(abft_report), sizeof(abft_fault_record));return 0;}\n")
    exe = tmp_path / "sz"
    subprocess.check_call(["gcc", f"-I{_build.INCLUDE_DIR}", str(src), "-o", str(exe)])
    vals = [int(x) for x in subprocess.check_output([str(exe)]).split()]
    assert vals == [ctypes.sizeof(N.GemmArgs), N.GemmArgs.report.offset, N.GemmArgs.batch.offset,
                    N.GemmArgs.stride_c.offset, ctypes.sizeof(N.CheckArgs), N.CheckArgs.workspace.offset,
                    N.REPORT_HEADER_BYTES, N.RECORD_BYTES]


def test_report_parsing_round_trip():
    import struct

    hdr = struct.pack("<8I4fi3I", 3, 2, 1, 1, 0, 4, 128, 248, 1.5, 2.5, 1.0, 0.4, 0, 0, 0, 0)
    rec = struct.pack("<iifffI", 7, 9, 3.0, 30.0, 0.1, 7) + struct.pack("<iifffI", 8, -1, 2.0, 5.0, 0.1, 1)
    rep = N.FaultReport.from_bytes(hdr + rec + bytes(48))
    assert rep.status == 3 and rep.n_faults == 2 and rep.tile_n == 248 and rep.ref_ok == 0
    assert rep.coords() == [(7, 9), (8, -1)]
    assert rep.records[0].corrected and not rep.records[1].located


def test_batched_report_parsing_and_views():
    """A batched report: records with rows flattened over the batch, then
    {faults, located, corrected, 0} per batch after the record slots."""
    import struct

    cap, nb, rows = 4, 3, 10
    hdr = struct.pack("<8I4fi3I", 3, 3, 2, 2, 0, cap, 128, 248, 0.0, 0.0, 0.0, 0.0, -1, nb, 0, 0)
    recs = (struct.pack("<iifffI", 12, 5, 3.0, 18.0, 0.1, 7) + struct.pack("<iifffI", 25, -1, 2.0, 5.0, 0.1, 1)
            + struct.pack("<iifffI", 3, 0, 1.0, 1.0, 0.1, 7) + bytes(24))
    counts = struct.pack("<4I", 1, 1, 1, 0) + struct.pack("<4I", 1, 1, 1, 0) + struct.pack("<4I", 1, 0, 0, 0)
    rep = N.FaultReport.from_bytes(hdr + recs + counts)
    assert rep.batch_counts == [(1, 1, 1), (1, 1, 1), (1, 0, 0)]
    v0, v1, v2 = (rep.batch_view(b, rows) for b in range(nb))
    assert [(r.row, r.col) for r in v0.records] == [(3, 0)]
    assert [(r.row, r.col) for r in v1.records] == [(2, 5)]
    assert [(r.row, r.col) for r in v2.records] == [(5, -1)]
    assert v2.status == N.STATUS_FAULT | N.STATUS_UNLOCATED and v2.n_located == 0
    assert v0.status == N.STATUS_FAULT and v0.n_corrected == 1
    # a one-product report has no counters: batch 0 carries the header counts
    single = N.FaultReport.from_bytes(struct.pack("<8I4fi3I", 1, 1, 1, 0, 0, 0, 128, 248, 0, 0, 0, 0, -1, 0, 0, 0))
    assert single.batch_counts == [] and single.batch_view(0, 5).n_faults == 1
    assert single.batch_view(1, 5).n_faults == 0
