"""The kernel's multiply-shift division (tile coordinates) on the host.

tile_coords divides tile indices by launch constants with FastDiv; this
compiles a host program against the kernel header with nvcc (no GPU needed)
and compares fast_div with integer division over edge and random cases.
"""
import subprocess

import pytest

from vla_abft_estimate_b200 import _build

PROGRAM = r"""
#include <cstdio>
#include <random>
#include "gemm_kernel.cuh"
int main() {
  std::mt19937_64 rng(7);
  const long long ds[] = {1, 2, 3, 5, 7, 16, 17, 31, 32, 33, 148, 152, 153, 255, 256, 1000, 4095, 65535,
                          65536, 1 << 20, (1 << 30) - 1, 1 << 30, 2147483647LL};
  long bad = 0, tot = 0;
  for (long long d : ds) {
    const abft::FastDiv f = abft::make_fast_div(d);
    for (int i = 0; i < 200000; ++i) {
      int n = static_cast<int>(rng() & 0x7FFFFFFF);
      if (i < 1000) n = i;
      else if (i < 2000) n = 0x7FFFFFFF - (i - 1000);
      ++tot;
      bad += abft::fast_div(n, f) != static_cast<int>(n / d);
    }
    for (long long k = 1; k < 2000 && d * k <= 0x7FFFFFFF; ++k)
      for (long long e = -1; e <= 1; ++e) {
        const long long n = d * k + e;
        if (n < 0 || n > 0x7FFFFFFF) continue;
        ++tot;
        bad += abft::fast_div(static_cast<int>(n), f) != static_cast<int>(n / d);
      }
  }
  std::printf("%ld %ld\n", tot, bad);
  return 0;
}
"""


def _have_nvcc() -> bool:
    try:
        _build._nvcc()
        return True
    except RuntimeError:
        return False


@pytest.mark.skipif(not _have_nvcc(), reason="needs nvcc")
def test_fast_div_matches_integer_division(tmp_path):
    src = tmp_path / "fd.cu"
    src.write_text(PROGRAM)
    exe = tmp_path / "fd"
    subprocess.check_call([_build._nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O2",
                           f"-I{_build.CSRC_DIR}", f"-I{_build.INCLUDE_DIR}", str(src), "-o", str(exe)])
    tot, bad = (int(x) for x in subprocess.check_output([str(exe)]).split())
    assert tot > 4_000_000 and bad == 0
