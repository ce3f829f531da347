"""The host constant that replaces the kernels' per-sample division by the
point count (``msda::points_magic`` in ``muspace_b200/csrc/msda_kernels.h``).

The kernels take the level of sample s as ``__umulhi(s, magic)`` whenever the
host returns a non-zero magic, so for every (levels, points) the C-ABI accepts
(L, P <= 4096), a non-zero magic must give floor(s / P) for every sample index
s < L * P. A small C++ program compiled against the header checks every
level boundary (s = k P - 1, k P, k P + P - 1) for every P and the largest L
that still gets a magic, and that the magic is 0 where it would not be exact.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
HEADER_DIR = REPO / "muspace_b200" / "csrc"

PROGRAM = r"""
#include <cstdint>
#include <cstdio>
#include "msda_kernels.h"

static uint32_t umulhi(uint32_t a, uint32_t b) { return static_cast<uint32_t>((uint64_t{a} * b) >> 32); }

int main() {
  long checked = 0;
  for (int p = 1; p <= 4096; ++p) {
    // the largest level count that still gets a magic, capped at the C-ABI's 4096
    const uint64_t lmax = p > 1 ? ((uint64_t{1} << 32) - 1) / (uint64_t(p) * p) : 4096;
    const int levels[3] = {1, static_cast<int>(lmax < 4096 ? lmax : 4096), 4096};
    for (int li = 0; li < 3; ++li) {
      const int l = levels[li];
      if (l < 1) continue;
      const uint32_t m = msda::points_magic(l, p);
      const bool exact_range = p > 1 && uint64_t(l) * p * p < (uint64_t{1} << 32);
      if (!exact_range) {
        if (m != 0) { std::printf("L=%d P=%d: magic %u outside the exact range\n", l, p, m); return 1; }
        continue;
      }
      if (m == 0) { std::printf("L=%d P=%d: no magic inside the exact range\n", l, p); return 1; }
      const uint32_t n = uint32_t(l) * p;
      const uint32_t step = l > 2048 ? l / 2048 : 1;
      for (uint32_t k = 0; k <= uint32_t(l); k += (k + step < uint32_t(l) ? step : 1)) {
        const uint32_t cand[3] = {k * p - 1, k * p, k * p + p - 1};
        for (uint32_t s : cand) {
          if (s >= n) continue;
          ++checked;
          if (umulhi(s, m) != s / p) {
            std::printf("L=%d P=%d s=%u: %u != %u\n", l, p, s, umulhi(s, m), s / p);
            return 1;
          }
        }
        if (k == uint32_t(l)) break;
      }
    }
  }
  std::printf("ok %ld\n", checked);
  return 0;
}
"""


def _cuda_include() -> Path | None:
    for cand in (Path("/usr/local/cuda/include"),):
        if (cand / "cuda_runtime.h").exists():
            return cand
    return None


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_points_magic_equals_the_division_for_every_sample_index(tmp_path):
    inc = _cuda_include()
    if inc is None:
        pytest.skip("cuda_runtime.h not found")
    src = tmp_path / "magic.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "magic"
    subprocess.run(["g++", "-O2", "-std=c++17", f"-I{HEADER_DIR}", f"-I{inc}", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.startswith("ok ")
