"""CPU: the device forward's exp (csrc/kernels/expf_exact.h, yl_expf) against
the C library, over every float input.

yl_expf evaluates e^x in double precision and rounds once, so it must equal
the correctly rounded e^x. Two independent references are used: the C
library's double exp rounded to float (what the oracle uses) and, on x86, an
x87 long-double expl rounded to float. The C library's own expf (what the
reference's f32::exp calls on glibc) is within 0.502 ulp; the test records on
how many inputs it differs (by exactly one ulp) from the correctly rounded
value. The header is compiled with g++ exactly as the device compiles it
(plain IEEE double adds, multiplies and fused multiply-adds).
"""
from __future__ import annotations

import os
import platform
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HDR = ROOT / "yallma3-mini-inference_b200" / "csrc" / "kernels" / "expf_exact.h"

PROG = r"""
#include <cmath>
#include <cstdio>
#include <cstring>
#include <cstdint>
#include "expf_exact.h"
static uint32_t bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }
int main(int argc, char** argv) {
  const int use_expl = argc > 1 && argv[1][0] == '1';
  long long vs_double = 0, vs_expl = 0, glibc_off = 0, glibc_far = 0;
#pragma omp parallel for reduction(+ : vs_double, vs_expl, glibc_off, glibc_far) schedule(dynamic, 1 << 16)
  for (long long i = 0; i < (1LL << 32); ++i) {
    const uint32_t b = (uint32_t)i;
    float x;
    memcpy(&x, &b, 4);
    if (x != x) continue;
    const float ours = yl::yl_expf(x);
    const float ref = (float)exp((double)x);
    if (bits(ours) != bits(ref)) ++vs_double;
    if (use_expl && bits(ours) != bits((float)expl((long double)x))) ++vs_expl;
    const float g = expf(x);
    if (bits(g) != bits(ref)) {
      ++glibc_off;
      const uint32_t d = bits(g) > bits(ref) ? bits(g) - bits(ref) : bits(ref) - bits(g);
      if (d > 1) ++glibc_far;
    }
  }
  printf("%lld %lld %lld %lld\n", vs_double, vs_expl, glibc_off, glibc_far);
  return 0;
}
"""


@pytest.mark.timeout(900)
def test_yl_expf_is_correctly_rounded_for_every_float(tmp_path):
    src = tmp_path / "expcheck.cpp"
    src.write_text(PROG)
    exe = tmp_path / "expcheck"
    subprocess.run(["g++", "-O2", "-std=c++17", "-fopenmp", "-ffp-contract=off", f"-I{HDR.parent}", str(src),
                    "-o", str(exe), "-lm"], check=True)
    use_expl = platform.machine() in ("x86_64", "AMD64")
    env = dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count() or 1))
    out = subprocess.run([str(exe), "1" if use_expl else "0"], check=True, capture_output=True, text=True,
                         env=env).stdout.split()
    vs_double, vs_expl, glibc_off, glibc_far = map(int, out)
    print(f"yl_expf vs rounded double exp: {vs_double}; vs rounded x87 expl: {vs_expl}; "
          f"C library expf off by one ulp on {glibc_off} inputs, by more on {glibc_far}")
    assert vs_double == 0
    assert vs_expl == 0
    assert glibc_far == 0  # the library's expf is never more than one ulp away
