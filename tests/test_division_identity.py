"""The kernel scales logits by a per-row temperature with Markstein's division
by a constant (ns_device.cuh: div_by_const) instead of the divide
instruction.  This re-checks, on the CPU with the same fp32 FMA semantics,
that it equals IEEE x / t bit for bit: on a 2^24-element sample of all fp32
bit patterns for several divisors (an exhaustive 2^32 run per divisor was
done when the guard was chosen).
"""
import subprocess
from pathlib import Path

import pytest

SRC = r"""
#include <stdio.h>
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>
static float u2f(uint32_t u){float f; memcpy(&f,&u,4); return f;}
static uint32_t f2u(float f){uint32_t u; memcpy(&u,&f,4); return u;}
int main(int argc, char** argv){
  long bad = 0;
  for (int a = 1; a < argc; a++) {
    volatile float t = (float)atof(argv[a]);
    float r = 1.0f / t;
    for (uint64_t i = 0; i < (1ull << 32); i += 251) {
      float x = u2f((uint32_t)i);
      if (x != x) continue;
      float q0 = x * r, rem = fmaf(-q0, t, x), q = fmaf(rem, r, q0);
      float ax = fabsf(x), aq = fabsf(q0);
      if (!(fminf(ax, aq) >= 0x1p-60f && fmaxf(ax, aq) <= 0x1p+100f)) q = x / t;
      if (f2u(q) != f2u(x / t)) bad++;
    }
  }
  printf("%ld\n", bad);
  return bad != 0;
}
"""


def test_markstein_division_is_correctly_rounded(tmp_path: Path):
    src = tmp_path / "div.c"
    src.write_text(SRC)
    exe = tmp_path / "div"
    subprocess.run(["gcc", "-O2", "-mfma", "-ffp-contract=off", str(src), "-o", str(exe), "-lm"], check=True)
    res = subprocess.run([str(exe), "0.7", "1.3", "1e-6", "1.1", "123.456", "0.3"], capture_output=True, text=True)
    assert res.returncode == 0 and res.stdout.strip() == "0", res.stdout + res.stderr
