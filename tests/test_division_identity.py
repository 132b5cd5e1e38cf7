"""The LayerNorm kernels replace the per-element IEEE division delta / count of the
Welford mean update (segmented_rms_adaln.cu:262-265) by Markstein's correction step with
a correctly rounded reciprocal of the integer count (compile-time for the per-element
step, planned per CTA for the combine steps), and the quantizers form the row scale
absmax / qmax (convrot_quant.cu:475-478, qmax = 127 or 7) the same way.  tests/native/division_check.c
compares the two against C's IEEE division and fmaf -- every significand of two binades
of delta, both signs, every count 1..128, and a sample of the counts up to 16384."""

import shutil
import subprocess
from pathlib import Path

import pytest

SRC = Path(__file__).resolve().parent / "native" / "division_check.c"


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_markstein_step_equals_ieee_division_for_small_counts(tmp_path):
    exe = tmp_path / "division_check"
    subprocess.run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-o", str(exe), str(SRC), "-lm"],
                   check=True)
    res = subprocess.run([str(exe), "128"], capture_output=True, text=True, timeout=600)
    checked, mismatches = (int(v) for v in res.stdout.split())
    assert checked == 128 * 2 * 2 * (1 << 23)
    assert mismatches == 0
    assert res.returncode == 0
    # The combine steps divide by counts up to the row width (<= 16384 on the fast path).
    # Every significand of counts 129..16384 was checked once (5.45e11 cases, no
    # mismatch); here every 4099th significand of each.
    res = subprocess.run([str(exe), "16384", "4099", "129"], capture_output=True, text=True, timeout=600)
    checked, mismatches = (int(v) for v in res.stdout.split())
    assert checked == (16384 - 128) * 2 * 2 * ((1 << 23) // 4099 + 1)
    assert mismatches == 0
