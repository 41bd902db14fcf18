"""On-device checks of the sigmoid step's exp and reciprocal
(tt_lazy_b200/csrc/exp_cr.cuh), built from tests/native/exp_cr_gpu_check.cu:
the Markstein reciprocal equals the IEEE reciprocal (__frcp_rn) on every
float in [1, 2^126); exp_cr differs from CUDA's double exp rounded to float
only by single ulps at rounding midpoints; the vector sigmoid (one range test
for several values, packed pairs) equals the scalar one, NaN and infinities
included; the packed pair reciprocal equals __frcp_rn(1 + e) on every e in
[0, 2^126)."""
import os
import re
import shutil
import subprocess

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "tt_lazy_b200", "csrc")
NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")


def test_exp_and_reciprocal_on_device(tmp_path):
    if not os.path.exists(NVCC) and shutil.which("nvcc") is None:
        pytest.fail("nvcc is needed to build the device check")
    exe = str(tmp_path / "exp_cr_gpu_check")
    subprocess.check_call([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-fmad=false", "-std=c++17",
                           "-I" + CSRC, os.path.join(HERE, "native", "exp_cr_gpu_check.cu"), "-o", exe])
    out = subprocess.run([exe], check=True, capture_output=True, text=True, timeout=300).stdout
    m = re.search(r"rcp_mismatch=(\d+) exp_mismatch=(\d+) exp_over1ulp=(\d+) vec_mismatch=(\d+) "
                  r"rcp2_mismatch=(\d+)", out)
    assert m, out
    rcp, exp_bad, exp_far, vec, rcp2 = map(int, m.groups())
    assert rcp == 0
    assert exp_far == 0
    assert exp_bad <= 32, exp_bad
    assert vec == 0
    assert rcp2 == 0
