"""On-device checks of the sigmoid step's exp and reciprocal
(tt_lazy_b200/csrc/expf_ref.cuh), built from tests/native/expf_ref_gpu_check.cu:
the Markstein reciprocal equals the IEEE reciprocal (__frcp_rn) on every
float in [1, 2^126), as does the packed pair form of 1 / (1 + e) on every e in
[0, 2^126); the device exp equals this host's glibc expf, and the vector
sigmoid the kernels use equals the reference's formula 1.0f / (1.0f +
expf(-x)) evaluated on this host, on all 2^32 floats."""
import os
import re
import shutil
import subprocess

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "tt_lazy_b200", "csrc")
NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")


def test_exp_and_sigmoid_on_device_equal_host_glibc(tmp_path):
    if not os.path.exists(NVCC) and shutil.which("nvcc") is None:
        pytest.fail("nvcc is needed to build the device check")
    exe = str(tmp_path / "expf_ref_gpu_check")
    subprocess.check_call([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-fmad=false", "-std=c++17",
                           "-Xcompiler", "-fopenmp,-ffp-contract=off", "-lgomp", "-I" + CSRC,
                           os.path.join(HERE, "native", "expf_ref_gpu_check.cu"), "-o", exe])
    out = subprocess.run([exe], check=True, capture_output=True, text=True, timeout=600).stdout
    m = re.search(r"rcp_mismatch=(\d+) rcp2_mismatch=(\d+) exp_mismatch=(\d+) sig_mismatch=(\d+) "
                  r"sig_over1ulp=(\d+) fma_variant=(\d)", out)
    assert m, out
    rcp, rcp2, exp_bad, sig_bad, sig_far, fma_variant = map(int, m.groups())
    assert rcp == 0 and rcp2 == 0, out
    if fma_variant:
        assert (exp_bad, sig_bad) == (0, 0), out
    else:  # glibc's build without FMA: 2 floats of exp, 1 of sigmoid, 1 ulp
        assert exp_bad <= 2 and sig_bad <= 1 and sig_far == 0, out
