"""GPU check of the error bound behind the 256-expert biased-sigmoid router's preselection
(router_biased.cu): the approximate sigmoid 0.5 tanh.approx(x / 2) + 0.5 and exact_sigmoid are
swept over every finite fp32 input against a double-precision sigmoid.  The kernel's margin
kErrAbs = 1e-5 must be at least twice their sum (the bias roundings are covered by the relative
term), and +-inf must give exactly 1 and 0.  The probe is compiled with nvcc for sm_100a.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
K_ERR_ABS = 1.0e-5


def test_approx_sigmoid_error_bound(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "approx_sigmoid_bound"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    "--fmad=false", f"-I{ROOT / 'include'}",
                    f"-I{ROOT / 'exfold-moe_b200' / 'csrc'}",
                    str(ROOT / "tests" / "gpu_probes" / "approx_sigmoid_bound.cu"), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    approx, exact = float(out[1]), float(out[3])
    assert approx < 4.1e-6, approx
    assert exact < 1.0e-7, exact
    assert 2.0 * (approx + exact) <= K_ERR_ABS
    assert float(out[5]) == 1.0 and float(out[6]) == 0.0
