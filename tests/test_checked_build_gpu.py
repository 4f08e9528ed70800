"""The bounds-checked build (``ECZ_CHECK=1``: module ``economize_b200._C_check``, kernels check the indices they read
from device memory and report bad ones in the status word instead of addressing memory with them). Runs the canary
and paged-cache tests on it in a child process, and checks that a committed length past the cache is reported.
Skipped when the checked variant is not built (``ECZ_CHECK=1 python setup.py build_ext --inplace --build-temp
build/check``)."""

import glob
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _checked_env():
    if not glob.glob(os.path.join(ROOT, "economize_b200", "_C_check*.so")):
        pytest.skip("the bounds-checked build is not built")
    return dict(os.environ, ECZ_CHECK="1", PYTHONPATH=ROOT)


def test_kernel_tests_pass_on_the_checked_build(cuda):
    env = _checked_env()
    proc = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-m", "gpu",
                           "tests/test_canary_gpu.py", "tests/test_paged_cache_gpu.py",
                           "tests/test_attention_options_gpu.py::test_tree_pass_options"],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-2000:]


def test_checked_build_reports_a_length_past_the_cache(cuda):
    env = _checked_env()
    script = """
import torch
from economize_b200 import ops
assert ops._ext.module_name().endswith("_C_check")
q = torch.randn(1, 1, 4, 128, device="cuda").bfloat16()
k = torch.randn(1, 2, 256, 128, device="cuda").bfloat16()
ops.require().status(0)
bad = torch.tensor([300], dtype=torch.int32, device="cuda")  # committed length past the 256-slot cache
ops.attention(q, k, k, bad, torch.ones(1, dtype=torch.int32, device="cuda"))
torch.cuda.synchronize()
print("STATUS", ops.require().status(0))
"""
    proc = subprocess.run([sys.executable, "-c", script], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    status = int(proc.stdout.split("STATUS")[-1])
    assert status & 32, proc.stdout
