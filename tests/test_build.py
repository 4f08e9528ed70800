"""The compiled extension: errors raised inside it reach Python as exceptions (a broken C++ toolchain turns them
into process crashes), and every public op is exported."""

import subprocess
import sys

import pytest

from economize_b200.ops import _ext


@pytest.mark.skipif(not _ext.available(), reason="extension not built")
def test_formatted_errors_raise():
    code = ("from economize_b200 import _C\ntry:\n    _C.raise_formatted(3)\nexcept RuntimeError as e:\n"
            "    print('raised', e)\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "formatted error 3" in r.stdout


@pytest.mark.skipif(not _ext.available(), reason="extension not built")
def test_exports():
    from economize_b200 import _C

    for name in ("rmsnorm", "rope_store", "attention", "silu_mul", "linear", "linear_wq", "argmax", "greedy_accept",
                 "kv_compact", "sample", "rejection", "ngram"):
        assert hasattr(_C, name), name
