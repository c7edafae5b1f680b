"""The C ABI from C: `tests/c_abi_example.c` links `libsemblend_b200.so` without
Python or torch, runs one paged copy inject on the GPU and checks it bit for
bit on the host, plus the status code of an invalid call."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

from semblend_b200 import _lib

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def test_c_caller(tmp_path):
    lib = Path(_lib.LIB_PATH).resolve()
    if not lib.exists():
        pytest.fail(f"native library not built: {lib}")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "c_abi_example"
    subprocess.run([nvcc, "-O2", "-Wno-deprecated-gpu-targets", "-o", str(exe), str(ROOT / "tests/c_abi_example.c"),
                    "-I", str(ROOT / "include"), "-L", str(lib.parent), "-lsemblend_b200",
                    "-Xlinker", f"-rpath,{lib.parent}"], check=True, capture_output=True, text=True, timeout=300)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "c abi ok" in r.stdout
