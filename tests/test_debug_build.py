"""The bounds-checked debug build (-DNGL_BOUNDS_CHECK, selected by
NGL_BOUNDS_CHECK=1 at build time) compiles for sm_100a: its checks record a
bounds status and leave the kernel instead of touching memory outside a
slot (no GPU needed: nvcc cross-compiles)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="needs nvcc")
@pytest.mark.parametrize("src", ["fused_kernels.cu", "codec_kernels.cu"])
def test_bounds_checked_build_compiles(src, tmp_path):
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O1", "-std=c++17", "-DNGL_DEVICE_BUILD",
           "-DNGL_BOUNDS_CHECK", "-I" + os.path.join(ROOT, "csrc"), "-c", os.path.join(ROOT, "csrc", "cuda", src),
           "-o", str(tmp_path / "k.o")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
