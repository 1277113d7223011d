"""The host library's fast paths (csrc/host/fast_scalar.h) return the same
bits as the scalar Rust rules (csrc/common/ngl_scalar.h): Q8.23 conversion
and EB codes over all 2^32 float bit patterns, Q8.23 -> f32 over all 2^32
integers, stochastic rounding, absmax and u64 -> f32 on 10^8 samples
(csrc/host/selftest/fast_paths.cpp, compiled with the host build's flags)."""
import os
import platform
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_fast_paths_match_the_scalar_rules(tmp_path):
    exe = str(tmp_path / "fast_paths")
    flags = ["-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fno-trapping-math", "-pthread"]
    if platform.machine() in ("x86_64", "AMD64"):
        flags.append("-march=x86-64-v2")
    src = os.path.join(ROOT, "csrc", "host", "selftest", "fast_paths.cpp")
    r = subprocess.run(["g++", *flags, "-I" + os.path.join(ROOT, "csrc"), src, "-o", exe], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    r = subprocess.run([exe], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0 and "fast paths ok" in r.stdout, r.stdout + r.stderr
