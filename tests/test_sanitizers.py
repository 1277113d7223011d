"""The C++ host library under AddressSanitizer + UndefinedBehaviorSanitizer,
and under ThreadSanitizer: csrc/host/selftest/selftest.cpp drives every codec
(round trips, truncated and garbage streams), the NZCP container,
TopologyMask bincode and the product-format oracle at sizes that split its
block-parallel loops over several host threads; any out-of-bounds access,
undefined operation or data race between those threads aborts the run."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


SRC = [os.path.join(ROOT, "csrc", "host", f) for f in ("codecs.cpp", "pipeline.cpp", "product.cpp", "lammps_io.cpp",
                                                 "hdf5_io.cpp")]
SRC.append(os.path.join(ROOT, "csrc", "host", "selftest", "selftest.cpp"))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_host_library_clean_under_asan_ubsan(tmp_path):
    exe = str(tmp_path / "selftest")
    src = SRC
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
           "-fno-omit-frame-pointer", "-I" + os.path.join(ROOT, "csrc"), *src, "-o", exe]
    b = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    if b.returncode != 0 and "asan" in (b.stderr or "").lower():
        pytest.skip("sanitizer runtime not available: " + b.stderr[-200:])
    assert b.returncode == 0, b.stderr[-2000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=1", UBSAN_OPTIONS="print_stacktrace=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    assert "selftest ok" in r.stdout


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_host_threads_race_free_under_tsan(tmp_path):
    exe = str(tmp_path / "selftest_tsan")
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fsanitize=thread", "-fno-omit-frame-pointer", "-pthread",
           "-I" + os.path.join(ROOT, "csrc"), *SRC, "-o", exe]
    b = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    if b.returncode != 0 and "tsan" in (b.stderr or "").lower():
        pytest.skip("sanitizer runtime not available: " + b.stderr[-200:])
    assert b.returncode == 0, b.stderr[-2000:]
    env = dict(os.environ, NGL_HOST_THREADS="4", TSAN_OPTIONS="halt_on_error=1:exitcode=66")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    assert "selftest ok" in r.stdout and "ThreadSanitizer" not in r.stderr


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_tsan_sees_a_race_between_host_threads(tmp_path):
    """Control for the run above: a loop that writes one shared counter from
    every parallel_for range is reported, so a clean run means something."""
    src = tmp_path / "race.cpp"
    src.write_text('#include "host/parallel.h"\n#include <cstdio>\nint main() {\n  long shared = 0;\n'
                   '  ngl::host::parallel_for(1 << 20, 1 << 16, [&](size_t lo, size_t hi) {\n'
                   '    for (size_t i = lo; i < hi; ++i) shared += 1;\n  });\n  std::printf("%ld\\n", shared);\n}\n')
    exe = str(tmp_path / "race")
    b = subprocess.run(["g++", "-std=c++17", "-O1", "-g", "-fsanitize=thread", "-pthread",
                        "-I" + os.path.join(ROOT, "csrc"), str(src), "-o", exe], capture_output=True, text=True,
                       timeout=300)
    if b.returncode != 0 and "tsan" in (b.stderr or "").lower():
        pytest.skip("sanitizer runtime not available: " + b.stderr[-200:])
    assert b.returncode == 0, b.stderr[-2000:]
    env = dict(os.environ, NGL_HOST_THREADS="4", TSAN_OPTIONS="halt_on_error=1:exitcode=66")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 66 and "ThreadSanitizer: data race" in r.stderr, (r.returncode, r.stderr[-1500:])
