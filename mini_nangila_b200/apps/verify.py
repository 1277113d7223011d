"""One-command verification run (scripts/verify.sh): regenerate the
verification artifacts and check each against the reference's committed
result.

    python -m mini_nangila_b200.apps.verify [--out verification] [--skip-tests] [--gpu] [--quick]

Steps, with the reference's artifact names:

1. tests             ``tests.txt``  (``pytest -m "not gpu"``; ``--gpu`` runs the GPU tests too)
2. determinism hash  ``determinism_hash.txt``  must be the reference's Q8.23 hash
3. AI throughput     ``ai_throughput.txt``     INT4 ratio above 8x minus headers
4. HPC bench         ``hpc_bench.txt``         ratio 2.00x, max error within eps
5. topology          ``topology.txt``          30 % drop mask of 124 bytes, bincode round trip
6. rotor twin        ``rotor.txt``             3 s at 50 Hz, ratio 1.50x
7. device codecs     ``device_codecs.txt``     (``--gpu``) ``.nz`` bytes of the sm_100a pipeline
                                                equal to the host library's, for every codec

Writes ``checks.json`` (one entry per step: ok and the figures checked) and
exits non-zero when a check fails.  ``--quick`` shrinks the two benches.
"""
from __future__ import annotations

import argparse
import contextlib
import io
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
# verification/determinism_hash.txt of the reference
REFERENCE_HASH = "c18cd836f0cb712247e0ace683d710b8550f3e3f40a6a2998252df59498aab56"


def _capture(path: str, fn, *args):
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        out = fn(*args)
    with open(path, "w") as fh:
        fh.write(buf.getvalue())
    return out


def step_tests(out_dir: str, gpu: bool) -> dict:
    tests = os.path.join(ROOT, "tests")
    if not os.path.isdir(tests):
        return {"ok": True, "skipped": "no tests directory next to the package"}
    marker = [] if gpu else ["-m", "not gpu"]
    r = subprocess.run([sys.executable, "-m", "pytest", tests, "-q", *marker], cwd=ROOT, capture_output=True,
                       text=True)
    with open(os.path.join(out_dir, "tests.txt"), "w") as fh:
        fh.write(r.stdout + r.stderr)
    tail = (r.stdout.strip().splitlines() or [""])[-1]
    return {"ok": r.returncode == 0, "summary": tail}


def step_hash(out_dir: str) -> dict:
    from . import determinism_hash

    h = _capture(os.path.join(out_dir, "determinism_hash.txt"), determinism_hash.main, [])
    return {"ok": h == REFERENCE_HASH, "hash": h}


def step_throughput(out_dir: str, quick: bool) -> dict:
    from . import throughput_bench

    argv = ["--dim", "65536", "--steps", "10"] if quick else []
    r = _capture(os.path.join(out_dir, "ai_throughput.txt"), throughput_bench.main, argv)
    # INT4 packs two codes per byte: 8x less the 4-byte scale per step
    return {"ok": r["ratio"] > 7.9, "ratio": round(r["ratio"], 3), "MBps": round(r["mb_s"], 1)}


def step_hpc(out_dir: str, quick: bool) -> dict:
    from . import hpc_compress_bench

    argv = ["--particles", "20000", "--steps", "20"] if quick else []
    r = _capture(os.path.join(out_dir, "hpc_bench.txt"), hpc_compress_bench.main, argv)
    return {"ok": bool(r["ok"]) and abs(r["ratio"] - 2.0) < 0.01, "ratio": round(r["ratio"], 4),
            "max_abs_err": r["max_abs_err"], "MBps": round(r["mb_s"], 1)}


def step_topology(out_dir: str) -> dict:
    from ..core import TopologyMask
    from . import topology_calibration

    path = os.path.join(out_dir, "topology_mask.bin")
    m = _capture(os.path.join(out_dir, "topology.txt"), topology_calibration.main, ["--output", path])
    b = open(path, "rb").read()
    back = TopologyMask.from_bytes(b)
    return {"ok": len(b) == 124 and back.to_bytes() == b and len(m.driver_indices) == 9, "mask_bytes": len(b),
            "drivers": len(m.driver_indices)}


def step_rotor(out_dir: str) -> dict:
    from . import rotor_twin

    ratio, rms = _capture(os.path.join(out_dir, "rotor.txt"), rotor_twin.main,
                          ["--duration", "3", "--rate-hz", "50", "--no-sleep"])
    return {"ok": abs(ratio - 1.5) < 0.01 and rms < 0.05, "ratio": round(ratio, 4), "rms_err": round(rms, 5)}


def step_device_codecs(out_dir: str) -> dict:
    import torch

    from ..checkpoint import lammps, nzcp
    from ..ops import trajectory

    x = lammps.generate_brownian(20000, 12, seed=3)
    lines, ok = [], True
    for codec in ("eb", "rle", "bs", "bsrle"):
        host_blob, _ = nzcp.compress(x, x.shape[1], x.shape[0], codec, 1e-3)
        dev_blob, _ = trajectory.compress(torch.from_numpy(np.ascontiguousarray(x)).cuda(), codec, 1e-3)
        same = host_blob == dev_blob
        ok &= same
        lines.append(f"{codec}: host {len(host_blob)} B, device {len(dev_blob)} B, identical={same}")
    with open(os.path.join(out_dir, "device_codecs.txt"), "w") as fh:
        fh.write("\n".join(lines) + "\n")
    return {"ok": ok, "codecs": lines}


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", default="verification")
    ap.add_argument("--skip-tests", action="store_true")
    ap.add_argument("--gpu", action="store_true", help="also run the GPU tests and the device codec check")
    ap.add_argument("--quick", action="store_true", help="smaller AI and HPC benches")
    a = ap.parse_args(argv)
    os.makedirs(a.out, exist_ok=True)
    steps = [
        ("tests", lambda: {"ok": True, "skipped": "--skip-tests"} if a.skip_tests else step_tests(a.out, a.gpu)),
        ("determinism_hash", lambda: step_hash(a.out)),
        ("ai_throughput", lambda: step_throughput(a.out, a.quick)),
        ("hpc_bench", lambda: step_hpc(a.out, a.quick)),
        ("topology", lambda: step_topology(a.out)),
        ("rotor", lambda: step_rotor(a.out)),
    ]
    if a.gpu:
        steps.append(("device_codecs", lambda: step_device_codecs(a.out)))
    checks = {}
    for i, (name, fn) in enumerate(steps, 1):
        print(f"[{i}/{len(steps)}] {name}", flush=True)
        checks[name] = fn()
        print(f"      {'ok' if checks[name]['ok'] else 'FAILED'}  "
              f"{ {k: v for k, v in checks[name].items() if k != 'ok'} }", flush=True)
    with open(os.path.join(a.out, "checks.json"), "w") as fh:
        json.dump(checks, fh, indent=1)
    print(f"Verification outputs in {a.out}/")
    if not all(c["ok"] for c in checks.values()):
        raise SystemExit(1)
    return checks


if __name__ == "__main__":
    main()
