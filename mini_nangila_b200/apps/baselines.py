"""Compression baselines on a LAMMPS trajectory dump
(benchmarks/run_baselines.sh, benchmarks/plot_baselines.py).

    python -m mini_nangila_b200.apps.baselines [--data large.dump] [--results-dir baseline_results]
        [--particles 100000] [--steps 100] [--device cpu|cuda|both] [--plot]

Compresses one LAMMPS ASCII dump (generated with the reference's synthetic
writer when ``--data`` does not exist) with

* the general-purpose compressors of the reference script: gzip -1, -6 and
  -9, bzip2 and xz, through Python's zlib/gzip, bz2 and lzma modules (the
  same formats and levels as the command-line tools);
* this package's ``.nz`` codecs with the LinearPredictor closed loop:
  EB, EB+RLE, EB+BlockSparse and EB+BlockSparse+RLE at eps = 1e-3, EB and
  EB+RLE at eps = 1e-2, on the host library (``--device cpu``, single
  thread like the reference's binary), on the GPU pipeline (``cuda``), or
  both;
* SZ and ZFP when ``SZ_CMD`` / ``ZFP_CMD`` hold a command template with
  ``{in}``, ``{out}`` and ``{eps}`` placeholders (eps 1e-3); a run that
  leaves no output file is recorded as SKIPPED.

Ratio = dump bytes / compressed file bytes.  Time = wall clock of the whole
tool run: read the input, compress, write the output (the ``.nz`` rows
include parsing the dump, as the reference times its ``lammps-compress``
binary); ``codec_time_s`` is the compression alone.  Throughput = dump MiB
per second.  Writes ``baseline_comparison.txt`` and
``baseline_comparison.csv`` (the reference's columns ``tool, epsilon,
codec, compressed_bytes, ratio, comp_time_s, throughput_MBps, status`` plus
``codec_time_s`` and ``device``) into the results directory; ``--plot``
also writes ``baseline_comparison.png``.
"""
from __future__ import annotations

import argparse
import bz2
import csv
import gzip
import lzma
import os
import shlex
import subprocess
import time

import numpy as np

from ..checkpoint import lammps, nzcp

CSV_FIELDS = ["tool", "epsilon", "codec", "compressed_bytes", "ratio", "comp_time_s", "throughput_MBps", "status",
              "codec_time_s", "device"]
MIB = 1048576.0

GENERAL = [
    ("gzip -1 (fast)", "gz1", lambda b: gzip.compress(b, compresslevel=1, mtime=0)),
    ("gzip -6 (default)", "gz6", lambda b: gzip.compress(b, compresslevel=6, mtime=0)),
    ("gzip -9 (best)", "gz9", lambda b: gzip.compress(b, compresslevel=9, mtime=0)),
    ("bzip2", "bz2", lambda b: bz2.compress(b, 9)),
    ("xz", "xz", lambda b: lzma.compress(b, preset=6)),
]
# (codec key, label used in the tool name and codec column, epsilon)
NZ_RUNS = [
    ("eb", "EB", 1e-3),
    ("rle", "EB+RLE", 1e-3),
    ("bs", "BlockSparse", 1e-3),
    ("bsrle", "BlockSparse+RLE", 1e-3),
    ("eb", "EB", 1e-2),
    ("rle", "EB+RLE", 1e-2),
]
SUFFIX = {"eb": "", "rle": ".rle", "bs": ".bs", "bsrle": ".bsrle"}


def _row(tool, eps, codec, nbytes, orig, total_s, codec_s, status="OK", device=""):
    ok = status == "OK" and nbytes > 0 and total_s > 0
    return {
        "tool": tool,
        "epsilon": "" if eps is None else f"{eps:g}",
        "codec": codec,
        "compressed_bytes": int(nbytes) if ok else 0,
        "ratio": f"{orig / nbytes:.2f}" if ok else "0",
        "comp_time_s": f"{total_s:.3f}" if ok else "0",
        "throughput_MBps": f"{orig / MIB / total_s:.2f}" if ok else "0",
        "status": status,
        "codec_time_s": f"{codec_s:.3f}" if ok else "0",
        "device": device,
    }


def run_general(data_path: str, out_dir: str, orig: int) -> list[dict]:
    rows = []
    base = os.path.join(out_dir, os.path.basename(data_path))
    for label, ext, fn in GENERAL:
        t0 = time.perf_counter()
        with open(data_path, "rb") as fh:
            raw = fh.read()
        t1 = time.perf_counter()
        comp = fn(raw)
        t2 = time.perf_counter()
        with open(f"{base}.{ext}", "wb") as fh:
            fh.write(comp)
        t3 = time.perf_counter()
        rows.append(_row(label, None, "", len(comp), orig, t3 - t0, t2 - t1, device="cpu"))
    return rows


def _nz_compress(data: np.ndarray, particles: int, steps: int, codec: str, eps: float, device: str):
    if device == "cuda":
        import torch

        from ..ops import trajectory

        torch.cuda.synchronize()
        t0 = time.perf_counter()
        x = torch.from_numpy(data).to("cuda").view(steps, particles)
        blob, _ = trajectory.compress(x, codec, eps)
        torch.cuda.synchronize()
        return blob, time.perf_counter() - t0
    t0 = time.perf_counter()
    blob, _ = nzcp.compress(data, particles, steps, codec, eps)
    return blob, time.perf_counter() - t0


def run_nz(data_path: str, out_dir: str, orig: int, devices: list[str]) -> list[dict]:
    rows = []
    base = os.path.join(out_dir, os.path.splitext(os.path.basename(data_path))[0] + ".nz")
    for device in devices:
        if device == "cuda":  # first CUDA use (context, module load) outside the timed runs
            import torch

            torch.zeros(1, device="cuda")
            _nz_compress(np.zeros(2 * 3, np.float32), 3, 2, "bsrle", 1e-3, "cuda")
        for codec, label, eps in NZ_RUNS:
            t0 = time.perf_counter()
            snaps = lammps.read_dump(data_path)
            particles, steps = snaps[0].size, len(snaps)
            data = np.concatenate(snaps)
            blob, codec_s = _nz_compress(data, particles, steps, codec, eps, device)
            path = f"{base}.{str(eps).replace('0.', '')}{SUFFIX[codec]}"
            with open(path, "wb") as fh:
                fh.write(blob)
            total = time.perf_counter() - t0
            tool = f"Mini-Nangila ({label})" + (" [cuda]" if device == "cuda" else "")
            rows.append(_row(tool, eps, label, len(blob), orig, total, codec_s, device=device))
    return rows


def run_external(name: str, template: str, data_path: str, out_dir: str, orig: int, eps: float = 1e-3) -> dict:
    """One SZ/ZFP run from a command template; SKIPPED when no output appears."""
    out = os.path.join(out_dir, os.path.basename(data_path) + "." + name.lower())
    if os.path.exists(out):
        os.remove(out)
    cmd = template.replace("{in}", data_path).replace("{out}", out).replace("{eps}", f"{eps:g}")
    t0 = time.perf_counter()
    try:
        subprocess.run(shlex.split(cmd), stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL, check=False)
    except OSError:
        pass
    dt = time.perf_counter() - t0
    if not os.path.isfile(out) or os.path.getsize(out) == 0:
        return _row(name, eps, "NA", 0, orig, 0.0, 0.0, status="SKIPPED")
    return _row(name, eps, "NA", os.path.getsize(out), orig, dt, dt, device="cpu")


def write_results(rows: list[dict], out_dir: str, orig: int) -> tuple[str, str]:
    txt = os.path.join(out_dir, "baseline_comparison.txt")
    csv_path = os.path.join(out_dir, "baseline_comparison.csv")
    with open(csv_path, "w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=CSV_FIELDS)
        w.writeheader()
        w.writerows(rows)
    with open(txt, "w") as fh:
        fh.write("Baseline Compression Comparison\n")
        fh.write(f"Generated: {time.strftime('%a %b %d %H:%M:%S %Z %Y')}\n")
        fh.write(f"Original size: {orig / MIB:.2f} MB ({orig} bytes)\n\n")
        for r in rows:
            if r["status"] != "OK":
                fh.write(f"{r['tool']}: {r['status']}\n\n")
                continue
            label = r["tool"] if not r["epsilon"] else f"{r['tool']} (eps={r['epsilon']})"
            fh.write(f"{label}:\n")
            fh.write(f"  Compressed size: {r['compressed_bytes'] / MIB:.2f} MB ({r['compressed_bytes']} bytes)\n")
            fh.write(f"  Compression ratio: {r['ratio']}×\n")
            fh.write(f"  Compression time: {r['comp_time_s']}s\n")
            fh.write(f"  Throughput: {r['throughput_MBps']} MB/s\n\n")
    return txt, csv_path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--data", default=os.path.join("baseline_results", "data", "large.dump"))
    ap.add_argument("--results-dir", default="baseline_results")
    ap.add_argument("--particles", type=int, default=100_000, help="atoms of a generated dump")
    ap.add_argument("--steps", type=int, default=100, help="snapshots of a generated dump")
    ap.add_argument("--device", choices=["cpu", "cuda", "both"], default="cpu")
    ap.add_argument("--skip-general", action="store_true", help="only the .nz (and SZ/ZFP) rows")
    ap.add_argument("--plot", action="store_true")
    a = ap.parse_args(argv)
    os.makedirs(a.results_dir, exist_ok=True)
    if not os.path.isfile(a.data):
        os.makedirs(os.path.dirname(a.data) or ".", exist_ok=True)
        print(f"Generating synthetic dataset {a.data} ({a.particles} atoms, {a.steps} steps)")
        lammps.write_dump(a.data, a.particles, a.steps)
    orig = os.path.getsize(a.data)
    print(f"Original file: {a.data}  Size: {orig / MIB:.2f} MB ({orig} bytes)")
    rows = [] if a.skip_general else run_general(a.data, a.results_dir, orig)
    devices = ["cpu", "cuda"] if a.device == "both" else [a.device]
    rows += run_nz(a.data, a.results_dir, orig, devices)
    for name, var in (("ZFP", "ZFP_CMD"), ("SZ", "SZ_CMD")):
        if os.environ.get(var):
            rows.append(run_external(name, os.environ[var], a.data, a.results_dir, orig))
    txt, csv_path = write_results(rows, a.results_dir, orig)
    for r in rows:
        print(f"{r['tool']:<36} eps={r['epsilon'] or '-':<6} ratio {r['ratio']:>7}x  "
              f"{r['throughput_MBps']:>9} MB/s  {r['status']}")
    print(f"Results saved to: {txt}\nCSV: {csv_path}")
    if a.plot:
        from ..utils import analysis

        try:
            print("Saved:", analysis.plot_baselines(csv_path, os.path.join(a.results_dir, "baseline_comparison.png")))
        except RuntimeError as e:
            print(e)
    return rows


if __name__ == "__main__":
    main()
