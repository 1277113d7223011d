"""High-ratio compression benchmark (examples/cpu_compression_bench/src/main.rs):
Top-K 5 % on 1M synthetic gradients (5 % signal spikes) and RLE on 100k
trajectory residuals that are 99 % zero.  ``--device cuda`` runs the
sm_100a radix-select top-k and RLE encoder (identical bytes)."""
from __future__ import annotations

import argparse
import time

import numpy as np

from ..ai import TopKQuantizer
from ..core import FixedPointBuffer
from ..hpc import RunLengthQuantizer


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", default="cpu")
    a = ap.parse_args(argv)
    out = {}
    print("Running Mini-Nangila CPU Compression Benchmark (High Ratio Targets)")
    print("\n[Scenario 1: AI Gradient Compression (Target: >20x)]")
    i = np.arange(1_000_000)
    ai = np.where(i % 20 == 0, np.sin(i.astype(np.float32) * np.float32(0.001)),
                  (i % 100).astype(np.float32) * np.float32(0.0001)).astype(np.float32)
    buf = FixedPointBuffer.from_f32(ai)
    if a.device.startswith("cuda"):
        buf = buf.cuda(a.device)
    q = TopKQuantizer(0.05)
    q.quantize(buf)  # warm-up (device kernels)
    t0 = time.perf_counter()
    b, _ = q.quantize(buf)
    dt = time.perf_counter() - t0
    raw, comp = ai.size * 4, len(b)
    print(f"Raw Size: {raw / 2**20:.2f} MB\nCompressed Size: {comp / 2**20:.2f} MB")
    print(f"Compression Ratio: {raw / comp:.2f}x\nThroughput: {raw / 2**20 / dt:.2f} MB/s")
    print("SUCCESS: AI Target Met (>18x)" if raw / comp > 18.0 else "FAILURE: AI Target Missed")
    out["topk"] = (raw / comp, raw / 2**20 / dt)
    print("\n[Scenario 2: HPC/Twin Trajectory (Target: >100x)]")
    j = np.arange(100_000)
    hpc = np.where(j % 100 == 0, 1.0, 0.0).astype(np.float32)
    hb = FixedPointBuffer.from_f32(hpc)
    if a.device.startswith("cuda"):
        hb = hb.cuda(a.device)
    r = RunLengthQuantizer(0.01)
    r.quantize(hb)
    t0 = time.perf_counter()
    b, _ = r.quantize(hb)
    dt = time.perf_counter() - t0
    raw, comp = hpc.size * 4, len(b)
    print(f"Raw Size: {raw / 2**20:.2f} MB\nCompressed Size: {comp / 2**20:.2f} MB")
    print(f"Compression Ratio: {raw / comp:.2f}x\nThroughput: {raw / 2**20 / dt:.2f} MB/s")
    print("SUCCESS: HPC Target Met (>50x)" if raw / comp > 50.0 else "FAILURE: HPC Target Missed")
    out["rle"] = (raw / comp, raw / 2**20 / dt)
    return out


if __name__ == "__main__":
    main()
