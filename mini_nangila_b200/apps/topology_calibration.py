"""Topology calibration (examples/topology_calibration/src/main.rs): collect
per-layer gradient-norm statistics over calibration steps, build
Driver/Passenger masks for several drop fractions and save the recommended
(30 % drop) mask in the reference's bincode layout (topology_mask.bin)."""
from __future__ import annotations

import argparse

import numpy as np

from ..core import TopologyMask


def collect(num_layers=12, steps=100, seed=0):
    rng = np.random.default_rng(seed)
    out = np.zeros((num_layers, steps), np.float32)
    for step in range(steps):
        for layer in range(num_layers):
            base = 0.5 if layer < 4 else (0.3 if layer < 8 else 0.1)
            out[layer, step] = np.float32(rng.random()) * np.float32(base) + np.float32(np.sin(step * 0.1) * 0.1)
    mean = out.mean(axis=1, keepdims=True)
    return ((out - mean) ** 2).mean(axis=1).astype(np.float32)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--layer-size", type=int, default=1024)
    ap.add_argument("--output", default="topology_mask.bin")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    print("=== Topology Calibration Example ===\n")
    v = collect(a.layers, a.steps, a.seed)
    for i, x in enumerate(v):
        print(f"  Layer {i:2d}: variance = {x:.6f}")
    for drop in (0.0, 0.2, 0.3, 0.4, 0.5):
        m = TopologyMask.from_variance_threshold(v, drop)
        print(f"Drop Percentage: {drop * 100:.0f}%")
        print(f"  Drivers: {len(m.driver_indices)} layers {m.driver_indices}")
        print(f"  Passengers: {len(m.passenger_indices)} layers {m.passenger_indices}")
        print(f"  Compression Factor: {m.compression_factor():.2f}×\n  Threshold Variance: {m.threshold:.6f}\n")
    rec = TopologyMask.from_variance_threshold(v, 0.3)
    b = rec.to_bytes()
    with open(a.output, "wb") as fh:
        fh.write(b)
    assert TopologyMask.from_bytes(b).driver_indices == rec.driver_indices
    print(f"✓ Saved recommended mask (30% drop) to {a.output}\n  Size: {len(b)} bytes")
    return rec


if __name__ == "__main__":
    main()
