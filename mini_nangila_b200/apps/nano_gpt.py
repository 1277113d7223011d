"""Simulated NanoGPT gradient compression (examples/nano_gpt/src/main.rs):
per-layer synthetic gradients (sparsity growing with steps, early layers
noisier), a variance-calibrated topology mask (30 % passengers), Q8.23
momentum prediction and top-k 10 % residual compression; overall ratio.
Passenger layers update their predictor with the raw gradient, as the
reference does (their receivers would drift)."""
from __future__ import annotations

import argparse
import time

import numpy as np

from ..ai import MomentumPredictor
from ..core import FixedPointBuffer, QuantizationMode, TopologyMask, UnifiedQuantizer


def gradients(rng, layers, size, step, loss):
    out = []
    for layer in range(layers):
        lf = 1.0 if layer < 4 else (0.6 if layer < 8 else 0.3)
        sparsity = 0.5 + min(step / 2000.0, 0.4)
        i = np.arange(size, dtype=np.float32)
        mag = np.float32((loss / 10.0) * lf * 0.1)
        g = np.sin(np.float32(step) * np.float32(0.1) + i * np.float32(0.001)) * mag
        g = g + rng.uniform(-1, 1, size).astype(np.float32) * mag * np.float32(0.1)
        g[rng.random(size) < sparsity] = 0.0
        out.append(g.astype(np.float32))
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--num-steps", type=int, default=50)
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--hidden", type=int, default=768)
    ap.add_argument("--calibration-steps", type=int, default=20)
    ap.add_argument("--topk", type=float, default=0.10)
    ap.add_argument("--drop", type=float, default=0.30)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    rng = np.random.default_rng(a.seed)
    size = 4 * a.hidden * a.hidden
    norms = np.array([[np.linalg.norm(g) for g in gradients(rng, a.layers, size, s, 10.0 - s * 0.01)]
                      for s in range(a.calibration_steps)], np.float32)
    mask = TopologyMask.from_variance_threshold(norms.var(axis=0), a.drop)
    print(f"Topology: {len(mask.driver_indices)} drivers, {len(mask.passenger_indices)} passengers, "
          f"factor {mask.compression_factor():.2f}×")
    preds = [MomentumPredictor(0.9) for _ in range(a.layers)]
    q = UnifiedQuantizer(QuantizationMode.TopK(a.topk))
    raw = comp = 0
    t0 = time.perf_counter()
    for step in range(a.num_steps):
        loss = 10.0 * (1 - step / a.num_steps) ** 2 + 2.5 * step / a.num_steps
        for layer, g in enumerate(gradients(rng, a.layers, size, step, loss)):
            gb = FixedPointBuffer.from_f32(g)
            raw += g.size * 4
            if mask.is_passenger(layer):
                preds[layer].update(gb)
                continue
            p = preds[layer].predict()
            r = gb.clone() if p.is_empty() else gb.sub(p)
            b, s = q.quantize(r)
            comp += len(b) + 4
            d = q.dequantize(b, s)
            preds[layer].update(d if p.is_empty() else p.add(d))
    dt = time.perf_counter() - t0
    ratio = raw / max(comp, 1)
    print(f"Overall Compression: {ratio:.2f}×  ({raw / 1e9:.2f} GB raw, {dt:.1f} s)")
    print(("✓" if ratio >= 20 else "✗") + f" Compression target {'met' if ratio >= 20 else 'missed'}: {ratio:.2f}× vs 20×")
    return ratio


if __name__ == "__main__":
    main()
