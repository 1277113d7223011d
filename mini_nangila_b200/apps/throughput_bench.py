"""AI-mode throughput benchmark (examples/throughput_bench/src/main.rs):
1M-element gradients sin(0.1 t + (i % 100) 0.001) for 100 steps through the
Q8.23 momentum predictor and stochastic INT4 (global scale) closed loop;
compression ratio and MB/s of raw data.  ``--device cuda`` keeps every
buffer on the GPU (sm_100a Q8.23 and stochastic-codec kernels)."""
from __future__ import annotations

import argparse
import time

import numpy as np

from ..ai import MomentumPredictor, StochasticQuantizer
from ..core import FixedPointBuffer


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--dim", type=int, default=1024 * 1024)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--device", default="cpu")
    a = ap.parse_args(argv)
    print("Running Mini-Nangila Throughput Benchmark (AI Mode)")
    cuda = a.device.startswith("cuda")
    if cuda:
        import torch

        noise = (torch.arange(a.dim, device=a.device) % 100).float() * 0.001
    else:
        noise = (np.arange(a.dim) % 100).astype(np.float32) * np.float32(0.001)
    pred, q = MomentumPredictor(0.9), StochasticQuantizer(42)
    raw = comp = 0
    if cuda:
        torch.cuda.synchronize()
    t0 = time.perf_counter()
    for t in range(a.steps):
        phase = np.float32(t) * np.float32(0.1)
        data = (noise + float(phase)).sin() if cuda else np.sin(np.float32(phase) + noise).astype(np.float32)
        g = FixedPointBuffer.from_f32(data)
        raw += a.dim * 4
        p = pred.predict()
        r = g.clone() if p.is_empty() else g.sub(p)
        b, s = q.quantize(r)
        comp += len(b) + 4
        d = q.dequantize(b, s, device=a.device if cuda else None)
        pred.update(d if p.is_empty() else p.add(d))
        if t % 10 == 0:
            print(f"Step {t}: Compression Ratio {raw / comp:.2f}x")
    if cuda:
        torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    print("--------------------------------------------------")
    print(f"Total Raw Data: {raw / 2**20:.2f} MB\nTotal Compressed: {comp / 2**20:.2f} MB")
    print(f"Final Compression Ratio: {raw / comp:.2f}x (Target: >8x for INT4)")
    print(f"Throughput (Raw): {raw / 2**20 / dt:.2f} MB/s")
    return {"ratio": raw / comp, "mb_s": raw / 2**20 / dt}


if __name__ == "__main__":
    main()
