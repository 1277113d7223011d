"""HPC compression benchmark (examples/hpc_compress_bench/src/main.rs):
100k particles x 100 steps of cos(0.1 t + 0.01 i) + (i % 100) 1e-4 through
the LinearPredictor + ErrorBounded(1e-3) closed loop; ratio, max error, MB/s.
``--device cuda`` runs the fused sm_100a step kernel."""
from __future__ import annotations

import argparse
import time

from ..checkpoint import lammps, nzcp


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--particles", type=int, default=100_000)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--epsilon", type=float, default=1e-3)
    ap.add_argument("--device", default="cpu")
    a = ap.parse_args(argv)
    print("Running Mini-Nangila HPC Compression Benchmark (Mock LAMMPS)")
    data = lammps.generate_synthetic(a.particles, a.steps)
    t0 = time.perf_counter()
    if a.device.startswith("cuda"):
        import torch

        from ..ops import trajectory

        x = torch.from_numpy(data).to(a.device).view(a.steps, a.particles)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _, stats = trajectory.compress(x, "eb", a.epsilon)
    else:
        _, stats = nzcp.compress(data, a.particles, a.steps, "eb", a.epsilon)
    dt = time.perf_counter() - t0
    raw = stats["total_raw"]
    comp = stats["total_comp"] - 4 * a.steps  # the reference counts payload + f32 scale per step
    print("--------------------------------------------------")
    print("Benchmark Complete")
    print(f"Total Raw Data: {raw / 2**20:.2f} MB")
    print(f"Total Compressed: {comp / 2**20:.2f} MB")
    print(f"Final Compression Ratio: {raw / comp:.2f}x")
    print(f"Max Absolute Error: {stats['max_abs_err']:.6f}")
    print(f"Throughput: {raw / 2**20 / dt:.2f} MB/s")
    ok = stats["max_abs_err"] <= a.epsilon + 1e-5
    print("SUCCESS: Error bound respected." if ok else "FAILURE: Error bound violated!")
    return {"ratio": raw / comp, "max_abs_err": stats["max_abs_err"], "mb_s": raw / 2**20 / dt, "ok": ok}


if __name__ == "__main__":
    main()
