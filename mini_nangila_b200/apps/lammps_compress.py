"""LAMMPS trajectory compression CLI (examples/lammps_compress/src/main.rs).

    python -m mini_nangila_b200.apps.lammps_compress [--input dump] [--output compressed.nz]
        [--epsilon 1e-3] [--use-rle | --use-block-sparse | --use-block-sparse-rle]
        [--particles 100000] [--steps 100] [--generate path] [--decompress] [--device cpu|cuda]

Writes the NZCP container (``b"NZCP" v1 codec particles steps`` then per step
``f32 scale, u32 nbytes, payload``) with the LinearPredictor closed loop.
``--device cuda`` runs the sm_100a pipeline (byte-identical output).
``--decompress`` reconstructs values (``--residuals`` returns the residual
stream as the reference's decoder does).
"""
from __future__ import annotations

import argparse
import time

import numpy as np

from ..checkpoint import lammps, nzcp


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--input")
    ap.add_argument("--output", default="compressed.nz")
    ap.add_argument("--decompress", action="store_true")
    ap.add_argument("--residuals", action="store_true")
    ap.add_argument("--epsilon", type=float, default=1e-3)
    ap.add_argument("--use-rle", action="store_true")
    ap.add_argument("--use-block-sparse", action="store_true")
    ap.add_argument("--use-block-sparse-rle", action="store_true")
    ap.add_argument("--particles", type=int, default=100_000)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--generate")
    ap.add_argument("--device", default="cpu")
    a = ap.parse_args(argv)
    if a.decompress:
        if a.device.startswith("cuda") and not a.residuals:
            from ..ops import trajectory

            with open(a.output, "rb") as fh:
                vals = trajectory.decompress(fh.read()).cpu().numpy().reshape(-1)
        else:
            vals = nzcp.read(a.output, add_back=not a.residuals)
        print(f"Decompressed {vals.size} values")
        return vals
    if a.generate:
        print(f"Generating synthetic LAMMPS dump: {a.generate} ({a.particles} atoms, {a.steps} steps)")
        lammps.write_dump(a.generate, a.particles, a.steps)
        print("✓ Wrote synthetic dump")
        return None
    if a.input:
        print(f"Reading LAMMPS dump: {a.input}")
        snaps = lammps.read_dump(a.input)
        if not snaps:
            raise SystemExit("No snapshots parsed from dump")
        particles, steps = snaps[0].size, len(snaps)
        data = np.concatenate(snaps)
    else:
        particles, steps = a.particles, a.steps
        data = lammps.generate_synthetic(particles, steps)
    codec = "bsrle" if a.use_block_sparse_rle else "bs" if a.use_block_sparse else "rle" if a.use_rle else "eb"
    print(f"Codec: {nzcp.CODEC_NAMES[nzcp.CODECS[codec]]} (ε = {a.epsilon:.3e})")
    t0 = time.perf_counter()
    if a.device.startswith("cuda"):
        import torch

        from ..ops import trajectory

        b, stats = trajectory.compress(torch.from_numpy(data).to(a.device).view(steps, particles), codec, a.epsilon)
    else:
        b, stats = nzcp.compress(data, particles, steps, codec, a.epsilon)
    dt = time.perf_counter() - t0
    with open(a.output, "wb") as fh:
        fh.write(b)
    ratio = stats["total_raw"] / max(1, stats["total_comp"])
    print(f"DONE  compressed={stats['total_comp'] / 1e6:.2f} MB  raw={stats['total_raw'] / 1e6:.2f} MB  "
          f"ratio={ratio:.2f}×  max_err={stats['max_abs_err']:.6f}  ({stats['total_raw'] / dt / 1e6:.1f} MB/s)")
    return stats


if __name__ == "__main__":
    main()
