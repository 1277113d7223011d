"""LAMMPS ASCII dump reader/writer and synthetic trajectories
(examples/lammps_compress/src/main.rs:311-419).

``read_dump`` returns one flattened ``[x0, y0, z0, x1, ...]`` float32 array
per ``ITEM: TIMESTEP`` block, locating the x/y/z columns by name.
"""
from __future__ import annotations


import numpy as np

from .._ext import host


class DumpFormatError(ValueError):
    pass


def read_dump(path: str) -> list[np.ndarray]:
    snaps = []
    with open(path) as fh:
        lines = iter(fh)
        for line in lines:
            if not line.strip().startswith("ITEM: TIMESTEP"):
                continue
            next(lines, None)  # timestep value
            hdr = next(lines, "")
            if not hdr.startswith("ITEM: NUMBER OF ATOMS"):
                raise DumpFormatError("unexpected format, expected NUMBER OF ATOMS line")
            natoms = int(next(lines).strip())
            hdr = next(lines, "")
            if not hdr.startswith("ITEM: BOX BOUNDS"):
                raise DumpFormatError("unexpected format, expected BOX BOUNDS line")
            for _ in range(3):
                next(lines, None)
            hdr = next(lines, "")
            if not hdr.startswith("ITEM: ATOMS"):
                raise DumpFormatError("expected ATOMS header")
            fields = hdr.split()[2:]
            try:
                xi, yi, zi = fields.index("x"), fields.index("y"), fields.index("z")
            except ValueError:
                raise DumpFormatError("x/y/z column not found") from None
            snap = np.empty(natoms * 3, dtype=np.float32)
            for a in range(natoms):
                row = next(lines, None)
                if row is None:
                    raise DumpFormatError("unexpected EOF reading atoms")
                t = row.split()
                snap[3 * a] = np.float32(t[xi])
                snap[3 * a + 1] = np.float32(t[yi])
                snap[3 * a + 2] = np.float32(t[zi])
            snaps.append(snap)
    return snaps


def write_dump(path: str, atoms: int, steps: int) -> None:
    """The reference's generator: cos/sin/cos(0.5) of phase 0.1 t + 0.001 i."""
    with open(path, "w") as fh:
        for t in range(steps):
            fh.write(f"ITEM: TIMESTEP\n{t}\nITEM: NUMBER OF ATOMS\n{atoms}\nITEM: BOX BOUNDS xx yy zz\n")
            fh.write("0 10\n0 10\n0 10\nITEM: ATOMS id type x y z\n")
            tt = np.float32(t) * np.float32(0.1)
            ph = (tt + np.arange(atoms, dtype=np.float32) * np.float32(0.001)).astype(np.float32)
            x, y, z = np.cos(ph), np.sin(ph), np.cos(ph * np.float32(0.5))
            for i in range(atoms):
                fh.write(f"{i + 1} 1 {x[i]:.6f} {y[i]:.6f} {z[i]:.6f}\n")


def generate_synthetic(particles: int, steps: int) -> np.ndarray:
    """``cos(0.1 t + 0.01 i) + (i % 100) * 1e-4`` (reference's in-memory generator)."""
    return host().lammps_generate_synthetic(int(particles), int(steps))


def generate_brownian(atoms: int, steps: int, sigma: float = 0.01, box: float = 100.0, seed: int = 0,
                      with_velocities: bool = False):
    """1M-atom-scale trajectory generator: uniform positions in a box, a
    Gaussian displacement of ``sigma`` per step under periodic wrap; returns
    ``steps`` x (3 * atoms) positions (and N(0,1) velocities if asked)."""
    rng = np.random.default_rng(seed)
    pos = (rng.random(atoms * 3, dtype=np.float32) * np.float32(box)).astype(np.float32)
    out = np.empty((steps, atoms * 3), dtype=np.float32)
    vel = np.empty((steps, atoms * 3), dtype=np.float32) if with_velocities else None
    for t in range(steps):
        if t:
            pos = np.mod(pos + rng.standard_normal(atoms * 3, dtype=np.float32) * np.float32(sigma),
                         np.float32(box)).astype(np.float32)
        out[t] = pos
        if vel is not None:
            vel[t] = rng.standard_normal(atoms * 3, dtype=np.float32)
    return (out, vel) if with_velocities else out
