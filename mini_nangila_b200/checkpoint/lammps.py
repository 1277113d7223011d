"""LAMMPS ASCII dump reader/writer and synthetic trajectories
(examples/lammps_compress/src/main.rs:311-419).

``read_dump`` returns one flattened ``[x0, y0, z0, x1, ...]`` float32 array
per ``ITEM: TIMESTEP`` block, locating the x/y/z columns by name.  Reading
and writing run in the native host library (``csrc/host/lammps_io.cpp``),
like the reference's Rust reader; malformed input raises
``DumpFormatError`` with the reference's message.
"""
from __future__ import annotations

import os

import numpy as np

from .._ext import host


class DumpFormatError(ValueError):
    """A malformed LAMMPS dump; the message is the reference reader's."""
    pass


def read_dump(path: str) -> list[np.ndarray]:
    """One flattened ``[x0, y0, z0, ...]`` snapshot per ``ITEM: TIMESTEP`` block of a dump file."""
    if not os.path.isfile(path):
        raise FileNotFoundError(path)
    try:
        return list(host().lammps_read_dump(str(path)))
    except RuntimeError as e:
        raise DumpFormatError(str(e)) from None


def read_dump_text(text: str | bytes) -> list[np.ndarray]:
    """``read_dump`` of an in-memory dump."""
    data = text.encode() if isinstance(text, str) else bytes(text)
    try:
        return list(host().lammps_read_dump_text(data))
    except RuntimeError as e:
        raise DumpFormatError(str(e)) from None


def write_dump(path: str, atoms: int, steps: int) -> None:
    """The reference's generator: cos/sin/cos(0.5) of phase 0.1 t + 0.001 i,
    six decimals, ``id type x y z`` rows."""
    host().lammps_write_dump(str(path), int(atoms), int(steps))


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
