"""Checkpoint / trajectory I/O: the ``.nz`` container, LAMMPS dumps, the
chunked error-bounded checkpoint layout (nangila-checkpoint) and
error-bounded model / optimizer state checkpoints."""
from . import hdf5, lammps, nzcp, tensor_ckpt

__all__ = ["hdf5", "lammps", "nzcp", "tensor_ckpt"]
