"""Checkpoint / trajectory I/O: the ``.nz`` container, LAMMPS dumps and the
chunked error-bounded checkpoint layout (nangila-checkpoint)."""
from . import hdf5, lammps, nzcp

__all__ = ["hdf5", "lammps", "nzcp"]
from . import tensor_ckpt  # noqa: E402,F401  error-bounded model/optimizer checkpoints
