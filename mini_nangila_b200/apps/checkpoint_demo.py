"""Chunked error-bounded checkpoint demo (examples/checkpoint_demo/src/main.rs):
write ``--len`` values of cos(0.005 i) + (i % 100) 1e-4 in ``--chunk`` pieces
(LinearPredictor across chunks + ErrorBounded INT16), read them back, report
the max error.  HDF5 when h5py is installed, else the same layout in .npz."""
from __future__ import annotations

import argparse

import numpy as np

from ..checkpoint import hdf5


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--output", default="traj_ckpt.h5")
    ap.add_argument("--dataset", default="traj")
    ap.add_argument("--len", type=int, default=50_000)
    ap.add_argument("--chunk", type=int, default=1024)
    ap.add_argument("--epsilon", type=float, default=1e-3)
    a = ap.parse_args(argv)
    i = np.arange(a.len)
    data = (np.cos(i.astype(np.float32) * np.float32(0.01) * np.float32(0.5))
            + (i % 100).astype(np.float32) * np.float32(1e-4)).astype(np.float32)
    hdf5.write_chunked_dataset(a.output, a.dataset, data, a.chunk, a.epsilon, "ErrorBoundedINT16")
    out = hdf5.read_compressed_1d(a.output, a.dataset)
    err = float(np.abs(out - data).max())
    fmt = "hdf5" if hdf5.h5py is not None else "npz"
    print(f"Wrote {a.output} ({fmt}, dataset '{a.dataset}'), len={a.len} chunk={a.chunk} eps={a.epsilon}  "
          f"max_err={err:.6f}")
    return err


if __name__ == "__main__":
    main()
