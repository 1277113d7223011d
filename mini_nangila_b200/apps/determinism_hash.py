"""Q8.23 determinism hash (nangila-math/examples/determinism_hash.rs:4-11).

    python -m mini_nangila_b200.apps.determinism_hash [--device cuda]

SHA-256 of the little-endian i32 Q8.23 encodings of 13 rationals, printed as
``Q823_HASH <hex>``; the conversion runs in the C++ host library or, with
``--device cuda``, in the sm_100a conversion kernel.  Any platform that
follows the Q8.23 rounding rules prints the same digest.
"""
from __future__ import annotations

import argparse
import hashlib

import numpy as np

VALUES = [0.0, 1.0, -1.0, 0.5, -0.5, 0.25, -0.25, 0.75, -0.75, 1.25, -1.25, 127.0, -128.0]


def digest(device: str = "cpu") -> str:
    x = np.asarray(VALUES, np.float32)
    if device == "cpu":
        from .._ext import host

        q = np.asarray(host().q823_from_f32(x), np.int32)
    else:
        import torch

        from .._ext import cuda

        q = cuda().q823_from_f32(torch.from_numpy(x).to(device)).cpu().numpy()
    return hashlib.sha256(q.astype("<i4").tobytes()).hexdigest()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--device", default="cpu")
    a = ap.parse_args(argv)
    h = digest(a.device)
    print(f"Q823_HASH {h}")
    return h


if __name__ == "__main__":
    main()
