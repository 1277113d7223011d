"""``.nz`` trajectory container (examples/lammps_compress/src/main.rs:90-127).

Layout, little-endian::

    b"NZCP" | u8 version=1 | u8 codec | u32 particles | u32 steps
    steps x ( f32 scale | u32 nbytes | nbytes of quantizer payload )

codec 1 = ErrorBounded INT16, 2 = EB + RLE, 3 = EB + BlockSparse,
4 = EB + BlockSparse + RLE.  Each step's payload is the closed-loop
LinearPredictor residual of that snapshot.  ``read`` returns reconstructed
values by default (predictor add-back); ``add_back=False`` returns the
residual stream, which is what the reference's decoder returns.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

from .._ext import host

CODECS = {"eb": 1, "rle": 2, "bs": 3, "bsrle": 4}
CODEC_NAMES = {1: "ErrorBoundedINT16", 2: "ErrorBoundedINT16_RLE", 3: "ErrorBoundedINT16_BlockSparse",
               4: "ErrorBoundedINT16_BlockSparse_RLE"}


@dataclass
class NzHeader:
    """The 14-byte ``.nz`` header (examples/lammps_compress/src/main.rs:90-99)."""
    version: int
    codec: int
    particles: int
    steps: int


def codec_id(codec) -> int:
    """``"eb" | "rle" | "bs" | "bsrle"`` or 1-4 -> the header's codec byte."""
    if isinstance(codec, str):
        return CODECS[codec]
    return int(codec)


def compress(data, particles: int, steps: int, codec="eb", epsilon: float = 1e-3) -> tuple[bytes, dict]:
    """Compress ``steps`` snapshots of ``particles`` floats (host, single thread)."""
    d = np.ascontiguousarray(np.asarray(data, dtype=np.float32).reshape(-1))
    b, stats = host().nz_compress(d, int(particles), int(steps), codec_id(codec), float(np.float32(epsilon)))
    return b.tobytes(), dict(stats)


def read_header(b) -> NzHeader:
    """Parse the header of an ``.nz`` image (raises on a bad magic)."""
    v, c, p, s = host().nz_read_header(np.frombuffer(bytes(b[:14]), dtype=np.uint8))
    return NzHeader(v, c, p, s)


def decompress(b, add_back: bool = True) -> np.ndarray:
    """All steps of an ``.nz`` image as f32: reconstructed values, or with ``add_back=False``
    the residual stream the reference's decoder returns (main.rs:249-309)."""
    return host().nz_decompress(np.frombuffer(bytes(b), dtype=np.uint8), bool(add_back))


def write(path: str, data, particles: int, steps: int, codec="eb", epsilon: float = 1e-3) -> dict:
    """``compress`` to a file; returns the stats."""
    b, stats = compress(data, particles, steps, codec, epsilon)
    with open(path, "wb") as fh:
        fh.write(b)
    return stats


def read(path: str, add_back: bool = True) -> np.ndarray:
    """``decompress`` of a file."""
    with open(path, "rb") as fh:
        return decompress(fh.read(), add_back)


def iter_steps(b):
    """Yield (scale, payload bytes) per step of an in-memory .nz image."""
    h = read_header(b)
    off = 14
    for _ in range(h.steps):
        scale, n = struct.unpack_from("<fI", b, off)
        off += 8
        yield scale, bytes(b[off:off + n])
        off += n


def build(header: NzHeader, steps) -> bytes:
    """Assemble an .nz image from (scale, payload) pairs."""
    out = bytearray(b"NZCP")
    out += struct.pack("<BBII", header.version, header.codec, header.particles, header.steps)
    for scale, payload in steps:
        out += struct.pack("<fI", scale, len(payload))
        out += payload
    return bytes(out)
