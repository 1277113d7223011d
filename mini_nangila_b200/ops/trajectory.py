"""Device ``.nz`` trajectory pipeline (examples/lammps_compress on the GPU).

``compress`` runs the LinearPredictor closed loop for every snapshot on the
device (one fused kernel per step plus the codec's packer, no host sync
between steps) and assembles a ``.nz`` image byte-identical to the host
library's.  ``decompress`` decodes all steps' payloads in parallel and
applies the predictor add-back chain on the device.
"""
from __future__ import annotations

import struct

import numpy as np
import torch

from .._ext import cuda
from ..checkpoint.nzcp import CODECS, NzHeader, read_header


def encode_steps(x: torch.Tensor, codec, epsilon: float):
    """x: [steps, particles] fp32 CUDA.  Returns (payloads, lengths, maxerr, status) on the device."""
    cid = CODECS[codec] if isinstance(codec, str) else int(codec)
    return cuda().nz_encode_steps(x.contiguous(), cid, float(np.float32(epsilon)))


def compress(x: torch.Tensor, codec="eb", epsilon: float = 1e-3) -> tuple[bytes, dict]:
    cid = CODECS[codec] if isinstance(codec, str) else int(codec)
    T, P = x.shape
    payload, lens, maxerr, st = encode_steps(x, cid, epsilon)
    lens_h = lens.cpu().numpy()
    if int(st[0]) != 0:
        raise RuntimeError(f"device encoder failed with status {st.cpu().tolist()}")
    scale = float(np.float32(2.0) * np.float32(epsilon))
    if cid == 2 and P == 0:
        scale = 1.0
    host = payload.cpu().numpy()
    out = bytearray(b"NZCP") + struct.pack("<BBII", 1, cid, P, T)
    for t in range(T):
        out += struct.pack("<fI", scale, int(lens_h[t]))
        out += host[t, : int(lens_h[t])].tobytes()
    stats = {"total_raw": T * P * 4, "total_comp": int(lens_h.sum()) + 8 * T, "max_abs_err": float(maxerr.item())}
    return bytes(out), stats


def decompress(b: bytes, device="cuda") -> torch.Tensor:
    """Decode an ``.nz`` image to fp32 values [steps, particles] on ``device``
    (reconstructed values: the predictor add-back runs on the device)."""
    h: NzHeader = read_header(b)
    off = 14
    spans, scales = [], []
    for _ in range(h.steps):
        scale, n = struct.unpack_from("<fI", b, off)
        spans.append(bytes(b[off + 8: off + 8 + n]))
        scales.append(scale)
        off += 8 + n
    offs = np.zeros(h.steps + 1, np.int64)
    offs[1:] = np.cumsum([len(x) for x in spans])
    data = torch.frombuffer(bytearray(b"".join(spans)) or bytearray(1), dtype=torch.uint8).to(device)
    sc = torch.tensor(scales or [1.0], dtype=torch.float32, device=device)
    out = cuda().nz_decode_steps(data, torch.from_numpy(offs).to(device), sc, h.codec, h.particles)
    return out.view(h.steps, h.particles)
