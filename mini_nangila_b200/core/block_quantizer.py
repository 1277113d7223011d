"""Block-scaled stochastic INT4/INT8 quantizer (the product wire format of the
fused all-reduce, usable on its own).

Per 256-element block one fp32 scale ``absmax / 7`` (INT4) or ``/127``
(INT8) and codes ``floor(x / s + U)`` with ``U`` from Philox4x32-10 keyed by
(seed, rank) and counted by (element / 4, stream, call).  The byte stream is
``[u32 n][chunk records]`` where a chunk record holds 8 block scales then the
8 blocks' codes (element 2i in the high nibble).  Unlike the reference's
global-scale INT4 it is unbiased (no -0.5 LSB offset) and one large element
only coarsens its own block.
"""
from __future__ import annotations

import struct

import numpy as np

from .._ext import host
from .fixed_point import FixedPointBuffer
from .quantizer import as_u8


class BlockStochasticQuantizer:
    """The fused hook's per-256-block INT4/INT8 format as a standalone quantizer (see the module docstring)."""
    def __init__(self, seed: int = 0, bits: int = 4, stochastic: bool = True, rank: int = 0, stream: int = 0):
        if bits not in (4, 8):
            raise ValueError("bits must be 4 or 8")
        self.seed, self.bits, self.stochastic = int(seed), bits, stochastic
        self.rank, self.stream = int(rank), int(stream)
        self.calls = 0

    def quantize(self, residual: FixedPointBuffer):
        x = residual.to_f32()
        if not isinstance(x, np.ndarray):
            x = x.cpu().numpy()
        wire, _ = host().product_encode(np.ascontiguousarray(x, np.float32), None, None, self.bits, self.stochastic,
                                        False, self.seed & 0xFFFFFFFFFFFFFFFF, self.rank, self.stream, self.calls)
        self.calls += 1
        return struct.pack("<I", x.size) + wire.tobytes(), 1.0

    def dequantize(self, compressed, scale: float = 1.0) -> FixedPointBuffer:
        b = as_u8(compressed)
        if b.size < 4:
            return FixedPointBuffer.new(0)
        n = int(b[:4].view("<u4")[0])
        wire = np.ascontiguousarray(b[4:])
        need = host().product_wire_bytes(n, 0 if self.bits == 4 else 1, 0)
        if wire.size < need:
            raise ValueError(f"truncated block payload: {wire.size} < {need} bytes")
        vals = host().product_reduce([wire], n, self.bits, None, 1.0)
        return FixedPointBuffer.from_f32(vals)
