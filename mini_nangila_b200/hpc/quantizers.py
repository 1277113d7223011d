"""HPC-domain error-bounded codecs (nangila-hpc): all quantize with
``q = round(x / 2eps)`` to INT16 (|err| <= eps while |q| fits), then:

* ``ErrorBoundedQuantizer``: q as little-endian i16 (error_bounded.rs);
* ``RunLengthQuantizer``: opcode stream, ``0x80+count-1`` for a run of up to
  128 zeros, ``count-1`` followed by up to 128 i16 literals (rle.rs);
* ``BlockSparseQuantizer``: ``[u32 n]`` then per 32-block ``[u32 mask]`` and an
  i16 per non-zero (block_sparse.rs);
* ``BlockSparseRleQuantizer``: ``[u32 n]`` then runs of zero-mask blocks
  ``0x80|(count-1)`` or literal runs ``count-1`` + count x ``[mask][i16...]``
  (block_sparse_rle.rs).

Device buffers (``residual.data.is_cuda``) run the sm_100a codec kernels
and produce the same bytes.
"""
from __future__ import annotations

import numpy as np

from .._ext import host
from ..core.fixed_point import FixedPointBuffer
from ..core.quantizer import as_u8, host_i32, to_bytes


def _dev():
    from ..ops import codecs

    return codecs


class _EBBase:
    """``strict=True`` raises ``QuantizerError`` instead of writing a code
    that saturated at the INT16 ends, where the error bound no longer holds
    (the reference declares ``FallbackRequired`` for this at
    nangila-hpc/src/error_bounded.rs:5-11 but clamps silently,
    :43-46)."""
    _name = ""

    def __init__(self, epsilon: float, strict: bool = False):
        self.epsilon = float(np.float32(epsilon))
        self.strict = strict

    def clamp_count(self, residual: FixedPointBuffer) -> int:
        """How many codes of ``residual`` saturate: ``round(v / 2eps)``
        (half away from zero) outside [-32768, 32767], i.e. the f32 quotient
        at or beyond 32767.5 / -32768.5.  ``v`` is the Q8.23 value as f32,
        as the quantizers see it; runs where the buffer lives."""
        import torch

        scale = np.float32(2.0) * np.float32(self.epsilon)
        x = residual.data.to(torch.float32).mul_(2.0 ** -23)
        # a divisor tensor on the buffer's device: a correctly rounded f32
        # division, as the quantizers do (a Python scalar divisor may be
        # applied as a multiply by its reciprocal)
        x = x / torch.full((1,), float(scale), dtype=torch.float32, device=x.device)
        return int(((x >= 32767.5) | (x <= -32768.5)).sum())

    def quantize(self, residual: FixedPointBuffer):
        if self.strict:
            k = self.clamp_count(residual)
            if k:
                raise QuantizerError(f"FallbackRequired: {k} of {residual.data.numel()} residuals exceed "
                                     f"the INT16 code range at epsilon={self.epsilon:g}")
        if residual.data.is_cuda:
            return getattr(_dev(), f"{self._name}_quantize")(residual.data, self.epsilon)
        b, s = getattr(host(), f"{self._name}_quantize")(host_i32(residual), self.epsilon)
        return to_bytes(b), float(s)

    def dequantize(self, compressed, scale: float, device=None) -> FixedPointBuffer:
        b = as_u8(compressed)
        if device is not None and str(device).startswith("cuda"):
            import torch

            # a writable copy: torch.from_numpy of a read-only array (bytes
            # from a file or a bytes object) is undefined if written
            w = np.require(b, requirements="W")
            return FixedPointBuffer(getattr(_dev(), f"{self._name}_dequantize")(torch.from_numpy(w).to(device),
                                                                               float(scale)))
        return FixedPointBuffer(getattr(host(), f"{self._name}_dequantize")(b, float(np.float32(scale))))


class ErrorBoundedQuantizer(_EBBase):
    """INT16 codes ``round(r / 2eps)``, little endian (nangila-hpc/src/error_bounded.rs:29-68)."""
    _name = "eb"


class RunLengthQuantizer(_EBBase):
    """EB codes as runs of zeros / literals of up to 128, no header (nangila-hpc/src/rle.rs:21-99)."""
    _name = "rle"


class BlockSparseQuantizer(_EBBase):
    """``[u32 n]`` then per 32 codes a mask and the nonzero i16 codes (nangila-hpc/src/block_sparse.rs:21-92)."""
    _name = "bs"
    block_size = 32


class BlockSparseRleQuantizer(_EBBase):
    """BlockSparse blocks grouped into zero-mask runs and literal runs (nangila-hpc/src/block_sparse_rle.rs:26-131)."""
    _name = "bsrle"
    block_size = 32


class QuantizerError(ValueError):
    """``FallbackRequired``: raised by a ``strict`` error-bounded quantizer
    when a residual is outside the INT16 code range."""


def rle_encode_i16(q) -> bytes:
    """Element RLE of raw i16 codes (the rotor twin's top-k path, rotor_twin_net client.rs:41-66)."""
    return to_bytes(host().rle_encode_i16(np.ascontiguousarray(np.asarray(q, dtype=np.int16))))


def rle_decode_i16(b) -> np.ndarray:
    """Inverse of ``rle_encode_i16``."""
    return host().rle_decode_i16(as_u8(b))
