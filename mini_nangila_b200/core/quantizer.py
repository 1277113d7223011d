"""Quantizer interface (nangila-core/src/quantizer.rs:9-12).

``quantize(residual) -> (bytes, scale)`` and ``dequantize(bytes, scale)``.
Stochastic quantizers keep a deterministic counter PRNG so the same inputs
give the same bytes on every platform.
"""
from __future__ import annotations

from typing import Protocol, runtime_checkable

import numpy as np
import torch

from .fixed_point import FixedPointBuffer


@runtime_checkable
class Quantizer(Protocol):
    """``quantize(residual) -> (bytes, scale)`` and ``dequantize(bytes, scale)``
    (nangila-core/src/quantizer.rs:3-12)."""
    def quantize(self, residual: FixedPointBuffer) -> tuple[bytes, float]:
        ...

    def dequantize(self, compressed, scale: float) -> FixedPointBuffer:
        ...


def as_u8(b) -> np.ndarray:
    """bytes-like / numpy / torch uint8 -> contiguous numpy uint8 (no copy when possible)."""
    if isinstance(b, torch.Tensor):
        return b.detach().cpu().contiguous().view(torch.uint8).numpy()
    if isinstance(b, np.ndarray):
        return np.ascontiguousarray(b.view(np.uint8).reshape(-1))
    return np.frombuffer(bytes(b), dtype=np.uint8)


def to_bytes(a) -> bytes:
    """numpy array or bytes-like -> ``bytes``."""
    return a.tobytes() if isinstance(a, np.ndarray) else bytes(a)


def host_i32(r: FixedPointBuffer) -> np.ndarray:
    """The buffer's Q8.23 values as a host int32 array."""
    return r.data.cpu().numpy()
