"""Runtime-switchable quantizer (nangila-core/src/unified_quantizer.rs).

Modes and their wire formats (bit-exact with the reference):

* ``Stochastic(seed, bits)``: global scale ``max|x| / ((2^bits - 1) / 2)``
  (``max/7.5`` for INT4); stochastic rounding with the counter PRNG
  ``fmix64(seed ^ counter)`` (one counter step per element, persistent across
  calls); INT4 packs element 2i in the high nibble, INT8 one byte each;
  other widths fall back to deterministic INT8.
* ``ErrorBounded(epsilon)``: INT16 little-endian, ``round(x / 2eps)``.
* ``TopK(k_percent)``: ``[u32 n]`` then per 32-element block ``[u32 mask]``
  and one int8 ``round(x / (max/127))`` per set bit; the threshold is the
  ``floor(n*k)``-th largest ``|x|`` and ties are all kept.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .._ext import host
from .fixed_point import FixedPointBuffer
from .quantizer import as_u8, host_i32, to_bytes


@dataclass(frozen=True)
class Stochastic:
    """Stochastic INT4/INT8 with the fmix64 counter PRNG (unified_quantizer.rs:171-250)."""
    seed: int = 0
    bits: int = 4


@dataclass(frozen=True)
class ErrorBounded:
    """INT16 codes with scale 2 * epsilon (unified_quantizer.rs:253-279)."""
    epsilon: float = 1e-3


@dataclass(frozen=True)
class TopK:
    """Keep the |x| >= k-th largest, ``[u32 n]`` + per-32 masks + int8 (unified_quantizer.rs:285-375)."""
    k_percent: float = 0.1


class QuantizationMode:
    """Namespace mirroring the Rust enum: ``QuantizationMode.Stochastic(...)``."""

    Stochastic = Stochastic
    ErrorBounded = ErrorBounded
    TopK = TopK


def _rust_exp2(x: float) -> str:
    m, e = f"{x:.2e}".split("e")
    return f"{m}e{int(e)}"


def _dev_codecs():
    from ..ops import codecs

    return codecs


class UnifiedQuantizer:
    """One quantizer whose mode switches at runtime (nangila-core/src/unified_quantizer.rs:68-166).

    The stochastic mode's counter persists across calls and restarts at 0 on
    ``set_mode``; element i of a call uses counter (elements quantized before) + i.
    CUDA residuals are quantized by the sm_100a kernels (same bytes)."""
    def __init__(self, mode):
        self._mode = mode
        self._counter = 0  # persistent PRNG counter of the stochastic mode

    @property
    def counter(self) -> int:
        return self._counter

    def mode(self):
        return self._mode

    def set_mode(self, mode) -> None:
        """Switch modes at runtime; the stochastic counter restarts at 0."""
        self._mode = mode
        self._counter = 0

    def mode_description(self) -> str:
        m = self._mode
        if isinstance(m, Stochastic):
            return f"Stochastic (seed={m.seed}, bits={m.bits})"
        if isinstance(m, ErrorBounded):
            return f"ErrorBounded (ε={_rust_exp2(float(np.float32(m.epsilon)))})"
        return f"TopK (k={float(np.float32(m.k_percent) * np.float32(100.0)):.1f}%)"

    def quantize(self, residual: FixedPointBuffer):
        m = self._mode
        if residual.data.is_cuda:
            return self._quantize_device(residual)
        q = host_i32(residual)
        if isinstance(m, Stochastic):
            b, s, self._counter = host().stochastic_quantize(q, int(m.bits), int(m.seed) & 0xFFFFFFFFFFFFFFFF,
                                                             self._counter)
            return to_bytes(b), float(s)
        if isinstance(m, ErrorBounded):
            b, s = host().eb_quantize(q, float(np.float32(m.epsilon)))
            return to_bytes(b), float(s)
        b, s = host().topk_quantize(q, float(np.float32(m.k_percent)))
        return to_bytes(b), float(s)

    def dequantize(self, compressed, scale: float, device=None) -> FixedPointBuffer:
        m = self._mode
        b = as_u8(compressed)
        if device is not None and str(device).startswith("cuda"):
            return self._dequantize_device(b, scale, device)
        s = float(np.float32(scale))
        if isinstance(m, Stochastic):
            return FixedPointBuffer(host().stochastic_dequantize(b, s, int(m.bits)))
        if isinstance(m, ErrorBounded):
            return FixedPointBuffer(host().eb_dequantize(b, s))
        return FixedPointBuffer(host().topk_dequantize(b, s))

    # ---- device paths (sm_100a kernels); same bytes as the host paths
    def _quantize_device(self, residual: FixedPointBuffer):
        m = self._mode
        c = _dev_codecs()
        if isinstance(m, Stochastic):
            b, s = c.stochastic_quantize(residual.data, int(m.bits), int(m.seed), self._counter)
            if int(m.bits) in (4, 8):  # other widths round deterministically (no PRNG draws)
                self._counter += residual.len()
            return b, s
        if isinstance(m, ErrorBounded):
            return c.eb_quantize(residual.data, float(np.float32(m.epsilon)))
        return c.topk_quantize(residual.data, float(np.float32(m.k_percent)))

    def _dequantize_device(self, b: np.ndarray, scale: float, device) -> FixedPointBuffer:
        import torch

        m = self._mode
        c = _dev_codecs()
        t = torch.from_numpy(np.require(b, requirements="W")).to(device)  # bytes-backed arrays are read-only
        if isinstance(m, Stochastic):
            return FixedPointBuffer(c.stochastic_dequantize(t, float(scale), int(m.bits)))
        if isinstance(m, ErrorBounded):
            return FixedPointBuffer(c.eb_dequantize(t, float(scale)))
        return FixedPointBuffer(c.topk_dequantize(t, float(scale)))
