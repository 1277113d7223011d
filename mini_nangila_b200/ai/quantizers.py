"""AI-domain quantizers (nangila-ai/src/quantizer.rs, topk.rs): thin wrappers
over ``UnifiedQuantizer``."""
from __future__ import annotations

import warnings

from ..core.unified import Stochastic, TopK, UnifiedQuantizer


class StochasticQuantizer:
    """Stochastic INT4 (0.5 byte per value) with the hash counter PRNG."""

    def __init__(self, seed: int):
        self.inner = UnifiedQuantizer(Stochastic(seed=seed, bits=4))

    def quantize(self, residual):
        return self.inner.quantize(residual)

    def dequantize(self, compressed, scale, device=None):
        return self.inner.dequantize(compressed, scale, device)


class RefCellQuantizer(StochasticQuantizer):
    """Deprecated alias kept for compatibility: stochastic INT8."""

    def __init__(self, seed: int):
        warnings.warn("RefCellQuantizer is deprecated; use StochasticQuantizer", DeprecationWarning, stacklevel=2)
        self.inner = UnifiedQuantizer(Stochastic(seed=seed, bits=8))


class TopKQuantizer:
    """Keep the top k fraction by magnitude: ``[u32 n][u32 mask][i8...]``."""

    def __init__(self, k_percent: float):
        self.inner = UnifiedQuantizer(TopK(k_percent=k_percent))

    def quantize(self, residual):
        return self.inner.quantize(residual)

    def dequantize(self, compressed, scale, device=None):
        return self.inner.dequantize(compressed, scale, device)
