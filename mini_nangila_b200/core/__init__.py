"""Core abstractions: Q8.23 math, Predictor/Quantizer interfaces, the
runtime-switchable UnifiedQuantizer and the TopologyMask (nangila-math,
nangila-core, nangila-edge)."""
from .fixed_point import FRACTIONAL_BITS, FixedPointBuffer, FixedPointError, FixedQ, ShapeMismatch
from .predictor import Predictor, PredictorError
from .quantizer import Quantizer
from .topology import TopologyMask
from .unified import ErrorBounded, QuantizationMode, Stochastic, TopK, UnifiedQuantizer

__all__ = [
    "FRACTIONAL_BITS", "FixedPointBuffer", "FixedPointError", "FixedQ", "ShapeMismatch", "Predictor",
    "PredictorError", "Quantizer", "TopologyMask", "ErrorBounded", "QuantizationMode", "Stochastic", "TopK",
    "UnifiedQuantizer",
]
