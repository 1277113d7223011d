"""AI domain: EMA momentum predictor, stochastic INT4/INT8 and top-k
quantizers (nangila-ai)."""
from .momentum import MomentumPredictor
from .quantizers import RefCellQuantizer, StochasticQuantizer, TopKQuantizer

__all__ = ["MomentumPredictor", "RefCellQuantizer", "StochasticQuantizer", "TopKQuantizer"]
