"""Linear extrapolation predictor (nangila-hpc/src/linear.rs):
``predict = s_t + (s_t - s_{t-1})`` with saturating Q8.23 ops; one snapshot
predicts itself; none predicts an empty buffer."""
from __future__ import annotations

from ..core.fixed_point import FixedPointBuffer, ShapeMismatch
from ..core.predictor import PredictorShapeMismatch


class LinearPredictor:
    """``2 s_t - s_{t-1}`` extrapolation (nangila-hpc/src/linear.rs:10-57)."""
    def __init__(self):
        self.s_t: FixedPointBuffer | None = None
        self.s_t_minus_1: FixedPointBuffer | None = None

    def predict(self) -> FixedPointBuffer:
        if self.s_t is not None and self.s_t_minus_1 is not None:
            try:
                return self.s_t.add(self.s_t.sub(self.s_t_minus_1))
            except ShapeMismatch as e:
                raise PredictorShapeMismatch(str(e)) from e
        if self.s_t is not None:
            return self.s_t.clone()
        return FixedPointBuffer.new(0)

    def update(self, observation: FixedPointBuffer) -> None:
        self.s_t_minus_1 = self.s_t
        self.s_t = observation.clone()

    def reset(self) -> None:
        self.s_t = None
        self.s_t_minus_1 = None
