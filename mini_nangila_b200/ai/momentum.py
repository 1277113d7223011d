"""EMA momentum predictor in Q8.23 (nangila-ai/src/momentum.rs).

``update`` copies the first observation, then
``state = state.mul_scalar(beta).add(obs.mul_scalar(1 - beta))`` with the
saturating fixed-point ops; ``predict`` returns the state (empty before the
first update).  Works on host and device buffers.
"""
from __future__ import annotations

import numpy as np

from ..core.fixed_point import FixedPointBuffer, ShapeMismatch
from ..core.predictor import PredictorShapeMismatch


class MomentumPredictor:
    """EMA predictor in Q8.23 (nangila-ai/src/momentum.rs:9-61): the first update copies
    the observation, later ones ``state * beta + obs * (1 - beta)`` with ``mul_scalar``."""
    def __init__(self, beta: float):
        self.beta = float(np.float32(beta))
        self._state: FixedPointBuffer | None = None

    def predict(self) -> FixedPointBuffer:
        if self._state is None:
            return FixedPointBuffer.new(0)
        return self._state.clone()

    def update(self, observation: FixedPointBuffer) -> None:
        if self._state is None:
            self._state = observation.clone()
            return
        decayed = self._state.mul_scalar(self.beta)
        scaled = observation.to(self._state.device).mul_scalar(float(np.float32(1.0) - np.float32(self.beta)))
        try:
            self._state = decayed.add(scaled)
        except ShapeMismatch as e:
            raise PredictorShapeMismatch(str(e)) from e

    def reset(self) -> None:
        self._state = None

    def state_dict(self) -> dict:
        return {"beta": self.beta, "state": None if self._state is None else self._state.data.cpu().clone()}

    def load_state_dict(self, sd: dict, device=None) -> None:
        self.beta = sd["beta"]
        self._state = None if sd["state"] is None else FixedPointBuffer(sd["state"].to(device or "cpu"))
