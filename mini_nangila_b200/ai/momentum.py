"""EMA momentum predictor in Q8.23 (nangila-ai/src/momentum.rs).

``update`` copies the first observation, then
``state = state.mul_scalar(beta).add(obs.mul_scalar(1 - beta))`` with the
saturating fixed-point ops; ``predict`` returns the state (empty before the
first update).  Works on host and device buffers.
"""
from __future__ import annotations

import numpy as np
import torch

from .._ext import host
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
        omb = float(np.float32(1.0) - np.float32(self.beta))
        obs = observation.to(self._state.device)
        if self._state.device.type == "cpu":
            # the same three ops fused in one host pass
            if len(self._state) != len(obs):
                raise PredictorShapeMismatch(f"Shape mismatch: {len(self._state)} vs {len(obs)}")
            self._state = FixedPointBuffer(torch.from_numpy(host().q823_momentum_update(
                self._state.numpy(), obs.numpy(), self.beta, omb)))
            return
        decayed = self._state.mul_scalar(self.beta)
        scaled = obs.mul_scalar(omb)
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
