"""Predictor interface (nangila-core/src/predictor.rs:4-21)."""
from __future__ import annotations

from typing import Protocol, runtime_checkable

from .fixed_point import FixedPointBuffer, FixedPointError


class PredictorError(ValueError):
    pass


class PredictorShapeMismatch(PredictorError):
    pass


@runtime_checkable
class Predictor(Protocol):
    def predict(self) -> FixedPointBuffer:
        """Prediction from the internal state (empty before any update)."""

    def update(self, observation: FixedPointBuffer) -> None:
        """Fold an observation into the state."""

    def reset(self) -> None:
        """Forget all history."""


__all__ = ["Predictor", "PredictorError", "PredictorShapeMismatch", "FixedPointError"]
