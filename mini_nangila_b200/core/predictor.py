"""Predictor interface (nangila-core/src/predictor.rs:4-21)."""
from __future__ import annotations

from typing import Protocol, runtime_checkable

from .fixed_point import FixedPointBuffer, FixedPointError


class PredictorError(ValueError):
    """Predictor failure (``NangilaError`` of nangila-core/src/predictor.rs)."""
    pass


class PredictorShapeMismatch(PredictorError):
    """An observation of another length than the predictor's state."""
    pass


@runtime_checkable
class Predictor(Protocol):
    """``predict`` / ``update`` / ``reset`` (nangila-core/src/predictor.rs:4-21)."""
    def predict(self) -> FixedPointBuffer:
        """Prediction from the internal state (empty before any update)."""

    def update(self, observation: FixedPointBuffer) -> None:
        """Fold an observation into the state."""

    def reset(self) -> None:
        """Forget all history."""


__all__ = ["Predictor", "PredictorError", "PredictorShapeMismatch", "FixedPointError"]
