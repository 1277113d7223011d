"""Closed-loop edge -> cloud sync (nangila-twin/src/edge_sync.rs).

Both ends run the same predictor.  The edge sends the quantized residual
``x - predict()`` and updates its predictor with the *reconstruction*
``predict() + dequantize(q)`` (what the cloud will see), so the two
predictors never drift.  An empty prediction (first frame) sends ``x``.
"""
from __future__ import annotations

from ..core.fixed_point import FixedPointBuffer, ShapeMismatch


class SyncError(ValueError):
    """A closed-loop step failed (shape mismatch or a malformed payload)."""
    pass


class EdgeNode:
    """Sender of the closed loop (nangila-twin/src/edge_sync.rs:29-63): predict, quantize
    the residual, and update the predictor with the reconstruction the receiver computes."""
    def __init__(self, predictor, quantizer):
        self.predictor = predictor
        self.quantizer = quantizer

    def send(self, sensor: FixedPointBuffer):
        try:
            pred = self.predictor.predict()
            residual = sensor.clone() if pred.is_empty() else sensor.sub(pred)
            compressed, scale = self.quantizer.quantize(residual)
            deq = self.quantizer.dequantize(compressed, scale)
            recon = deq if pred.is_empty() else pred.add(deq)
            self.predictor.update(recon)
        except (ShapeMismatch, ValueError) as e:
            raise SyncError(str(e)) from e
        return compressed, scale


class CloudNode:
    """Receiver of the closed loop (nangila-twin/src/edge_sync.rs:83-102); mirrors ``EdgeNode``."""
    def __init__(self, predictor, quantizer):
        self.predictor = predictor
        self.quantizer = quantizer
        self.current_state: FixedPointBuffer | None = None

    def receive(self, compressed, scale: float) -> FixedPointBuffer:
        try:
            pred = self.predictor.predict()
            residual = self.quantizer.dequantize(compressed, scale)
            recon = residual if pred.is_empty() else pred.add(residual)
            self.predictor.update(recon)
        except (ShapeMismatch, ValueError) as e:
            raise SyncError(str(e)) from e
        self.current_state = recon.clone()
        return recon
