"""Per-step training log in the reference trainer's CSV layout.

``TrainLog`` writes ``ts,step,loss,lr,tokens_per_sec,step_ms`` rows (the
header of python/nangila_ddp/train_nano.py:150-151, so the reference's plot
scripts read our logs) from rank 0 only.  ``StepTimer`` measures one step's
duration: CUDA events on the current stream for a CUDA device (the device
time of the queued work, read when the step's loss is read anyway), a
monotonic host clock otherwise.

Used by the app trainers (``apps.train_nano``, ``apps.minigpt_train``,
``apps.loss_curves``) and by ``DDPTrainer.fit``.
"""
from __future__ import annotations

import os
import time

import torch

HEADER = "ts,step,loss,lr,tokens_per_sec,step_ms"


class TrainLog:
    """Append-only CSV of training steps; a no-op unless ``enabled``."""

    def __init__(self, path: str | None, enabled: bool = True, echo_every: int = 0):
        self.path = path if (path and enabled) else None
        self.echo_every = int(echo_every)
        self.rows: list[tuple] = []
        if self.path:
            d = os.path.dirname(self.path)
            if d:
                os.makedirs(d, exist_ok=True)
            with open(self.path, "w") as fh:
                fh.write(HEADER + "\n")

    def row(self, step: int, loss: float, lr: float, tokens: int, step_ms: float) -> None:
        tps = tokens / max(step_ms / 1000.0, 1e-9)
        rec = (time.time(), int(step), float(loss), float(lr), tps, float(step_ms))
        self.rows.append(rec)
        if self.path:
            with open(self.path, "a") as fh:
                fh.write(f"{rec[0]:.6f},{rec[1]},{rec[2]:.6f},{rec[3]},{rec[4]:.2f},{rec[5]:.2f}\n")
        if self.echo_every and step % self.echo_every == 0:
            print(f"step {step} loss {loss:.4f} tps {tps:.1f} tokens/s", flush=True)


class StepTimer:
    """Duration of one step: CUDA events on the device, else a host clock."""

    def __init__(self, device: torch.device):
        self.cuda = device.type == "cuda"
        self._t0 = 0.0
        if self.cuda:
            self._s = torch.cuda.Event(enable_timing=True)
            self._e = torch.cuda.Event(enable_timing=True)

    def start(self) -> None:
        if self.cuda:
            self._s.record()
        else:
            self._t0 = time.perf_counter()

    def stop_ms(self) -> float:
        """Milliseconds since ``start`` (waits for the step on CUDA)."""
        if self.cuda:
            self._e.record()
            self._e.synchronize()
            return float(self._s.elapsed_time(self._e))
        return (time.perf_counter() - self._t0) * 1000.0
