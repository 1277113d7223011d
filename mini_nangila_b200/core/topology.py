"""Static Driver/Passenger layer mask (nangila-core/src/topology.rs).

``from_variance_threshold`` sorts layers by variance (descending, stable),
keeps ``ceil(L * (1 - drop))`` (clamped to [1, L]) as drivers, stores sorted
index lists and the weakest driver's variance as ``threshold``.
``to_bytes``/``from_bytes`` use the bincode 1.3 default layout of the Rust
struct (u64 lengths, usize as u64, f32), e.g. 124 bytes for 12 layers.
"""
from __future__ import annotations

import numpy as np

from .._ext import host


class TopologyMask:
    """Driver / passenger split of a model's layers (nangila-core/src/topology.rs:11-163),
    backed by the C++ host library; fields and bincode bytes as the Rust struct."""
    def __init__(self, native=None):
        self._m = native if native is not None else host().TopologyMask()

    @classmethod
    def from_variance_threshold(cls, layer_variances, drop_percent: float) -> "TopologyMask":
        v = np.ascontiguousarray(np.asarray(layer_variances, dtype=np.float32))
        return cls(host().TopologyMask.from_variance_threshold(v, float(np.float32(drop_percent))))

    @classmethod
    def all_drivers(cls, num_layers: int) -> "TopologyMask":
        return cls(host().TopologyMask.all_drivers(int(num_layers)))

    @property
    def driver_indices(self) -> list[int]:
        return list(self._m.driver_indices)

    @property
    def passenger_indices(self) -> list[int]:
        return list(self._m.passenger_indices)

    @property
    def threshold(self) -> float:
        return self._m.threshold

    @property
    def total_layers(self) -> int:
        return self._m.total_layers

    def is_driver(self, layer_id: int) -> bool:
        return self._m.is_driver(int(layer_id))

    def is_passenger(self, layer_id: int) -> bool:
        return self._m.is_passenger(int(layer_id))

    def compression_factor(self) -> float:
        return self._m.compression_factor()

    def passenger_percentage(self) -> float:
        return self._m.passenger_percentage()

    def to_bytes(self) -> bytes:
        return self._m.to_bytes()

    @classmethod
    def from_bytes(cls, b: bytes) -> "TopologyMask":
        try:
            return cls(host().TopologyMask.from_bytes(bytes(b)))
        except RuntimeError as e:
            raise ValueError(str(e)) from None

    def __repr__(self) -> str:
        return (f"TopologyMask(drivers={self.driver_indices}, passengers={self.passenger_indices}, "
                f"threshold={self.threshold}, total_layers={self.total_layers})")
