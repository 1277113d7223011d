"""Q8.23 fixed-point buffers (nangila-math: fixed_point.rs, ops.rs).

``FixedPointBuffer.data`` is an int32 ``torch.Tensor`` on the CPU or on a
CUDA device.  Host buffers run the C++ host library, device buffers run the
sm_100a kernels; both are bit-identical to the Rust semantics:

* ``from_f32``: ``round(x * 2^23)`` half away from zero, saturating, NaN -> 0;
* ``to_f32``: ``q as f32 / 2^23``;
* ``add``/``sub``: saturating, ``ShapeMismatch`` on length mismatch;
* ``mul_scalar(s)``: ``((q as i64) * ((s * 2^23) as i64)) >> 23`` clamped.
"""
from __future__ import annotations

import numpy as np
import torch

from .._ext import host

FRACTIONAL_BITS = 23
SCALE_FACTOR = float(1 << FRACTIONAL_BITS)


class FixedPointError(ValueError):
    """Base error of the Q8.23 layer (``MathError`` in nangila-math)."""
    pass


class ShapeMismatch(FixedPointError):
    """Element-wise op on buffers of different lengths (ops.rs:7-9)."""
    def __init__(self, a: int, b: int):
        super().__init__(f"Shape mismatch: {a} vs {b}")
        self.a, self.b = a, b


def _as_f32_tensor(values, device=None) -> torch.Tensor:
    if isinstance(values, torch.Tensor):
        t = values.detach()
        if t.dtype != torch.float32:
            t = t.float()
    else:
        t = torch.from_numpy(np.ascontiguousarray(np.asarray(values, dtype=np.float32)))
    if device is not None:
        t = t.to(device)
    return t.contiguous().reshape(-1)


def _dev_ops():
    from ..ops import codecs

    return codecs


class FixedPointBuffer:
    """Q8.23 values as an int32 tensor (nangila-math/src/fixed_point.rs:14-17).

    ``from_f32`` / ``to_f32`` convert (fixed_point.rs:34-60); ``add``, ``sub`` and
    ``mul_scalar`` are the saturating ops of ops.rs:6-49.  A CPU buffer runs the
    C++ host library, a CUDA buffer the sm_100a kernels; both give the same bits."""
    __slots__ = ("data",)

    def __init__(self, data):
        if isinstance(data, torch.Tensor):
            t = data
        else:
            t = torch.from_numpy(np.ascontiguousarray(np.asarray(data, dtype=np.int32)))
        if t.dtype != torch.int32:
            raise TypeError("FixedPointBuffer holds int32 Q8.23 values")
        self.data = t.contiguous().reshape(-1)

    # ---- construction / conversion
    @classmethod
    def new(cls, size: int, device=None) -> "FixedPointBuffer":
        return cls(torch.zeros(int(size), dtype=torch.int32, device=device))

    @classmethod
    def from_f32(cls, values, device=None) -> "FixedPointBuffer":
        t = _as_f32_tensor(values, device)
        if t.is_cuda:
            return cls(_dev_ops().q823_from_f32(t))
        return cls(torch.from_numpy(host().q823_from_f32(t.numpy())))

    def to_f32(self):
        """numpy float32 array for host buffers, float32 tensor for device buffers."""
        if self.data.is_cuda:
            return _dev_ops().q823_to_f32(self.data)
        return host().q823_to_f32(self.data.numpy())

    # ---- Rust-style accessors
    def len(self) -> int:
        return int(self.data.numel())

    def __len__(self) -> int:
        return self.len()

    def is_empty(self) -> bool:
        return self.len() == 0

    @property
    def device(self) -> torch.device:
        return self.data.device

    def to(self, device) -> "FixedPointBuffer":
        return FixedPointBuffer(self.data.to(device))

    def cpu(self) -> "FixedPointBuffer":
        return self.to("cpu")

    def cuda(self, device=None) -> "FixedPointBuffer":
        return self.to(device or "cuda")

    def clone(self) -> "FixedPointBuffer":
        return FixedPointBuffer(self.data.clone())

    def numpy(self) -> np.ndarray:
        return self.data.cpu().numpy()

    def __eq__(self, other) -> bool:
        return isinstance(other, FixedPointBuffer) and self.len() == other.len() and bool(
            torch.equal(self.data.cpu(), other.data.cpu()))

    def __repr__(self) -> str:
        return f"FixedPointBuffer(len={self.len()}, device={self.device})"

    # ---- ops (ops.rs)
    def _check(self, other: "FixedPointBuffer") -> None:
        if self.len() != other.len():
            raise ShapeMismatch(self.len(), other.len())

    def add(self, other: "FixedPointBuffer") -> "FixedPointBuffer":
        self._check(other)
        if self.data.is_cuda:
            return FixedPointBuffer(_dev_ops().q823_add(self.data, other.data.to(self.device)))
        return FixedPointBuffer(torch.from_numpy(host().q823_add(self.data.numpy(), other.data.cpu().numpy())))

    def sub(self, other: "FixedPointBuffer") -> "FixedPointBuffer":
        self._check(other)
        if self.data.is_cuda:
            return FixedPointBuffer(_dev_ops().q823_sub(self.data, other.data.to(self.device)))
        return FixedPointBuffer(torch.from_numpy(host().q823_sub(self.data.numpy(), other.data.cpu().numpy())))

    def mul_scalar(self, scalar: float) -> "FixedPointBuffer":
        s = float(np.float32(scalar))
        if self.data.is_cuda:
            return FixedPointBuffer(_dev_ops().q823_mul_scalar(self.data, s))
        return FixedPointBuffer(torch.from_numpy(host().q823_mul_scalar(self.data.numpy(), s)))


class FixedQ:
    """no_std edge encoding (nangila-edge/src/lib.rs): ``s +/- 0.5`` in f32,
    then truncation; differs from ``FixedPointBuffer`` for some odd values in
    [2^23, 2^24) where the f32 addition rounds to even."""

    FRACTIONAL_BITS = 23

    def __init__(self, data):
        self.data = np.ascontiguousarray(np.asarray(data, dtype=np.int32))

    @classmethod
    def from_f32(cls, values) -> "FixedQ":
        return cls(host().fixedq_from_f32(np.ascontiguousarray(np.asarray(values, dtype=np.float32))))

    def to_f32(self) -> np.ndarray:
        return host().fixedq_to_f32(self.data)
