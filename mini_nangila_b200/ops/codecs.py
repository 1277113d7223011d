"""Device (sm_100a) codecs with the reference's byte formats.

Every encoder returns ``(uint8 CUDA tensor, scale)`` holding exactly the
bytes the host library (and the reference) produce for the same input;
decoders take a uint8 CUDA tensor and return int32 Q8.23 values.  The
extension must be built: there is no PyTorch fallback.
"""
from __future__ import annotations

import numpy as np
import torch

from .._ext import cuda

KIND_BS, KIND_TOPK, KIND_BSRLE, KIND_RLE = 0, 1, 2, 3


def _f32(x) -> float:
    return float(np.float32(x))


def _i64(v: int) -> int:
    """u64 value as the signed int64 with the same bits (pybind int64_t)."""
    v = int(v) & 0xFFFFFFFFFFFFFFFF
    return v - (1 << 64) if v >= (1 << 63) else v


def _eps_scale(eps: float) -> float:
    return float(np.float32(2.0) * np.float32(eps))


# ---- Q8.23
def q823_from_f32(x: torch.Tensor) -> torch.Tensor:
    return cuda().q823_from_f32(x.contiguous())


def q823_to_f32(q: torch.Tensor) -> torch.Tensor:
    return cuda().q823_to_f32(q.contiguous())


def q823_add(a, b):
    return cuda().q823_addsub(a.contiguous(), b.contiguous(), False)


def q823_sub(a, b):
    return cuda().q823_addsub(a.contiguous(), b.contiguous(), True)


def q823_mul_scalar(a, s: float):
    return cuda().q823_mul_scalar(a.contiguous(), _f32(s))


# ---- error-bounded family
def eb_codes(r: torch.Tensor, scale: float) -> torch.Tensor:
    return cuda().eb_codes(r.contiguous(), _f32(scale))


def eb_quantize(r: torch.Tensor, eps: float):
    s = _eps_scale(eps)
    return eb_codes(r, s).view(torch.uint8), s


def eb_dequantize(b: torch.Tensor, scale: float) -> torch.Tensor:
    return cuda().eb_decode(b.contiguous(), _f32(scale))


def bs_quantize(r: torch.Tensor, eps: float):
    s = _eps_scale(eps)
    return cuda().pack_codes(eb_codes(r, s), KIND_BS), s


def bsrle_quantize(r: torch.Tensor, eps: float):
    s = _eps_scale(eps)
    return cuda().pack_codes(eb_codes(r, s), KIND_BSRLE), s


def rle_quantize(r: torch.Tensor, eps: float):
    if r.numel() == 0:
        return torch.empty(0, dtype=torch.uint8, device=r.device), 1.0
    s = _eps_scale(eps)
    return cuda().pack_codes(eb_codes(r, s), KIND_RLE), s


def _header_n(b: torch.Tensor) -> int:
    if b.numel() < 4:
        return -1
    return int(np.frombuffer(b[:4].cpu().numpy().tobytes(), "<u4")[0])


def decode_one(b: torch.Tensor, scale: float, kind: int, out_cap: int, table_cap: int) -> torch.Tensor:
    off = torch.tensor([0, b.numel()], dtype=torch.int64, device=b.device)
    sc = torch.tensor([_f32(scale)], dtype=torch.float32, device=b.device)
    out, ln = cuda().decode_streams(b.contiguous(), off, sc, kind, max(out_cap, 1), max(table_cap, 1))
    return out[: int(ln[0])]


def bs_dequantize(b: torch.Tensor, scale: float) -> torch.Tensor:
    n = _header_n(b)
    if n < 0:
        return torch.empty(0, dtype=torch.int32, device=b.device)
    return decode_one(b, scale, KIND_BS, n, (n + 31) // 32)


def bsrle_dequantize(b: torch.Tensor, scale: float) -> torch.Tensor:
    n = _header_n(b)
    if n < 0:
        return torch.empty(0, dtype=torch.int32, device=b.device)
    return decode_one(b, scale, KIND_BSRLE, n, (n + 31) // 32)


def topk_dequantize(b: torch.Tensor, scale: float) -> torch.Tensor:
    n = _header_n(b)
    if n < 0:
        return torch.empty(0, dtype=torch.int32, device=b.device)
    return decode_one(b, scale, KIND_TOPK, n, (n + 31) // 32)


def rle_dequantize(b: torch.Tensor, scale: float, n_hint: int | None = None) -> torch.Tensor:
    cap = n_hint if n_hint is not None else 128 * b.numel()
    return decode_one(b, scale, KIND_RLE, cap, b.numel())


# ---- reference stochastic INT4/INT8 and top-k
def stochastic_quantize(r: torch.Tensor, bits: int, seed: int, counter: int):
    b, s = cuda().stochastic_quantize(r.contiguous(), int(bits), _i64(seed), _i64(counter))
    return b, float(s)


def stochastic_dequantize(b: torch.Tensor, scale: float, bits: int) -> torch.Tensor:
    return cuda().stochastic_dequantize(b.contiguous(), _f32(scale), int(bits))


def topk_quantize(r: torch.Tensor, k_percent: float):
    b, s = cuda().topk_quantize(r.contiguous(), _f32(k_percent))
    return b, float(s)


def topk_threshold(r: torch.Tensor, k_percent: float) -> tuple[float, float]:
    t = cuda().topk_threshold(r.contiguous(), _f32(k_percent)).cpu().numpy()
    return float(t[0]), float(t[1])
