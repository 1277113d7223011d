"""Error-bounded checkpoints of model and optimizer state.

``save(path, state, eps, codec)`` writes every floating-point tensor of a
(nested) state dict as the error-bounded code of its Q8.23 residual against
an optional ``base`` checkpoint (delta coding between successive
checkpoints, the predictive-residual idea applied to training state):

    residual = Q8.23(x) - Q8.23(base)        (Q8.23(x) when no base)
    payload  = EB | BlockSparse | BlockSparse+RLE codec of the residual

so every restored value is within ``eps`` of the saved one (plus the fp32
rounding of the value itself).  Tensors on a CUDA device are encoded by the
sm_100a codec kernels (same bytes as the C++ library).  Values outside the
Q8.23 range (|x| >= 255) or non-finite, and every non-float tensor, are
stored raw: this is the fallback the reference declares but never produces
(nangila-hpc/src/error_bounded.rs:5-11, ``FallbackRequired``).

File layout (little endian): ``b"NZTS"``, u8 version 1, u32 entry count,
then per entry: u16 name length + UTF-8 name, u8 dtype code, u8 ndim,
ndim x u64 dims, u8 codec (0 raw, 1 EB, 3 BlockSparse, 4 BlockSparse+RLE;
the .nz codec numbers), u8 has_base, f32 eps, f32 scale, u64 payload
bytes, payload.  Non-tensor leaves (ints, floats, strings, lists) are kept
in a trailing pickled dict.
"""
from __future__ import annotations

import io
import pickle
import struct

import numpy as np
import torch

from ..core import FixedPointBuffer
from ..hpc import BlockSparseQuantizer, BlockSparseRleQuantizer, ErrorBoundedQuantizer

MAGIC = b"NZTS"
CODECS = {"raw": 0, "eb": 1, "bs": 3, "bsrle": 4}
_QUANT = {1: ErrorBoundedQuantizer, 3: BlockSparseQuantizer, 4: BlockSparseRleQuantizer}
_DTYPES = [torch.float32, torch.float16, torch.bfloat16, torch.float64, torch.int64, torch.int32, torch.int16,
           torch.int8, torch.uint8, torch.bool]
_Q823_LIMIT = 255.0


def _flatten(state, prefix=""):
    """(name, tensor) pairs and the non-tensor leaves of a nested dict/list."""
    tensors, other = [], {}
    if isinstance(state, dict):
        items = state.items()
    elif isinstance(state, (list, tuple)):
        items = enumerate(state)
    else:
        return [], {prefix: state}
    for k, v in items:
        name = f"{prefix}/{k}" if prefix else str(k)
        if isinstance(v, torch.Tensor):
            tensors.append((name, v))
        elif isinstance(v, (dict, list, tuple)):
            t, o = _flatten(v, name)
            tensors += t
            other.update(o)
        else:
            other[name] = v
    return tensors, other


def _encode(x: torch.Tensor, base: torch.Tensor | None, eps: float, codec: int):
    """Returns (codec used, scale, payload bytes)."""
    xf = x.detach().float().reshape(-1)
    if codec == 0 or xf.numel() == 0:
        return 0, 1.0, _raw(x)
    if not bool(torch.isfinite(xf).all()) or float(xf.abs().max()) >= _Q823_LIMIT:
        return 0, 1.0, _raw(x)
    if base is not None:
        bf = base.detach().float().reshape(-1).to(xf.device)
        if bf.numel() != xf.numel() or not bool(torch.isfinite(bf).all()) or float(bf.abs().max()) >= _Q823_LIMIT:
            return 0, 1.0, _raw(x)
        r = FixedPointBuffer.from_f32(xf).sub(FixedPointBuffer.from_f32(bf))
    else:
        r = FixedPointBuffer.from_f32(xf)
    q = _QUANT[codec](eps)
    payload, scale = q.quantize(r)
    return codec, float(scale), _as_bytes(payload)


def _as_bytes(payload) -> bytes:
    if isinstance(payload, (bytes, bytearray)):
        return bytes(payload)
    if isinstance(payload, torch.Tensor):
        return payload.cpu().numpy().tobytes()
    return np.asarray(payload, dtype=np.uint8).tobytes()


def _raw(x: torch.Tensor) -> bytes:
    t = x.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return t.numpy().tobytes()


def save(path_or_file, state, eps: float = 1e-3, codec: str = "bs", base=None) -> dict:
    """Write ``state`` (nested dict/list of tensors and plain values).

    ``base``: a state with the same tensor names (for instance the previous
    checkpoint as restored by ``load``) to delta-code against.  Returns
    byte counts ``{"raw": ..., "compressed": ..., "fallback_tensors": ...}``.
    """
    cid = CODECS[codec]
    tensors, other = _flatten(state)
    base_t = dict(_flatten(base)[0]) if base is not None else {}
    out = io.BytesIO()
    out.write(MAGIC + struct.pack("<BI", 1, len(tensors)))
    raw_bytes = comp_bytes = 0
    fallback = 0
    for name, x in tensors:
        if x.dtype not in _DTYPES:
            raise TypeError(f"unsupported dtype {x.dtype} for {name}")
        is_float = x.dtype.is_floating_point
        b = base_t.get(name) if is_float else None
        c, scale, payload = _encode(x, b, eps, cid if is_float else 0)
        if is_float and cid != 0 and c == 0:
            fallback += 1
        nb = name.encode()
        out.write(struct.pack("<H", len(nb)) + nb)
        out.write(struct.pack("<BB", _DTYPES.index(x.dtype), x.dim()))
        out.write(struct.pack(f"<{x.dim()}Q", *x.shape))
        out.write(struct.pack("<BBffQ", c, 1 if (c and b is not None) else 0, float(eps), scale, len(payload)))
        out.write(payload)
        raw_bytes += x.numel() * x.element_size()
        comp_bytes += len(payload)
    extra = pickle.dumps(other)
    out.write(struct.pack("<Q", len(extra)) + extra)
    data = out.getvalue()
    if hasattr(path_or_file, "write"):
        path_or_file.write(data)
    else:
        with open(path_or_file, "wb") as fh:
            fh.write(data)
    return {"raw": raw_bytes, "compressed": comp_bytes, "fallback_tensors": fallback, "file": len(data)}


def load(path_or_bytes, base=None, device=None) -> dict:
    """Read a checkpoint into a flat ``{name: tensor or value}`` dict (names
    joined with "/"); ``base`` must be the state the file was delta-coded
    against.  ``device="cuda"`` decodes on the GPU."""
    if isinstance(path_or_bytes, (bytes, bytearray)):
        data = bytes(path_or_bytes)
    else:
        with open(path_or_bytes, "rb") as fh:
            data = fh.read()
    if data[:4] != MAGIC:
        raise ValueError("not a tensor checkpoint (bad magic)")
    ver, count = struct.unpack_from("<BI", data, 4)
    if ver != 1:
        raise ValueError(f"unsupported version {ver}")
    off = 9
    base_t = dict(_flatten(base)[0]) if base is not None else {}
    out = {}
    for _ in range(count):
        (ln,) = struct.unpack_from("<H", data, off)
        name = data[off + 2: off + 2 + ln].decode()
        off += 2 + ln
        dti, nd = struct.unpack_from("<BB", data, off)
        off += 2
        shape = struct.unpack_from(f"<{nd}Q", data, off)
        off += 8 * nd
        c, has_base, eps, scale, nb = struct.unpack_from("<BBffQ", data, off)
        off += struct.calcsize("<BBffQ")
        payload = data[off: off + nb]
        off += nb
        dtype = _DTYPES[dti]
        if c == 0:
            if dtype == torch.bfloat16:
                t = torch.from_numpy(np.frombuffer(payload, np.int16).copy()).view(torch.bfloat16)
            else:
                npd = torch.empty(0, dtype=dtype).numpy().dtype
                t = torch.from_numpy(np.frombuffer(payload, npd).copy())
            t = t.reshape(shape)
        else:
            q = _QUANT[c](eps)
            n = int(np.prod(shape)) if nd else 1
            r = FixedPointBuffer(q.dequantize(payload, scale, device=device).data[:n])
            if has_base:
                b = base_t.get(name)
                if b is None:
                    raise KeyError(f"{name} was delta-coded: pass the base state")
                r = r.add(FixedPointBuffer.from_f32(b.detach().float().reshape(-1).to(r.device)))
            v = r.to_f32()
            vals = v.cpu() if isinstance(v, torch.Tensor) else torch.from_numpy(np.asarray(v, np.float32))
            t = vals.reshape(shape).to(dtype)
        out[name] = t
    (ln,) = struct.unpack_from("<Q", data, off)
    out.update(pickle.loads(data[off + 8: off + 8 + ln]))
    return out
