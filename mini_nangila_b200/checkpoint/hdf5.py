"""Chunked error-bounded checkpoint layout (nangila-checkpoint/src/lib.rs).

``write_chunked_dataset`` splits a 1-D float array into ``chunk``-sized
pieces (the last zero-padded), runs the LinearPredictor closed loop across
chunks with the ErrorBounded INT16 quantizer (the codec string is only a
label) and stores, under group ``dataset``:

* ``blob``   u8[]                    concatenated payloads
* ``offsets`` u64[num_chunks + 1]    payload boundaries in ``blob``
* ``scales`` f32[num_chunks]
* attrs ``total_len`` (u64), ``chunk`` (u64), ``codec`` (str), ``epsilon`` (f32)

``read_compressed_1d`` reverses it.  The file is always HDF5 with exactly
these names: through h5py when it is installed, otherwise through this
framework's native HDF5 writer and reader (``checkpoint.h5file``, no libhdf5
needed), whose files h5py reads and which reads files libhdf5 wrote.  Like
the reference's ``File::create``, the writers replace an existing file.
"""
from __future__ import annotations

import numpy as np

from ..core.fixed_point import FixedPointBuffer
from ..hpc import ErrorBoundedQuantizer, LinearPredictor

from . import h5file

try:  # optional dependency
    import h5py  # type: ignore
except ImportError:  # pragma: no cover - depends on the environment
    h5py = None


def _encode_chunks(data: np.ndarray, chunk: int, epsilon: float):
    chunk = max(1, int(chunk))
    total = data.size
    nch = (total + chunk - 1) // chunk
    pred = LinearPredictor()
    q = ErrorBoundedQuantizer(epsilon)
    blob, offsets, scales = bytearray(), [0], []
    for c in range(nch):
        buf = np.zeros(chunk, np.float32)
        seg = data[c * chunk:(c + 1) * chunk]
        buf[: seg.size] = seg
        x = FixedPointBuffer.from_f32(buf)
        p = pred.predict()
        r = x.clone() if p.is_empty() else x.sub(p)
        b, s = q.quantize(r)
        scales.append(s)
        d = q.dequantize(b, s)
        pred.update(d if p.is_empty() else p.add(d))
        blob += b
        offsets.append(len(blob))
    return np.frombuffer(bytes(blob), np.uint8), np.asarray(offsets, np.uint64), np.asarray(scales, np.float32)


def _decode_chunks(blob, offsets, scales, total_len: int, epsilon: float) -> np.ndarray:
    pred = LinearPredictor()
    q = ErrorBoundedQuantizer(epsilon)
    out = []
    for c in range(len(scales)):
        b = blob[int(offsets[c]):int(offsets[c + 1])]
        p = pred.predict()
        d = q.dequantize(b, float(scales[c]))
        r = d if p.is_empty() else p.add(d)
        pred.update(r)
        out.append(r.to_f32())
    v = np.concatenate(out) if out else np.zeros(0, np.float32)
    return v[:total_len]


def write_chunked_dataset(path: str, dataset: str, data, chunk: int, epsilon: float, codec: str) -> None:
    """Chunked error-bounded dataset (nangila-checkpoint/src/lib.rs:29-83): group ``dataset`` with
    ``blob``, ``offsets``, ``scales`` and attributes; the codes are always EB INT16."""
    data = np.ascontiguousarray(np.asarray(data, np.float32).reshape(-1))
    blob, offsets, scales = _encode_chunks(data, chunk, epsilon)
    attrs = {"total_len": np.uint64(data.size), "chunk": np.uint64(max(1, int(chunk))), "codec": codec,
             "epsilon": np.float32(epsilon)}
    if h5py is not None:
        with h5py.File(path, "w") as f:
            g = f.create_group(dataset)
            g.create_dataset("blob", data=blob)
            g.create_dataset("offsets", data=offsets)
            g.create_dataset("scales", data=scales)
            for k, v in attrs.items():
                g.attrs[k] = v
        return
    root = h5file.Group()
    g = root.create_group(dataset)
    g.create_dataset("blob", blob)
    g.create_dataset("offsets", offsets)
    g.create_dataset("scales", scales)
    g.attrs.update(attrs)
    h5file.save(path, root)


def read_compressed_1d(path: str, dataset: str) -> np.ndarray:
    """Decode a chunked dataset back to f32 (nangila-checkpoint/src/lib.rs:94-133)."""
    if h5py is not None:
        with h5py.File(path, "r") as f:
            g = f[dataset]
            return _decode_chunks(g["blob"][()], g["offsets"][()], g["scales"][()], int(g.attrs["total_len"]),
                                  float(g.attrs["epsilon"]))
    g = h5file.load(path)[dataset]
    return _decode_chunks(g["blob"].data, g["offsets"].data, g["scales"].data, int(g.attrs["total_len"]),
                          float(g.attrs["epsilon"]))


def write_dataset(path: str, dataset: str, data, epsilon: float, codec: str) -> None:
    """Plain 1-D f32 dataset with ``epsilon`` and ``codec`` attributes (nangila-checkpoint/src/lib.rs:14-26)."""
    data = np.asarray(data, np.float32).reshape(-1)
    if h5py is not None:
        with h5py.File(path, "w") as f:
            ds = f.create_dataset(dataset, data=data)
            ds.attrs["epsilon"] = np.float32(epsilon)
            ds.attrs["codec"] = codec
        return
    root = h5file.Group()
    root.create_dataset(dataset, data, attrs={"epsilon": np.float32(epsilon), "codec": codec})
    h5file.save(path, root)


def read_dataset(path: str, dataset: str) -> np.ndarray:
    """Read a plain dataset written by ``write_dataset``."""
    if h5py is not None:
        with h5py.File(path, "r") as f:
            return f[dataset][()]
    return h5file.load(path)[dataset].data
