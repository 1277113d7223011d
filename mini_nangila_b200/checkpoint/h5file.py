"""HDF5 files without libhdf5 or h5py: a small h5py-like tree over the native
writer and reader of the host library (``csrc/host/hdf5_io.cpp``).

    root = Group()
    g = root.create_group("traj")
    g.create_dataset("scales", np.ones(4, np.float32))
    g.attrs["codec"] = "ErrorBoundedINT16"
    save("ckpt.h5", root)
    load("ckpt.h5")["traj"]["scales"].data

Element types: little-endian integers (u1..u8, i1..i8), float32/float64 and
fixed-length byte strings; Python ``str`` values are stored as ASCII/UTF-8
bytes.  The writer produces the layout libhdf5 writes by default (superblock
0, version-1 object headers, symbol-table groups, contiguous datasets), so
h5py and the HDF5 tools read these files.  The reader also accepts the newer
object-header and link-message formats; chunked datasets and dense link
storage are reported as unsupported.
"""
from __future__ import annotations

import numpy as np

from .._ext import host


class Dataset:
    """An array with attributes."""

    def __init__(self, data, attrs: dict | None = None):
        self.data = data
        self.attrs = dict(attrs or {})

    def __getitem__(self, key):
        return self.data[key]

    @property
    def shape(self):
        return np.shape(self.data)


class Group(dict):
    """Named children (groups or datasets) with attributes; ``g["a/b"]`` walks paths."""

    def __init__(self, attrs: dict | None = None):
        super().__init__()
        self.attrs = dict(attrs or {})

    def create_group(self, name: str) -> "Group":
        g = Group()
        self[name] = g
        return g

    def create_dataset(self, name: str, data, attrs: dict | None = None) -> Dataset:
        d = Dataset(np.asarray(data) if not isinstance(data, (bytes, str)) else data, attrs)
        self[name] = d
        return d

    def __getitem__(self, key):
        node = self
        for part in str(key).strip("/").split("/"):
            node = dict.__getitem__(node, part)
        return node


def _value(x) -> tuple:
    """(kind, size, shape, bytes) of an attribute or dataset value."""
    if isinstance(x, str):
        x = x.encode("utf-8")
    if isinstance(x, (bytes, np.bytes_)):
        b = bytes(x)
        return ("S", max(1, len(b)), [], b if b else b"\0")
    if isinstance(x, bool):
        x = np.uint8(x)
    elif isinstance(x, int):
        x = np.int64(x) if x < 0 else np.uint64(x)
    elif isinstance(x, float):
        x = np.float64(x)
    a = np.asarray(x)
    if a.dtype.kind == "U":
        a = np.char.encode(a, "utf-8")
    if a.dtype.kind == "S":
        size = max(1, a.dtype.itemsize)
        a = a.astype(f"S{size}")
        return ("S", size, list(a.shape), a.tobytes(order="C"))
    if a.dtype.kind == "b":
        a = a.astype(np.uint8)
    if a.dtype.kind not in "uif" or (a.dtype.kind == "f" and a.dtype.itemsize not in (4, 8)):
        raise TypeError(f"unsupported HDF5 element type {a.dtype}")
    shape = list(a.shape)  # np.ascontiguousarray would turn a 0-d value into shape [1]
    a = a.astype(a.dtype.newbyteorder("<"), copy=False)
    return (a.dtype.kind, a.dtype.itemsize, shape, a.tobytes(order="C"))


def _array(v: tuple):
    kind, size, shape, raw = v
    dt = (np.dtype(f"S{size}") if kind == "S" else np.dtype((np.void, size)) if kind == "V"
          else np.dtype(f"<{kind}{size}"))
    a = np.frombuffer(raw, dtype=dt).reshape(shape) if shape else np.frombuffer(raw, dtype=dt)[0]
    return a.copy() if isinstance(a, np.ndarray) else a


def to_bytes(root: Group) -> bytes:
    objs: list = []

    def add(node, name, parent):
        attrs = [(k, _value(v)) for k, v in node.attrs.items()]
        if isinstance(node, Group):
            me = len(objs)
            objs.append((True, name, parent, None, attrs))
            for k, child in node.items():
                add(child, k, me)
        else:
            objs.append((False, name, parent, _value(node.data), attrs))

    add(root, "", -1)
    return host().h5_write(objs)


def from_bytes(b: bytes) -> Group:
    objs = host().h5_read(bytes(b))
    nodes: list = []
    for is_group, name, parent, value, attrs in objs:
        a = {k: _array(v) for k, v in attrs}
        node = Group(a) if is_group else Dataset(_array(value), a)
        nodes.append(node)
        if parent >= 0:
            dict.__setitem__(nodes[parent], name, node)
    return nodes[0]


def save(path: str, root: Group) -> None:
    with open(path, "wb") as fh:
        fh.write(to_bytes(root))


def load(path: str) -> Group:
    with open(path, "rb") as fh:
        return from_bytes(fh.read())


def is_hdf5(path: str) -> bool:
    """True if the file carries an HDF5 superblock signature (at 0 or after a user block)."""
    sig = b"\x89HDF\r\n\x1a\n"
    try:
        with open(path, "rb") as fh:
            data = fh.read(1 << 16)
    except OSError:
        return False
    off = 0
    while off + 8 <= len(data):
        if data[off:off + 8] == sig:
            return True
        off = 512 if off == 0 else off * 2
    return False
