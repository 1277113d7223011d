"""Native HDF5 files (csrc/host/hdf5_io.cpp through checkpoint.h5file):

* the reference's checkpoint round trip (nangila-checkpoint/tests/h5.rs:1-36:
  12,345 elements, chunk 1024, error <= eps + 1e-6; a raw dataset too);
* an independent walk of the written bytes, written here in Python from the
  HDF5 File Format Specification (superblock 0, symbol table entries,
  version-1 object headers, group B-tree, symbol table nodes, local heap,
  dataspace / datatype / layout / attribute messages), so the writer is not
  only checked by its own reader;
* a file written by libhdf5 itself (MATLAB's v7.3 format, shipped as test
  data with scipy) read by the native reader;
* trees with nested groups, more links than one symbol table node holds,
  every element type, scalars and empty datasets; corrupt files raise.
"""
import glob
import os
import struct

import numpy as np
import pytest

from mini_nangila_b200.checkpoint import h5file, hdf5


def _data(n):
    i = np.arange(n)
    t = i.astype(np.float32) * np.float32(0.01)
    return (np.cos(t * np.float32(0.5)) + (i % 100).astype(np.float32) * np.float32(1e-4)).astype(np.float32)


def test_reference_checkpoint_roundtrip(tmp_path):
    path = str(tmp_path / "ck.h5")
    data = _data(12345)
    hdf5.write_chunked_dataset(path, "traj", data, 1024, 1e-3, "ErrorBoundedINT16")
    assert h5file.is_hdf5(path)
    out = hdf5.read_compressed_1d(path, "traj")
    assert out.shape == data.shape
    assert float(np.abs(out - data).max()) <= 1e-3 + 1e-6
    raw = str(tmp_path / "raw.h5")
    hdf5.write_dataset(raw, "traj_raw", data, 0.0, "raw")
    assert h5file.is_hdf5(raw)
    back = hdf5.read_dataset(raw, "traj_raw")
    assert back.dtype == np.float32 and np.array_equal(back, data)
    g = h5file.load(path)["traj"]
    assert g.attrs["total_len"] == 12345 and g.attrs["chunk"] == 1024
    assert g.attrs["codec"].astype(str) == "ErrorBoundedINT16"  # as the reference's reader reads it
    assert g.attrs["epsilon"] == np.float32(1e-3)
    assert g["offsets"].data.dtype == np.uint64 and g["offsets"].data.shape == (14,)
    assert g["scales"].data.dtype == np.float32 and g["blob"].data.dtype == np.uint8


# ----------------------------------------------- independent structure walk
def _u(b, at, n):
    return int.from_bytes(b[at:at + n], "little")


def _messages(b, oh):
    assert b[oh] == 1, "object header version 1"
    count, size = _u(b, oh + 2, 2), _u(b, oh + 8, 4)
    p, end, out = oh + 16, oh + 16 + size, []
    while p < end:
        t, s = _u(b, p, 2), _u(b, p + 2, 2)
        assert s % 8 == 0, "version-1 messages are 8-byte aligned"
        out.append((t, p + 8, s))
        p += 8 + s
    assert p == end and len(out) == count
    return out


def _walk_group(b, btree, heap):
    assert b[heap:heap + 4] == b"HEAP" and b[heap + 4] == 0
    data_size, free, data_at = _u(b, heap + 8, 8), _u(b, heap + 16, 8), _u(b, heap + 24, 8)
    assert free == 1  # no free block
    assert b[data_at] == 0  # offset 0 is the empty name

    def name(off):
        assert off < data_size
        return b[data_at + off: b.index(b"\0", data_at + off)].decode()

    assert b[btree:btree + 4] == b"TREE" and b[btree + 4] == 0 and b[btree + 5] == 0
    used = _u(b, btree + 6, 2)
    assert _u(b, btree + 24, 8) == 0  # key 0: the empty name
    entries = []
    for i in range(used):
        child = _u(b, btree + 32 + 16 * i, 8)
        key = _u(b, btree + 40 + 16 * i, 8)
        assert b[child:child + 4] == b"SNOD" and b[child + 4] == 1
        nsym = _u(b, child + 6, 2)
        assert 1 <= nsym <= 8
        syms = []
        for k in range(nsym):
            e = child + 8 + 40 * k
            syms.append((name(_u(b, e, 8)), _u(b, e + 8, 8), _u(b, e + 16, 4), _u(b, e + 24, 8), _u(b, e + 32, 8)))
        assert [s[0] for s in syms] == sorted(s[0] for s in syms)
        assert name(key) == syms[-1][0]  # key i+1: the greatest name of child i
        entries += syms
    return entries


def _dataset(b, oh):
    msgs = {t: (at, s) for t, at, s in _messages(b, oh)}
    assert {1, 3, 5, 8} <= set(msgs)
    at, _ = msgs[1]
    assert b[at] == 1
    rank = b[at + 1]
    shape = tuple(_u(b, at + 8 + 8 * i, 8) for i in range(rank))
    at, _ = msgs[3]
    cls, size = b[at] & 0x0F, _u(b, at + 4, 4)
    at, _ = msgs[8]
    assert b[at] == 3 and b[at + 1] == 1  # layout version 3, contiguous
    addr, nbytes = _u(b, at + 2, 8), _u(b, at + 10, 8)
    return cls, size, shape, b[addr:addr + nbytes]


def test_written_bytes_follow_the_specification(tmp_path):
    path = str(tmp_path / "ck.h5")
    data = _data(5000)
    hdf5.write_chunked_dataset(path, "traj", data, 1024, 1e-3, "EB")
    b = open(path, "rb").read()
    assert b[:8] == b"\x89HDF\r\n\x1a\n"
    assert b[8:16] == bytes([0, 0, 0, 0, 0, 8, 8, 0])  # versions, 8-byte offsets and lengths
    assert _u(b, 16, 2) == 4 and _u(b, 18, 2) == 16  # group leaf / internal node K
    assert _u(b, 24, 8) == 0 and _u(b, 32, 8) == (1 << 64) - 1 and _u(b, 40, 8) == len(b)
    root_oh, cache, rbtree, rheap = _u(b, 64, 8), _u(b, 72, 4), _u(b, 80, 8), _u(b, 88, 8)
    assert cache == 1
    (t, at, _), = _messages(b, root_oh)
    assert t == 0x11 and (_u(b, at, 8), _u(b, at + 8, 8)) == (rbtree, rheap)
    (name, goh, gcache, gbtree, gheap), = _walk_group(b, rbtree, rheap)
    assert name == "traj" and gcache == 1
    msgs = _messages(b, goh)
    assert msgs[0][0] == 0x11 and (_u(b, msgs[0][1], 8), _u(b, msgs[0][1] + 8, 8)) == (gbtree, gheap)
    attrs = {}
    for t, at, _ in msgs[1:]:
        assert t == 0x0C and b[at] == 1
        nlen, dlen, slen = _u(b, at + 2, 2), _u(b, at + 4, 2), _u(b, at + 6, 2)
        p = at + 8
        aname = b[p:p + nlen - 1].decode()
        p += (nlen + 7) // 8 * 8
        cls, size = b[p] & 0x0F, _u(b, p + 4, 4)
        p += (dlen + 7) // 8 * 8
        assert b[p] == 1 and b[p + 1] == 0  # scalar dataspace
        p += (slen + 7) // 8 * 8
        attrs[aname] = (cls, size, b[p:p + size])
    assert attrs["total_len"] == (0, 8, struct.pack("<Q", 5000))
    assert attrs["chunk"] == (0, 8, struct.pack("<Q", 1024))
    assert attrs["codec"] == (3, 2, b"EB")
    assert attrs["epsilon"] == (1, 4, struct.pack("<f", np.float32(1e-3)))
    ds = {n: _dataset(b, oh) for n, oh, cache, _, _ in _walk_group(b, gbtree, gheap)}
    assert sorted(ds) == ["blob", "offsets", "scales"]
    ref = h5file.load(path)["traj"]
    assert ds["blob"][:3] == (0, 1, ref["blob"].data.shape) and ds["blob"][3] == ref["blob"].data.tobytes()
    assert ds["offsets"][:3] == (0, 8, (6,)) and ds["offsets"][3] == ref["offsets"].data.tobytes()
    assert ds["scales"][:3] == (1, 4, (5,)) and ds["scales"][3] == ref["scales"].data.tobytes()


# ----------------------------------------------------- a libhdf5-made file
def _matlab_hdf5_file():
    try:
        import scipy.io.matlab as m
    except ImportError:
        return None
    hits = glob.glob(os.path.join(os.path.dirname(m.__file__), "tests", "data", "testhdf5_7.4_GLNX86.mat"))
    return hits[0] if hits else None


def test_reads_a_file_written_by_libhdf5():
    """MATLAB v7.3 files are HDF5 written by libhdf5 after a 512-byte user
    block: superblock 0, symbol-table groups, a float64 dataset with a
    string attribute.  The data is the scipy test value pi/4 * arange(9)."""
    path = _matlab_hdf5_file()
    if path is None:
        pytest.skip("scipy's MATLAB test data is not installed")
    assert h5file.is_hdf5(path)
    root = h5file.load(path)
    assert list(root.keys()) == ["testdouble"]
    d = root["testdouble"]
    assert d.data.dtype == np.float64 and d.data.shape == (9, 1)
    assert np.array_equal(d.data.reshape(-1), np.pi / 4 * np.arange(9))
    assert d.attrs["MATLAB_class"] == b"double"


# --------------------------------------------------------- general trees
def test_tree_roundtrip_every_type(tmp_path):
    root = h5file.Group({"title": "run 7", "seed": 42, "neg": -3, "lr": 6e-4})
    g = root.create_group("model")
    sub = g.create_group("layer0")
    sub.create_dataset("w", np.arange(12, dtype=np.float32).reshape(3, 4), attrs={"shape_note": b"3x4"})
    for i, dt in enumerate((np.uint8, np.int8, np.uint16, np.int16, np.uint32, np.int32, np.uint64, np.int64,
                            np.float32, np.float64)):
        g.create_dataset(f"t{i:02d}", (np.arange(7) * (i + 1) - 5).astype(dt))
    g.create_dataset("empty", np.zeros(0, np.float32))
    g.create_dataset("scalar", np.float64(2.5))
    g.create_dataset("names", np.array([b"ab", b"cde", b""], dtype="S3"))
    path = str(tmp_path / "tree.h5")
    h5file.save(path, root)
    back = h5file.load(path)
    assert back.attrs["title"] == b"run 7" and back.attrs["seed"] == 42 and back.attrs["neg"] == -3
    assert back.attrs["lr"] == 6e-4
    m = back["model"]
    assert sorted(m.keys()) == sorted(["layer0", "empty", "scalar", "names"] + [f"t{i:02d}" for i in range(10)])
    assert np.array_equal(back["model/layer0/w"].data, np.arange(12, dtype=np.float32).reshape(3, 4))
    assert back["model/layer0/w"].attrs["shape_note"] == b"3x4"
    for i, dt in enumerate((np.uint8, np.int8, np.uint16, np.int16, np.uint32, np.int32, np.uint64, np.int64,
                            np.float32, np.float64)):
        a = m[f"t{i:02d}"].data
        assert a.dtype == np.dtype(dt) and np.array_equal(a, (np.arange(7) * (i + 1) - 5).astype(dt))
    assert m["empty"].data.shape == (0,)
    assert m["scalar"].data == 2.5
    assert list(m["names"].data) == [b"ab", b"cde", b""]


def test_many_links_span_several_symbol_table_nodes(tmp_path):
    root = h5file.Group()
    vals = {}
    for i in range(100):
        name = f"p{(i * 37) % 100:03d}"
        vals[name] = np.full(3, i, np.int32)
        root.create_dataset(name, vals[name])
    path = str(tmp_path / "many.h5")
    h5file.save(path, root)
    b = open(path, "rb").read()
    entries = _walk_group(b, _u(b, 80, 8), _u(b, 88, 8))
    assert [e[0] for e in entries] == sorted(vals)  # 13 symbol table nodes, in name order
    back = h5file.load(path)
    assert all(np.array_equal(back[k].data, v) for k, v in vals.items())


def test_corrupt_files_raise(tmp_path):
    path = str(tmp_path / "ck.h5")
    hdf5.write_chunked_dataset(path, "traj", _data(3000), 512, 1e-3, "EB")
    b = open(path, "rb").read()
    for cut in (0, 7, 50, 95, 200, len(b) // 2, len(b) - 1):
        with pytest.raises(ValueError):
            h5file.from_bytes(b[:cut])
    rng = np.random.default_rng(0)
    for _ in range(300):
        c = bytearray(b)
        for _ in range(3):
            c[int(rng.integers(len(c)))] = int(rng.integers(256))
        try:
            h5file.from_bytes(bytes(c))
        except ValueError:
            pass


def test_unsupported_values_are_rejected():
    root = h5file.Group()
    root.create_dataset("c", np.zeros(3, np.complex64))
    with pytest.raises(TypeError):
        h5file.to_bytes(root)
