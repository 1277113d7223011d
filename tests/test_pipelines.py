"""Integration tests (tests/test_ai_pipeline.rs, tests/test_hpc_pipeline.rs,
nangila-twin edge_sync.rs, nangila-checkpoint tests/h5.rs) and the .nz
container."""
import struct

import numpy as np
import pytest

from mini_nangila_b200.ai import MomentumPredictor, TopKQuantizer
from mini_nangila_b200.checkpoint import hdf5, lammps, nzcp
from mini_nangila_b200.core import FixedPointBuffer, TopologyMask
from mini_nangila_b200.hpc import (BlockSparseQuantizer, BlockSparseRleQuantizer, ErrorBoundedQuantizer,
                                   LinearPredictor)
from mini_nangila_b200.twin import CloudNode, EdgeNode

F = FixedPointBuffer.from_f32


def test_ai_compression_end_to_end():
    L, n, steps = 100, 1000, 50
    preds = [MomentumPredictor(0.9) for _ in range(L)]
    q = TopKQuantizer(0.10)
    mask = TopologyMask.from_variance_threshold([100.0 / (1.0 + i / 10.0) for i in range(L)], 0.30)
    raw = comp = 0
    idx = np.arange(n)
    for step in range(steps):
        for layer in range(L):
            g = np.where((idx + step + layer) % 100 < 70, 0.0,
                         np.sin((idx + step).astype(np.float32)) * np.float32(0.1)).astype(np.float32)
            gb = F(g)
            raw += n * 4
            if mask.is_passenger(layer):
                preds[layer].update(gb)
                continue
            p = preds[layer].predict()
            r = gb.clone() if p.is_empty() else gb.sub(p)
            b, s = q.quantize(r)
            comp += len(b) + 4
            d = q.dequantize(b, s)
            preds[layer].update(d if p.is_empty() else p.add(d))
    assert raw / comp > 20.0


def test_ai_closed_loop_sync():
    ep, cp, q = MomentumPredictor(0.9), MomentumPredictor(0.9), TopKQuantizer(0.10)
    for step in range(100):
        g = F(np.sin((np.arange(500) + step).astype(np.float32) * np.float32(0.01)))
        p = ep.predict()
        b, s = q.quantize(g.clone() if p.is_empty() else g.sub(p))
        d = q.dequantize(b, s)
        er = d if p.is_empty() else p.add(d)
        ep.update(er)
        pc = cp.predict()
        d2 = q.dequantize(b, s)
        cr = d2 if pc.is_empty() else pc.add(d2)
        cp.update(cr)
        assert er == cr


def test_hpc_error_bounded_100_steps():
    eps, q = 1e-3, ErrorBoundedQuantizer(1e-3)
    sp, rp = LinearPredictor(), LinearPredictor()
    for step in range(100):
        sig = (np.sin(np.arange(500, dtype=np.float32) * np.float32(0.01) + np.float32(step) * np.float32(0.05))
               * np.float32(10.0)).astype(np.float32)
        x = F(sig)
        p = sp.predict()
        b, s = q.quantize(x.clone() if p.is_empty() else x.sub(p))
        d = q.dequantize(b, s)
        srec = d if p.is_empty() else p.add(d)
        sp.update(srec)
        pr = rp.predict()
        d2 = q.dequantize(b, s)
        rrec = d2 if pr.is_empty() else pr.add(d2)
        rp.update(rrec)
        assert srec == rrec
        if step > 2:
            assert np.all(np.abs(x.to_f32() - rrec.to_f32()) < eps * 5 + 1e-5)


def test_hpc_compression_ratio():
    b, _ = ErrorBoundedQuantizer(1e-3).quantize(F(np.sin(np.arange(10000, dtype=np.float32) * np.float32(0.01))))
    assert 40000 / len(b) >= 1.9


@pytest.mark.parametrize("cls", [BlockSparseQuantizer, BlockSparseRleQuantizer])
def test_hpc_sparse_pipelines(cls):
    eps, q, pred = 1e-3, cls(1e-3), LinearPredictor()
    raw = comp = 0
    for step in range(50):
        i = np.arange(1024)
        sig = np.where((i + step * 7) % 50 < 5, np.sin(((i + step).astype(np.float32)) * np.float32(0.1)), 0.0)
        x = F(sig.astype(np.float32))
        p = pred.predict()
        b, s = q.quantize(x.clone() if p.is_empty() else x.sub(p))
        raw += 4096
        comp += len(b)
        d = q.dequantize(b, s)
        rec = d if p.is_empty() else p.add(d)
        pred.update(rec)
        assert np.all(np.abs(x.to_f32() - rec.to_f32()) <= eps + 1e-5)


def test_twin_end_to_end_sync():
    edge = EdgeNode(MomentumPredictor(0.9), ErrorBoundedQuantizer(0.05))
    cloud = CloudNode(MomentumPredictor(0.9), ErrorBoundedQuantizer(0.05))
    x = F([10.0])
    for _ in range(2):
        b, s = edge.send(x)
        assert abs(cloud.receive(b, s).to_f32()[0] - 10.0) < 0.06


@pytest.mark.parametrize("codec", ["eb", "rle", "bs", "bsrle"])
def test_nz_roundtrip(codec, tmp_path):
    P, T = 3000, 12
    data = lammps.generate_synthetic(P, T)
    path = str(tmp_path / "t.nz")
    stats = nzcp.write(path, data, P, T, codec, 1e-3)
    assert stats["max_abs_err"] <= 1e-3 + 1e-6
    raw = open(path, "rb").read()
    assert raw[:4] == b"NZCP" and raw[4] == 1 and raw[5] == nzcp.CODECS[codec]
    assert struct.unpack_from("<II", raw, 6) == (P, T)
    h = nzcp.read_header(raw)
    assert (h.particles, h.steps, h.codec) == (P, T, nzcp.CODECS[codec])
    rec = nzcp.read(path)
    assert rec.size == P * T and np.abs(rec - data).max() <= 1e-3 + 1e-6
    res = nzcp.read(path, add_back=False)
    # residual stream: the first step's residual is the snapshot itself
    assert np.abs(res[:P] - data[:P]).max() <= 1e-3 + 1e-6
    steps = list(nzcp.iter_steps(raw))
    assert len(steps) == T and nzcp.build(h, steps) == raw
    assert stats["total_comp"] == sum(len(p) + 8 for _, p in steps)


def test_nz_bad_magic():
    with pytest.raises(RuntimeError):
        nzcp.decompress(b"XXXX" + bytes(10))


def test_lammps_dump_roundtrip(tmp_path):
    p = str(tmp_path / "d.dump")
    lammps.write_dump(p, 50, 3)
    snaps = lammps.read_dump(p)
    assert len(snaps) == 3 and snaps[0].size == 150
    ph = np.float32(0.1) + np.arange(50, dtype=np.float32) * np.float32(0.001)
    assert np.allclose(snaps[1][0::3], np.cos(ph), atol=1e-5)


def test_checkpoint_layout_roundtrip(tmp_path):
    n = 12345
    i = np.arange(n)
    data = (np.cos(i.astype(np.float32) * np.float32(0.01) * np.float32(0.5))
            + (i % 100).astype(np.float32) * np.float32(1e-4)).astype(np.float32)
    path = str(tmp_path / "ck.h5")
    hdf5.write_chunked_dataset(path, "traj", data, 1024, 1e-3, "ErrorBoundedINT16")
    out = hdf5.read_compressed_1d(path, "traj")
    assert out.size == n and np.abs(out - data).max() <= 1e-3 + 1e-6
    p2 = str(tmp_path / "raw.h5")
    hdf5.write_dataset(p2, "traj_raw", data, 0.0, "raw")
    assert hdf5.read_dataset(p2, "traj_raw").size == n


def test_nz_decoder_checks_step_sizes_like_the_predictor():
    """Steps of other sizes glued under one header: after an empty step the
    prediction is empty and the next step passes through; a step whose size
    differs from the history raises the predictor's shape error
    (LinearPredictor + FixedPointBuffer::add, main.rs:249-309)."""
    import struct

    def glue(*blobs):
        steps = sum(struct.unpack_from("<I", x, 10)[0] for x in blobs)
        return blobs[0][:10] + struct.pack("<I", steps) + b"".join(x[14:] for x in blobs)

    empty, _ = nzcp.compress(np.zeros(0, np.float32), 0, 1, "eb", 1e-3)
    six, _ = nzcp.compress(np.arange(6, dtype=np.float32), 6, 1, "eb", 1e-3)
    four, _ = nzcp.compress(np.arange(4, dtype=np.float32), 4, 1, "eb", 1e-3)
    out = nzcp.decompress(glue(empty, six))
    assert out.size == 6 and np.abs(out - np.arange(6)).max() <= 1e-3 + 1e-6
    with pytest.raises(ValueError, match="Shape mismatch: 6 vs 4"):  # the host library's ShapeMismatch
        nzcp.decompress(glue(six, four))
    assert nzcp.decompress(glue(six, four), add_back=False).size == 10  # residuals need no history
