"""nangila-ai and nangila-hpc unit tests + proptests (momentum.rs, linear.rs,
quantizer.rs, topk.rs, error_bounded.rs, rle.rs, block_sparse*.rs)."""
import struct

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from mini_nangila_b200.ai import MomentumPredictor, RefCellQuantizer, StochasticQuantizer, TopKQuantizer
from mini_nangila_b200.core import FixedPointBuffer, QuantizationMode, UnifiedQuantizer
from mini_nangila_b200.hpc import (BlockSparseQuantizer, BlockSparseRleQuantizer, ErrorBoundedQuantizer,
                                   LinearPredictor, RunLengthQuantizer, rle_decode_i16, rle_encode_i16)

from .rust_semantics import block_sparse, eb_quantize

F = FixedPointBuffer.from_f32


def test_momentum_update():
    p = MomentumPredictor(0.9)
    assert p.predict().is_empty()
    for v, e in ((10.0, 10.0), (10.0, 10.0), (20.0, 11.0)):
        p.update(F([v]))
        assert abs(p.predict().to_f32()[0] - e) < 1e-6
    p.reset()
    assert p.predict().is_empty()


def test_momentum_constants():
    # beta 0.9 in Q8.23: (0.9f32 * 2^23) as i64 = 7549747; (1 - 0.9f32) -> 838861
    p = MomentumPredictor(0.9)
    p.update(FixedPointBuffer(np.array([1 << 23], np.int32)))
    p.update(FixedPointBuffer(np.array([0], np.int32)))
    assert p.predict().numpy()[0] == ((1 << 23) * 7549747) >> 23


def test_linear_extrapolation():
    p = LinearPredictor()
    p.update(F([10.0]))
    assert abs(p.predict().to_f32()[0] - 10.0) < 1e-6
    p.update(F([12.0]))
    assert abs(p.predict().to_f32()[0] - 14.0) < 1e-6
    p.update(F([14.0]))
    assert abs(p.predict().to_f32()[0] - 16.0) < 1e-6


def test_stochastic_unbiased_int8():
    with pytest.warns(DeprecationWarning):
        q = RefCellQuantizer(42)
    b, s = q.quantize(F(np.full(1000, 0.5, np.float32)))
    mean = np.frombuffer(b, np.int8).astype(np.float32).sum() * s / 1000
    assert abs(mean - 0.5) < 0.1


def test_topk_compression_and_delegation():
    x = np.full(100, 0.01, np.float32)
    for i, v in ((10, 5.0), (20, -5.0), (50, 10.0), (80, -10.0), (90, 8.0)):
        x[i] = v
    q = TopKQuantizer(0.05)
    b, s = q.quantize(F(x))
    r = q.dequantize(b, s).to_f32()
    nz = np.nonzero(np.abs(r) > 0)[0]
    assert 5 <= nz.size <= 6
    assert np.all(np.abs(r[nz] - x[nz]) < s * 0.6)
    data = np.sin(np.arange(200, dtype=np.float32) * np.float32(0.05))
    t, u = TopKQuantizer(0.1), UnifiedQuantizer(QuantizationMode.TopK(0.1))
    assert t.quantize(F(data)) == u.quantize(F(data))


def test_stochastic_quantizer_is_int4():
    b, s = StochasticQuantizer(42).quantize(F(np.linspace(-1, 1, 10, dtype=np.float32)))
    assert len(b) == 5


def test_eb_error_bound():
    q = ErrorBoundedQuantizer(1e-3)
    d = F([0.0, 0.0005, -0.0005, 0.0015, -0.1])
    b, s = q.quantize(d)
    assert np.all(np.abs(d.to_f32() - q.dequantize(b, s).to_f32()) < 1e-3 + 1e-6)


def test_rle_compression():
    d = np.zeros(201, np.float32)
    d[100] = 10.0
    q = RunLengthQuantizer(0.01)
    b, s = q.quantize(F(d))
    assert len(b) <= 6
    r = q.dequantize(b, s).to_f32()
    assert r.size == 201 and abs(r[100] - 10.0) < s and r[0] == 0.0 and r[200] == 0.0
    assert b == bytes([0x80 + 99, 0x00]) + struct.pack("<h", 500) + bytes([0x80 + 99])


def test_rle_runs_capped_at_128():
    q = np.zeros(300, np.int16)
    q[150:290] = 7
    b = rle_encode_i16(q)
    assert b[0] == 0xFF and b[1] == 0x80 + 21 and b[2] == 127
    assert np.array_equal(rle_decode_i16(b), q)


def test_block_sparse_roundtrip_and_layout():
    q = BlockSparseQuantizer(1e-3)
    data = np.sin(np.arange(100, dtype=np.float32) * np.float32(0.01))
    b, s = q.quantize(F(data))
    assert struct.unpack_from("<I", b, 0)[0] == 100
    assert np.all(np.abs(data - q.dequantize(b, s).to_f32()) <= 1e-3 + 1e-6)


def test_bsrle_roundtrip():
    data = np.concatenate([np.sin(np.arange(1024, dtype=np.float32) * np.float32(0.005)) * np.float32(1e-4),
                           np.sin(np.arange(1024, dtype=np.float32) * np.float32(0.01))]).astype(np.float32)
    q = BlockSparseRleQuantizer(1e-3)
    b, s = q.quantize(F(data))
    assert b[4] == 0x80 | 31  # the first 32 blocks quantize to zero -> one zero-run opcode
    assert np.all(np.abs(data - q.dequantize(b, s).to_f32()) <= 1e-3 + 1e-6)


def test_block_sparse_empty_and_truncated():
    q = BlockSparseQuantizer(1e-3)
    b, _ = q.quantize(FixedPointBuffer.new(0))
    assert b == b"\x00\x00\x00\x00"
    assert q.dequantize(b"\x01", 1.0).len() == 0
    d = F(np.ones(64, np.float32))
    b, s = q.quantize(d)
    assert q.dequantize(b[:20], s).len() <= 64


@settings(max_examples=50, deadline=None)
@given(st.lists(st.floats(-50.0, 50.0, width=32), min_size=10, max_size=200), st.floats(0.015625, 0.5, width=32))
def test_prop_eb_bs_bsrle_bounds(vals, eps):
    d = F(vals)
    for q in (ErrorBoundedQuantizer(eps), BlockSparseQuantizer(eps), BlockSparseRleQuantizer(eps),
              RunLengthQuantizer(eps)):
        b, s = q.quantize(d)
        r = q.dequantize(b, s).to_f32()
        assert r.size == len(vals)
        assert np.all(np.abs(d.to_f32() - r) <= eps * 1.2)


@settings(max_examples=50, deadline=None)
@given(st.lists(st.floats(-10.0, 10.0, width=32), min_size=0, max_size=120), st.floats(0.0009765625, 0.5, width=32))
def test_prop_matches_python_restatement(vals, eps):
    d = F(vals)
    assert ErrorBoundedQuantizer(eps).quantize(d) == eb_quantize(d.numpy(), eps)
    assert BlockSparseQuantizer(eps).quantize(d) == block_sparse(d.numpy(), eps)


@settings(max_examples=30, deadline=None)
@given(st.floats(-100.0, 100.0, width=32), st.integers(10, 100))
def test_prop_predictors_converge(c, n):
    m, lin = MomentumPredictor(0.9), LinearPredictor()
    for _ in range(n):
        m.update(F([c]))
        lin.update(F([c]))
    assert abs(m.predict().to_f32()[0] - c) < 5.0
    assert abs(lin.predict().to_f32()[0] - c) < 1.0


@settings(max_examples=30, deadline=None)
@given(st.lists(st.floats(-100.0, 100.0, width=32), min_size=10, max_size=50))
def test_prop_momentum_stable(vals):
    p = MomentumPredictor(0.9)
    for v in vals:
        p.update(F([v]))
        assert abs(p.predict().to_f32()[0]) <= 300.0


@settings(max_examples=40, deadline=None)
@given(st.lists(st.floats(-50.0, 50.0, width=32), min_size=5, max_size=20))
def test_prop_predictor_reset(vals):
    """proptest_predictors.rs:66-89: after any history, reset leaves no
    prediction (both predictors)."""
    for p in (MomentumPredictor(0.9), LinearPredictor()):
        for v in vals:
            p.update(F([v]))
        assert not p.predict().is_empty()
        p.reset()
        assert p.predict().is_empty()


def test_eb_clamp_count_and_strict_fallback():
    """Codes that saturate at the INT16 ends are counted; a strict quantizer
    raises instead of writing them (error_bounded.rs:5-11,43-46)."""
    from mini_nangila_b200.hpc import QuantizerError

    eps = 1e-3  # scale 2e-3: |v| up to ~65.53 fits
    scale = np.float32(2) * np.float32(eps)
    edge = [32767.5, -32768.5, 32767.4, -32768.4]  # quotients at and just inside the ends
    vals = np.array([0.0, 1.0, -65.0, 70.0, -100.0, 255.0] + [np.float32(e) * scale for e in edge], np.float32)
    r = FixedPointBuffer.from_f32(vals)
    q = np.frombuffer(ErrorBoundedQuantizer(eps).quantize(r)[0], dtype="<i2")
    x = r.to_f32() / scale
    want = int(np.sum((x >= 32767.5) | (x <= -32768.5)))
    assert want == int(np.sum(np.where(x < 0, -np.floor(-x + 0.5), np.floor(x + 0.5)) != q))
    for cls in (ErrorBoundedQuantizer, RunLengthQuantizer, BlockSparseQuantizer, BlockSparseRleQuantizer):
        assert cls(eps).clamp_count(r) == want >= 3
        with pytest.raises(QuantizerError, match="FallbackRequired"):
            cls(eps, strict=True).quantize(r)
        ok = FixedPointBuffer.from_f32(vals[np.abs(x) < 32767])
        assert cls(eps, strict=True).quantize(ok) == cls(eps).quantize(ok)
