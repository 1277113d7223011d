"""nangila-core: UnifiedQuantizer (unified_quantizer.rs tests), TopologyMask
(topology.rs tests + doc test), bincode layout, proptests."""
import struct

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from mini_nangila_b200.core import FixedPointBuffer, QuantizationMode, TopologyMask, UnifiedQuantizer

from .rust_semantics import stochastic_int4


def F(x):
    return FixedPointBuffer.from_f32(x)


def test_mode_switching():
    q = UnifiedQuantizer(QuantizationMode.Stochastic(seed=42, bits=4))
    assert isinstance(q.mode(), QuantizationMode.Stochastic)
    q.set_mode(QuantizationMode.ErrorBounded(1e-3))
    assert isinstance(q.mode(), QuantizationMode.ErrorBounded)


def test_stochastic_mode_error():
    q = UnifiedQuantizer(QuantizationMode.Stochastic(seed=42, bits=4))
    d = F([1.0, 2.0, 3.0, 4.0])
    b, s = q.quantize(d)
    r = q.dequantize(b, s).to_f32()
    assert np.all(np.abs(d.to_f32() - r) < s * 0.6 + 1e-6) or np.all(np.abs(d.to_f32() - r[:4]) <= s)
    assert abs(s - 4.0 / 7.5) < 1e-6  # scale = max / 7.5 for INT4


def test_error_bounded_mode():
    q = UnifiedQuantizer(QuantizationMode.ErrorBounded(1e-3))
    d = F([0.5, -0.5, 0.001, -0.001])
    b, s = q.quantize(d)
    assert np.all(np.abs(d.to_f32() - q.dequantize(b, s).to_f32()) < 1e-3 + 1e-6)


def test_topk_mode():
    q = UnifiedQuantizer(QuantizationMode.TopK(0.25))
    x = np.full(100, 0.01, np.float32)
    x[10], x[20], x[50] = 5.0, -5.0, 10.0
    b, s = q.quantize(F(x))
    r = q.dequantize(b, s).to_f32()
    assert abs(r[10] - 5.0) < 0.5 and abs(r[20] + 5.0) < 0.5 and abs(r[50] - 10.0) < 0.5
    assert np.sum(np.abs(r) > 0.1) <= 30


def test_topk_stream_layout_and_ties():
    # 25% of 8 -> keep 2; ties at the threshold are all kept (>= threshold)
    x = np.array([1.0, 3.0, 3.0, 3.0, 0.5, 0.0, 0.0, 0.0], np.float32)
    q = UnifiedQuantizer(QuantizationMode.TopK(0.25))
    b, s = q.quantize(F(x))
    n, mask = struct.unpack_from("<II", b, 0)
    assert n == 8 and mask == 0b1110  # three 3.0 values (ties) kept
    assert abs(s - 3.0 / 127.0) < 1e-7
    assert list(np.frombuffer(b[8:], np.int8)) == [127, 127, 127]


def test_topk_preserves_length_odd():
    q = UnifiedQuantizer(QuantizationMode.TopK(0.2))
    d = F(np.sin(np.arange(45, dtype=np.float32) * np.float32(0.1)))
    b, s = q.quantize(d)
    assert q.dequantize(b, s).len() == 45


def test_topk_malformed_graceful():
    q = UnifiedQuantizer(QuantizationMode.TopK(0.5))
    r = q.dequantize(struct.pack("<II", 10, 0), 1.0)
    assert r.len() == 10 and np.all(r.to_f32() == 0.0)
    g = q.dequantize(struct.pack("<I", 1000) + bytes([0xDE, 0xAD, 0xBE, 0xEF]), 1.0)
    assert g.len() <= 1000


def test_mode_descriptions():
    assert UnifiedQuantizer(QuantizationMode.Stochastic(42, 4)).mode_description() == "Stochastic (seed=42, bits=4)"
    assert UnifiedQuantizer(QuantizationMode.ErrorBounded(1e-3)).mode_description() == "ErrorBounded (ε=1.00e-3)"
    assert UnifiedQuantizer(QuantizationMode.TopK(0.1)).mode_description() == "TopK (k=10.0%)"


@pytest.mark.parametrize("mode", [QuantizationMode.Stochastic(0, 8), QuantizationMode.Stochastic(0, 4),
                                  QuantizationMode.ErrorBounded(1e-3)])
def test_dequantize_empty(mode):
    assert UnifiedQuantizer(mode).dequantize(b"", 1.0).len() == 0


def test_dequantize_truncated_error_bounded():
    assert UnifiedQuantizer(QuantizationMode.ErrorBounded(1e-3)).dequantize(b"\xff", 1.0).len() == 0


@pytest.mark.parametrize("mode", [QuantizationMode.Stochastic(0, 4), QuantizationMode.ErrorBounded(1e-3),
                                  QuantizationMode.TopK(0.1)])
def test_quantize_empty(mode):
    b, _ = UnifiedQuantizer(mode).quantize(FixedPointBuffer.new(0))
    assert b == b""


def test_int4_odd_length_gains_trailing_zero():
    q = UnifiedQuantizer(QuantizationMode.Stochastic(1, 4))
    b, s = q.quantize(F([1.0, 2.0, 3.0]))
    assert len(b) == 2 and q.dequantize(b, s).len() == 4


def test_counter_persists_and_resets():
    q = UnifiedQuantizer(QuantizationMode.Stochastic(7, 4))
    x = F(np.linspace(-1, 1, 33, dtype=np.float32))
    b1, _ = q.quantize(x)
    assert q.counter == 33
    b2, _ = q.quantize(x)
    assert q.counter == 66 and b1 != b2
    q.set_mode(QuantizationMode.Stochastic(7, 4))
    assert q.counter == 0 and q.quantize(x)[0] == b1


@settings(max_examples=50, deadline=None)
@given(st.lists(st.floats(-100.0, 100.0, width=32), min_size=1, max_size=64), st.integers(0, 2**64 - 1),
       st.integers(0, 1000))
def test_stochastic_matches_python_restatement(vals, seed, counter):
    q = UnifiedQuantizer(QuantizationMode.Stochastic(seed, 4))
    q._counter = counter
    d = F(vals)
    b, s = q.quantize(d)
    pb, ps, pc = stochastic_int4(d.numpy(), seed, counter)
    assert b == pb and abs(s - ps) == 0.0 and q.counter == pc


@settings(max_examples=40, deadline=None)
@given(st.lists(st.floats(-100.0, 100.0, width=32), min_size=10, max_size=100))
def test_prop_int8_roundtrip_and_dimension(vals):
    q = UnifiedQuantizer(QuantizationMode.Stochastic(0, 8))
    d = F(vals)
    b, s = q.quantize(d)
    r = q.dequantize(b, s)
    assert r.len() == d.len()
    err = np.abs(d.to_f32() - r.to_f32())
    rel = err / np.maximum(np.abs(d.to_f32()), 1e-6)
    assert np.all((rel < 0.2) | (err < 1.0))


# ------------------------------------------------------------- TopologyMask
def test_variance_threshold_basic_and_doc():
    m = TopologyMask.from_variance_threshold([0.5, 0.1, 0.8, 0.05, 0.6], 0.4)
    assert m.driver_indices == [0, 2, 4] and m.passenger_indices == [1, 3] and m.total_layers == 5
    assert abs(m.compression_factor() - 1.67) < 0.01
    assert abs(m.passenger_percentage() - 40.0) < 0.1
    assert m.is_driver(0) and m.is_passenger(1) and m.is_driver(2) and m.is_passenger(3) and m.is_driver(4)
    assert m.threshold == np.float32(0.5)


def test_edge_cases():
    m = TopologyMask.from_variance_threshold([0.5, 0.1, 0.8], 1.0)
    assert m.driver_indices == [2]
    m = TopologyMask.from_variance_threshold([0.5, 0.1, 0.8], 0.0)
    assert m.driver_indices == [0, 1, 2] and m.passenger_indices == [] and m.compression_factor() == 1.0
    m = TopologyMask.from_variance_threshold([], 0.5)
    assert m.driver_indices == [] and m.total_layers == 0
    a = TopologyMask.all_drivers(10)
    assert len(a.driver_indices) == 10 and a.compression_factor() == 1.0
    assert all(a.is_driver(i) and not a.is_passenger(i) for i in range(10))


def test_bincode_layout_124_bytes_for_12_layers():
    m = TopologyMask.from_variance_threshold(np.arange(12, dtype=np.float32), 0.3)
    b = m.to_bytes()
    assert len(b) == 124
    nd = struct.unpack_from("<Q", b, 0)[0]
    assert nd == 9 and list(struct.unpack_from("<9Q", b, 8)) == m.driver_indices
    np_ = struct.unpack_from("<Q", b, 8 + 72)[0]
    assert np_ == 3
    thr, total = struct.unpack_from("<fQ", b, 8 + 72 + 8 + 24)
    assert total == 12 and thr == np.float32(3.0)
    r = TopologyMask.from_bytes(b)
    assert r.driver_indices == m.driver_indices and r.passenger_indices == m.passenger_indices
    with pytest.raises(ValueError):
        TopologyMask.from_bytes(b[:50])


def test_stable_sort_ties():
    m = TopologyMask.from_variance_threshold([1.0, 1.0, 1.0, 1.0], 0.5)
    assert m.driver_indices == [0, 1]


@settings(max_examples=40, deadline=None)
@given(st.lists(st.floats(0.0, 100.0, width=32), min_size=5, max_size=20), st.floats(0.125, 0.875, width=32))
def test_prop_topology_determinism_coverage(v, drop):
    a = TopologyMask.from_variance_threshold(v, drop)
    b = TopologyMask.from_variance_threshold(v, drop)
    assert a.driver_indices == b.driver_indices and a.passenger_indices == b.passenger_indices
    assert len(a.driver_indices) + len(a.passenger_indices) == len(v)
    assert not set(a.driver_indices) & set(a.passenger_indices)


@settings(max_examples=200, deadline=None)
@given(st.lists(st.integers(-2**31, 2**31 - 1), min_size=0, max_size=200), st.integers(0, 2**32 - 1),
       st.sampled_from([0.9, 0.5, 0.0, 1.0, 0.999, -0.3, 1.7, 1e6, 3e-8]))
def test_fused_momentum_update_matches_the_three_ops(state, seed, beta):
    """The host's one-pass momentum update equals
    state.mul_scalar(beta).add(obs.mul_scalar(1 - beta)) bit for bit."""
    from mini_nangila_b200 import _ext

    h = _ext.host()
    s = np.array(state, np.int32)
    o = np.random.default_rng(seed).integers(-2**31, 2**31, s.size, dtype=np.int64).astype(np.int32)
    b = float(np.float32(beta))
    omb = float(np.float32(1.0) - np.float32(b))
    want = h.q823_add(h.q823_mul_scalar(s, b), h.q823_mul_scalar(o, omb))
    assert np.array_equal(h.q823_momentum_update(s, o, b, omb), want)
