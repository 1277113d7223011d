"""Q8.23 math (nangila-math tests: fixed_point.rs, ops.rs, determinism.rs,
proptest_fixed_point.rs; determinism_hash example)."""
import hashlib

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from mini_nangila_b200.core import FixedPointBuffer, FixedQ, ShapeMismatch

from .rust_semantics import from_f32 as py_from_f32

Q = 1 << 23
RATIONALS = [0.0, 1.0, -1.0, 0.5, -0.5, 0.25, -0.25, 0.75, -0.75, 1.25, -1.25, 127.0, -128.0]


def f32s(lo, hi, min_size=1, max_size=100):
    return st.lists(st.floats(lo, hi, width=32, allow_nan=False), min_size=min_size, max_size=max_size)


def test_determinism_hash():
    b = FixedPointBuffer.from_f32(RATIONALS).numpy().astype("<i4").tobytes()
    assert hashlib.sha256(b).hexdigest() == "c18cd836f0cb712247e0ace683d710b8550f3e3f40a6a2998252df59498aab56"


def test_rationals_exact():
    exp = [0, Q, -Q, Q // 2, -Q // 2, Q // 4, -Q // 4, 3 * Q // 4, -3 * Q // 4, Q + Q // 4, -Q - Q // 4, 127 * Q,
           -128 * Q]
    buf = FixedPointBuffer.from_f32(RATIONALS)
    assert buf.numpy().tolist() == exp
    assert np.allclose(buf.to_f32(), RATIONALS, atol=1e-6)


def test_add_sub_mul_scalar_determinism():
    a = FixedPointBuffer.from_f32([1.25, -0.75])
    b = FixedPointBuffer.from_f32([0.25, 0.5])
    assert a.add(b).numpy().tolist() == [3 * Q // 2, -Q // 4]
    assert a.sub(b).numpy().tolist() == [Q, -Q - Q // 4]
    assert a.mul_scalar(0.5).numpy().tolist() == [(Q + Q // 4) // 2, -((3 * Q) // 4) // 2]


def test_roundtrip_and_saturation():
    inp = [0.0, 1.0, -1.0, 0.5, -0.5, 127.0, -128.0]
    assert np.allclose(FixedPointBuffer.from_f32(inp).to_f32(), inp, atol=1e-6)
    out = FixedPointBuffer.from_f32([200.0, -200.0]).to_f32()
    assert out[0] > 127.0 and out[1] < -127.0
    sat = FixedPointBuffer.from_f32([1e30, -1e30, float("inf"), float("-inf"), float("nan")]).numpy()
    assert sat.tolist() == [2**31 - 1, -(2**31), 2**31 - 1, -(2**31), 0]


def test_add_mul_examples():
    c = FixedPointBuffer.from_f32([1.0, 2.0]).add(FixedPointBuffer.from_f32([0.5, -0.5])).to_f32()
    assert np.allclose(c, [1.5, 1.5], atol=1e-6)
    d = FixedPointBuffer.from_f32([10.0, -10.0]).mul_scalar(0.5).to_f32()
    assert np.allclose(d, [5.0, -5.0], atol=1e-6)


def test_shape_mismatch():
    a, b = FixedPointBuffer.from_f32([1.0]), FixedPointBuffer.from_f32([1.0, 2.0])
    for op in (a.add, a.sub):
        try:
            op(b)
        except ShapeMismatch as e:
            assert "1 vs 2" in str(e)
        else:
            raise AssertionError("expected ShapeMismatch")


def test_saturating_add_edges():
    big = FixedPointBuffer(np.array([2**31 - 1, -(2**31)], np.int32))
    one = FixedPointBuffer(np.array([1, -1], np.int32))
    assert big.add(one).numpy().tolist() == [2**31 - 1, -(2**31)]
    assert big.sub(FixedPointBuffer(np.array([-1, 1], np.int32))).numpy().tolist() == [2**31 - 1, -(2**31)]


def test_fixedq_rounding_quirk():
    # nangila-edge adds +-0.5 in f32: for odd s in [2^23, 2^24) the sum rounds to even.
    x = np.float32((2**23 + 1) / 2**23)  # s = 2^23 + 1 (odd)
    a = FixedPointBuffer.from_f32([x]).numpy()[0]
    b = FixedQ.from_f32([x]).data[0]
    assert a == 2**23 + 1 and b == 2**23 + 2
    assert FixedQ.from_f32([1.0, -1.0]).to_f32().tolist() == [1.0, -1.0]


@settings(max_examples=60, deadline=None)
@given(f32s(-255.0, 255.0, 1, 200))
def test_prop_roundtrip(vals):
    out = FixedPointBuffer.from_f32(vals).to_f32()
    assert np.all(np.abs(np.asarray(vals, np.float32) - out) < 2e-6)


@settings(max_examples=40, deadline=None)
@given(f32s(-100.0, 100.0, 1, 60), f32s(-100.0, 100.0, 1, 60))
def test_prop_commutative_and_inverse(a, b):
    n = min(len(a), len(b))
    A, B = FixedPointBuffer.from_f32(a[:n]), FixedPointBuffer.from_f32(b[:n])
    assert A.add(B) == B.add(A)
    assert np.all(np.abs(A.add(B).sub(B).to_f32() - A.to_f32()) < 1e-5)


@settings(max_examples=40, deadline=None)
@given(f32s(-50.0, 50.0, 1, 40), f32s(-50.0, 50.0, 1, 40), st.floats(-2.0, 2.0, width=32))
def test_prop_distributive(a, b, k):
    n = min(len(a), len(b))
    A, B = FixedPointBuffer.from_f32(a[:n]), FixedPointBuffer.from_f32(b[:n])
    lhs = A.add(B).mul_scalar(k).to_f32()
    rhs = A.mul_scalar(k).add(B.mul_scalar(k)).to_f32()
    assert np.all(np.abs(lhs - rhs) < 1e-4)


@settings(max_examples=40, deadline=None)
@given(st.lists(st.floats(allow_nan=False, width=32), min_size=1, max_size=10))
def test_prop_saturation(vals):
    out = FixedPointBuffer.from_f32(vals).to_f32()
    assert np.all((out >= -256.0) & (out <= 256.0))


def test_regression_extreme_value():
    # proptest regression seed: extreme_vals = [6.2555353e16]
    assert FixedPointBuffer.from_f32([6.2555353e16]).numpy().tolist() == [2**31 - 1]


@settings(max_examples=60, deadline=None)
@given(st.lists(st.one_of(st.floats(-300.0, 300.0, width=32), st.just(float("nan"))), min_size=1, max_size=64))
def test_prop_matches_python_restatement(vals):
    assert FixedPointBuffer.from_f32(vals).numpy().tolist() == py_from_f32(vals).tolist()
