"""Cross-decoder fuzzing: random byte strings (and random cuts of valid
streams) decode to the same values on the sm_100a decoders as in the C++
host library, for every stream codec.  Header-carrying formats get a small
element count in their first four bytes (decoders size their output from
it)."""
import numpy as np
import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from mini_nangila_b200.core import FixedPointBuffer, QuantizationMode, UnifiedQuantizer
from mini_nangila_b200.hpc import (BlockSparseQuantizer, BlockSparseRleQuantizer, ErrorBoundedQuantizer,
                                   RunLengthQuantizer)

pytestmark = pytest.mark.gpu

CODECS = {
    "eb": (lambda: ErrorBoundedQuantizer(1e-3), False),
    "rle": (lambda: RunLengthQuantizer(1e-3), False),
    "bs": (lambda: BlockSparseQuantizer(1e-3), True),
    "bsrle": (lambda: BlockSparseRleQuantizer(1e-3), True),
    "topk": (lambda: UnifiedQuantizer(QuantizationMode.TopK(0.1)), True),
    "int4": (lambda: UnifiedQuantizer(QuantizationMode.Stochastic(seed=3, bits=4)), False),
    "int8": (lambda: UnifiedQuantizer(QuantizationMode.Stochastic(seed=3, bits=8)), False),
}


def _bytes(draw_bytes, header, n_header):
    b = bytearray(draw_bytes)
    if header and len(b) >= 4:
        b[0:4] = int(n_header).to_bytes(4, "little")
    return bytes(b)


@pytest.mark.parametrize("codec", sorted(CODECS))
@settings(max_examples=60, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(data=st.binary(min_size=0, max_size=3000), n_header=st.integers(0, 6000),
       scale=st.sampled_from([0.002, 1.0, 0.013]))
def test_random_bytes_decode_like_host(codec, data, n_header, scale):
    make, header = CODECS[codec]
    q = make()
    b = _bytes(data, header, n_header)
    host = q.dequantize(b, scale).numpy()
    dev = q.dequantize(b, scale, device="cuda").numpy()
    assert np.array_equal(dev, host)


@pytest.mark.parametrize("codec", sorted(CODECS))
@settings(max_examples=40, deadline=None)
@given(n=st.integers(1, 20000), sparsity=st.sampled_from([0.0, 0.5, 0.95]), cut=st.floats(0.0, 1.0),
       seed=st.integers(0, 1000))
def test_cut_streams_decode_like_host(codec, n, sparsity, cut, seed):
    make, _ = CODECS[codec]
    q = make()
    g = np.random.default_rng(seed)
    x = (g.standard_normal(n) * 0.01).astype(np.float32)
    x[g.random(n) < sparsity] = 0.0
    b, s = q.quantize(FixedPointBuffer.from_f32(x))
    b = bytes(np.asarray(b, dtype=np.uint8).tobytes() if not isinstance(b, (bytes, bytearray)) else b)
    b = b[: int(len(b) * cut)]
    assert np.array_equal(q.dequantize(b, s, device="cuda").numpy(), q.dequantize(b, s).numpy())
