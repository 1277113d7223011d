"""BlockStochasticQuantizer: the fused hook's per-256-block format as a
standalone quantizer (host).  Per-block error within one quantization step,
unbiased stochastic rounding, reproducible bytes per (seed, rank, stream,
call), truncation rejected."""
import numpy as np
import pytest

from mini_nangila_b200.core import FixedPointBuffer
from mini_nangila_b200.core.block_quantizer import BlockStochasticQuantizer


@pytest.mark.parametrize("bits,levels", [(4, 7.0), (8, 127.0)])
@pytest.mark.parametrize("n", [1, 255, 256, 257, 5000])
def test_error_within_one_step_per_block(bits, levels, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * np.exp(rng.uniform(-6, 0, n))).astype(np.float32)
    q = BlockStochasticQuantizer(seed=3, bits=bits)
    b, scale = q.quantize(FixedPointBuffer.from_f32(x))
    y = q.dequantize(b, scale).to_f32()
    assert y.size == n
    for s in range(0, n, 256):
        blk = x[s:s + 256]
        step = np.abs(blk).max() / levels
        assert np.abs(y[s:s + 256] - blk).max() <= step * (1 + 1e-5) + 2.0 ** -22


def test_unbiased_and_reproducible():
    x = np.full(256, 0.3, np.float32)
    x[0] = 1.0  # block scale 1/7: 0.3 sits between codes 2 and 3
    acc = np.zeros(256)
    q = BlockStochasticQuantizer(seed=11)
    for _ in range(400):
        acc += q.dequantize(*q.quantize(FixedPointBuffer.from_f32(x))).to_f32()
    assert abs(acc[1:].mean() / 400 - 0.3) < 2e-3
    a = BlockStochasticQuantizer(seed=5, rank=1, stream=2).quantize(FixedPointBuffer.from_f32(x))[0]
    b = BlockStochasticQuantizer(seed=5, rank=1, stream=2).quantize(FixedPointBuffer.from_f32(x))[0]
    c = BlockStochasticQuantizer(seed=5, rank=2, stream=2).quantize(FixedPointBuffer.from_f32(x))[0]
    assert a == b and a != c


def test_truncated_payload_is_rejected():
    q = BlockStochasticQuantizer()
    b, _ = q.quantize(FixedPointBuffer.from_f32(np.ones(1000, np.float32)))
    with pytest.raises(ValueError, match="truncated"):
        q.dequantize(b[:-10])
    assert q.dequantize(b[:3]).len() == 0
