"""Accuracy of the product format against a float64 reduction (host oracle,
CPU): the averaged gradient is within one quantization step per rank of the
exact mean, stochastic rounding is unbiased, and with error feedback the
accumulated error over many steps stays bounded by one step's residual."""
import numpy as np
import pytest

from mini_nangila_b200 import _ext


def _ranks(W, n, seed):
    g = np.random.default_rng(seed)
    return [(g.standard_normal(n) * 1e-3 * (1 + r)).astype(np.float32) for r in range(W)]


def _scales(wire, n, bits):
    """Per-256-block scales of a dense chunked payload."""
    rec = 32 + 8 * (128 if bits == 4 else 256)
    nblk = (n + 255) // 256
    out = np.empty(nblk, np.float32)
    for b in range(nblk):
        c, j = divmod(b, 8)
        out[b] = np.frombuffer(wire[c * rec + 4 * j: c * rec + 4 * j + 4].tobytes(), np.float32)[0]
    return out


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("W", [2, 4, 8])
def test_average_within_one_step_per_rank(bits, W):
    h = _ext.host()
    n = 5000
    gs = _ranks(W, n, 1)
    wires = [h.product_encode(gs[r], None, None, bits, True, False, 7, r, 0, 0)[0] for r in range(W)]
    avg = h.product_reduce(wires, n, bits, None, float(np.float32(1) / np.float32(W)))
    exact = np.mean(np.stack(gs).astype(np.float64), axis=0)
    bound = np.zeros(n)
    for r in range(W):
        bound += np.repeat(_scales(wires[r], n, bits).astype(np.float64), 256)[:n]
    bound /= W
    assert np.all(np.abs(avg - exact) <= bound * (1 + 1e-5) + 1e-9)


def test_stochastic_rounding_unbiased():
    h = _ext.host()
    n = 4096
    g = (np.random.default_rng(3).standard_normal(n) * 1e-3).astype(np.float32)
    acc = np.zeros(n)
    steps = 400
    for s in range(steps):
        w, _ = h.product_encode(g, None, None, 4, True, False, 11, 0, 0, s)
        acc += h.product_reduce([w], n, 4, None, 1.0)
    err = acc / steps - g.astype(np.float64)
    step = np.repeat(_scales(w, n, 4).astype(np.float64), 256)[:n]
    # mean error over 400 independent roundings: ~ step / sqrt(400) per element
    assert abs(err.mean()) < 0.01 * step.mean()
    assert np.abs(err).max() < 0.2 * step.max()


def test_error_feedback_bounds_accumulated_error():
    h = _ext.host()
    n = 4096
    g = (np.random.default_rng(4).standard_normal(n) * 1e-3).astype(np.float32)
    ef = np.zeros(n, np.float32)
    sent = np.zeros(n)
    steps = 200
    for s in range(steps):
        w, ef = h.product_encode(g, None, ef, 4, True, True, 5, 0, 0, s)
        sent += h.product_reduce([w], n, 4, None, 1.0)
    # what was sent + what is still owed = what was produced, exactly up to fp32
    total = steps * g.astype(np.float64)
    assert np.abs(sent + ef - total).max() < 1e-6 * steps
    assert np.abs(ef).max() < 3 * np.abs(g).max()


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("W", [2, 4, 8])
def test_twoshot_average_within_both_stages_bound(bits, W):
    """Two-shot: each chunk owner sums the ranks' stochastic codes, then
    re-encodes the mean as INT8 with round-to-nearest and one scale per
    256-block, which every rank decodes.  Against the float64 mean, the error
    is at most the first stage's one step per rank (averaged) plus half a
    step of the second stage (block absmax of the mean / 127).  That second
    rounding is not seen by error feedback, so its bound is checked alone too:
    the two-shot result is within half a second-stage step of the one-shot
    average that it re-encodes."""
    h = _ext.host()
    n = 5000
    gs = _ranks(W, n, 2)
    wires = [h.product_encode(gs[r], None, None, bits, True, False, 13, r, 0, 0)[0] for r in range(W)]
    inv = float(np.float32(1) / np.float32(W))
    one = h.product_reduce(wires, n, bits, None, inv).astype(np.float64)
    two = h.product_reduce_twoshot(wires, n, bits, None, inv).astype(np.float64)
    exact = np.mean(np.stack(gs).astype(np.float64), axis=0)
    nblk = (n + 255) // 256
    amax = np.array([np.abs(one[b * 256:(b + 1) * 256]).max() for b in range(nblk)])
    half2 = np.repeat(amax / 127.0 / 2.0, 256)[:n]
    stage1 = np.zeros(n)
    for r in range(W):
        stage1 += np.repeat(_scales(wires[r], n, bits).astype(np.float64), 256)[:n]
    stage1 /= W
    assert np.all(np.abs(two - one) <= half2 * (1 + 1e-5) + 1e-12)
    assert np.all(np.abs(two - exact) <= (stage1 + half2) * (1 + 1e-5) + 1e-12)
    # the second stage is round-to-nearest: its error is no larger than the
    # first stage's stochastic error on average
    assert np.abs(two - one).mean() < np.abs(one - exact).mean()
