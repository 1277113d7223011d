"""Chunk-granular static topology drop of the product format (host oracle):
exactly the requested number of passenger chunks, identical on every rank,
passengers send a zero record and keep their residual as error feedback,
kept chunks are byte-identical to an encode without topology."""
import math

import numpy as np
import pytest

from mini_nangila_b200 import _ext
from mini_nangila_b200.parallel.fused import nchunks_of, topology, wire_bytes

CH = 2048


def _passengers(nch, t):
    a, b, nd = t
    return np.array([((c * a + b) % nch) < nd for c in range(nch)], bool)


@pytest.mark.parametrize("nch", [1, 2, 3, 7, 64, 1000, 4096])
@pytest.mark.parametrize("drop", [0.0, 0.1, 0.3, 0.5, 0.99, 1.0])
def test_exact_passenger_count(nch, drop):
    t = _ext.host().product_topology(nch, drop, 424242, 5)
    a, b, nd = t
    keep = max(1, math.floor(nch * (1 - drop)))
    assert nd == nch - keep
    assert math.gcd(a, nch) == 1 and 0 < a and (a < nch or nch == 1) and 0 <= b < nch
    assert _passengers(nch, t).sum() == nd
    # same parameters for the same (seed, stream) -> every rank agrees
    assert tuple(_ext.host().product_topology(nch, drop, 424242, 5)) == tuple(t)


def test_streams_differ():
    a = _passengers(1000, _ext.host().product_topology(1000, 0.3, 1, 0))
    b = _passengers(1000, _ext.host().product_topology(1000, 0.3, 1, 1))
    assert not np.array_equal(a, b)


@pytest.mark.parametrize("mode", ["int4", "int8", "topk"])
def test_passenger_records_and_error_feedback(mode):
    h = _ext.host()
    n = 37 * CH + 100
    rng = np.random.default_rng(0)
    g = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    pred = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    ef = (rng.standard_normal(n) * 1e-4).astype(np.float32)
    t = topology(n, 0.3, 7, 2)
    k = 13
    if mode == "topk":
        w0, e0 = h.product_topk_encode(g, pred, ef, k, True)
        w1, e1 = h.product_topk_encode(g, pred, ef, k, True, t)
        rec = 8 * ((4 + 2 * k + 3) & ~3)
    else:
        bits = 4 if mode == "int4" else 8
        w0, e0 = h.product_encode(g, pred, ef, bits, True, True, 3, 0, 2, 1)
        w1, e1 = h.product_encode(g, pred, ef, bits, True, True, 3, 0, 2, 1, t)
        rec = 32 + 8 * (128 if bits == 4 else 256)
    nch = nchunks_of(n)
    pas = _passengers(nch, t)
    assert pas.sum() == t[2] > 0
    resid = ((g - pred).astype(np.float32) + ef).astype(np.float32)
    for c in range(nch):
        r0, r1 = w0[c * rec:(c + 1) * rec], w1[c * rec:(c + 1) * rec]
        sl = slice(c * CH, min(n, (c + 1) * CH))
        if pas[c]:
            assert not r1.any()
            assert np.array_equal(e1[sl].view(np.uint32), resid[sl].view(np.uint32))
        else:
            assert np.array_equal(r0, r1)
            assert np.array_equal(e0[sl].view(np.uint32), e1[sl].view(np.uint32))
    assert wire_bytes(n, mode, k, 0.3, 7, 2) == (nch - t[2]) * rec
    # the reduction of passenger chunks is the prediction itself
    if mode != "topk":
        avg = h.product_reduce([w1, w1], n, bits, pred, 0.5)
        for c in np.flatnonzero(pas):
            sl = slice(c * CH, min(n, (c + 1) * CH))
            assert np.array_equal(avg[sl].view(np.uint32), pred[sl].view(np.uint32))
