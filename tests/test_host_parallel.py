"""Host product oracle on several threads and with in-place outputs: the
bytes do not depend on the thread count (NGL_HOST_THREADS), and writing the
error feedback, the average or the EMA state in place gives the same values
as the returning calls (the host DDP hook uses the in-place forms)."""
import numpy as np
import pytest

from mini_nangila_b200 import _ext


def _inputs(n, seed=0):
    rng = np.random.default_rng(seed)
    return [(rng.standard_normal(n) * 1e-3).astype(np.float32) for _ in range(4)]


def _run_all(h, n):
    g, pred, ef, g2 = _inputs(n)
    out = []
    for bits in (4, 8):
        w, e = h.product_encode(g, pred, ef, bits, True, True, 3, 0, 1, 7)
        w2, _ = h.product_encode(g2, pred, ef, bits, True, True, 3, 1, 1, 7)
        out += [w, e, h.product_reduce([w, w2], n, bits, pred, 0.5), h.product_reduce_twoshot([w, w2], n, bits, pred, 0.5)]
    r1, e1 = h.product_topk_encode(g, pred, ef, 13, True)
    r2, _ = h.product_topk_encode(g2, pred, ef, 13, True)
    out += [r1, e1, h.product_topk_reduce([r1, r2], n, 13, pred, 0.5), h.product_ema(pred, g, 0.9, False)]
    return [np.asarray(x).tobytes() for x in out]


def test_results_do_not_depend_on_the_thread_count(monkeypatch):
    h = _ext.host()
    n = 300_001
    runs = []
    for t in ("1", "3", "8"):
        monkeypatch.setenv("NGL_HOST_THREADS", t)
        runs.append(_run_all(h, n))
    assert runs[0] == runs[1] == runs[2]


def test_in_place_outputs_match_the_returning_calls():
    h = _ext.host()
    n = 70_000
    g, pred, ef, g2 = _inputs(n, 1)
    w, e = h.product_encode(g, pred, ef, 4, True, True, 5, 0, 2, 3)
    ef_inout = ef.copy()  # the new error feedback overwrites the old one
    w_in, e_in = h.product_encode(g, pred, ef_inout, 4, True, True, 5, 0, 2, 3, e_out=ef_inout)
    assert e_in is ef_inout and np.array_equal(w, w_in) and np.array_equal(e.view(np.uint32), ef_inout.view(np.uint32))
    avg = h.product_reduce([w, w], n, 4, pred, 0.5)
    out = np.empty(n, np.float32)
    assert h.product_reduce([w, w], n, 4, pred, 0.5, out=out) is out
    assert np.array_equal(avg.view(np.uint32), out.view(np.uint32))
    state = pred.copy()
    h.product_ema_(state, avg, 0.9, False)
    assert np.array_equal(state.view(np.uint32), h.product_ema(pred, avg, 0.9, False).view(np.uint32))


@pytest.mark.parametrize("bad", [np.zeros(10, np.float64), np.zeros(20, np.float32)[::2], np.zeros(9, np.float32)])
def test_in_place_outputs_reject_arrays_they_cannot_write(bad):
    h = _ext.host()
    g, pred, ef, _ = _inputs(10, 2)
    with pytest.raises((RuntimeError, TypeError)):
        h.product_encode(g, pred, ef, 4, True, True, 5, 0, 0, 1, e_out=bad)
    w, _ = h.product_encode(g, pred, ef, 4, True, True, 5, 0, 0, 1)
    with pytest.raises((RuntimeError, TypeError)):
        h.product_reduce([w], 10, 4, pred, 1.0, out=bad)
    ro = np.zeros(10, np.float32)
    ro.flags.writeable = False
    with pytest.raises((RuntimeError, TypeError)):
        h.product_ema_(ro, pred, 0.9, False)
