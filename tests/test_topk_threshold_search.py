"""The per-block top-k threshold search of the fused kernels
(``topk_threshold_bits`` in csrc/cuda/fused_kernels.cu), restated in numpy
over many blocks at once and checked against the C++ oracle
(``product_topk_encode``, whose search is a plain bit-at-a-time greedy): the
bracket search may stop at a different threshold, but the kept index set
must be the same on every block.  The GPU tests compare the kernel's records
with the same oracle byte for byte; this test covers the search on inputs
the kernel tests do not reach (heavy ties, denormals, inf/NaN, all-zero and
partial blocks, k from 1 to 256)."""
import numpy as np
import pytest

from mini_nangila_b200 import _ext

BLOCK = 256


def _bracket_threshold(m: np.ndarray, keff: np.ndarray) -> np.ndarray:
    """m: [B, 256] |c| bit patterns (int64), keff: [B] -> thresholds [B]."""
    M = m.max(axis=1)
    lo = np.zeros_like(M)
    hi = M + 1
    done = hi - lo <= 1
    first = True
    while not done.all():
        if first:
            c3 = np.where(M > (1 << 22), M - (1 << 22), 0)
            c2 = np.where(M > (1 << 23), M - (1 << 23), 0)
            c1 = np.where(M > (2 << 23), M - (2 << 23), 0)
            first = False
        else:
            d = hi - lo
            c1, c2, c3 = lo + (d >> 2), lo + (d >> 1), hi - (d >> 2)
        n1, n2, n3 = ((m >= c[:, None]).sum(axis=1) for c in (c1, c2, c3))
        a = ~done
        t3, t2, t1 = a & (n3 >= keff), a & (n3 < keff) & (n2 >= keff), a & (n2 < keff) & (n1 >= keff)
        t0 = a & (n1 < keff)
        nlo = np.full_like(lo, -1)
        lo = np.where(t3, c3, np.where(t2, c2, np.where(t1, c1, lo)))
        hi = np.where(t2, c3, np.where(t1, c2, np.where(t0, c1, hi)))
        nlo = np.where(t3, n3, np.where(t2, n2, np.where(t1, n1, nlo)))
        done = done | (a & (nlo == keff)) | (hi - lo <= 1)
    return lo


def _kept(m: np.ndarray, T: np.ndarray, keff: np.ndarray, length: np.ndarray) -> list[np.ndarray]:
    valid = np.arange(BLOCK)[None, :] < length[:, None]
    gt = (m > T[:, None]) & valid
    eq = (m == T[:, None]) & valid
    budget = keff - gt.sum(axis=1)
    rank = np.cumsum(eq, axis=1) - 1
    sel = gt | (eq & (rank < budget[:, None]))
    return [np.flatnonzero(s) for s in sel]


def _blocks(rng, nblk: int) -> np.ndarray:
    out = []
    for b in range(nblk):
        kind = b % 8
        if kind == 0:
            x = rng.standard_normal(BLOCK) * 1e-3
        elif kind == 1:
            x = rng.integers(-3, 4, BLOCK) * 0.5  # heavy ties
        elif kind == 2:
            x = np.zeros(BLOCK)
        elif kind == 3:
            x = rng.standard_normal(BLOCK) * 1e-41  # denormals
        elif kind == 4:
            x = rng.standard_normal(BLOCK)
            x[rng.integers(0, BLOCK, 3)] = np.inf
            x[rng.integers(0, BLOCK, 2)] = np.nan
        elif kind == 5:
            x = rng.standard_cauchy(BLOCK) * 1e-5
        elif kind == 6:
            x = np.exp(rng.uniform(-80, 80, BLOCK)) * rng.choice([-1, 1], BLOCK)
        else:
            x = np.full(BLOCK, 0.25)
            x[rng.integers(0, BLOCK, 10)] = 1.0
        out.append(x)
    with np.errstate(over="ignore"):
        return np.concatenate(out).astype(np.float32)


def _oracle_kept(g: np.ndarray, k: int) -> list[np.ndarray]:
    n = g.size
    rec, _ = _ext.host().product_topk_encode(g, None, None, k, False)
    rb = (4 + 2 * k + 3) & ~3
    out = []
    for b in range((n + BLOCK - 1) // BLOCK):
        keff = min(k, n - b * BLOCK)
        r = rec[b * rb:(b + 1) * rb]
        out.append(np.sort(r[4:4 + keff].astype(np.int64)))
    return out


@pytest.mark.parametrize("k", [1, 3, 13, 26, 64, 128, 255, 256])
@pytest.mark.parametrize("tail", [0, 1, 77, 255])
def test_bracket_search_keeps_the_oracle_set(k, tail):
    rng = np.random.default_rng(1000 * k + tail)
    g = _blocks(rng, 48)
    if tail:
        g = np.concatenate([g, _blocks(rng, 1)[:tail]])
    n = g.size
    nblk = (n + BLOCK - 1) // BLOCK
    m = np.zeros((nblk, BLOCK), np.int64)
    bits = (g.view(np.uint32) & 0x7FFFFFFF).astype(np.int64)
    m.reshape(-1)[:n] = bits
    length = np.minimum(BLOCK, n - np.arange(nblk) * BLOCK)
    keff = np.minimum(k, length)
    T = _bracket_threshold(m, keff)
    got = _kept(m, T, keff, length)
    want = _oracle_kept(g, k)
    for b in range(nblk):
        assert np.array_equal(got[b], want[b]), (b, b % 8, k, tail)
