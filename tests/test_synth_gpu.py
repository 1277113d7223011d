"""Device workload generators vs a numpy restatement of the same Philox4x32-10
counters and Box-Muller transform (float64 math; the device uses CUDA's
float32 log/sqrt/sincospi, so values agree to float32 rounding)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

M0, M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
W0, W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)


def philox(c0, c1, c2, c3, k0, k1):
    c = [np.asarray(x, np.uint32).copy() for x in (c0, c1, c2, c3)]
    k0, k1 = np.uint32(k0), np.uint32(k1)
    for _ in range(10):
        p0 = M0 * c[0].astype(np.uint64)
        p1 = M1 * c[2].astype(np.uint64)
        hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), (p0 & np.uint64(0xFFFFFFFF)).astype(np.uint32)
        hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), (p1 & np.uint64(0xFFFFFFFF)).astype(np.uint32)
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
        k0 = np.uint32((int(k0) + int(W0)) & 0xFFFFFFFF)
        k1 = np.uint32((int(k1) + int(W1)) & 0xFFFFFFFF)
    return c


def u01(b):
    return ((b >> np.uint32(8)).astype(np.float64) + 1.0) / 16777216.0


def gauss(r):
    return np.sqrt(-2.0 * np.log(u01(r[0]))) * np.cos(2.0 * np.pi * u01(r[1]))


def draw(seed, i, step, stream):
    i = np.asarray(i, np.uint64)
    return philox((i & np.uint64(0xFFFFFFFF)).astype(np.uint32), (i >> np.uint64(32)).astype(np.uint32),
                  np.full(i.shape, step, np.uint32), np.full(i.shape, stream, np.uint32),
                  seed & 0xFFFFFFFF, seed >> 32)


def test_philox_restatement_matches_product_noise():
    # The same Philox drives the product format's stochastic rounding; its
    # host implementation is the oracle for this restatement.
    from mini_nangila_b200 import _ext

    c = _ext.cuda()
    x = c.synth_brownian(5, 1, seed=7, sigma=0.0, box=1.0, lo=0.0, periodic=False).cpu().numpy()[0]
    r = draw(7, np.arange(5), 0, 0x4C4D5000)
    assert np.allclose(x, u01(r[0]) - 2.0 ** -24, rtol=0, atol=1e-7)


def test_ar1_matches_reference_math():
    from mini_nangila_b200 import _ext

    n, T, seed = 4097, 6, 123
    out = _ext.cuda().synth_ar1(n, T, seed=seed, rho=0.9, sigma=1e-3, sigma0=1e-2, sparse_frac=0.7,
                                sparse_scale=0.01).cpu().numpy()
    i = np.arange(n)
    r0 = draw(seed, i, 0, 0x41523100)
    scale = np.where(u01(r0[2]) <= 0.7, 0.01, 1.0)
    g = 1e-2 * gauss(r0)
    for t in range(T):
        if t:
            g = 0.9 * g + 1e-3 * gauss(draw(seed, i, t, 0x41523101))
        np.testing.assert_allclose(out[t], g * scale, rtol=2e-4, atol=1e-9)
    # the distribution: AR(1) with rho 0.9 keeps a std near sigma0 * rho^t
    assert 0.6 < np.std(out[0][scale == 1.0]) / 1e-2 < 1.4


@pytest.mark.parametrize("periodic", [True, False])
def test_brownian_matches_reference_math(periodic):
    from mini_nangila_b200 import _ext

    n, T, seed, box, lo, sigma = 3 * 1001, 5, 9, 100.0, -50.0, 0.5
    out = _ext.cuda().synth_brownian(n, T, seed=seed, sigma=sigma, box=box, lo=lo, periodic=periodic).cpu().numpy()
    i = np.arange(n)
    x = lo + box * (u01(draw(seed, i, 0, 0x4C4D5000)[0]) - 2.0 ** -24)
    for t in range(T):
        if t:
            x = x + sigma * gauss(draw(seed, i, t, 0x4C4D5001))
            if periodic:
                x = lo + np.mod(x - lo, box)
        d = out[t] - x
        if periodic:
            d = (d + box / 2) % box - box / 2  # distance on the circle
            assert out[t].min() >= lo and out[t].max() < lo + box
        assert np.abs(d).max() < 1e-3
