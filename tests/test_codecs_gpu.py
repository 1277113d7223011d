"""sm_100a codec kernels vs the C++ host library: identical bytes and
identical decoded Q8.23 values for every reference format."""
import numpy as np
import pytest
import torch

from mini_nangila_b200 import _ext
from mini_nangila_b200.checkpoint import lammps, nzcp
from mini_nangila_b200.core import FixedPointBuffer, QuantizationMode, UnifiedQuantizer
from mini_nangila_b200.hpc import BlockSparseQuantizer, BlockSparseRleQuantizer, ErrorBoundedQuantizer, \
    RunLengthQuantizer
from mini_nangila_b200.ops import trajectory

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 31, 32, 33, 255, 256, 257, 4095, 4096, 4097, 100003]


def _resid(n, seed, sparsity=0.7, scale=0.01):
    g = np.random.default_rng(seed)
    x = (g.standard_normal(n) * scale).astype(np.float32)
    x[g.random(n) < sparsity] = 0.0
    return FixedPointBuffer.from_f32(x)


def _host_bytes(b):
    return b if isinstance(b, bytes) else b.tobytes()


@pytest.mark.parametrize("n", SIZES)
def test_q823_ops(n):
    g = np.random.default_rng(n)
    x = (g.standard_normal(n) * 50).astype(np.float32)
    x[: min(n, 3)] = [1e30, -1e30, np.nan][: min(n, 3)]
    h = FixedPointBuffer.from_f32(x)
    d = FixedPointBuffer.from_f32(torch.from_numpy(x).cuda())
    assert np.array_equal(d.numpy(), h.numpy())
    assert np.array_equal(d.to_f32().cpu().numpy().view(np.uint32), h.to_f32().view(np.uint32))
    y = FixedPointBuffer.from_f32((g.standard_normal(n) * 50).astype(np.float32))
    assert np.array_equal(d.add(y.cuda()).numpy(), h.add(y).numpy())
    assert np.array_equal(d.sub(y.cuda()).numpy(), h.sub(y).numpy())
    for s in (0.9, np.float32(1.0) - np.float32(0.9), -1.5, 0.5):
        assert np.array_equal(d.mul_scalar(s).numpy(), h.mul_scalar(s).numpy())


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("cls", [ErrorBoundedQuantizer, BlockSparseQuantizer, BlockSparseRleQuantizer,
                                 RunLengthQuantizer])
@pytest.mark.parametrize("sparsity", [0.0, 0.7, 0.99])
def test_eb_family_bytes_and_decode(n, cls, sparsity):
    q = cls(1e-3)
    r = _resid(n, 11, sparsity)
    hb, hs = q.quantize(r)
    db, ds = q.quantize(r.cuda())
    assert ds == hs
    assert db.cpu().numpy().tobytes() == _host_bytes(hb)
    hr = q.dequantize(hb, hs)
    dr = q.dequantize(hb, hs, device="cuda")
    assert np.array_equal(dr.numpy(), hr.numpy())


@pytest.mark.parametrize("cls", [BlockSparseQuantizer, BlockSparseRleQuantizer, RunLengthQuantizer])
def test_truncated_streams_decode_like_host(cls):
    q = cls(1e-3)
    r = _resid(3000, 5, 0.5)
    hb, hs = q.quantize(r)
    for cut in (1, 3, 4, 5, 7, 40, len(hb) // 2, len(hb) - 1):
        b = hb[:cut]
        assert np.array_equal(q.dequantize(b, hs, device="cuda").numpy(), q.dequantize(b, hs).numpy()), cut


@pytest.mark.parametrize("sparsity", [0.0, 0.5, 0.99])
def test_truncated_multiwindow_blocksparse(sparsity):
    # Streams longer than the 16 KB decode windows, cut at and around window
    # boundaries and inside blocks: the window-parallel decoder must follow
    # the reference's tolerant decode exactly.
    q = BlockSparseQuantizer(1e-3)
    r = _resid(120001, 9, sparsity)
    hb, hs = q.quantize(r)
    W = 16384
    cuts = {len(hb), len(hb) - 1, len(hb) - 3, len(hb) // 3}
    for k in (1, 2, 3):
        for d in (-5, -4, -2, -1, 0, 1, 2, 3, 4, 5, 37):
            c = 4 + k * W + d
            if 0 < c <= len(hb):
                cuts.add(c)
    for cut in sorted(cuts):
        b = hb[:cut]
        assert np.array_equal(q.dequantize(b, hs, device="cuda").numpy(), q.dequantize(b, hs).numpy()), cut


def test_topk_compat_truncated_multiwindow():
    g = np.random.default_rng(3)
    x = g.standard_normal(400000).astype(np.float32)
    r = FixedPointBuffer.from_f32(x)
    q = UnifiedQuantizer(QuantizationMode.TopK(0.5))
    hb, hs = q.quantize(r)
    for cut in (len(hb), len(hb) - 1, 4 + 16384 + 1, 4 + 2 * 16384 - 2, len(hb) // 2 + 1):
        b = hb[:cut]
        assert np.array_equal(q.dequantize(b, hs, device="cuda").numpy(), q.dequantize(b, hs).numpy()), cut


def test_long_zero_runs():
    x = np.zeros(200000, np.float32)
    x[::50000] = 1.0
    r = FixedPointBuffer.from_f32(x)
    for cls in (BlockSparseRleQuantizer, RunLengthQuantizer):
        q = cls(1e-3)
        hb, hs = q.quantize(r)
        db, _ = q.quantize(r.cuda())
        assert db.cpu().numpy().tobytes() == hb


@pytest.mark.parametrize("n", [1, 2, 3, 31, 1000, 65537])
@pytest.mark.parametrize("bits", [4, 8, 3])
def test_stochastic_compat(n, bits):
    r = _resid(n, 3, 0.2, 1.0)
    hq = UnifiedQuantizer(QuantizationMode.Stochastic(seed=2**63 + 5, bits=bits))
    dq = UnifiedQuantizer(QuantizationMode.Stochastic(seed=2**63 + 5, bits=bits))
    for _ in range(2):  # counter persists across calls
        hb, hs = hq.quantize(r)
        db, ds = dq.quantize(r.cuda())
        assert ds == hs and db.cpu().numpy().tobytes() == hb
    assert hq.counter == dq.counter
    assert np.array_equal(dq.dequantize(hb, hs, device="cuda").numpy(), hq.dequantize(hb, hs).numpy())


@pytest.mark.parametrize("n", [1, 7, 32, 100, 1000, 65537, 300000])
@pytest.mark.parametrize("k", [0.0, 0.001, 0.05, 0.1, 0.25, 1.0, 1.5])
def test_topk_compat(n, k):
    g = np.random.default_rng(n)
    x = (g.standard_normal(n)).astype(np.float32)
    x[g.random(n) < 0.3] = 0.25  # ties
    r = FixedPointBuffer.from_f32(x)
    q = UnifiedQuantizer(QuantizationMode.TopK(k))
    hb, hs = q.quantize(r)
    db, ds = q.quantize(r.cuda())
    assert ds == hs
    assert db.cpu().numpy().tobytes() == hb
    assert np.array_equal(q.dequantize(hb, hs, device="cuda").numpy(), q.dequantize(hb, hs).numpy())


@pytest.mark.parametrize("codec", ["eb", "rle", "bs", "bsrle"])
@pytest.mark.parametrize("P,T,eps", [(30001, 7, 1e-3), (300007, 3, 1e-3), (300007, 3, 0.05), (1, 3, 1e-3),
                                     (33, 2, 1e-3), (131073, 2, 1e-2)])
def test_nz_pipeline_device_matches_host(codec, P, T, eps):
    # Multi-tile streams (BlockSparse tiles of 16384 codes, run tiles of 4096
    # items), dense and sparse codes, and one- and two-block snapshots.
    data = lammps.generate_synthetic(P, T)
    hb, hst = nzcp.compress(data, P, T, codec, eps)
    db, dst = trajectory.compress(torch.from_numpy(data).cuda().view(T, P), codec, eps)
    assert db == hb
    assert dst["total_comp"] == hst["total_comp"]
    assert abs(dst["max_abs_err"] - hst["max_abs_err"]) == 0.0
    host_vals = nzcp.decompress(hb)
    dev_vals = trajectory.decompress(hb).cpu().numpy().reshape(-1)
    assert np.array_equal(dev_vals.view(np.uint32), host_vals.view(np.uint32))


@pytest.mark.parametrize("eps", [1e-3, 5e-7, 0.05, 1.5, 3e-5, 1e-35])
def test_eb_codes_match_host_at_near_ties(eps):
    """Device EB codes equal the host library's on quotients placed at and
    around half-integers (where round-half-away after the f32 division
    decides), across the clamp boundary, and on random residuals."""
    from mini_nangila_b200 import _ext

    h, c = _ext.host(), _ext.cuda()
    g = np.random.default_rng(int(eps * 1e9) % 1000)
    s = float(np.float32(2.0) * np.float32(eps))
    k = g.integers(-45000, 45000, 300000).astype(np.float64)
    d = g.integers(-12, 13, k.size).astype(np.float64)
    v = (k + 0.5) * s + d * 2.0 ** -23  # near-ties, a few Q8.23 steps apart
    r_near = np.clip(np.round(v * 2.0 ** 23), -2 ** 31, 2 ** 31 - 1).astype(np.int32)
    r_rand = g.integers(-2 ** 31, 2 ** 31 - 1, 300000, dtype=np.int64).astype(np.int32)
    r_small = g.integers(-2 ** 16, 2 ** 16, 300000).astype(np.int32)
    for r in (r_near, r_rand, r_small):
        hb, _ = h.eb_quantize(r, float(np.float32(eps)))
        host = np.frombuffer(bytes(hb), dtype="<i2")
        dev = c.eb_codes(torch.from_numpy(r).cuda(), s).cpu().numpy()
        bad = np.flatnonzero(host != dev)
        assert bad.size == 0, (bad[:5], r[bad[:5]], host[bad[:5]], dev[bad[:5]])


def test_eb_clamp_count_on_the_device_matches_the_host():
    from mini_nangila_b200.hpc import QuantizerError

    r = _resid(100003, 5, 0.5, scale=40.0)  # |v| up to ~200: many codes saturate at eps 1e-3
    q = ErrorBoundedQuantizer(1e-3)
    k = q.clamp_count(r)
    assert k > 0 and q.clamp_count(r.cuda()) == k
    with pytest.raises(QuantizerError, match=f"FallbackRequired: {k} of"):
        ErrorBoundedQuantizer(1e-3, strict=True).quantize(r.cuda())
