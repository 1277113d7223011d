"""Golden digest of the host library: SHA-256 over the outputs of every
codec entry point (Q8.23 ops, stochastic INT4/INT8 and the deterministic
fallback, top-k, EB / RLE / BlockSparse / BlockSparse+RLE both ways, `.nz`
compress and decompress, the product-format oracle) on seeded random inputs
with NaN, inf, signed zeros, denormals and values at the Q8.23 range mixed
in.  The digest was recorded from the scalar implementation, before the
host fast paths, threads and vector clones; any change to a single output
bit fails it."""
import hashlib

import numpy as np

GOLDEN = "911e8eb33d9da559373f1ee94597a5d16bdfe8463b2f3a9250ce68ae4023e7f9"


def outputs_digest(h) -> str:
    rng = np.random.default_rng(2024)
    sha = hashlib.sha256()

    def f32(n, special):
        x = (rng.standard_normal(n) * np.exp(rng.uniform(-10, 4, n))).astype(np.float32)
        if special and n:
            idx = rng.integers(0, n, max(1, n // 40))
            x[idx] = rng.choice(np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 3e38, -3e38, 1e-42, 255.9, -256.0, 0.5,
                                          2.5], np.float32), idx.size)
        return x

    def add(*xs):
        for x in xs:
            if isinstance(x, np.ndarray):
                sha.update(np.ascontiguousarray(x).tobytes())
            elif isinstance(x, float):
                sha.update(np.float32(x).tobytes())
            elif isinstance(x, (bytes, bytearray)):
                sha.update(bytes(x))
            else:
                sha.update(repr(x).encode())

    for trial in range(24):
        n = int(rng.integers(0, 20000)) if trial % 4 else int(rng.integers(0, 70))
        sp = trial % 2 == 1
        x = f32(n, sp)
        q = h.q823_from_f32(x)
        q2 = h.q823_from_f32(f32(n, sp))
        add(q, h.q823_to_f32(q), h.q823_add(q, q2), h.q823_sub(q, q2), h.q823_mul_scalar(q, 0.9),
            h.fixedq_from_f32(x))
        for bits in (4, 8, 3):
            for c0 in (0, 2**63 + 7):
                qb, s, c = h.stochastic_quantize(q, bits, 42 if c0 == 0 else 2**64 - 99, c0)
                add(qb, s, c, h.stochastic_dequantize(qb, s, bits))
        for k in (0.0, 0.05, 1.0):
            qb, s = h.topk_quantize(q, k)
            add(qb, s, h.topk_dequantize(qb, s))
        for eps in (1e-3, 0.05):
            for name in ("eb", "rle", "bs", "bsrle"):
                qb, s = getattr(h, name + "_quantize")(q, eps)
                add(qb, s, getattr(h, name + "_dequantize")(qb, s))
        P, T = max(1, n // 10), 10 if n >= 10 else 1
        data = f32(P * T, False)
        for codec in (1, 2, 3, 4):
            blob, st = h.nz_compress(data, P, T, codec, 1e-3)
            add(blob, repr(sorted(dict(st).items())), h.nz_decompress(blob, True), h.nz_decompress(blob, False))
        g, pred, ef, g2 = x, f32(n, False), f32(n, False), f32(n, False)
        for bits in (4, 8):
            w, e = h.product_encode(g, pred, ef, bits, True, True, 9, 1, 2, trial)
            w2, _ = h.product_encode(g2, pred, ef, bits, True, True, 9, 0, 2, trial)
            add(w, e, h.product_reduce([w, w2], n, bits, pred, 0.5), h.product_reduce_twoshot([w, w2], n, bits, pred, 0.5))
        r1, e1 = h.product_topk_encode(g, pred, ef, 13, True)
        add(r1, e1, h.product_topk_reduce([r1, r1], n, 13, pred, 0.5), h.product_ema(pred, g, 0.9, False))
    return sha.hexdigest()


def test_host_outputs_match_the_golden_digest(monkeypatch):
    from mini_nangila_b200 import _ext

    for threads in ("1", "4"):
        monkeypatch.setenv("NGL_HOST_THREADS", threads)
        assert outputs_digest(_ext.host()) == GOLDEN
