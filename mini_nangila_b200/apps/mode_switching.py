"""Runtime mode switching between AI and HPC quantization
(examples/mode_switching/src/main.rs).

Training steps compress the momentum-predicted residual with a training
quantizer; every ``--checkpoint-interval`` steps the residual is encoded
with an error-bounded checkpoint codec instead.  The predictor is updated
with the reconstruction (closed loop) in Q8.23 either way.

Defaults reproduce the reference example (sin gradients, global-scale
stochastic INT4, BlockSparse checkpoints — ``--checkpoint-block-sparse`` is
always on there).  ``--preset ar1-block-int4`` runs AR(1) gradients with
block-scaled INT4 and EB checkpoints:
10,000 elements, 50 steps, checkpoint every 10, AR(1) gradients
g_t = 0.9 g_{t-1} + N(0, 1e-3^2) from seed 0 with g_0 ~ N(0, 1e-2^2) and 70 %
of coordinates scaled by 0.01, momentum beta 0.9, stochastic INT4 with one
fp32 scale per 256-element block, error-bounded eps 1e-3 checkpoints.
It prints the overall compression ratio and a determinism hash (SHA-256 of
every step's scale and payload bytes).
"""
from __future__ import annotations

import argparse
import hashlib
import struct
import time

import numpy as np

from ..ai import MomentumPredictor
from ..core import FixedPointBuffer, QuantizationMode, UnifiedQuantizer
from ..core.block_quantizer import BlockStochasticQuantizer
from ..hpc import BlockSparseQuantizer, BlockSparseRleQuantizer


def sin_gradients(n, steps):
    i = np.arange(n, dtype=np.float32)
    for step in range(steps):
        yield (np.sin(np.float32(step) * np.float32(0.1) + i * np.float32(0.001)) * np.float32(0.5)).astype(np.float32)


def ar1_gradients(n, steps, seed=0, rho=0.9, sigma=1e-3, sigma0=1e-2, sparse_frac=0.7, sparse_scale=0.01):
    rng = np.random.default_rng(seed)
    g = rng.normal(0.0, sigma0, n).astype(np.float32)
    scale = np.where(rng.random(n) < sparse_frac, np.float32(sparse_scale), np.float32(1.0)).astype(np.float32)
    for step in range(steps):
        if step:
            g = (np.float32(rho) * g + rng.normal(0.0, sigma, n).astype(np.float32)).astype(np.float32)
        yield (g * scale).astype(np.float32)


def run(num_steps=50, checkpoint_interval=10, gradient_size=10_000, epsilon=1e-3, checkpoint_codec="bs",
        train="rust-int4", train_topk=0.0, generator="sin", seed=42, verbose=True):
    pred = MomentumPredictor(0.9)
    if train_topk > 0.0:
        tq = UnifiedQuantizer(QuantizationMode.TopK(train_topk))
        train_desc = tq.mode_description()
    elif train == "block-int4":
        tq = BlockStochasticQuantizer(seed=seed, bits=4)
        train_desc = f"BlockStochastic (seed={seed}, bits=4, block=256)"
    else:
        tq = UnifiedQuantizer(QuantizationMode.Stochastic(seed=seed, bits=4))
        train_desc = tq.mode_description()
    if checkpoint_codec == "bsrle":
        cq, ck_label = BlockSparseRleQuantizer(epsilon), "ErrorBounded+BlockSparse+RLE"
    elif checkpoint_codec == "bs":
        cq, ck_label = BlockSparseQuantizer(epsilon), "ErrorBounded+BlockSparse"
    else:
        cq, ck_label = UnifiedQuantizer(QuantizationMode.ErrorBounded(epsilon)), "ErrorBounded"
    gen = ar1_gradients(gradient_size, num_steps) if generator == "ar1" else sin_gradients(gradient_size, num_steps)
    h = hashlib.sha256()
    tb = cb = 0
    tt = ct = 0.0
    max_ck_err = 0.0
    if verbose:
        print("=== Unified Quantizer Mode Switching Example ===\n")
        print(f"Initial mode: {train_desc}\n")
    for step, g in enumerate(gen):
        grad = FixedPointBuffer.from_f32(g)
        is_ck = (step + 1) % checkpoint_interval == 0
        t0 = time.perf_counter()
        p = pred.predict()
        resid = grad.clone() if p.is_empty() else grad.sub(p)
        q = cq if is_ck else tq
        b, s = q.quantize(resid)
        dt = time.perf_counter() - t0
        h.update(struct.pack("<f", s))
        h.update(b)
        d = q.dequantize(b, s)
        rec = d if p.is_empty() else p.add(d)
        if is_ck:
            cb += len(b)
            ct += dt
            err = float(np.abs(grad.to_f32() - rec.to_f32()).max())
            max_ck_err = max(max_ck_err, err)
            if verbose:
                print(f"Step {step}: CHECKPOINT")
                print(f"  Codec: {ck_label} | Compressed: {len(b)} bytes (raw: {gradient_size * 4} bytes)")
                print(f"  Compression ratio: {gradient_size * 4 / len(b):.2f}×")
                print(f"  Max error: {err:.2e} (bound: {epsilon:.1e})")
        else:
            tb += len(b)
            tt += dt
        pred.update(rec)
    raw = num_steps * gradient_size * 4
    ratio = raw / max(1, tb + cb)
    out = {"ratio": ratio, "training_bytes": tb, "checkpoint_bytes": cb, "raw_bytes": raw,
           "max_checkpoint_err": max_ck_err, "determinism_hash": h.hexdigest(),
           "training_ms_per_step": 1e3 * tt / max(1, num_steps - num_steps // checkpoint_interval)}
    if verbose:
        print("\n=== Summary ===\n")
        print(f"Overall:\n  Raw data: {raw / 2**20:.2f} MB\n  Compressed: {(tb + cb) / 1024:.1f} KB")
        print(f"  Compression ratio: {ratio:.2f}×")
        print(f"  Determinism hash: {out['determinism_hash']}")
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--preset", choices=["reference", "ar1-block-int4"], default="reference")
    ap.add_argument("--num-steps", type=int, default=50)
    ap.add_argument("--checkpoint-interval", type=int, default=10)
    ap.add_argument("--gradient-size", type=int, default=10_000)
    ap.add_argument("--epsilon", type=float, default=1e-3)
    ap.add_argument("--checkpoint-block-sparse", action="store_true", default=True)
    ap.add_argument("--checkpoint-bsrle", action="store_true")
    ap.add_argument("--checkpoint-codec", choices=["eb", "bs", "bsrle"])
    ap.add_argument("--train-topk", type=float, default=0.0)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    if a.preset == "ar1-block-int4":
        kw = dict(generator="ar1", train="block-int4", checkpoint_codec="eb")
    else:
        kw = dict(generator="sin", train="rust-int4", checkpoint_codec="bsrle" if a.checkpoint_bsrle else "bs")
    if a.checkpoint_codec:
        kw["checkpoint_codec"] = a.checkpoint_codec
    out = run(a.num_steps, a.checkpoint_interval, a.gradient_size, a.epsilon, train_topk=a.train_topk,
              verbose=not a.json, **kw)
    if a.json:
        import json

        print(json.dumps(out))
    return out


if __name__ == "__main__":
    main()
