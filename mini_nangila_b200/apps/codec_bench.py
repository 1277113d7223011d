"""GPU error-bounded trajectory codec benchmark (1 GPU).

    python -m mini_nangila_b200.apps.codec_bench [--atoms 1000000] [--steps 100] [--epsilon 1e-3]

Synthetic LAMMPS-style trajectory from the device generator (Philox +
Box-Muller, ``csrc/cuda/synth_kernels.cu``): positions uniform in a 100^3
box centred on the origin ([-50, 50)^3), each step adds an N(0, 0.01^2)
displacement per coordinate; fp32 x/y/z of every atom form one snapshot
(3 * atoms values).  ``--fields pos,vel`` adds the velocity field, N(0, 1)
per coordinate and step, and reports both fields and their total.  The first snapshot has no prediction, so its codes are
the coordinates themselves: a box reaching 100 would exceed the INT16 code
range at eps 1e-3 (+-65.5) in the reference's format.  The codec sees unwrapped
coordinates (LAMMPS xu/yu/zu): with periodic wrap a boundary crossing is a
~100-unit residual, beyond INT16 range at eps 1e-3 (32767 * 2 eps = 65.5) in
the reference's format, which has no escape code; ``--wrapped`` runs the
wrapped positions (the max error then shows the clamping).

For EB, EB+BlockSparse and EB+BlockSparse+RLE it reports device encode and
decode GB/s (raw fp32 bytes / CUDA-event time of the device pipeline: the
closed loop of every step and the packers; all step payloads decoded and the
predictor add-back chain), the compression ratio, the max error, byte
identity with the C++ host library on the first steps, and the host
library's single-thread MB/s on the same data as the CPU baseline.
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np
import torch

from ..checkpoint import nzcp
from ..ops import trajectory


def make_positions(atoms, steps, sigma, box, seed, wrapped, device):
    """[steps, 3 * atoms] positions from the device Brownian generator
    (Philox + Box-Muller), uniform start in [-box/2, box/2)."""
    from .._ext import cuda

    dev = torch.device(device)
    return cuda().synth_brownian(3 * atoms, steps, seed=seed, sigma=sigma, box=box, lo=-box / 2, periodic=wrapped,
                                 device=dev.index if dev.index is not None else torch.cuda.current_device())


def make_velocities(atoms, steps, seed, device):
    """[steps, 3 * atoms] N(0, 1) velocities, independent per step (the device
    AR(1) generator with rho 0)."""
    from .._ext import cuda

    dev = torch.device(device)
    return cuda().synth_ar1(3 * atoms, steps, seed=seed + 1, rho=0.0, sigma=1.0, sigma0=1.0, sparse_frac=0.0,
                            sparse_scale=1.0, device=dev.index if dev.index is not None else torch.cuda.current_device())


def _median_ms(fn, warmup=2, iters=5):
    """Median CUDA-event time of fn() on the current stream (outputs dropped)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out = fn()
        e.record()
        e.synchronize()
        del out
        times.append(s.elapsed_time(e))
    return float(np.median(times))


def run_codec(x, codec, eps, verify_steps, cpu_steps):
    dev = x.device
    T, P = x.shape
    raw = T * P * 4
    # Each call's outputs are released before the next call, so the timed
    # calls reuse the allocator's cached blocks instead of new cudaMallocs.
    enc_ms = _median_ms(lambda: trajectory.encode_steps(x, codec, eps))
    payload, lens, maxerr, st = trajectory.encode_steps(x, codec, eps)
    lens_h = lens.cpu().numpy()
    assert int(st[0]) == 0, st.tolist()
    comp = int(lens_h.sum()) + 8 * T + 14
    # decode all steps on the device from the packed payloads
    offs = np.zeros(T + 1, np.int64)
    offs[1:] = np.cumsum(lens_h)
    host = payload.cpu().numpy()
    data = torch.from_numpy(np.concatenate([host[t, : lens_h[t]] for t in range(T)])).to(dev)
    offs_d = torch.from_numpy(offs).to(dev)
    scale = float(np.float32(2.0) * np.float32(eps))
    sc = torch.full((T,), scale, dtype=torch.float32, device=dev)
    from .._ext import cuda

    cid = nzcp.CODECS[codec]
    dec_ms = _median_ms(lambda: cuda().nz_decode_steps(data, offs_d, sc, cid, P))
    vals = cuda().nz_decode_steps(data, offs_d, sc, cid, P)
    # decoded values vs the original snapshots
    dec_err = float((vals.view(T, P) - x).abs().max())
    # byte identity and CPU baseline on a prefix of the steps
    xs = x[:verify_steps].contiguous().cpu().numpy()
    hb, hstats = nzcp.compress(xs.reshape(-1), P, verify_steps, codec, eps)
    db, _ = trajectory.compress(x[:verify_steps].contiguous(), codec, eps)
    xc = x[:cpu_steps].contiguous().cpu().numpy().reshape(-1)
    t0 = time.perf_counter()
    nzcp.compress(xc, P, cpu_steps, codec, eps)
    cpu_s = time.perf_counter() - t0
    return {
        "codec": codec, "encode_GBps": raw / (enc_ms * 1e6), "decode_GBps": raw / (dec_ms * 1e6),
        "encode_ms": enc_ms, "decode_ms": dec_ms, "ratio": raw / comp, "max_abs_err": float(maxerr.item()),
        "decode_max_abs_err": dec_err, "bytes_identical_to_host_on_first_steps": db == hb,
        "cpu_single_thread_MBps": cpu_steps * P * 4 / cpu_s / 1e6,
    }


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--atoms", type=int, default=1_000_000)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--epsilon", type=float, default=1e-3)
    ap.add_argument("--sigma", type=float, default=0.01)
    ap.add_argument("--box", type=float, default=100.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--wrapped", action="store_true")
    ap.add_argument("--codecs", default="eb,bs,bsrle")
    ap.add_argument("--verify-steps", type=int, default=3)
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--fields", default="pos,vel", help="pos (positions), vel (N(0,1) velocities)")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    rows = []
    for field in a.fields.split(","):
        if field == "pos":
            x = make_positions(a.atoms, a.steps, a.sigma, a.box, a.seed, a.wrapped, dev)
        elif field == "vel":
            x = make_velocities(a.atoms, a.steps, a.seed, dev)
        else:
            raise SystemExit(f"unknown field {field}")
        for codec in a.codecs.split(","):
            r = run_codec(x, codec, a.epsilon, a.verify_steps, a.cpu_steps)
            r.update(field=field, atoms=a.atoms, steps=a.steps, epsilon=a.epsilon, wrapped=a.wrapped,
                     raw_GB=a.steps * 3 * a.atoms * 4 / 1e9)
            rows.append(r)
            print(json.dumps(r), flush=True)
        del x
    # both fields together, as one 1M-atom x 100-step dump of positions + velocities
    for codec in a.codecs.split(","):
        rs = [r for r in rows if r["codec"] == codec]
        if len(rs) > 1:
            raw = sum(r["raw_GB"] for r in rs)
            enc = sum(r["encode_ms"] for r in rs)
            dec = sum(r["decode_ms"] for r in rs)
            comp = sum(r["raw_GB"] / r["ratio"] for r in rs)
            tot = {"codec": codec, "field": "+".join(r["field"] for r in rs), "raw_GB": raw,
                   "encode_GBps": raw / (enc * 1e-3), "decode_GBps": raw / (dec * 1e-3), "ratio": raw / comp,
                   "max_abs_err": max(r["max_abs_err"] for r in rs)}
            rows.append(tot)
            print(json.dumps(tot), flush=True)
    return rows


if __name__ == "__main__":
    main()
