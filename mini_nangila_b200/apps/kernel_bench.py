"""Time one sm_100a kernel on a synthetic input (single GPU).

    python -m mini_nangila_b200.apps.kernel_bench --op fused_oneshot --n 67108864

Ops: fused_single (INT4, world 1), fused_oneshot (rank 0 of a --world-rank
one-shot all-reduce, 2 by default, with the peers' payloads and flags
pre-delivered into local memory, so the exchange kernel runs in full on one
GPU; --dtype bf16 and --no-pred give the top-k configuration of a bf16
model), fused_twoshot (rank 0 of a
--world-rank two-shot all-reduce: every peer's phase-A records, its INT8
result records and both kinds of flags pre-delivered), fused_topk_single,
fused_topk_oneshot, hpc_step, bs_encode, bsrle_encode, rle_encode,
bs_decode, bsrle_decode, stochastic_encode, topk_encode, nz_encode_eb / nz_encode_bs /
nz_encode_bsrle (whole-trajectory device .nz encode, --steps snapshots of
n / steps values), synth_brownian (device trajectory generator).

Inputs are larger than the 126 MB L2 for the default n.  Each timed launch is
bracketed by CUDA events on the launching stream after warm-up; the figure
reported is the median.  Algorithmic bytes / time is compared with the
measured HBM copy bandwidth of MEASURED_PEAKS.json.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def hbm_peak() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def _time(fn, iters, warmup, setup=None):
    for _ in range(warmup):
        if setup:
            setup()
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        if setup:
            setup()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        out.append(s.elapsed_time(e))
    return statistics.median(out)


def _emulated_oneshot(n, mode, k, world=2, dtype=torch.float32, use_pred=True):
    """Rank 0 of a ``world``-rank one-shot launch; every peer's record and
    column flag are written into rank 0's region before every call, so the
    kernel runs in full (encode, pushes, waits, rank-ordered decode of all
    ``world`` records) on one GPU.  ``dtype`` is the bucket's; without
    ``use_pred`` there is no predictor state (the top-k configuration)."""
    from mini_nangila_b200 import _ext
    from mini_nangila_b200.parallel.fused import MAX_COLS, MODES, VARIANTS, FusedAllReduce, make_layout

    c = _ext.cuda()
    dev = torch.device("cuda")
    L = make_layout(world, n, k, (mode,))
    regs = [torch.zeros(L.total, dtype=torch.uint8, device=dev) for _ in range(world)]
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    comm = c.FusedComm(world, 0, [r.data_ptr() for r in regs], L.flags_off, L.inbox_off, L.slot_bytes,
                       L.result_off, L.result_bytes, status)
    mcode = MODES[mode]
    grid = c.fused_grid(n, mcode, dtype == torch.bfloat16, VARIANTS["oneshot"], 0, 0)
    tag = FusedAllReduce.tag_for(n, 0)
    reg0 = regs[0]
    g1 = torch.randn(n, device=dev) * 1e-3
    p1, _ = c.product_encode(g1, None, None, mcode, k, True, 3, 1, 0, 0)
    g = (torch.randn(n, device=dev) * 1e-3).to(dtype)
    pred = torch.zeros(n, device=dev) if use_pred else None
    ef = torch.zeros(n, device=dev)
    flags = reg0[L.flags_off:].view(torch.int64)
    ftag = tag ^ ((grid * 0x9E3779B1) & 0xFFFFFFFF)
    for par in (0, 1):
        for src in range(1, world):
            slot = L.inbox_off + (par * world + src) * L.slot_bytes
            reg0[slot: slot + p1.numel()] = p1

    def setup():
        epoch = comm.epoch + 1
        par = epoch & 1
        val = (ftag << 32) | epoch
        if val >= 1 << 63:
            val -= 1 << 64
        for src in range(1, world):
            base = ((par * 2 + 0) * world + src) * MAX_COLS
            flags[base: base + grid] = val

    def run():
        comm.run(g, pred, ef, mcode, k, VARIANTS["oneshot"], True, 3, 0, 1, 0.9, False, 0, int(5e9), tag)

    wire = p1.numel()
    es = g.element_size()
    # g read and written back (the average), ef read and written, pred read
    # and written; own record written to every slot (world copies, the
    # peers' over NVLink in a real run), world records read.
    algo = 2 * es * n + 8 * n + (8 * n if use_pred else 0) + 2 * world * wire
    return setup, run, algo, status


def _emulated_twoshot(n, world, l2_keep_mb):
    """Rank 0 of a ``world``-rank two-shot launch.  Rank 0's region holds
    every peer's payload (phase A reads the chunks rank 0 owns) and INT8
    result records (phase C reads the chunks the peers own); the payload
    and result flags of every peer are written before every call."""
    from mini_nangila_b200 import _ext
    from mini_nangila_b200.parallel.fused import MAX_COLS, MODES, VARIANTS, FusedAllReduce, make_layout

    c = _ext.cuda()
    dev = torch.device("cuda")
    L = make_layout(world, n, 1, ("int4",))
    regs = [torch.zeros(L.total, dtype=torch.uint8, device=dev) for _ in range(world)]
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    comm = c.FusedComm(world, 0, [r.data_ptr() for r in regs], L.flags_off, L.inbox_off, L.slot_bytes,
                       L.result_off, L.result_bytes, status)
    comm.l2_keep_bytes = int(l2_keep_mb * (1 << 20))
    mcode = MODES["int4"]
    grid = c.fused_grid(n, mcode, False, VARIANTS["twoshot"], 0, 0)
    tag = FusedAllReduce.tag_for(n, 0)
    reg0 = regs[0]
    peer = torch.randn(n, device=dev) * 1e-3
    p1, _ = c.product_encode(peer, None, None, mcode, 1, True, 3, 1, 0, 0)
    res, _ = c.product_encode(peer * 0.5, None, None, MODES["int8"], 1, False, 3, 1, 0, 0)
    for par in (0, 1):
        for src in range(1, world):
            slot = L.inbox_off + (par * world + src) * L.slot_bytes
            reg0[slot: slot + p1.numel()] = p1
        r0 = L.result_off + par * L.result_bytes
        reg0[r0: r0 + res.numel()] = res
    g = torch.randn(n, device=dev) * 1e-3
    pred = torch.randn(n, device=dev) * 1e-3
    ef = torch.zeros(n, device=dev)
    flags = reg0[L.flags_off:].view(torch.int64)
    ftag = tag ^ ((grid * 0x9E3779B1) & 0xFFFFFFFF)

    def setup():
        epoch = comm.epoch + 1
        par = epoch & 1
        val = (ftag << 32) | epoch
        if val >= 1 << 63:
            val -= 1 << 64
        for kind in (0, 1):
            for src in range(1, world):
                base = ((par * 2 + kind) * world + src) * MAX_COLS
                flags[base: base + grid] = val

    def run():
        comm.run(g, pred, ef, mcode, 1, VARIANTS["twoshot"], True, 3, 0, 1, 0.9, False, 0, int(5e9), tag)

    P, R = p1.numel(), res.numel()
    # g, pred, ef read, ef written (16n); own records (P) written; the owned
    # chunks' W records read (P); INT8 results written to every rank (R) and
    # read back (R); pred read again and grad, pred written (12n)
    algo = 28 * n + 2 * P + 2 * R
    return setup, run, algo, status


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", required=True)
    ap.add_argument("--n", type=int, default=64 << 20)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--k", type=int, default=13, help="top-k kept per 256-block")
    ap.add_argument("--steps", type=int, default=100, help="snapshots for the trajectory ops")
    ap.add_argument("--world", type=int, default=None,
                    help="emulated ranks of fused_twoshot (default 8) / fused_oneshot (default 2)")
    ap.add_argument("--dtype", choices=["fp32", "bf16"], default="fp32", help="bucket dtype of fused_oneshot")
    ap.add_argument("--no-pred", action="store_true", help="fused_oneshot without predictor state")
    ap.add_argument("--l2-keep-mb", type=float, default=48.0,
                    help="fused_twoshot: predictor MB kept in L2 between phases (0: no L2 policy)")
    args = ap.parse_args()
    torch.cuda.set_device(0)
    from mini_nangila_b200 import _ext
    from mini_nangila_b200.parallel.fused import FusedAllReduce

    c = _ext.cuda()
    n, dev = args.n, torch.device("cuda")
    setup, status = None, None
    if args.op in ("fused_single", "fused_topk_single"):
        mode = "topk" if "topk" in args.op else "int4"
        comm = FusedAllReduce(n, device=dev)
        g = torch.randn(n, device=dev) * 1e-3
        pred = torch.zeros(n, device=dev)
        ef = torch.zeros(n, device=dev)
        run = lambda: comm.allreduce_(g, pred, ef, mode=mode, k=args.k, step=1)  # noqa: E731
        algo = 24 * n
        status = comm.status
    elif args.op in ("fused_oneshot", "fused_topk_oneshot"):
        mode = "topk" if "topk" in args.op else "int4"
        setup, run, algo, status = _emulated_oneshot(
            n, mode, args.k, args.world or 2, torch.bfloat16 if args.dtype == "bf16" else torch.float32,
            not args.no_pred)
    elif args.op == "fused_twoshot":
        setup, run, algo, status = _emulated_twoshot(n, args.world or 8, args.l2_keep_mb)
    elif args.op == "hpc_step":
        x = torch.rand(n, device=dev) * 100
        st = c.q823_from_f32(x)
        stm1 = c.q823_from_f32(x * 0.999)
        codes = torch.empty(n, dtype=torch.int16, device=dev)
        recon = torch.empty(n, dtype=torch.int32, device=dev)
        mx = torch.zeros(1, dtype=torch.int32, device=dev)
        run = lambda: c.hpc_step(x, st, stm1, 2, 2e-3, codes, recon, mx)  # noqa: E731
        algo = 4 * n * 3 + 2 * n + 4 * n
    elif args.op in ("bs_encode", "bsrle_encode", "rle_encode"):
        kind = {"bs_encode": 0, "bsrle_encode": 2, "rle_encode": 3}[args.op]
        g = np.random.default_rng(0)
        q = torch.from_numpy((g.standard_normal(n) * 50).astype(np.int16)).to(dev)
        q[torch.rand(n, device=dev) < 0.7] = 0
        out_len = c.pack_codes(q, kind).numel()
        run = lambda: c.pack_codes(q, kind)  # noqa: E731
        algo = 2 * n + out_len
    elif args.op == "bsrle_decode":
        q = (torch.randn(n, device=dev) * 50).to(torch.int16)
        q[torch.rand(n, device=dev) < 0.3] = 0
        b = c.pack_codes(q, 2)
        off = torch.tensor([0, b.numel()], dtype=torch.int64, device=dev)
        sc = torch.tensor([2e-3], device=dev)
        run = lambda: c.decode_streams(b, off, sc, 2, n, (n + 31) // 32)  # noqa: E731
        algo = b.numel() + 4 * n
    elif args.op == "bs_decode":
        q = (torch.randn(n, device=dev) * 50).to(torch.int16)
        q[torch.rand(n, device=dev) < 0.7] = 0
        b = c.pack_codes(q, 0)
        off = torch.tensor([0, b.numel()], dtype=torch.int64, device=dev)
        sc = torch.tensor([2e-3], device=dev)
        run = lambda: c.decode_streams(b, off, sc, 0, n, (n + 31) // 32)  # noqa: E731
        algo = b.numel() + 4 * n
    elif args.op in ("nz_encode_eb", "nz_encode_bs", "nz_encode_bsrle"):
        # Whole-trajectory device .nz encode: T steps of P values (Brownian
        # positions from the device generator), closed loop + packer.
        from ..ops import trajectory

        codec = args.op.split("_")[-1]
        T = args.steps
        P = max(1, n // T)
        x = c.synth_brownian(P, T, seed=1, sigma=0.01, box=100.0, lo=-50.0, periodic=False)
        run = lambda: trajectory.encode_steps(x, codec, 1e-3)  # noqa: E731
        algo = 4 * T * P + 2 * T * P
    elif args.op == "synth_brownian":
        T = args.steps
        run = lambda: c.synth_brownian(max(1, n // T), T, seed=1)  # noqa: E731
        algo = 4 * (n // T) * T
    elif args.op == "stochastic_encode":
        r = c.q823_from_f32(torch.randn(n, device=dev))
        run = lambda: c.stochastic_quantize(r, 4, 42, 0)  # noqa: E731
        algo = 2 * 4 * n + n // 2
    elif args.op == "topk_encode":
        r = c.q823_from_f32(torch.randn(n, device=dev))
        run = lambda: c.topk_quantize(r, 0.05)  # noqa: E731
        algo = 6 * 4 * n + n // 10
    else:
        raise SystemExit(f"unknown op {args.op}")
    ms = _time(run, args.iters, args.warmup, setup)
    torch.cuda.synchronize()
    if status is not None and int(status[0]) != 0:
        raise SystemExit(f"kernel reported status {status.tolist()}")
    peak, src = hbm_peak()
    gbs = algo / (ms * 1e6)
    print(json.dumps({"op": args.op, "n": n, "ms": ms, "algo_bytes": algo, "GBps": gbs,
                      f"frac_of_{src}_hbm": gbs / peak, "hbm_peak_gbs": peak}), flush=True)


if __name__ == "__main__":
    main()
