"""Exchange kernels of several ranks, run on one GPU.

The one-shot and two-shot kernels wait for flags that other ranks' kernels
set over NVLink.  Two kernels that wait on each other must never share a
GPU (nothing guarantees they run at the same time), so these helpers never
launch one: every rank's region is a buffer on the local GPU, and what the
other ranks would have stored into it (payload records, two-shot INT8
results, flags) is written before the launch, so each launch finds
everything it waits for already delivered.

* ``oneshot(n, mode, k, drop)``: rank 0 of a 2-rank one-shot launch, the
  peer's payload and payload flags pre-delivered.
* ``twoshot(n, mode, world, drop, grid_cap)``: ranks world-1 .. 1 run first,
  each with every other rank's payload and every flag pre-delivered into its
  own region; their phase-A records, phase-B results and flags land in rank
  0's region through the kernel's own stores; rank 0 runs last.

Both return the launch's status word and outputs with the host library's
results for the same inputs (``csrc/host/product.cpp``), which must agree
bit for bit.
"""
from __future__ import annotations

import numpy as np
import torch

from .._ext import cuda as _cuda
from .._ext import host as _host
from .fused import MAX_COLS, MODES, VARIANTS, FusedAllReduce, make_layout, topology


def _data(n: int, seed: int, scale: float = 1e-3) -> np.ndarray:
    g = np.random.default_rng(seed)
    x = (g.standard_normal(n) * scale).astype(np.float32)
    x[g.random(n) < 0.3] *= 0.01
    return x


def _flag_value(tag: int, grid: int, epoch: int) -> int:
    v = (((tag ^ ((grid * 0x9E3779B1) & 0xFFFFFFFF)) & 0xFFFFFFFF) << 32) | epoch
    return v - (1 << 64) if v >= 1 << 63 else v


def oneshot(n: int, mode: str = "int4", k: int = 13, drop: float = 0.0, bad_tag: bool = False,
            deliver: bool = True, timeout_s: float = 0.2) -> dict:
    """Rank 0 of a 2-rank one-shot all-reduce.  ``deliver=False`` leaves the
    peer's flags unset (the bounded wait then gives up: status 1);
    ``bad_tag`` delivers them with a wrong tag (status 3)."""
    h, c = _host(), _cuda()
    dev = torch.device("cuda")
    topo = topology(n, drop, 3, 4)
    tl = list(topo) if drop else []
    L = make_layout(2, n, k)
    regs = [torch.zeros(L.total, dtype=torch.uint8, device=dev) for _ in range(2)]
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    comm = c.FusedComm(2, 0, [r.data_ptr() for r in regs], L.flags_off, L.inbox_off, L.slot_bytes, L.result_off,
                       L.result_bytes, status)
    epoch, parity = comm.epoch + 1, (comm.epoch + 1) & 1
    tag = FusedAllReduce.tag_for(n, 4)
    g0, g1 = _data(n, 1), _data(n, 2)
    mcode = MODES[mode]
    grid = c.fused_grid(n, mcode, False, VARIANTS["oneshot"], 0, 0)
    if deliver:
        p1, _ = c.product_encode(torch.from_numpy(g1).to(dev), None, None, mcode, k, True, 99, 1, 4, 7, tl)
        slot = L.inbox_off + (parity * 2 + 1) * L.slot_bytes
        regs[0][slot: slot + p1.numel()] = p1
        flags = regs[0][L.flags_off:].view(torch.int64)
        base = ((parity * 2 + 0) * 2 + 1) * MAX_COLS  # payload flags from rank 1
        flags[base: base + grid] = _flag_value(tag ^ (1 if bad_tag else 0), grid, epoch)
    torch.cuda.synchronize()
    gd = torch.from_numpy(g0).to(dev)
    comm.run(gd, None, None, mcode, k, VARIANTS["oneshot"], True, 99, 4, 7, 0.9, True, 0, int(timeout_s * 1e9), tag,
             tl)
    torch.cuda.synchronize()
    inv = float(np.float32(0.5))
    if mode == "topk":
        recs = [h.product_topk_encode(g, None, None, k, False, topo)[0] for g in (g0, g1)]
        ref = h.product_topk_reduce(recs, n, k, None, inv)
    else:
        bits = 8 if mode == "int8" else 4
        wires = [h.product_encode(g, None, None, bits, True, False, 99, r, 4, 7, topo)[0]
                 for r, g in enumerate((g0, g1))]
        ref = h.product_reduce(wires, n, bits, None, inv)
    return {"status": status.cpu().tolist(), "avg": gd.cpu().numpy(), "ref_avg": np.asarray(ref, np.float32)}


def adamw_reference(p, m, v, g, hyper):
    """AdamW with decoupled weight decay in float64, with the scalars of
    ``parallel.fused.FusedOpt.hyper`` as the kernel receives them: rounded to
    float32, and 1 - beta formed in float32."""
    b1, b2, eps, decay, step_size, inv_bc2 = (float(np.float32(x)) for x in hyper)
    omb1 = float(np.float32(1) - np.float32(b1))
    omb2 = float(np.float32(1) - np.float32(b2))
    p, m, v, g = (np.asarray(a, np.float64) for a in (p, m, v, g))
    p = p * decay
    m = b1 * m + omb1 * g
    v = b2 * v + omb2 * g * g
    p = p - step_size * m / (np.sqrt(v) * inv_bc2 + eps)
    return p, m, v


def _opt_segments(n: int, dev, seed: int = 9):
    """Parameters covering the bucket in four segments, one boundary not
    on a multiple of 8 elements (the element-by-element path), with random
    weights and moments; returns (FusedOpt without scalars, tensors)."""
    from .fused import FusedOpt

    cuts = sorted({0, n // 3, n // 3 + 13, (2 * n) // 3, n})
    rng = np.random.default_rng(seed)
    rows, tensors = [], []
    for a, b in zip(cuts[:-1], cuts[1:]):
        if b <= a:
            continue
        p = torch.from_numpy((rng.standard_normal(b - a) * 0.02).astype(np.float32)).to(dev)
        m = torch.from_numpy((rng.standard_normal(b - a) * 1e-4).astype(np.float32)).to(dev)
        v = torch.from_numpy((rng.random(b - a) * 1e-7).astype(np.float32)).to(dev)
        rows.append((a, b - a, p.data_ptr(), m.data_ptr(), v.data_ptr()))
        tensors.append((a, b, p, m, v))
    table = np.array(rows, dtype=[("off", "<i8"), ("numel", "<i8"), ("p", "<u8"), ("m", "<u8"), ("v", "<u8")])
    segs = torch.from_numpy(np.frombuffer(table.tobytes(), np.uint8).copy()).to(dev)
    t = 3
    hyper = [0.9, 0.999, 1e-8, 1.0 - 6e-4 * 0.01, 6e-4 / (1 - 0.9 ** t), 1.0 / np.sqrt(1 - 0.999 ** t)]
    return FusedOpt(segs, len(rows), hyper), tensors


def twoshot(n: int, mode: str = "int4", world: int = 4, drop: float = 0.0, grid_cap: int = 0,
            optimizer: bool = False) -> dict:
    """Rank 0 of a ``world``-rank two-shot all-reduce with a predictor and
    error feedback (see the module docstring).  ``optimizer`` also applies
    AdamW in rank 0's decode phase; the result then carries the updated and
    the float64 reference parameters and moments."""
    h, c = _host(), _cuda()
    dev = torch.device("cuda")
    k = 13
    topo = topology(n, drop, 5, 6)
    tl = list(topo) if drop else []
    L = make_layout(world, n, k, modes=(mode,))
    regs = [torch.zeros(L.total, dtype=torch.uint8, device=dev) for _ in range(world)]
    ptrs = [r.data_ptr() for r in regs]
    mcode = MODES[mode]
    tag = FusedAllReduce.tag_for(n, 6)
    # the optimizer instance has its own occupancy, hence grid; every rank
    # runs the same instance, as in a real run
    grid = c.fused_grid(n, mcode, False, VARIANTS["twoshot"], grid_cap, 0, optimizer)
    epoch, parity = 1, 1  # every communicator below is new: its first launch
    val = _flag_value(tag, grid, epoch)
    pred = _data(n, 40)
    efs = [_data(n, 50 + r, 1e-4) for r in range(world)]
    gs = [_data(n, 60 + r) for r in range(world)]
    seed, bucket, step = 21, 6, 3
    payloads = [c.product_encode(torch.from_numpy(gs[r]).to(dev), torch.from_numpy(pred).to(dev),
                                 torch.from_numpy(efs[r]).to(dev), mcode, k, True, seed, r, bucket, step, tl)[0]
                for r in range(world)]
    out = None
    for r in list(range(world - 1, 0, -1)) + [0]:
        if r != 0:
            reg = regs[r]
            flags = reg[L.flags_off:].view(torch.int64)
            for src in range(world):
                if src == r:
                    continue
                slot = L.inbox_off + (parity * world + src) * L.slot_bytes
                reg[slot: slot + payloads[src].numel()] = payloads[src]
                for kind in (0, 1):
                    base = ((parity * 2 + kind) * world + src) * MAX_COLS
                    flags[base: base + grid] = val
        status = torch.zeros(4, dtype=torch.int32, device=dev)
        comm = c.FusedComm(world, r, ptrs, L.flags_off, L.inbox_off, L.slot_bytes, L.result_off, L.result_bytes,
                           status)
        gd = torch.from_numpy(gs[r].copy()).to(dev)
        pd = torch.from_numpy(pred.copy()).to(dev)
        ed = torch.from_numpy(efs[r].copy()).to(dev)
        opt, tensors = _opt_segments(n, dev, seed=9 + r) if optimizer else (None, [])
        before = [(a, b, p.cpu().numpy(), m.cpu().numpy(), v.cpu().numpy()) for a, b, p, m, v in tensors]
        torch.cuda.synchronize()
        comm.run(gd, pd, ed, mcode, k, VARIANTS["twoshot"], True, seed, bucket, step, 0.9, False, grid_cap,
                 int(2e9), tag, tl, None if opt is None else opt.segs, 0 if opt is None else opt.nsegs, 0,
                 [] if opt is None else opt.hyper)
        torch.cuda.synchronize()
        if r == 0:
            out = {"status": status.cpu().tolist(), "avg": gd.cpu().numpy(), "pred": pd.cpu().numpy(),
                   "ef": ed.cpu().numpy()}
            if opt is not None:
                out["opt"] = [(a, b, p.cpu().numpy(), m.cpu().numpy(), v.cpu().numpy(), before[i][2:])
                              for i, (a, b, p, m, v) in enumerate(tensors)]
                out["opt_hyper"] = opt.hyper
    bits = 8 if mode == "int8" else 4
    inv = float(np.float32(1.0) / np.float32(world))
    encs = [h.product_encode(gs[r], pred, efs[r], bits, True, True, seed, r, bucket, step, topo) for r in range(world)]
    avg = h.product_reduce_twoshot([e[0] for e in encs], n, bits, pred, inv)
    out.update(ref_avg=np.asarray(avg, np.float32), ref_pred=np.asarray(h.product_ema(pred, avg, 0.9, False)),
               ref_ef=np.asarray(encs[0][1], np.float32))
    return out


def bit_equal(a, b) -> bool:
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))
