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


def twoshot(n: int, mode: str = "int4", world: int = 4, drop: float = 0.0, grid_cap: int = 0) -> dict:
    """Rank 0 of a ``world``-rank two-shot all-reduce with a predictor and
    error feedback (see the module docstring)."""
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
    grid = c.fused_grid(n, mcode, False, VARIANTS["twoshot"], grid_cap, 0)
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
        torch.cuda.synchronize()
        comm.run(gd, pd, ed, mcode, k, VARIANTS["twoshot"], True, seed, bucket, step, 0.9, False, grid_cap,
                 int(2e9), tag, tl)
        torch.cuda.synchronize()
        if r == 0:
            out = {"status": status.cpu().tolist(), "avg": gd.cpu().numpy(), "pred": pd.cpu().numpy(),
                   "ef": ed.cpu().numpy()}
    bits = 8 if mode == "int8" else 4
    inv = float(np.float32(1.0) / np.float32(world))
    encs = [h.product_encode(gs[r], pred, efs[r], bits, True, True, seed, r, bucket, step, topo) for r in range(world)]
    avg = h.product_reduce_twoshot([e[0] for e in encs], n, bits, pred, inv)
    out.update(ref_avg=np.asarray(avg, np.float32), ref_pred=np.asarray(h.product_ema(pred, avg, 0.9, False)),
               ref_ef=np.asarray(encs[0][1], np.float32))
    return out


def bit_equal(a, b) -> bool:
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))
