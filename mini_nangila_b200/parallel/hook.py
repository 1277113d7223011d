"""PyTorch DDP communication hook with predictive-residual compression.

``register_nangila_hook`` accepts the keyword arguments of the reference's
hook (``python/nangila_ddp/comm_hook.py:47-60``) and adds:

* ``impl``: ``"fused"`` (default on CUDA) runs one sm_100a kernel per bucket
  that predicts, compresses, exchanges over NVLink, decodes, sums, adds the
  prediction back and updates the predictor and the error feedback; the
  returned future completes on the communication stream, so the exchange
  overlaps the rest of backward.  ``"host"`` runs the same product format
  through the C++ oracle and ``all_gather`` (CPU / gloo ranks).  ``"compat"``
  reproduces the reference's algorithm and payload (global absmax scale,
  ``floor(x + U - 0.5)`` rounding, hi/lo nibbles, LSB-first top-k mask,
  static randperm topology) with torch ops.
* ``error_feedback`` (fused/host; the reference has none), ``variant``
  (``auto|oneshot|twoshot``, or ``nccl`` for the uncompressed averaged
  all-reduce behind the same API), ``timeout_s``, ``verbose``, ``max_ctas``,
  ``autotune`` (fused, more than 2 ranks: the first bucket times one-shot
  against two-shot on this box and sets the size from which two-shot runs).

``topo_drop_percent`` (a fraction, as in the reference) selects passengers
per bucket.  fused/host drop whole 2048-element chunks by a keyed
permutation that every rank computes alike: passengers are neither encoded
nor sent, reconstruct to the prediction, and (with error feedback) carry
their residual to the next step.  The reference drops single elements with a
seeded ``randperm`` (``comm_hook.py:149-174``); ``impl="compat"`` does that.

The hook state object returned by ``register_nangila_hook`` exposes
``state_dict()/load_state_dict()``: the predictor and error-feedback
buffers, the call counters (the noise keys), and each bucket's parameter
layout. A resumed run continues bit-identically while the bucket layout
matches. Otherwise each parameter's state follows it into the new buckets;
this also happens in a live run when DDP rebuilds its buckets after the
first iteration.

With ``metrics_path`` set, rank 0 appends one line per bucket in the
reference's ``key,value`` layout. Its ``res_mean_abs`` (mean |g - pred|) is
computed on the device and written once it has landed, so logging adds no
host sync.
"""
from __future__ import annotations

import atexit
import os
import time
import zlib
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.distributed as dist

from ..utils.nvtx import nvtx_range
from .fused import CommError, FusedAllReduce, autotune_twoshot, topk_per_block, topology, wire_bytes


@dataclass
class _BucketState:
    numel: int
    sig: tuple
    pred: torch.Tensor | None
    ef: torch.Tensor | None
    calls: int = 0
    # ((parameter index, offset, numel), ...) of the bucket's gradients when
    # DDP names them; lets a state follow its parameters into another layout
    layout: tuple | None = None


@dataclass
class HookConfig:
    """Keyword arguments of ``register_nangila_hook`` (python/nangila_ddp/comm_hook.py:47-60, plus this framework's)."""
    beta: float = 0.9
    bits: int = 4
    stochastic: bool = True
    use_fp16_transport: bool = True  # accepted for API compatibility; unused (as in the reference)
    seed: int = 12345
    metrics_path: str | None = None
    use_momentum: bool = False
    topk_percent: float = 0.0
    topo_drop_percent: float = 0.0
    topo_seed: int = 424242
    impl: str = "fused"
    error_feedback: bool = True
    variant: str = "auto"
    timeout_s: float = 10.0
    verbose: bool = False
    max_ctas: int = 0
    # CTAs of the exchange kernels of buckets that are not the last one,
    # which run while backward still computes (0: the whole grid)
    inflight_ctas: int = 0

    @property
    def mode(self) -> str:
        if self.topk_percent > 0.0:
            return "topk"
        return "int8" if self.bits == 8 else "int4"

    @property
    def k(self) -> int:
        return topk_per_block(self.topk_percent) if self.topk_percent > 0.0 else 0


@dataclass
class NangilaHookState:
    """What ``register_nangila_hook`` returns: per-bucket predictor / EF state,
    byte counters, metrics and the communicator."""
    config: HookConfig
    group: object = None
    comm: FusedAllReduce | None = None
    buckets: dict = field(default_factory=dict)
    stream: torch.cuda.Stream | None = None
    raw_bytes: int = 0
    comp_bytes: int = 0
    calls: int = 0
    last_variant: str = ""
    # metrics lines whose res_mean_abs is still being computed on the
    # device: (ts, hook_idx, numel, comp_bytes, pinned scalar, event)
    pending_metrics: list = field(default_factory=list)
    # parameter data_ptr -> index in model.parameters()
    param_index: dict = field(default_factory=dict)
    # bucket states (a loaded state_dict, or the buckets DDP just replaced)
    # that new buckets take their predictor / EF state from, per parameter
    restore: dict | None = None
    # fused: called as after_reduce(bucket) on the hook stream right after
    # the bucket's exchange kernel, before its future completes (the
    # trainer's per-bucket optimizer update)
    after_reduce: object = None
    # fused: a utils.timeline.StepTimeline that receives each bucket's events
    timeline: object = None
    # fused: kernel_opt(bucket) -> parallel.fused.FusedOpt or None (AdamW in
    # the exchange kernel's decode phase), then kernel_opt_done(bucket)
    kernel_opt: object = None
    kernel_opt_done: object = None

    def compression_ratio(self) -> float:
        return self.raw_bytes / max(1, self.comp_bytes)

    def flush_metrics(self, wait: bool = True) -> int:
        """Write the metrics lines whose device statistic has landed (all of
        them with ``wait``, which waits for each one's event).  Returns the
        number of lines written."""
        lines = []
        while self.pending_metrics:
            ts, idx, numel, comp, val, ev = self.pending_metrics[0]
            if not wait and not ev.query():
                break
            ev.synchronize()
            self.pending_metrics.pop(0)
            lines.append(_metrics_line(ts, idx, numel, comp, float(val)))
        _append(self.config.metrics_path, lines)
        return len(lines)

    def state_dict(self) -> dict:
        """Predictor and error-feedback state of every bucket (CPU copies),
        call counters (the stochastic-rounding step keys) and the exchange
        epoch.  With the same bucket layout a resumed run is bit-identical
        to an uninterrupted one; with another layout (a new DDP instance
        whose buckets differ), each parameter's state is carried over
        through the saved layouts."""
        out = {"calls": self.calls, "buckets": {}}
        for b, st in self.buckets.items():
            out["buckets"][b] = {
                "numel": st.numel,
                "calls": st.calls,
                "pred": None if st.pred is None else st.pred.detach().cpu().clone(),
                "ef": None if st.ef is None else st.ef.detach().cpu().clone(),
                "layout": None if st.layout is None else [list(x) for x in st.layout],
            }
        if self.comm is not None:
            out["epoch"] = int(self.comm.comm.epoch)
        return out

    def load_state_dict(self, sd: dict) -> None:
        """Restore a ``state_dict``; each bucket takes its state when the hook
        next sees it (a bucket of the same index, size and layout whole, any
        other bucket parameter by parameter)."""
        self.calls = int(sd.get("calls", 0))
        self.buckets = {}
        self.restore = {"buckets": {int(b): d for b, d in sd["buckets"].items()}}
        if self.comm is not None and "epoch" in sd:
            self.comm.comm.epoch = int(sd["epoch"])

    def _snapshot(self) -> dict:
        """The current bucket states as a restore source (no copies)."""
        return {"buckets": {b: {"numel": st.numel, "calls": st.calls, "pred": st.pred, "ef": st.ef,
                                "layout": st.layout} for b, st in self.buckets.items()}}


def _bucket_sig(bucket) -> tuple:
    try:
        ps = bucket.parameters()
        return (bucket.buffer().numel(), tuple(p.data_ptr() for p in ps[:2]), len(ps))
    except Exception:
        return (bucket.buffer().numel(),)


def _layout(bucket, buf: torch.Tensor, param_index: dict) -> tuple | None:
    """((parameter index, offset, numel), ...) of a DDP bucket from its
    gradient views into the flat buffer; None when the bucket does not name
    its parameters or a view lies outside the buffer."""
    if not param_index:
        return None
    try:
        params, grads = bucket.parameters(), bucket.gradients()
    except Exception:
        return None
    if not params or len(params) != len(grads):
        return None
    base, es, n = buf.data_ptr(), buf.element_size(), buf.numel()
    out = []
    for p, g in zip(params, grads):
        pi = param_index.get(p.data_ptr())
        off, rem = divmod(g.data_ptr() - base, es)
        if pi is None or rem or off < 0 or off + g.numel() > n:
            return None
        out.append((pi, off, g.numel()))
    return tuple(out)


def _restored(hs: NangilaHookState, bidx: int, buf: torch.Tensor, layout, want_pred: bool,
              want_ef: bool) -> _BucketState | None:
    src = hs.restore
    if not src:
        return None
    saved = src["buckets"]
    n, dev = buf.numel(), buf.device

    def dev_copy(t, want):
        return t.to(dev, torch.float32).clone() if (want and t is not None) else (
            torch.zeros(n, dtype=torch.float32, device=dev) if want else None)

    d = saved.get(bidx)
    if d is not None and d["numel"] == n:
        sl = d.get("layout")
        if layout is None or sl is None or tuple(tuple(x) for x in sl) == layout:
            return _BucketState(n, (), dev_copy(d["pred"], want_pred), dev_copy(d["ef"], want_ef),
                                int(d["calls"]), layout)
    if layout is None:
        return None
    where = src.get("where")
    if where is None:
        where = {pi: (b, off, num) for b, dd in saved.items() for pi, off, num in (dd.get("layout") or ())}
        src["where"] = where
    if not all(pi in where and where[pi][2] == num for pi, _, num in layout):
        return None
    pred = torch.zeros(n, dtype=torch.float32, device=dev) if want_pred else None
    ef = torch.zeros(n, dtype=torch.float32, device=dev) if want_ef else None
    calls = 0
    for pi, off, num in layout:
        b, soff, _ = where[pi]
        dd = saved[b]
        for dst, key in ((pred, "pred"), (ef, "ef")):
            if dst is not None and dd[key] is not None:
                dst[off:off + num].copy_(dd[key][soff:soff + num])
        calls = max(calls, int(dd["calls"]))
    return _BucketState(n, (), pred, ef, calls, layout)


def _get_state(hs: NangilaHookState, bidx: int, buf: torch.Tensor, bucket, want_pred: bool,
               want_ef: bool) -> tuple[_BucketState, bool]:
    sig = _bucket_sig(bucket)
    st = hs.buckets.get(bidx)
    if hs.restore is not None:
        served = hs.restore.setdefault("served", set())
        if bidx in served:
            hs.restore = None  # a bucket index came round again: a new step, all states taken over
        else:
            served.add(bidx)
    if st is None or st.numel != buf.numel() or st.sig != sig:
        if st is not None and hs.restore is None:
            # DDP replaced its buckets (the rebuild after the first iteration):
            # the new ones take their parameters' state from the old ones
            hs.restore = hs._snapshot()
            hs.restore["served"] = {bidx}
        layout = _layout(bucket, buf, hs.param_index)
        st = _restored(hs, bidx, buf, layout, want_pred, want_ef)
        if st is None:
            pred = torch.zeros(buf.numel(), dtype=torch.float32, device=buf.device) if want_pred else None
            ef = torch.zeros(buf.numel(), dtype=torch.float32, device=buf.device) if want_ef else None
            st = _BucketState(buf.numel(), sig, pred, ef, 0, layout)
        st.sig = sig
        hs.buckets[bidx] = st
    first = st.calls == 0
    st.calls += 1
    return st, first


def _metrics_line(ts: float, idx: int, numel: int, comp: int, res_mean_abs: float) -> str:
    # Same key,value layout as the reference's metrics CSV (comm_hook.py:307-319)
    raw = numel * 4
    return (f"ts,{ts:.6f},hook_idx,{idx},bucket_elems,{numel},raw_bytes,{raw},"
            f"comp_bytes,{comp},ratio,{raw / max(comp, 1):.6f},res_mean_abs,{res_mean_abs:.6e}\n")


def _append(path: str | None, lines: list[str]) -> None:
    if not path or not lines:
        return
    try:
        with open(path, "a") as fh:
            fh.write("".join(lines))
    except OSError:
        pass


def _wants_metrics(hs: NangilaHookState) -> bool:
    cfg = hs.config
    return bool(cfg.metrics_path) and (dist.get_rank(hs.group) if dist.is_initialized() else 0) == 0


def _log(hs: NangilaHookState, bidx: int, numel: int, comp: int, res_mean_abs=float("nan")) -> None:
    """One metrics line for this hook call (rank 0).  ``res_mean_abs`` is a
    float, or a CUDA scalar still being computed: its line is queued with an
    event and written once the value has landed, so logging adds no host
    sync to the step."""
    cfg = hs.config
    rank = dist.get_rank(hs.group) if dist.is_initialized() else 0
    if rank != 0 or not (cfg.metrics_path or cfg.verbose):
        return
    raw = numel * 4
    if cfg.verbose:
        print(f"[nangila-b200-{cfg.mode}] bucket={numel} raw={raw/1e6:.3f}MB comp_local={comp/1e6:.3f}MB "
              f"ratio={raw / max(comp, 1):.2f}x pred_mode={'EMA' if cfg.use_momentum else 'none'} bits={cfg.bits}")
    if not cfg.metrics_path:
        return
    if isinstance(res_mean_abs, torch.Tensor) and res_mean_abs.is_cuda:
        val = torch.empty((), dtype=torch.float32, pin_memory=True)
        val.copy_(res_mean_abs, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        hs.pending_metrics.append((time.time(), hs.calls, numel, comp, val, ev))
        hs.flush_metrics(wait=False)
        return
    hs.flush_metrics(wait=True)  # keep the file in call order
    _append(cfg.metrics_path, [_metrics_line(time.time(), hs.calls, numel, comp, float(res_mean_abs))])


# --------------------------------------------------------------- fused (GPU)
def _fused_hook(hs: NangilaHookState, bucket):
    cfg = hs.config
    buf = bucket.buffer()
    bidx = bucket.index()
    # A launch that gave up (a peer's flag never came, a tag mismatch) left
    # its bucket unreduced; its status reaches the host asynchronously.
    st_code = hs.comm.poll_status()
    if st_code != 0:
        hs.comm.check()  # synchronizes and raises CommError with the details
    st, first = _get_state(hs, bidx, buf, bucket, cfg.use_momentum, cfg.error_feedback)
    hs.calls += 1
    if getattr(hs, "autotune_pending", False):
        # First bucket: time one-shot vs two-shot at bucket-like sizes on this
        # box (every rank runs the same sequence; max over ranks decides).
        hs.autotune_pending = False
        with nvtx_range("nangila/autotune"):
            autotune_twoshot(hs.comm, sizes_mb=(4, 16, 32, 64, 128, 256))
    cur = torch.cuda.current_stream(buf.device)
    # Buckets before the last one run while backward still computes: their
    # kernels get a capped grid so backward keeps most SMs.  The last bucket
    # (the first layers' gradients) runs when backward is over and gets the
    # whole grid.  is_last() is the same on every rank, so the grids (part
    # of the flag tags) agree.
    last = bool(bucket.is_last()) if hasattr(bucket, "is_last") else True
    ctas = cfg.max_ctas if (last or not cfg.inflight_ctas) else cfg.inflight_ctas
    # AdamW in the kernel's decode phase: dense (INT4/INT8) fp32 buckets only
    kopt = hs.kernel_opt(bucket) if (hs.kernel_opt is not None and cfg.mode != "topk") else None
    tl = hs.timeline
    trec = None
    if tl is not None:
        variant = hs.comm.choose_variant(buf.numel(), cfg.mode, cfg.variant)
        from .._ext import cuda as _cuda

        grid = _cuda().fused_grid(buf.numel(), {"int4": 0, "int8": 1, "topk": 2}[cfg.mode],
                                  buf.dtype == torch.bfloat16, {"single": 0, "oneshot": 1, "twoshot": 2}[variant],
                                  ctas, buf.device.index, kopt is not None)
        trec = tl.bucket(bucket=bidx, numel=buf.numel(), variant=variant, grid=grid, last=last,
                         optimizer_in_kernel=kopt is not None)
        tl.event(trec, "ready", cur)
    hs.stream.wait_stream(cur)
    with torch.cuda.stream(hs.stream), nvtx_range(f"nangila/bucket{bidx}/{buf.numel()}"):
        # mean |g - pred| of this rank's bucket, the reference's res_mean_abs
        # (comm_hook.py:146,178); computed only when it is logged
        res = None
        if _wants_metrics(hs):
            # out of place: buf.float() of an fp32 bucket is the bucket itself
            if st.pred is not None and not first:
                res = (buf.float() - st.pred).abs_().mean()
            else:
                res = buf.float().abs().mean()
        if trec is not None:
            tl.event(trec, "start", hs.stream)
        hs.last_variant = hs.comm.allreduce_(
            buf, st.pred, st.ef, mode=cfg.mode, k=cfg.k, variant=cfg.variant, stochastic=cfg.stochastic,
            seed=cfg.seed, bucket=bidx, step=st.calls, beta=cfg.beta, first=first,
            topo_drop=cfg.topo_drop_percent, topo_seed=cfg.topo_seed, max_ctas=ctas, opt=kopt,
        )
        if trec is not None:
            tl.event(trec, "end", hs.stream)
        if kopt is not None:
            hs.kernel_opt_done(bucket)
        elif hs.after_reduce is not None:
            hs.after_reduce(bucket)
            if trec is not None:
                tl.event(trec, "opt_end", hs.stream)
        fut = torch.futures.Future(devices=[buf.device])
        fut.set_result(buf)
        comp = wire_bytes(buf.numel(), cfg.mode, cfg.k, cfg.topo_drop_percent, cfg.topo_seed, bidx)
        hs.raw_bytes += buf.numel() * 4
        hs.comp_bytes += comp
        _log(hs, bidx, buf.numel(), comp, res if res is not None else float("nan"))
    return fut


# ------------------------------------------------------- host (CPU, gloo)
_MAGIC = 0x504C474E  # "NGLP"


def _fault(rank: int, call: int) -> str | None:
    """Host-side fault injection for tests: NGL_FAULT="<kind>:<rank>:<call>"
    with kind corrupt (flip a payload byte after its checksum) or mismatch
    (announce another bucket) applies to that rank's hook call."""
    spec = os.environ.get("NGL_FAULT", "")
    if not spec:
        return None
    kind, r, c = (spec.split(":") + ["", "", ""])[:3]
    return kind if (r == str(rank) and c == str(call)) else None


def _frame(wire: np.ndarray, n: int, step: int, bucket: int, fault: str | None) -> torch.Tensor:
    """Payload = [magic, n lo, n hi, step, bucket, crc32(wire)] (u32) + wire."""
    w = np.ascontiguousarray(wire, dtype=np.uint8)
    crc = zlib.crc32(w.tobytes()) & 0xFFFFFFFF
    hdr = np.array([_MAGIC, n & 0xFFFFFFFF, n >> 32, step & 0xFFFFFFFF, bucket & 0xFFFFFFFF, crc], dtype=np.uint32)
    if fault == "corrupt" and w.size:
        w = w.copy()
        w[w.size // 2] ^= 0xFF
    elif fault == "mismatch":
        hdr[4] ^= 1
    return torch.from_numpy(np.concatenate([hdr.view(np.uint8), w]))


def _unframe(x: torch.Tensor, src: int, n: int, step: int, bucket: int) -> np.ndarray:
    b = x.numpy()
    hdr = b[:24].view(np.uint32)
    w = b[24:]
    if hdr[0] != _MAGIC or (int(hdr[1]) | (int(hdr[2]) << 32)) != n:
        raise CommError(f"rank {src}: bad payload header (magic/length) for bucket {bucket}")
    if int(hdr[3]) != (step & 0xFFFFFFFF) or int(hdr[4]) != (bucket & 0xFFFFFFFF):
        raise CommError(f"rank {src}: payload of bucket {int(hdr[4])} step {int(hdr[3])}, expected bucket {bucket} "
                        f"step {step} (ranks disagree on bucket order)")
    if (zlib.crc32(w.tobytes()) & 0xFFFFFFFF) != int(hdr[5]):
        raise CommError(f"rank {src}: payload checksum mismatch in bucket {bucket} step {step}")
    return w


def _np_view(t: torch.Tensor | None) -> np.ndarray | None:
    """A writable numpy view of a CPU, contiguous fp32 tensor (None otherwise):
    the host calls then write their outputs straight into the tensor."""
    if t is None or t.device.type != "cpu" or t.dtype != torch.float32 or not t.is_contiguous():
        return None
    return t.detach().numpy()


def _host_hook(hs: NangilaHookState, bucket):
    from .._ext import host

    h = host()
    cfg = hs.config
    buf = bucket.buffer()
    bidx = bucket.index()
    world = dist.get_world_size(hs.group)
    rank = dist.get_rank(hs.group)
    st, first = _get_state(hs, bidx, buf, bucket, cfg.use_momentum, cfg.error_feedback)
    hs.calls += 1
    g = buf.detach().float().cpu().numpy()
    pred = st.pred.cpu().numpy() if st.pred is not None else None
    ef = st.ef.cpu().numpy() if st.ef is not None else None
    n = g.size
    # mean |g - pred| (comm_hook.py:146,178), before g (a view of the bucket
    # on CPU) is overwritten with the average
    res = float("nan")
    if _wants_metrics(hs):
        r = g - pred if (pred is not None and not first) else g
        res = float(np.abs(r, dtype=np.float64).mean()) if n else 0.0
    topo = topology(n, cfg.topo_drop_percent, cfg.topo_seed, bidx)
    ef_view = _np_view(st.ef) if cfg.error_feedback else None
    if cfg.mode == "topk":
        wire, e_out = h.product_topk_encode(g, pred, ef, cfg.k, cfg.error_feedback, topo)
    else:
        bits = 4 if cfg.mode == "int4" else 8
        # the new error feedback is written over the old one when it lives in
        # a CPU fp32 tensor (each block is read before it is written)
        wire, e_out = h.product_encode(g, pred, ef, bits, cfg.stochastic, cfg.error_feedback,
                                       cfg.seed & 0x7FFFFFFFFFFFFFFF, rank, bidx, st.calls, topo, e_out=ef_view)
    payload = _frame(wire, n, st.calls, bidx, _fault(rank, hs.calls))
    gathered = [torch.empty_like(payload) for _ in range(world)]
    dist.all_gather(gathered, payload, group=hs.group)
    inv_world = np.float32(1.0) / np.float32(world)
    # every rank checks every payload after the same collective, so all of
    # them raise together on a corrupt or mismatched one
    wires = [_unframe(x, r, n, st.calls, bidx) for r, x in enumerate(gathered)]
    # the average is written straight into a CPU fp32 bucket (g, its view,
    # is no longer needed)
    out_view = _np_view(buf)
    if cfg.mode == "topk":
        avg = h.product_topk_reduce(wires, n, cfg.k, pred, float(inv_world))
    else:
        avg = h.product_reduce(wires, n, bits, pred, float(inv_world), out=out_view)
    if st.pred is not None:
        pred_view = _np_view(st.pred)
        if pred_view is not None:
            h.product_ema_(pred_view, avg, cfg.beta, first)
        else:
            st.pred.copy_(torch.from_numpy(h.product_ema(st.pred.cpu().numpy(), avg, cfg.beta, first)))
    if st.ef is not None and e_out is not ef_view:
        st.ef.copy_(torch.from_numpy(e_out))
    if avg is not out_view:
        buf.copy_(torch.from_numpy(avg).to(buf.dtype))
    comp = wire_bytes(n, cfg.mode, cfg.k, cfg.topo_drop_percent, cfg.topo_seed, bidx)
    hs.raw_bytes += n * 4
    hs.comp_bytes += comp
    _log(hs, bidx, n, comp, res)
    if hs.after_reduce is not None:
        hs.after_reduce(bucket)
    fut = torch.futures.Future()
    fut.set_result(buf)
    return fut


# ------------------------------------------------ uncompressed (baseline)
def _nccl_hook(hs: NangilaHookState, bucket):
    """Plain averaged all-reduce of the bucket (the stock DDP path), behind
    the same API and metrics for A/B runs."""
    buf = bucket.buffer()
    world = dist.get_world_size(hs.group)
    hs.calls += 1
    hs.raw_bytes += buf.numel() * buf.element_size()
    hs.comp_bytes += buf.numel() * buf.element_size()
    with nvtx_range(f"nccl/bucket{bucket.index()}"):
        fut = dist.all_reduce(buf.div_(world), group=hs.group, async_op=True).get_future()
    return fut.then(lambda f: f.value()[0])


def register_nangila_hook(
    model: torch.nn.Module,
    *,
    beta: float = 0.9,
    bits: int = 4,
    stochastic: bool = True,
    use_fp16_transport: bool = True,
    seed: int = 12345,
    metrics_path: str | None = None,
    use_momentum: bool = False,
    topk_percent: float = 0.0,
    topo_drop_percent: float = 0.0,
    topo_seed: int = 424242,
    impl: str | None = None,
    error_feedback: bool | None = None,
    variant: str = "auto",
    timeout_s: float = 10.0,
    verbose: bool = False,
    max_ctas: int = 0,
    process_group=None,
    autotune: bool = True,
    inflight_ctas: int = 0,
    stream_priority: int = -1,
    l2_keep_mb: float = 0.0,
) -> NangilaHookState:
    """Register a predictive-residual compression comm hook on a DDP model.

    ``inflight_ctas`` caps the grid of the exchange kernels of every bucket
    but the last (they overlap backward); 0 (the default) leaves them the
    whole grid, which measured fastest on B200s: a capped exchange kernel
    lacks the memory parallelism to finish early and holds its SMs longer.
    ``stream_priority`` is the hook stream's CUDA priority (-1 high, 0
    normal).  ``l2_keep_mb`` bounds the predictor bytes an exchange kernel
    keeps in L2 between its two phases; 0, the default, turns the L2 policy
    off: it makes the kernel alone faster, but in GPT-2 training at 2 GPUs
    the kept lines cost the concurrent backward more (19.88 against 20.23
    ms per step with 48 MB kept).

    Returns the hook state (metrics, ``state_dict``/``load_state_dict``).
    """
    if not hasattr(model, "register_comm_hook"):
        raise RuntimeError("Model is not DDP-wrapped; call torch.nn.parallel.DistributedDataParallel first.")
    if bits not in (4, 8):
        raise ValueError("bits must be 4 or 8")
    dev = next(model.parameters()).device
    if impl is None:
        impl = "fused" if dev.type == "cuda" else "host"
    if variant == "nccl":  # uncompressed all-reduce through the same hook API
        impl = "nccl"
    if impl == "compat":
        from .compat_hook import make_compat_hook

        cfg = HookConfig(beta, bits, stochastic, use_fp16_transport, seed, metrics_path, use_momentum, topk_percent,
                         topo_drop_percent, topo_seed, impl, bool(error_feedback), variant, timeout_s, verbose)
        hs = NangilaHookState(cfg, process_group)
        model.register_comm_hook(state=None, hook=make_compat_hook(hs))
        return hs
    cfg = HookConfig(beta, bits, stochastic, use_fp16_transport, seed, metrics_path, use_momentum, topk_percent,
                     topo_drop_percent, topo_seed, impl, True if error_feedback is None else bool(error_feedback),
                     variant, timeout_s, verbose, max_ctas, int(inflight_ctas))
    hs = NangilaHookState(cfg, process_group)
    hs.param_index = {p.data_ptr(): i for i, p in enumerate(model.parameters())}
    if impl == "fused":
        if dev.type != "cuda":
            raise RuntimeError("impl='fused' needs a CUDA model; use impl='host' on CPU")
        bucket_cap = int(getattr(model, "bucket_bytes_cap", 25 * 1024 * 1024))
        # A bucket holds up to the cap plus one parameter; longer buckets (DDP's
        # first iteration reduces the whole model as one) run in segments.
        max_numel = bucket_cap // 4 + max(p.numel() for p in model.parameters()) + 8192
        hs.comm = FusedAllReduce(max_numel, group=process_group, device=dev, topk_k=max(cfg.k, 1),
                                 timeout_s=timeout_s, max_ctas=max_ctas, modes=(cfg.mode,))
        hs.comm.comm.l2_keep_bytes = int(max(0.0, l2_keep_mb) * (1 << 20))
        hs.stream = torch.cuda.Stream(device=dev, priority=int(stream_priority))
        hs.autotune_pending = bool(autotune) and hs.comm.world > 2 and variant == "auto" and cfg.mode != "topk"

        def hook(_state, bucket):
            return _fused_hook(hs, bucket)
    elif impl == "host":
        def hook(_state, bucket):
            return _host_hook(hs, bucket)
    elif impl == "nccl":
        def hook(_state, bucket):
            return _nccl_hook(hs, bucket)
    else:
        raise ValueError(f"unknown impl {impl!r}")
    model.register_comm_hook(state=None, hook=hook)
    if cfg.metrics_path and impl == "fused":
        atexit.register(_flush_at_exit, hs)
    return hs


def _flush_at_exit(hs: NangilaHookState) -> None:
    try:
        hs.flush_metrics(wait=True)
    except Exception:  # the CUDA context may already be unusable at exit
        pass
