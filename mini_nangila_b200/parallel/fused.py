"""Fused compressed all-reduce communicator (one sm_100a kernel per bucket).

``FusedAllReduce`` owns, per process:

* one symmetric region (CUDA IPC, mapped by every rank) holding the u64
  arrival flags, two inbox generations of ``world`` payload slots and two
  two-shot result regions;
* the device status word the kernel writes instead of trapping;
* the epoch counter (one per call; every rank calls in the same order).

``allreduce_`` averages a bucket in place: predictor add-back, error
feedback and predictor update happen inside the same kernel.  Wire formats:

* INT4 / INT8: per 256-element block one fp32 scale (absmax/7 or /127) and
  two's-complement codes, element 2i in the high nibble;
* top-k: per 256-element block a fixed record ``[f32 scale][k u8 idx][k i8]``
  padded to 4 bytes, indices ascending.

Reference: ``python/nangila_ddp/comm_hook.py:125-324`` performs the same
reduction with eager ops and five ``all_gather`` calls.
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .._ext import cuda as _cuda
from .symm import SymmetricRegion

MODES = {"int4": 0, "int8": 1, "topk": 2}
VARIANTS = {"single": 0, "oneshot": 1, "twoshot": 2}
BLOCK = 256
CHUNK_BLOCKS = 8
STATUS_NAMES = {
    0: "ok",
    1: "timeout waiting for a peer's payload",
    2: "timeout waiting for a two-shot result",
    5: "timeout of a bulk copy into shared memory",
    3: "payload tag mismatch (ranks disagree on bucket size or order)",
    4: "bounds check",
    6: "timeout of a scan's look-back wait",
}


@dataclass
class FusedOpt:
    """AdamW fused into the decode phase of one launch: ``segs`` is a uint8
    CUDA tensor of ``nsegs`` packed segment records (bucket offset, numel,
    parameter / first-moment / second-moment pointers), ``hyper`` the step's
    (beta1, beta2, eps, 1 - lr*wd, lr / (1 - beta1^t), 1 / sqrt(1 - beta2^t)),
    ``base`` the bucket element of the launch's first element."""
    segs: torch.Tensor
    nsegs: int
    hyper: list
    base: int = 0


class CommError(RuntimeError):
    """A fused exchange gave up (a bounded wait expired, a tag or bounds check failed)."""
    pass


def topk_per_block(frac: float) -> int:
    """Kept elements per 256-block for a keep fraction (at least 1)."""
    return max(1, min(BLOCK, int(frac * BLOCK + 0.5)))


def topk_record_bytes(k: int) -> int:
    return (4 + 2 * k + 3) & ~3


def chunk_record_bytes(mode: str, k: int = 0) -> int:
    """Wire bytes of one chunk record (8 blocks of 256 elements)."""
    if mode == "int4":
        return 4 * CHUNK_BLOCKS + CHUNK_BLOCKS * 128
    if mode == "int8":
        return 4 * CHUNK_BLOCKS + CHUNK_BLOCKS * 256
    return CHUNK_BLOCKS * topk_record_bytes(k)


def nchunks_of(n: int) -> int:
    return ((n + BLOCK - 1) // BLOCK + CHUNK_BLOCKS - 1) // CHUNK_BLOCKS


def payload_bytes(n: int, mode: str, k: int = 0) -> int:
    """Wire bytes one rank sends per bucket of n elements."""
    return nchunks_of(n) * chunk_record_bytes(mode, k)


_TOPO_CACHE: dict = {}


def topology(n: int, drop: float, seed: int, stream: int) -> tuple[int, int, int]:
    """Chunk-granular static topology drop of a bucket of n elements:
    (a, b, ndrop) such that chunk c is a passenger iff
    (c * a + b) mod nchunks < ndrop.  Identical on every rank."""
    if drop <= 0.0:
        return (1, 0, 0)
    key = (nchunks_of(n), float(drop), int(seed), int(stream))
    t = _TOPO_CACHE.get(key)
    if t is None:
        from .._ext import host

        t = tuple(int(x) for x in host().product_topology(key[0], key[1], key[2] & 0xFFFFFFFFFFFFFFFF,
                                                          key[3] & 0xFFFFFFFFFFFFFFFF))
        if len(_TOPO_CACHE) > 4096:
            _TOPO_CACHE.clear()
        _TOPO_CACHE[key] = t
    return t


def wire_bytes(n: int, mode: str, k: int = 0, drop: float = 0.0, seed: int = 0, stream: int = 0) -> int:
    """Bytes one rank actually sends for a bucket (passenger chunks are not sent)."""
    ndrop = topology(n, drop, seed, stream)[2]
    return (nchunks_of(n) - ndrop) * chunk_record_bytes(mode, k)


def dense_payload_bytes(n: int, bits: int) -> int:
    return payload_bytes(n, "int4" if bits == 4 else "int8")


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


MAX_COLS = 2048  # flag columns (max CTAs of one launch)


@dataclass
class Layout:
    """Offsets of the flags, inboxes and result slots inside each rank's symmetric region."""
    max_numel: int
    flags_off: int
    inbox_off: int
    slot_bytes: int
    result_off: int
    result_bytes: int
    total: int


def make_layout(world: int, max_numel: int, topk_k: int, modes=("int4", "int8", "topk")) -> Layout:
    slot = _align(max(payload_bytes(max_numel, m, max(1, topk_k)) for m in modes))
    result = _align(payload_bytes(max_numel, "int8"))
    flags_off = 0
    inbox_off = _align(flags_off + 2 * 2 * world * MAX_COLS * 8)
    result_off = _align(inbox_off + 2 * world * slot)
    total = _align(result_off + 2 * result)
    return Layout(max_numel, flags_off, inbox_off, slot, result_off, result, total)


class FusedAllReduce:
    """Process-level communicator for the fused compressed all-reduce."""

    def __init__(
        self,
        max_numel: int,
        group=None,
        device: torch.device | None = None,
        topk_k: int = 26,
        timeout_s: float = 10.0,
        max_ctas: int = 0,
        twoshot_min_bytes: int | None = None,
        modes=("int4", "int8", "topk"),
    ):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("the fused communicator spans one node (at most 8 ranks)")
        # Largest segment one launch handles; longer buckets are split into
        # segments of this many elements (a multiple of one chunk).
        self.capacity = int(max_numel)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.timeout_ns = int(timeout_s * 1e9)
        self.max_ctas = int(max_ctas)
        self.status = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._status_host = torch.zeros(4, dtype=torch.int32, pin_memory=True)
        self.launches = 0
        # Bucket-size threshold (fp32 bytes) above which dense modes use
        # the two-shot kernel; set by autotune() from measured timings.
        self.twoshot_min_bytes = twoshot_min_bytes if twoshot_min_bytes is not None else self._default_twoshot()
        self.region = None
        if self.world > 1:
            self.layout = make_layout(self.world, max_numel, topk_k, modes)
            self.region = SymmetricRegion(self.layout.total, group=group, device=self.device)
            ptrs = self.region.ptrs
            L = self.layout
            self.comm = _cuda().FusedComm(
                self.world, self.rank, ptrs, L.flags_off, L.inbox_off, L.slot_bytes, L.result_off, L.result_bytes,
                self.status,
            )
        else:
            self.layout = None
            self.comm = _cuda().FusedComm(1, 0, [], 0, 0, 0, 0, 0, self.status)

    def _default_twoshot(self) -> int:
        # One-shot moves (W-1)*P bytes per rank, two-shot about 2*P*(W-1)/W
        # plus one more flag round trip; from 4 ranks up two-shot wins for
        # buckets large enough to amortize the extra phase.
        if self.world <= 2:
            return 1 << 62
        # measured at 8 ranks: one-shot still wins at 16 MB, two-shot at 256 MB;
        # the hook refines this on its first call (autotune_twoshot)
        return 64 << 20

    def choose_variant(self, numel: int, mode: str, variant: str = "auto") -> str:
        if self.world == 1:
            return "single"
        if variant != "auto":
            return variant
        if mode == "topk":
            return "oneshot"
        return "twoshot" if numel * 4 >= self.twoshot_min_bytes else "oneshot"

    @staticmethod
    def tag_for(numel: int, bucket: int) -> int:
        return zlib.crc32(f"{numel}:{bucket}".encode()) & 0xFFFFFFFF

    def allreduce_(
        self,
        grad: torch.Tensor,
        pred: torch.Tensor | None,
        ef: torch.Tensor | None,
        *,
        mode: str = "int4",
        k: int = 26,
        variant: str = "auto",
        stochastic: bool = True,
        seed: int = 0,
        bucket: int = 0,
        step: int = 0,
        beta: float = 0.9,
        first: bool = False,
        tag: int | None = None,
        topo_drop: float = 0.0,
        topo_seed: int = 0,
        max_ctas: int | None = None,
        opt: FusedOpt | None = None,
    ) -> str:
        """Average ``grad`` across ranks in place on the current stream.

        ``max_ctas`` caps this launch's grid (default: the communicator's);
        every rank must pass the same value for the same bucket.  ``opt``
        applies AdamW to the bucket's parameters as each averaged gradient
        element is written (fp32 buckets).

        Buckets longer than ``capacity`` run as several launches over
        segments; segment s of bucket b draws its noise from stream
        ``b * 65536 + s``.  ``topo_drop`` > 0 makes that fraction of the
        bucket's 2048-element chunks passengers (see ``topology``).
        """
        n = grad.numel()
        if self.world > 1 and n > self.capacity:
            seg = max(CHUNK_BLOCKS * BLOCK, self.capacity // (CHUNK_BLOCKS * BLOCK) * (CHUNK_BLOCKS * BLOCK))
            v = ""
            for si, s0 in enumerate(range(0, n, seg)):
                s1 = min(n, s0 + seg)
                v = self.allreduce_(
                    grad[s0:s1], None if pred is None else pred[s0:s1], None if ef is None else ef[s0:s1],
                    mode=mode, k=k, variant=variant, stochastic=stochastic, seed=seed,
                    bucket=(bucket * 65536 + si) & 0xFFFFFFFF, step=step, beta=beta, first=first,
                    tag=None if tag is None else (tag + si) & 0xFFFFFFFF, topo_drop=topo_drop,
                    topo_seed=topo_seed, max_ctas=max_ctas,
                    opt=None if opt is None else FusedOpt(opt.segs, opt.nsegs, opt.hyper, opt.base + s0),
                )
            return v
        v = self.choose_variant(n, mode, variant)
        if tag is None:
            tag = self.tag_for(n, bucket)
        self.comm.run(
            grad, pred, ef, MODES[mode], int(k), VARIANTS[v], bool(stochastic), int(seed) & 0x7FFFFFFFFFFFFFFF,
            int(bucket), int(step), float(beta), bool(first), self.max_ctas if max_ctas is None else int(max_ctas),
            self.timeout_ns, int(tag),
            list(topology(n, topo_drop, topo_seed, bucket)) if topo_drop > 0.0 else [],
            None if opt is None else opt.segs, 0 if opt is None else int(opt.nsegs),
            0 if opt is None else int(opt.base), [] if opt is None else [float(x) for x in opt.hyper],
        )
        self.launches += 1
        self._status_host.copy_(self.status, non_blocking=True)
        return v

    def poll_status(self) -> int:
        """Status copied after the previous launches (no device sync)."""
        return int(self._status_host[0])

    def check(self) -> None:
        """Synchronize and raise ``CommError`` if any launch reported an error."""
        torch.cuda.synchronize(self.device)
        st = self.status.cpu().tolist()
        if st[0] != 0:
            raise CommError(f"fused all-reduce failed: {STATUS_NAMES.get(st[0], st[0])} (chunk {st[1]}, rank {st[2]})")

    def reset_status(self) -> None:
        self.status.zero_()

    def close(self) -> None:
        if self.region is not None:
            torch.cuda.synchronize(self.device)
            self.region.close()
            self.region = None


def autotune_twoshot(comm: FusedAllReduce, sizes_mb=(1, 4, 16, 64), iters: int = 5) -> int:
    """Time one-shot vs two-shot INT4 per bucket size; return the crossover.

    Every rank runs the same sequence; the decision uses the max over ranks
    so all ranks pick the same variant.
    """
    if comm.world == 1:
        return comm.twoshot_min_bytes
    dev = comm.device
    best_twoshot_from = None
    for mb in sizes_mb:
        n = min(mb * (1 << 20) // 4, comm.layout.max_numel)
        g = torch.randn(n, device=dev) * 1e-3
        times = {}
        for v in ("oneshot", "twoshot"):
            for _ in range(2):
                comm.allreduce_(g, None, None, variant=v, bucket=0, step=0)
            torch.cuda.synchronize(dev)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for i in range(iters):
                comm.allreduce_(g, None, None, variant=v, bucket=0, step=i)
            e.record()
            torch.cuda.synchronize(dev)
            t = torch.tensor([s.elapsed_time(e) / iters], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=comm.group)
            times[v] = float(t)
        if times["twoshot"] < times["oneshot"] and best_twoshot_from is None:
            best_twoshot_from = n * 4
        if times["twoshot"] >= times["oneshot"]:
            best_twoshot_from = None
    comm.check()
    comm.twoshot_min_bytes = best_twoshot_from if best_twoshot_from is not None else (1 << 62)
    return comm.twoshot_min_bytes
