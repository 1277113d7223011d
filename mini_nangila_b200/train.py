"""Data-parallel training engine: the public API a user calls.

``DDPTrainer`` wraps a model in ``DistributedDataParallel`` (25 MB buckets,
gradient buckets as views), registers a gradient communication hook and runs
AdamW steps under bf16 autocast with fp32 master weights:

* ``hook="fused"``: predictive-residual compression, one sm_100a kernel per
  bucket (``register_nangila_hook``);
* ``hook="nccl"``: stock DDP all-reduce (plain NCCL fp32), the baseline;
* ``hook="compat"`` / ``"host"``: the reference-compatible and the CPU paths.

``step(x, y)`` trains on device-resident tokens and returns the loss tensor;
``step_host(x_pinned, y_pinned)`` copies the step's inputs from pinned host
memory, trains, and reads the loss back (the end-to-end path).

Reference: python/nangila_ddp/train_nano.py:126-181 (DDP + hook + AdamW loop).
"""
from __future__ import annotations

import math
import os
from datetime import timedelta

import numpy as np
import torch

from .utils.nvtx import nvtx_range
import torch.distributed as dist
from torch.nn.parallel import DistributedDataParallel as DDP

from .parallel.hook import register_nangila_hook


def init_distributed(backend: str | None = None, timeout_s: float = 300.0) -> tuple[int, int, int]:
    """Initialise torch.distributed from torchrun's environment (or as a
    single rank on 127.0.0.1).  Returns (rank, world, local_rank)."""
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if "MASTER_PORT" not in os.environ:
            import socket

            s = socket.socket()
            s.bind(("127.0.0.1", 0))
            os.environ["MASTER_PORT"] = str(s.getsockname()[1])
            s.close()
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        os.environ.setdefault("LOCAL_RANK", "0")
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        local = int(os.environ["LOCAL_RANK"])
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s))
    return dist.get_rank(), dist.get_world_size(), int(os.environ.get("LOCAL_RANK", "0"))


class BucketAdamW:
    """The trainer's AdamW applied to one DDP bucket's parameters, from the
    gradient hook, with PyTorch's fused AdamW kernel on the current (hook)
    stream: each bucket's update runs as soon as its averaged gradients
    land, overlapping the rest of backward, and only the last bucket's
    update follows the end of backward.

    The state lives in the ``torch.optim.AdamW`` object (``exp_avg``,
    ``exp_avg_sq`` and a device ``step`` per parameter, created as that
    optimizer creates them for ``fused=True``), so its ``state_dict`` is
    unchanged and either path can resume the other.  Hyper-parameters are
    read from the parameter's group at every call (schedulers work).  What
    cannot work with an update per bucket: anything that needs every
    gradient before the first update (global-norm clipping, a skipped step).
    """

    def __init__(self, opt: torch.optim.Optimizer):
        self.opt = opt
        self.group_of = {id(p): g for g in opt.param_groups for p in g["params"]}
        self.updated: set[int] = set()  # ids of parameters updated in this step
        self._cache: dict = {}
        self._kcache: dict = {}
        self._pending = None

    def _lists(self, params, grads):
        key = tuple(p.data_ptr() for p in params) + tuple(g.data_ptr() for g in grads)
        hit = self._cache.get(key)
        if hit is not None:
            return hit
        by_group: dict[int, tuple] = {}
        for p, g in zip(params, grads):
            grp = self.group_of[id(p)]
            st = self.opt.state[p]
            if len(st) == 0:
                st["step"] = torch.zeros((), dtype=torch.float32, device=p.device)
                st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            lists = by_group.setdefault(id(grp), (grp, [], [], [], [], []))
            lists[1].append(p)
            lists[2].append(g.view_as(p))
            lists[3].append(st["exp_avg"])
            lists[4].append(st["exp_avg_sq"])
            lists[5].append(st["step"])
        out = list(by_group.values())
        if len(self._cache) > 4096:
            self._cache.clear()
        self._cache[key] = out
        return out

    def apply(self, params, grads) -> None:
        with torch.no_grad():
            for grp, ps, gs, ms, vs, steps in self._lists(params, grads):
                b1, b2 = grp["betas"]
                torch._foreach_add_(steps, 1)
                torch._fused_adamw_(ps, gs, ms, vs, [], steps, lr=float(grp["lr"]), beta1=float(b1),
                                    beta2=float(b2), weight_decay=float(grp["weight_decay"]), eps=float(grp["eps"]),
                                    amsgrad=False, maximize=bool(grp.get("maximize", False)))
        self.updated.update(id(p) for p in params)

    def __call__(self, bucket) -> None:
        self.apply(bucket.parameters(), bucket.gradients())

    # ------------------------------------------- AdamW inside the exchange kernel
    def kernel_args(self, bucket):
        """The bucket's update as a ``parallel.fused.FusedOpt`` for the
        exchange kernel to apply as it writes each averaged gradient, or
        None when the bucket does not qualify (parameters not fp32 CUDA
        tensors of one group, amsgrad or maximize, a non-float lr)."""
        from .parallel.fused import FusedOpt

        params, grads = bucket.parameters(), bucket.gradients()
        buf = bucket.buffer()
        if not params or buf.dtype != torch.float32 or not buf.is_cuda:
            return None
        key = (buf.data_ptr(), buf.numel()) + tuple(p.data_ptr() for p in params)
        hit = self._kcache.get(key)
        if hit is None:
            grp = self.group_of.get(id(params[0]))
            if grp is None or grp.get("amsgrad") or grp.get("maximize") or not isinstance(grp["lr"], float):
                return None
            rows = []
            steps = []
            for p, g in zip(params, grads):
                if (self.group_of.get(id(p)) is not grp or p.dtype != torch.float32 or not p.is_cuda
                        or not p.is_contiguous() or g.dtype != torch.float32):
                    return None
                off, rem = divmod(g.data_ptr() - buf.data_ptr(), 4)
                if rem or off < 0 or off + g.numel() > buf.numel() or g.numel() != p.numel():
                    return None
                st = self.opt.state[p]
                if len(st) == 0:
                    st["step"] = torch.zeros((), dtype=torch.float32, device=p.device)
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                rows.append((off, p.numel(), p.data_ptr(), st["exp_avg"].data_ptr(), st["exp_avg_sq"].data_ptr()))
                steps.append(st["step"])
            rows.sort()
            table = np.array(rows, dtype=[("off", "<i8"), ("numel", "<i8"), ("p", "<u8"), ("m", "<u8"),
                                          ("v", "<u8")])
            segs = torch.from_numpy(np.frombuffer(table.tobytes(), np.uint8).copy()).to(buf.device)
            # all of a bucket's parameters step together; the count is read
            # from the device once, then kept on the host
            t = int(steps[0].item())
            hit = {"segs": segs, "n": len(rows), "steps": steps, "t": t, "grp": grp, "params": list(params)}
            if len(self._kcache) > 4096:
                self._kcache.clear()
            self._kcache[key] = hit
        grp = hit["grp"]
        t = hit["t"] + 1
        b1, b2 = grp["betas"]
        lr, wd = float(grp["lr"]), float(grp["weight_decay"])
        hyper = [float(b1), float(b2), float(grp["eps"]), 1.0 - lr * wd, lr / (1.0 - float(b1) ** t),
                 1.0 / math.sqrt(1.0 - float(b2) ** t)]
        self._pending = hit
        return FusedOpt(hit["segs"], hit["n"], hyper)

    def kernel_done(self, bucket) -> None:
        """After the kernel launch that applied ``kernel_args``: advance the
        step counters (device tensors, as torch's AdamW keeps them)."""
        hit = self._pending
        self._pending = None
        hit["t"] += 1
        torch._foreach_add_(hit["steps"], 1)
        self.updated.update(id(p) for p in hit["params"])

    def finish_step(self, all_params) -> None:
        """Update the parameters no bucket carried this step (if any), then
        start the next step's bookkeeping."""
        rest = [p for p in all_params if p.grad is not None and id(p) not in self.updated]
        if rest:
            self.apply(rest, [p.grad for p in rest])
        self.updated.clear()


class DDPTrainer:
    """DDP + gradient hook + AdamW (+ bf16 autocast) training steps; see the module docstring.

    ``overlap_optimizer=True`` (fused hook on CUDA) applies AdamW per bucket
    from the hook (``BucketAdamW``) instead of once after backward; with
    ``optimizer_in_kernel`` (the default) the exchange kernel itself applies
    it to fp32 parameters as it writes each averaged gradient.
    ``timeline_next_step()`` records the next step's device timeline
    (``utils.timeline.StepTimeline``).
    """
    def __init__(
        self,
        model: torch.nn.Module,
        *,
        lr: float = 6e-4,
        hook: str = "fused",
        hook_kwargs: dict | None = None,
        bucket_cap_mb: float = 25.0,
        autocast_dtype: torch.dtype | None = torch.bfloat16,
        device: torch.device | None = None,
        fused_optimizer: bool = True,
        monitor: bool = False,
        overlap_optimizer: bool = False,
        optimizer_in_kernel: bool = True,
    ):
        self.device = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
                                 else torch.device("cpu"))
        model = model.to(self.device)
        kw = dict(bucket_cap_mb=bucket_cap_mb, gradient_as_bucket_view=True)
        if self.device.type == "cuda":
            kw["device_ids"] = [self.device.index]
        self.ddp = DDP(model, **kw)
        self.hook_state = None
        if hook in ("fused", "compat", "host"):
            hk = dict(hook_kwargs or {})
            hk.setdefault("impl", hook)
            self.hook_state = register_nangila_hook(self.ddp, **hk)
        elif hook != "nccl":
            raise ValueError(f"unknown hook {hook!r}")
        self.steps_done = 0
        self.monitor = None
        if monitor:
            from .parallel.monitor import RankMonitor

            comm = getattr(self.hook_state, "comm", None) if self.hook_state is not None else None
            self.monitor = RankMonitor(comms=[comm] if comm is not None else [])
        # PyTorch's fused AdamW on CUDA and on CPU.  On CPU it also keeps the
        # ranks' parameters bit-identical: the unfused CPU step runs its
        # square root through a vector-math library split over the intra-op
        # threads, and one thread's share of a tensor has been seen to come
        # out about 1e-4 off (relative) on one rank of two from identical
        # inputs, while a single-threaded replay of the same step was exact.
        use_fused = fused_optimizer and self.device.type in ("cuda", "cpu")
        self.opt = torch.optim.AdamW(self.ddp.parameters(), lr=lr, fused=use_fused)
        self.autocast_dtype = autocast_dtype if self.device.type == "cuda" else None
        self.bucket_opt = None
        if overlap_optimizer:
            if hook not in ("fused", "host"):
                raise ValueError("overlap_optimizer needs the fused (CUDA) or host (CPU) hook")
            self.bucket_opt = BucketAdamW(self.opt)
            self.hook_state.after_reduce = self.bucket_opt
            if optimizer_in_kernel and hook == "fused":
                # AdamW inside the exchange kernel's decode phase when the
                # bucket qualifies (fp32 parameters); the separate update
                # above otherwise
                self.hook_state.kernel_opt = self.bucket_opt.kernel_args
                self.hook_state.kernel_opt_done = self.bucket_opt.kernel_done
        self.timeline = None
        self._timeline_next = False

    def timeline_next_step(self) -> None:
        """Record the next ``step``'s timeline into ``self.timeline``."""
        self._timeline_next = True

    @property
    def model(self) -> torch.nn.Module:
        return self.ddp.module

    def step(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        if self.monitor is not None:
            self.monitor.check(self.steps_done)  # a peer that left is noticed before any launch
        tl = None
        if self._timeline_next and self.device.type == "cuda":
            from .utils.timeline import StepTimeline

            tl = self.timeline = StepTimeline()
            tl.mark("forward")
            if self.hook_state is not None and hasattr(self.hook_state, "timeline"):
                self.hook_state.timeline = tl
        self._timeline_next = False
        with nvtx_range("forward"):
            if self.autocast_dtype is not None:
                with torch.autocast(self.device.type, dtype=self.autocast_dtype):
                    loss = self.ddp(x, y)
            else:
                loss = self.ddp(x, y)
        self.opt.zero_grad(set_to_none=False)
        if tl is not None:
            tl.mark("backward")
        with nvtx_range("backward"):
            loss.backward()
        if tl is not None:
            tl.mark("backward_done")
        with nvtx_range("optimizer"):
            if self.bucket_opt is not None:
                self.bucket_opt.finish_step(self.opt.param_groups[0]["params"] if len(self.opt.param_groups) == 1
                                            else [p for g in self.opt.param_groups for p in g["params"]])
            else:
                self.opt.step()
        if tl is not None:
            tl.mark("step_done")
            if self.hook_state is not None and hasattr(self.hook_state, "timeline"):
                self.hook_state.timeline = None
        self.steps_done += 1
        return loss.detach()

    def step_host(self, x_host: torch.Tensor, y_host: torch.Tensor) -> float:
        x = x_host.to(self.device, non_blocking=True)
        y = y_host.to(self.device, non_blocking=True)
        return float(self.step(x, y).item())

    def step_host_async(self, x_host: torch.Tensor, y_host: torch.Tensor):
        """One step from pinned host tensors without waiting for it: the
        batch is copied to the device, the step is queued, and its loss is
        copied back into pinned host memory.  Returns ``(loss, event)``;
        ``event.synchronize()`` then ``float(loss)`` reads it, typically
        after the next step has been queued (``train_steps`` does this)."""
        x = x_host.to(self.device, non_blocking=True)
        y = y_host.to(self.device, non_blocking=True)
        loss = self.step(x, y)
        if self.device.type != "cuda":
            return loss.detach().clone(), None
        out = torch.empty((), dtype=loss.dtype, pin_memory=True)
        out.copy_(loss, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        return out, ev

    def train_steps(self, batches_host) -> list[float]:
        """Run one step per (x, y) pinned host batch, reading every step's loss
        one step late, so the host never waits for the step in flight."""
        losses: list[float] = []
        pending = None
        for x_host, y_host in batches_host:
            cur = self.step_host_async(x_host, y_host)
            if pending is not None:
                if pending[1] is not None:
                    pending[1].synchronize()
                losses.append(float(pending[0]))
            pending = cur
        if pending is not None:
            if pending[1] is not None:
                pending[1].synchronize()
            losses.append(float(pending[0]))
        return losses

    def fit(self, next_batch, steps: int, log=None, lr: float | None = None, first_step: int = 1) -> list[float]:
        """Run ``steps`` training steps.  ``next_batch(step)`` returns the
        step's (x, y) on the device; each step is timed on the device
        (``utils.trainlog.StepTimer``) and, with a ``TrainLog``, logged as one
        row.  Returns the losses (read every step, so this loop waits for
        each step; ``train_steps`` is the pipelined form)."""
        from .utils.trainlog import StepTimer

        timer = StepTimer(self.device)
        lr = lr if lr is not None else self.opt.param_groups[0]["lr"]
        losses = []
        for step in range(first_step, first_step + steps):
            x, y = next_batch(step)
            timer.start()
            loss = self.step(x, y)
            ms = timer.stop_ms()
            losses.append(float(loss))
            if log is not None:
                log.row(step, losses[-1], lr, x.numel(), ms)
        return losses

    def state_dict(self) -> dict:
        """Everything a resumed run needs: model, optimizer, the hook's
        predictor / error-feedback state and counters, steps done."""
        return {"model": self.model.state_dict(), "optimizer": self.opt.state_dict(),
                "hook": self.hook_state.state_dict() if self.hook_state is not None else None,
                "steps_done": self.steps_done}

    def load_state_dict(self, sd: dict) -> None:
        self.model.load_state_dict(sd["model"])
        self.opt.load_state_dict(sd["optimizer"])
        if self.hook_state is not None and sd.get("hook") is not None:
            self.hook_state.load_state_dict(sd["hook"])
        self.steps_done = int(sd.get("steps_done", 0))

    def kernel_launches(self) -> int:
        hs = self.hook_state
        if hs is not None and getattr(hs, "comm", None) is not None:
            return hs.comm.launches
        return 0
