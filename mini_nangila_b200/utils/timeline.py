"""Per-step device timeline of a DDP training step (CUDA events only).

A ``StepTimeline`` collects, for one training step:

* phase marks on the main stream: ``forward``, ``backward`` (after the
  forward), ``backward_done`` (after ``loss.backward()`` returned, which on
  the main stream includes the wait for every bucket's future), and
  ``step_done`` (after the optimizer);
* per gradient bucket, in call order: ``ready`` (main stream, when DDP
  handed the bucket to the hook: its gradients are complete up to there),
  ``start`` / ``end`` of its exchange kernel and, with the optimizer applied
  per bucket, ``opt_end`` (hook stream).

Recording adds no host synchronisation; ``collect`` waits for the last
event and returns every time in milliseconds since ``forward``.  The
summary names the exposed tail: the time from the end of the backward
compute (the last bucket's ``ready``) to ``step_done``.
"""
from __future__ import annotations

import torch


class StepTimeline:
    def __init__(self):
        self.marks: list[tuple[str, torch.cuda.Event]] = []
        self.buckets: list[dict] = []

    @staticmethod
    def _ev(stream=None) -> torch.cuda.Event:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        return ev

    def mark(self, name: str, stream=None) -> None:
        self.marks.append((name, self._ev(stream)))

    def bucket(self, **info) -> dict:
        """A new bucket record; ``event(rec, name, stream)`` adds its events."""
        rec = dict(info)
        rec["events"] = []
        self.buckets.append(rec)
        return rec

    def event(self, rec: dict, name: str, stream=None) -> None:
        rec["events"].append((name, self._ev(stream)))

    def collect(self) -> dict:
        if not self.marks:
            return {}
        last = self.marks[-1][1]
        for rec in self.buckets:
            for _, ev in rec["events"]:
                ev.synchronize()
        last.synchronize()
        t0 = self.marks[0][1]
        out = {"marks": {n: t0.elapsed_time(ev) for n, ev in self.marks}, "buckets": []}
        for rec in self.buckets:
            row = {k: v for k, v in rec.items() if k != "events"}
            for n, ev in rec["events"]:
                row[n] = t0.elapsed_time(ev)
            out["buckets"].append(row)
        return out


def summarize(tl: dict) -> dict:
    """Headline numbers of a collected timeline (ms): step time, backward
    compute end (last bucket ready), exposed tail after it, exchange kernel
    time in total and inside backward, and the last bucket's kernel and
    optimizer time."""
    m = tl.get("marks", {})
    bs = tl.get("buckets", [])
    if not m or not bs:
        return {}
    ready_last = max(b["ready"] for b in bs)
    step = m.get("step_done", m.get("backward_done"))
    kern = [b["end"] - b["start"] for b in bs if "end" in b and "start" in b]
    hidden = sum(max(0.0, min(b["end"], ready_last) - b["start"]) for b in bs if "end" in b)
    last = max(bs, key=lambda b: b["ready"])
    out = {
        "step_ms": step,
        "backward_compute_end_ms": ready_last,
        "exposed_tail_ms": step - ready_last,
        "kernel_ms_total": sum(kern),
        "kernel_ms_inside_backward": hidden,
        "buckets": len(bs),
        "last_bucket": {k: last[k] for k in ("bucket", "numel", "variant", "grid") if k in last},
        "last_bucket_kernel_ms": last.get("end", 0.0) - last.get("start", 0.0),
        "last_bucket_wait_ms": last.get("start", 0.0) - last["ready"],
    }
    if "opt_end" in last:
        out["last_bucket_optimizer_ms"] = last["opt_end"] - last["end"]
    if "backward_done" in m and "step_done" in m:
        out["optimizer_after_backward_ms"] = m["step_done"] - m["backward_done"]
    return out
