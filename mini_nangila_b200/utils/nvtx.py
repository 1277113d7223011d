"""NVTX ranges for timeline tools (no-ops without CUDA or with NGL_NVTX=0).

The hook marks each bucket's compressed exchange and the trainer marks the
forward, backward and optimizer phases, so a timeline shows how the
exchange overlaps backward."""
from __future__ import annotations

import contextlib
import os

import torch

_ON = os.environ.get("NGL_NVTX", "1") != "0"


def enabled() -> bool:
    return _ON and torch.cuda.is_available()


@contextlib.contextmanager
def nvtx_range(name: str):
    if not enabled():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
