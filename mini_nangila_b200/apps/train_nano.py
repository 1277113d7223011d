"""Character-level TinyGPT DDP training with the compression hook.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m mini_nangila_b200.apps.train_nano \\
        --device cpu --steps 50 --use_momentum

The command line and both CSV outputs are the reference trainer's
(python/nangila_ddp/train_nano.py:66-82 flags; ``train_log.csv`` with
``ts,step,loss,lr,tokens_per_sec,step_ms``; the hook's metrics CSV), so its
plot scripts read these logs.  The rest is this framework's:

* data: ``data.CharCorpus`` — every rank reads the same text (``--data``,
  else the reference's offline fallback text; there is no network here) and
  draws random windows keyed by (seed, rank, step), so no broadcast or
  sampler is needed;
* the step: ``train.DDPTrainer`` (DDP with bucket views, the hook, AdamW),
  fp32 like the reference;
* logging: ``utils.trainlog.TrainLog`` on rank 0, step time from CUDA events
  on GPUs.

``--impl`` picks the hook (fused sm_100a kernel on CUDA, the C++ host path
on CPU, or the reference-compatible ``compat``).  ``--topo_drop`` without
``--impl`` uses ``compat``, whose element-granular drop matches the
reference's; fused/host drop whole 2048-element chunks.
"""
from __future__ import annotations

import argparse

import torch
import torch.distributed as dist

from ..data import CharCorpus
from ..models import TinyGPT
from ..train import DDPTrainer, init_distributed
from ..utils.trainlog import TrainLog


def parse(argv=None):
    ap = argparse.ArgumentParser(description="TinyGPT DDP training with the compression hook")
    ap.add_argument("--data", default="", help="text file; empty: the offline fallback text")
    ap.add_argument("--block_size", type=int, default=128)
    ap.add_argument("--d_model", type=int, default=256)
    ap.add_argument("--nhead", type=int, default=4)
    ap.add_argument("--nlayers", type=int, default=4)
    ap.add_argument("--batch_size", type=int, default=16)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--metrics_path", default="ddp_metrics.csv")
    ap.add_argument("--train_log", default="train_log.csv")
    ap.add_argument("--device", default="auto", choices=["auto", "cuda", "cpu"])
    ap.add_argument("--seed", type=int, default=1337)
    ap.add_argument("--use_momentum", action="store_true")
    ap.add_argument("--topk", type=float, default=0.0)
    ap.add_argument("--topo_drop", type=float, default=0.0)
    ap.add_argument("--impl", default=None, choices=[None, "fused", "compat", "host"])
    return ap.parse_args(argv)


def main(argv=None):
    a = parse(argv)
    use_cuda = a.device == "cuda" or (a.device == "auto" and torch.cuda.is_available())
    rank, world, local = init_distributed("nccl" if use_cuda else "gloo")
    device = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    torch.manual_seed(a.seed)  # same initial weights on every rank (DDP also broadcasts them)
    corpus = CharCorpus.from_path(a.data or None)
    impl = a.impl or ("compat" if a.topo_drop > 0.0 else ("fused" if use_cuda else "host"))
    hook_kwargs = dict(beta=0.9, bits=4, stochastic=True, use_fp16_transport=False, metrics_path=a.metrics_path,
                       use_momentum=a.use_momentum, topk_percent=a.topk, topo_drop_percent=a.topo_drop)
    trainer = DDPTrainer(TinyGPT(a.d_model, a.nhead, a.nlayers, corpus.vocab, a.block_size), lr=a.lr, hook=impl,
                         hook_kwargs=hook_kwargs, autocast_dtype=None, device=device)
    log = TrainLog(a.train_log, enabled=rank == 0, echo_every=10 if rank == 0 else 0)

    def next_batch(step):
        return corpus.batch(a.batch_size, a.block_size, seed=a.seed, rank=rank, step=step, device=device)

    trainer.fit(next_batch, a.steps, log=log, lr=a.lr)
    if trainer.hook_state is not None and getattr(trainer.hook_state, "comm", None) is not None:
        trainer.hook_state.comm.check()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
