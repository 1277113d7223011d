"""Toy DDP training on random tokens with the compression hook
(python/nangila_ddp/examples/minigpt_train.py): a TinyGPT stepped by
``DDPTrainer``, on CUDA with the fused hook or on CPU with the host hook.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m mini_nangila_b200.apps.minigpt_train --steps 20
"""
from __future__ import annotations

import argparse

import torch
import torch.distributed as dist

from ..data import uniform_tokens
from ..models import TinyGPT
from ..train import DDPTrainer, init_distributed
from ..utils.trainlog import TrainLog


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--vocab", type=int, default=5000)
    ap.add_argument("--train_log", default="")
    a = ap.parse_args(argv)
    cuda = torch.cuda.is_available()
    rank, world, local = init_distributed("nccl" if cuda else "gloo")
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    tr = DDPTrainer(TinyGPT(vocab=a.vocab), lr=3e-4, hook="fused" if cuda else "host", device=dev,
                    hook_kwargs=dict(beta=0.9, bits=4, stochastic=True, use_fp16_transport=True),
                    autocast_dtype=None)
    log = TrainLog(a.train_log or None, enabled=rank == 0, echo_every=10 if rank == 0 else 0)
    tr.fit(lambda step: uniform_tokens(a.vocab, 8, 128, seed=1000 * step + rank, device=dev), a.steps, log=log,
           first_step=0)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
