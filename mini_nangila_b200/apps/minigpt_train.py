"""Toy DDP training on random tokens with the compression hook
(python/nangila_ddp/examples/minigpt_train.py); runs on CUDA (fused hook) or
CPU (host hook)."""
from __future__ import annotations

import argparse

import torch
import torch.distributed as dist

from ..models import TinyGPT
from ..train import DDPTrainer, init_distributed


class _LM(torch.nn.Module):
    def __init__(self, vocab):
        super().__init__()
        self.m = TinyGPT(vocab=vocab)
        self.vocab = vocab

    def forward(self, x, y):
        return torch.nn.functional.cross_entropy(self.m(x).reshape(-1, self.vocab), y.reshape(-1))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--vocab", type=int, default=5000)
    a = ap.parse_args(argv)
    cuda = torch.cuda.is_available()
    rank, world, local = init_distributed("nccl" if cuda else "gloo")
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    tr = DDPTrainer(_LM(a.vocab), lr=3e-4, hook="fused" if cuda else "host", device=dev,
                    hook_kwargs=dict(beta=0.9, bits=4, stochastic=True, use_fp16_transport=True),
                    autocast_dtype=None)
    g = torch.Generator(device=dev).manual_seed(rank)
    for step in range(a.steps):
        x = torch.randint(0, a.vocab, (8, 128), device=dev, generator=g)
        y = torch.randint(0, a.vocab, (8, 128), device=dev, generator=g)
        loss = tr.step(x, y)
        if rank == 0 and step % 10 == 0:
            print(f"step {step} loss {loss.item():.4f}")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
