"""Character-level TinyGPT DDP training with the compression hook
(python/nangila_ddp/train_nano.py).

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m mini_nangila_b200.apps.train_nano \
        --device cpu --steps 50 --use_momentum

Same flags and CSV outputs as the reference (``train_log.csv`` with
``ts,step,loss,lr,tokens_per_sec,step_ms``; the hook's metrics CSV).  There
is no network here: without ``--data`` the reference's synthetic fallback
text is used.  On CUDA the hook is the fused sm_100a kernel (``--impl``
selects fused / compat / host).
"""
from __future__ import annotations

import argparse
import os
import time

import torch
import torch.distributed as dist
from torch.nn.parallel import DistributedDataParallel as DDP
from torch.utils.data import DataLoader, Dataset

from ..models import TinyGPT
from ..parallel import register_nangila_hook
from ..train import init_distributed


class CharDataset(Dataset):
    def __init__(self, text: str, block_size: int):
        self.block = block_size
        self.chars = sorted(set(text))
        self.c2i = {c: i for i, c in enumerate(self.chars)}
        self.vocab = len(self.chars)
        self.data = torch.tensor([self.c2i[c] for c in text], dtype=torch.long)

    def __len__(self):
        return max(0, self.data.numel() - self.block - 1)

    def __getitem__(self, i):
        return self.data[i:i + self.block], self.data[i + 1:i + 1 + self.block]


def main(argv=None):
    ap = argparse.ArgumentParser(description="NanoGPT DDP with the compression hook")
    ap.add_argument("--data", default="")
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
    a = ap.parse_args(argv)
    dev = a.device if a.device != "auto" else ("cuda" if torch.cuda.is_available() else "cpu")
    rank, world, local = init_distributed("nccl" if dev == "cuda" else "gloo")
    device = torch.device("cuda", local) if dev == "cuda" else torch.device("cpu")
    torch.manual_seed(a.seed + rank)
    if rank == 0:
        if a.data and os.path.exists(a.data):
            text = open(a.data, encoding="utf-8").read()
        else:
            text = "abc def ghi " * 100000
    else:
        text = ""
    lens = torch.tensor([len(text)], dtype=torch.long, device=device)
    dist.broadcast(lens, src=0)
    buf = torch.empty(int(lens.item()), dtype=torch.uint8, device=device)
    if rank == 0:
        buf.copy_(torch.tensor(list(text.encode("utf-8")), dtype=torch.uint8, device=device))
    dist.broadcast(buf, src=0)
    text = bytes(buf.cpu().tolist()).decode("utf-8")
    ds = CharDataset(text, a.block_size)
    sampler = torch.utils.data.distributed.DistributedSampler(ds, num_replicas=world, rank=rank, shuffle=True)
    loader = DataLoader(ds, batch_size=a.batch_size, sampler=sampler, drop_last=True)
    model = TinyGPT(a.d_model, a.nhead, a.nlayers, ds.vocab, a.block_size).to(device)
    model = DDP(model, device_ids=[local]) if dev == "cuda" else DDP(model)
    impl = a.impl or ("fused" if dev == "cuda" else "host")
    if a.topo_drop > 0.0:
        impl = "compat"
    register_nangila_hook(model, beta=0.9, bits=4, stochastic=True, use_fp16_transport=False,
                          metrics_path=a.metrics_path, use_momentum=a.use_momentum, topk_percent=a.topk,
                          topo_drop_percent=a.topo_drop, impl=impl)
    opt = torch.optim.AdamW(model.parameters(), lr=a.lr)
    loss_fn = torch.nn.CrossEntropyLoss()
    if rank == 0:
        with open(a.train_log, "w") as fh:
            fh.write("ts,step,loss,lr,tokens_per_sec,step_ms\n")
    step, tok = 0, a.batch_size * a.block_size
    for epoch in range(1_000_000):
        sampler.set_epoch(epoch)
        for xb, yb in loader:
            step += 1
            xb, yb = xb.to(device), yb.to(device)
            t0 = time.time()
            logits = model(xb)
            loss = loss_fn(logits.view(-1, ds.vocab), yb.view(-1))
            opt.zero_grad(set_to_none=True)
            loss.backward()
            opt.step()
            ms = (time.time() - t0) * 1000.0
            if rank == 0:
                with open(a.train_log, "a") as fh:
                    fh.write(f"{time.time():.6f},{step},{loss.item():.6f},{a.lr},{tok / max(1e-6, ms / 1000):.2f},"
                             f"{ms:.2f}\n")
                if step % 10 == 0:
                    print(f"step {step} loss {loss.item():.4f} tps {tok / max(1e-6, ms / 1000):.1f} tokens/s")
            if step >= a.steps:
                break
        if step >= a.steps:
            break
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
