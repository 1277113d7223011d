"""Training curves of GPT-2 small under each gradient exchange, same seeds.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        -m mini_nangila_b200.apps.loss_curves --steps 300 --out curves.json

Every setting starts from the same weights (seed 0) and sees the same
batches (``data.MarkovTokens``: a learnable synthetic Markov stream over the
first ``--corpus-vocab`` token ids of the GPT-2 vocabulary, 2048 by default,
so that a few hundred steps reach the chain's entropy instead of stopping
on the plateau of a 50,257-token table; batches are keyed by (seed, rank,
step)); the optimizer is AdamW at
the workload's lr with a short linear warm-up, identical for all settings.
Settings (``--settings``, comma-separated):

* ``nccl``: DDP's uncompressed NCCL fp32 all-reduce (the baseline);
* ``int4-oneshot`` / ``int4-auto`` / ``int4-twoshot``: the fused INT4 +
  EMA + error-feedback hook, one-shot only, the size-based one-shot /
  two-shot choice, or two-shot only (every bucket takes the second,
  round-to-nearest INT8 stage, which error feedback does not see);
* ``topk5``: the fused per-block top-k 5 % + error-feedback hook;
* ``compat``: the reference-compatible hook (INT4, global scale, no EF).

Rank 0 writes JSON with the rank-mean loss of every step per setting and a
summary (loss at steps 0/100/200/..., the mean of the last 20 steps, and
its difference to ``nccl``); ``--log-dir`` adds one ``train_log.csv``-style
file per setting.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from ..data import MarkovTokens
from ..models import GPT2, GPT2Config
from ..train import DDPTrainer, init_distributed
from ..utils.trainlog import TrainLog

SETTINGS = {
    "nccl": dict(hook="nccl"),
    "int4-oneshot": dict(hook="fused", hook_kwargs=dict(use_momentum=True, error_feedback=True, variant="oneshot")),
    "int4-auto": dict(hook="fused", hook_kwargs=dict(use_momentum=True, error_feedback=True, variant="auto")),
    "int4-twoshot": dict(hook="fused", hook_kwargs=dict(use_momentum=True, error_feedback=True, variant="twoshot")),
    "topk5": dict(hook="fused", hook_kwargs=dict(use_momentum=False, error_feedback=True, topk_percent=0.05)),
    "compat": dict(hook="compat", hook_kwargs=dict(use_momentum=True, bits=4)),
}


def run_setting(name: str, a, corpus: MarkovTokens, rank: int, world: int, device) -> list[float]:
    spec = SETTINGS[name]
    torch.manual_seed(0)
    cfg = GPT2Config.small() if not a.tiny else GPT2Config.tiny()
    hk = dict(spec.get("hook_kwargs", {}))
    if spec["hook"] != "nccl":
        hk.setdefault("seed", 12345)
    # the fused kernel's format runs through the host library on CPU ranks
    hook = "host" if (spec["hook"] == "fused" and device.type != "cuda") else spec["hook"]
    if hook == "host":
        hk.pop("variant", None)
    tr = DDPTrainer(GPT2(cfg), lr=a.lr, hook=hook, hook_kwargs=hk or None, bucket_cap_mb=25.0,
                    autocast_dtype=torch.bfloat16 if device.type == "cuda" else None, device=device,
                    overlap_optimizer=hook in ("fused", "host"))
    log = TrainLog(os.path.join(a.log_dir, f"train_log_{name}.csv") if a.log_dir else None, enabled=rank == 0)
    losses = []
    for step in range(a.steps):
        lr = a.lr * min(1.0, (step + 1) / max(1, a.warmup))
        for g in tr.opt.param_groups:
            g["lr"] = lr
        x, y = corpus.batch(a.micro_batch, a.seq, seed=a.seed, rank=rank, step=step, device=device)
        loss = tr.step(x, y)
        t = loss.detach().float().reshape(1)
        dist.all_reduce(t)
        losses.append(float(t) / world)
        log.row(step, losses[-1], lr, x.numel() * world, 0.0)
    hs = tr.hook_state
    if hs is not None and getattr(hs, "comm", None) is not None:
        hs.comm.check()
        hs.comm.close()
    del tr
    torch.cuda.empty_cache() if device.type == "cuda" else None
    return losses


def summarize(curves: dict, every: int = 100, tail: int = 20) -> dict:
    out = {}
    base = None
    if "nccl" in curves:
        c = curves["nccl"]
        base = sum(c[-tail:]) / len(c[-tail:])
    for name, c in curves.items():
        final = sum(c[-tail:]) / len(c[-tail:])
        marks = {str(s): c[s] for s in range(0, len(c), every)}
        marks[str(len(c) - 1)] = c[-1]
        out[name] = {"loss_at": marks, f"mean_last_{tail}": final,
                     "delta_vs_nccl": None if base is None else final - base}
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--settings", default="nccl,int4-oneshot,int4-auto,int4-twoshot,topk5,compat")
    ap.add_argument("--micro-batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--lr", type=float, default=6e-4)
    ap.add_argument("--warmup", type=int, default=30, help="linear lr warm-up steps")
    ap.add_argument("--seed", type=int, default=7)
    ap.add_argument("--out", default="loss_curves.json")
    ap.add_argument("--log-dir", default="")
    ap.add_argument("--corpus-vocab", type=int, default=2048,
                    help="tokens the Markov chain uses (ids below this; the model keeps its full vocabulary)")
    ap.add_argument("--tiny", action="store_true", help="tiny GPT-2 (tests)")
    a = ap.parse_args(argv)
    use_cuda = torch.cuda.is_available()
    rank, world, local = init_distributed("nccl" if use_cuda else "gloo")
    device = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    cfg = GPT2Config.small() if not a.tiny else GPT2Config.tiny()
    corpus = MarkovTokens(min(a.corpus_vocab, cfg.vocab_size), seed=a.seed)
    curves = {}
    for name in [s for s in a.settings.split(",") if s]:
        if name not in SETTINGS:
            raise SystemExit(f"unknown setting {name!r}; choose from {sorted(SETTINGS)}")
        curves[name] = run_setting(name, a, corpus, rank, world, device)
    if rank == 0:
        res = {"world": world, "steps": a.steps, "micro_batch": a.micro_batch, "seq": a.seq, "lr": a.lr,
               "warmup": a.warmup, "data": "MarkovTokens(%d tokens of the model's %d, 4 successors, seed %d)" % (
                   corpus.vocab, cfg.vocab_size, a.seed),
               "entropy_floor_nats": corpus.entropy_nats, "summary": summarize(curves), "curves": curves}
        with open(a.out, "w") as fh:
            json.dump(res, fh)
        print(json.dumps(res["summary"]), flush=True)
    dist.destroy_process_group()
    return curves


if __name__ == "__main__":
    main()
