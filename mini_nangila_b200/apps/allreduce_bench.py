"""Compressed all-reduce bandwidth sweep (run under torchrun, one rank per GPU).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m mini_nangila_b200.apps.allreduce_bench \
        [--sizes-mb 1,4,16,64,256,1024] [--steps 20] [--out results.jsonl]

Bucket contents are N(0, 1e-3^2) and evolve as an AR(1) process with rho 0.9
over the steps (each rank its own stream), so the momentum predictor has
signal.  For every size it times, with CUDA events around each call and the
max over ranks: the fused kernel in INT4 (one-shot, two-shot and the auto
choice) and top-k 1/5/10 %, and NCCL all_reduce of the fp32 and bf16 bucket.

Reported per row: time per call, effective GB/s of uncompressed fp32 data
reduced, compressed bytes each rank sends over NVLink, and the fraction of
the roofline max(HBM bytes / measured HBM bandwidth, NVLink bytes / 900 GB/s
per direction, the nominal NVLink 5 figure), with the fraction against the
770 GB/s peer copy measured on these machines as a second column.  With
``--nvlink`` every rank also reads its GPU's NVLink data counters (NVML,
``utils.nvlink``) around the timed calls and the row carries the measured
bytes sent and received per call (mean and max over ranks).
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 900.0  # NVLink 5 per direction per GPU (nominal): the roofline
NVLINK_MEASURED_GBS = 770.0  # peer copy per direction measured on these B200s


def hbm_peak_gbs() -> float:
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            return float(json.load(fh)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def roofline_ms(n: int, world: int, mode: str, variant: str, k: int,
                link_gbs: float = NVLINK_GBS) -> tuple[float, int]:
    from ..parallel.fused import dense_payload_bytes, payload_bytes

    P = payload_bytes(n, mode, k)
    if variant == "twoshot":
        R = dense_payload_bytes(n, 8)
        nvl = (world - 1) * (P + R) // world
        hbm = 24 * n + 2 * P + 2 * R
    elif variant == "nccl_fp32":
        nvl = 2 * (world - 1) * n * 4 // world
        hbm = 3 * n * 4
    elif variant == "nccl_bf16":
        nvl = 2 * (world - 1) * n * 2 // world
        hbm = 3 * n * 2
    else:
        nvl = (world - 1) * P
        hbm = 24 * n + 2 * world * P
    t = max(hbm / (hbm_peak_gbs() * 1e6), nvl / (link_gbs * 1e6))
    return t, int(nvl)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-mb", default="1,4,16,25,64,154,256,1024")
    ap.add_argument("--nvlink", action="store_true", help="read NVLink data counters around the timed calls")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--modes", default="int4,topk1,topk5,topk10")
    ap.add_argument("--out", default="")
    ap.add_argument("--max-ctas", type=int, default=0)
    args = ap.parse_args()

    from ..parallel.fused import FusedAllReduce, topk_per_block
    from ..train import init_distributed

    rank, world, local = init_distributed("nccl", timeout_s=300)
    dev = torch.device("cuda", local)
    sizes = [int(float(s) * (1 << 20)) // 4 for s in args.sizes_mb.split(",")]
    comm = FusedAllReduce(max(sizes), device=dev, topk_k=topk_per_block(0.10), timeout_s=30.0,
                          max_ctas=args.max_ctas)
    counter = None
    if args.nvlink:
        from ..utils.nvlink import NvlinkCounter

        counter = NvlinkCounter(dev)
    rows = []
    g = torch.Generator(device=dev)
    for n in sizes:
        g.manual_seed(1000 + rank)
        sig = torch.randn(n, device=dev, generator=g) * 1e-3
        buf = torch.empty(n, device=dev)
        pred = torch.zeros(n, device=dev)
        ef = torch.zeros(n, device=dev)
        configs = []
        for m in args.modes.split(","):
            if m == "int4":
                for v in (["oneshot", "twoshot"] if world > 1 else ["single"]):
                    configs.append(("int4", 0, v))
            elif m.startswith("topk"):
                frac = float(m[4:]) / 100.0
                configs.append(("topk", topk_per_block(frac), "oneshot" if world > 1 else "single"))
        configs += [("nccl_fp32", 0, "nccl_fp32"), ("nccl_bf16", 0, "nccl_bf16")]
        for mode, k, variant in configs:
            pred.zero_()
            ef.zero_()
            total = 0.0
            link = [0, 0]
            for step in range(args.warmup + args.steps):
                # AR(1): sig <- 0.9 sig + sqrt(1 - 0.81) * N(0, 1e-3^2)
                sig.mul_(0.9).add_(torch.randn(n, device=dev, generator=g), alpha=math.sqrt(0.19) * 1e-3)
                if mode == "nccl_bf16":
                    xb = sig.to(torch.bfloat16)
                else:
                    buf.copy_(sig)
                torch.cuda.synchronize(dev)
                if counter is not None and step >= args.warmup:
                    dist.barrier()  # the peers' traffic of the previous call has ended
                    c0 = counter.read()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                if mode == "nccl_fp32":
                    dist.all_reduce(buf)
                    buf.div_(world)
                elif mode == "nccl_bf16":
                    dist.all_reduce(xb)
                    xb.div_(world)
                else:
                    comm.allreduce_(buf, pred, ef, mode=mode, k=max(k, 1), variant=variant, seed=7, bucket=0,
                                    step=step, beta=0.9, first=(step == 0))
                e.record()
                e.synchronize()
                if step >= args.warmup:
                    total += s.elapsed_time(e)
                    if counter is not None:
                        dist.barrier()  # every peer's stores into this GPU have landed
                        c1 = counter.read()
                        link[0] += c1[0] - c0[0]
                        link[1] += c1[1] - c0[1]
            ms = total / args.steps
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t)
            roof, nvl = roofline_ms(n, world, mode if mode in ("int4", "topk") else "int4",
                                    variant if world > 1 else "single", max(k, 1))
            if mode.startswith("nccl"):
                roof, nvl = roofline_ms(n, world, "int4", variant, 1)
            roof_meas, _ = roofline_ms(n, world, mode if mode in ("int4", "topk") else "int4",
                                       variant if world > 1 else "single", max(k, 1), NVLINK_MEASURED_GBS)
            if mode.startswith("nccl"):
                roof_meas, _ = roofline_ms(n, world, "int4", variant, 1, NVLINK_MEASURED_GBS)
            row = dict(n_gpus=world, bucket_mb=n * 4 / (1 << 20), mode=mode if mode != "topk" else f"topk_k{k}",
                       variant=variant, ms=ms, eff_gbs=n * 4 / (ms * 1e6), nvlink_bytes_per_rank=nvl,
                       roofline_ms=roof, roofline_frac=roof / ms if ms > 0 else None,
                       roofline_frac_measured_link=roof_meas / ms if ms > 0 else None)
            if counter is not None:
                lt = torch.tensor([link[0] / args.steps, link[1] / args.steps], device=dev, dtype=torch.float64)
                lmax = lt.clone()
                dist.all_reduce(lt)
                dist.all_reduce(lmax, op=dist.ReduceOp.MAX)
                row.update(nvlink_counters=counter.available, nvlink_counter_source=counter.source,
                           nvlink_tx_bytes_measured_mean=float(lt[0]) / world,
                           nvlink_rx_bytes_measured_mean=float(lt[1]) / world,
                           nvlink_tx_bytes_measured_max=float(lmax[0]))
            rows.append(row)
            if rank == 0:
                print(json.dumps(row), flush=True)
        del sig, buf, pred, ef
        torch.cuda.empty_cache()
    comm.check()
    if rank == 0 and args.out:
        with open(args.out, "w") as fh:
            for r in rows:
                fh.write(json.dumps(r) + "\n")
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
