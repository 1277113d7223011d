#!/usr/bin/env python
"""GPT-2 small DDP training throughput with the predictive-residual hook.

    python bench.py [--gpus N --steps K --warmup W]            # this framework
    python bench.py --impl reference ...                       # reference hook
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Workload: GPT-2 small (12 layers, d 768, 12 heads, FFN 3072, vocab 50257),
seq 1024, micro-batch 8 per GPU, fp32 master weights with bf16 autocast,
AdamW lr 6e-4, DDP buckets of 25 MB, random-init N(0, 0.02) weights,
tokens uniform over the vocabulary from a seed (synthetic data).

Timing: W untimed warm-up steps, then exactly K steps between a barrier +
synchronize on both sides, CUDA events on the launching stream, max over
ranks.  A step touches ~2 GB of weights, gradients and optimizer state, far
more than the 126 MB L2, so no flush is needed between steps.  The
end-to-end figure runs the same K steps through ``DDPTrainer.step_host``:
H2D copy of the step's tokens from pinned memory, the step, and a D2H read
of the loss, timed on the host between synchronized points (max over ranks).

The repo arm also times, on the same box and in the same process, two
comparison arms (``--no-arms`` skips them) and prints them as extra keys:

* ``nccl_fp32``: the same model, optimizer and DDP settings with DDP's own
  uncompressed NCCL fp32 all-reduce and AdamW after backward (the plain
  baseline);
* ``hook_on_reference_model``: this framework's fused hook on exactly the
  reference arm's setup (stock ``transformers`` model, foreach AdamW,
  default DDP arguments), so its ratio to the reference arm isolates the
  hook from the model and optimizer.

The product arm applies AdamW per bucket from the hook (``--overlap-opt``)
and caps the exchange grid of buckets that overlap backward
(``--inflight-ctas``).  ``--timeline FILE`` records one more step's
per-bucket device timeline on every rank (``utils.timeline``).

Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import sys

import torch
import torch.distributed as dist

METRIC = "GPT-2 DDP tokens/s + compressed-allreduce GB/s at 1–8 B200; compression ratio"
ROOT = os.path.dirname(os.path.abspath(__file__))


def parse():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--hook", choices=["fused", "nccl", "compat"], default="fused")
    ap.add_argument("--mode", choices=["int4", "int8", "topk"], default="int4")
    ap.add_argument("--topk", type=float, default=0.05, help="keep fraction for --mode topk")
    ap.add_argument("--variant", default="auto", choices=["auto", "oneshot", "twoshot"])
    ap.add_argument("--model", choices=["gpt2", "llama"], default="gpt2")
    ap.add_argument("--micro-batch", type=int, default=None)
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--clock-period-ms", type=int, default=100,
                    help="nvidia-smi sampling period (the samples of the timed region are kept)")
    ap.add_argument("--max-ctas", type=int, default=0)
    ap.add_argument("--momentum", choices=["auto", "on", "off"], default="auto",
                    help="EMA predictor in the hook (auto: on for int4/int8, off for top-k, which uses error feedback)")
    ap.add_argument("--overlap-opt", choices=["on", "off"], default="on",
                    help="fused hook: apply AdamW per bucket from the hook, overlapping backward")
    ap.add_argument("--opt-in-kernel", choices=["on", "off"], default="on",
                    help="with --overlap-opt: AdamW inside the exchange kernel (fp32 parameters)")
    ap.add_argument("--inflight-ctas", type=int, default=0,
                    help="grid cap of exchange kernels that overlap backward (0: the whole grid)")
    ap.add_argument("--stream-priority", type=int, default=-1, help="hook stream priority (-1 high, 0 normal)")
    ap.add_argument("--l2-keep-mb", type=float, default=0.0,
                    help="predictor MB an exchange kernel keeps in L2 between its phases (0: no L2 policy, the "
                         "default: the kept lines cost the concurrent backward more than they save)")
    ap.add_argument("--no-arms", action="store_true", help="skip the same-box NCCL and same-model comparison arms")
    ap.add_argument("--bucket-mb", type=float, default=25.0,
                    help="DDP bucket cap in MB for every arm (GPT-2's workload fixes 25)")
    ap.add_argument("--timeline", default="", help="write one step's per-bucket device timeline (JSON) here")
    return ap.parse_args()


def visible_gpu_indices(n: int) -> list[int] | None:
    v = os.environ.get("CUDA_VISIBLE_DEVICES")
    if v:
        parts = [p.strip() for p in v.split(",") if p.strip()]
        if all(p.isdigit() for p in parts):
            return [int(p) for p in parts[:n]]
        return None
    return list(range(n))


def make_batches(vocab: int, mb: int, seq: int, count: int, seed: int, device) -> list[tuple]:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = []
    for _ in range(count):
        t = torch.randint(0, vocab, (mb, seq + 1), generator=g, device=device)
        out.append((t[:, :-1].contiguous(), t[:, 1:].contiguous()))
    return out


class _HFLoss(torch.nn.Module):
    """forward(x, y) -> loss adapter around a transformers causal LM."""

    def __init__(self, m):
        super().__init__()
        self.m = m

    def forward(self, x, y):
        logits = self.m(input_ids=x).logits
        return torch.nn.functional.cross_entropy(logits.view(-1, logits.size(-1)).float(), y.reshape(-1))


def build_hf_model(args, device, tiny: bool = False):
    """The stock ``transformers`` model of the workload's family (the
    reference ships no GPT-2 or Llama model): GPT-2 small (fp32 weights, bf16
    autocast) or the Llama-style 1.1B (bf16 weights), each wrapped as
    forward(x, y) -> loss.  Returns (module, autocast)."""
    if args.model == "gpt2":
        from transformers import GPT2Config, GPT2LMHeadModel  # noqa: E402

        dims = dict(vocab_size=512, n_positions=64, n_embd=64, n_layer=2, n_head=4, n_inner=256) if tiny else \
            dict(vocab_size=50257, n_positions=1024, n_embd=768, n_layer=12, n_head=12, n_inner=3072)
        cfg = GPT2Config(**dims, resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0, initializer_range=0.02)
        cfg._attn_implementation = "sdpa"
        with torch.device(device):  # initialised on the device: every rank builds its copy in parallel
            model = _HFLoss(GPT2LMHeadModel(cfg))
        autocast = True
    else:
        from transformers import LlamaConfig as HFLlamaConfig  # noqa: E402
        from transformers import LlamaForCausalLM  # noqa: E402

        from mini_nangila_b200.models import LlamaConfig

        c = LlamaConfig.tiny() if tiny else LlamaConfig.b1_1()
        cfg = HFLlamaConfig(vocab_size=c.vocab_size, hidden_size=c.d_model, intermediate_size=c.d_ff,
                            num_hidden_layers=c.n_layer, num_attention_heads=c.n_head,
                            num_key_value_heads=c.n_kv_head, max_position_embeddings=c.max_seq,
                            rms_norm_eps=c.eps, rope_theta=c.rope_theta, initializer_range=c.init_std,
                            tie_word_embeddings=False)
        cfg._attn_implementation = "sdpa"
        with torch.device(device):
            model = _HFLoss(LlamaForCausalLM(cfg)).to(dtype=torch.bfloat16)
        autocast = False
    return model, autocast


def build_reference(args, device, tiny: bool = False):
    """Reference arm: the unmodified nangila_ddp hook from baseline/_ref on
    the stock model of ``build_hf_model``: GPT-2 small with the INT4 + EMA
    hook, or the Llama-style 1.1B with the hook in top-k mode.  ``tiny``
    swaps in small models of the same families (CPU tests of this arm)."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "nangila_ddp")):
        return None, "baseline/_ref/nangila_ddp is not installed", ""
    sys.path.insert(0, ref)
    from nangila_ddp import register_nangila_hook as ref_register  # noqa: E402

    model, autocast = build_hf_model(args, device, tiny)
    ddp = torch.nn.parallel.DistributedDataParallel(
        model, device_ids=[device.index] if device.type == "cuda" else None, bucket_cap_mb=args.bucket_mb)
    topk = args.topk if args.mode == "topk" else 0.0
    momentum = args.momentum == "on" or (args.momentum == "auto" and args.mode != "topk")
    # Same call the reference's trainer makes (train_nano.py:133-143)
    ref_register(ddp, beta=0.9, bits=4, stochastic=True, use_fp16_transport=False, use_momentum=momentum,
                 topk_percent=topk)
    opt = torch.optim.AdamW(ddp.parameters(), lr=6e-4)

    def step(x, y):
        with torch.autocast(device.type, dtype=torch.bfloat16, enabled=autocast):
            loss = ddp(x, y)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        return loss.detach()

    name = "reference-nangila_ddp-int4" + ("-ema" if momentum else "") + (f"-topk{topk:g}" if topk else "")
    return step, None, name


def build_hook_on_reference_model(args, device, tiny: bool = False):
    """This framework's fused hook on exactly the reference arm's setup:
    the same stock model, default DDP arguments and foreach AdamW, with the
    hook's mode set as the reference arm sets its own.  Returns (step, hook
    state, name)."""
    from mini_nangila_b200.parallel import register_nangila_hook

    model, autocast = build_hf_model(args, device, tiny)
    ddp = torch.nn.parallel.DistributedDataParallel(
        model, device_ids=[device.index] if device.type == "cuda" else None, bucket_cap_mb=args.bucket_mb)
    topk = args.topk if args.mode == "topk" else 0.0
    momentum = args.momentum == "on" or (args.momentum == "auto" and args.mode != "topk")
    hs = register_nangila_hook(ddp, beta=0.9, bits=4, stochastic=True, use_momentum=momentum, topk_percent=topk,
                               seed=12345, error_feedback=True, variant=args.variant,
                               impl="fused" if device.type == "cuda" else "host")
    opt = torch.optim.AdamW(ddp.parameters(), lr=6e-4)

    def step(x, y):
        with torch.autocast(device.type, dtype=torch.bfloat16, enabled=autocast):
            loss = ddp(x, y)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        return loss.detach()

    name = ("fused-topk" if topk else "fused-int4") + ("-ema" if momentum else "") + "-ef" + \
        (f"-keep{topk:g}" if topk else "")
    return step, hs, name


def time_steps(step_fn, batches, warmup: int, steps: int, device) -> float:
    """Milliseconds for ``steps`` steps after ``warmup`` (CUDA events, max over ranks)."""
    from mini_nangila_b200.utils import barrier_sync, max_over_ranks

    for i in range(warmup):
        step_fn(*batches[i % len(batches)])
    barrier_sync(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(steps):
        step_fn(*batches[i % len(batches)])
    e.record()
    barrier_sync(device)
    return max_over_ranks(s.elapsed_time(e), device)


def comparison_arms(args, device, world: int, mb: int, seq: int, batches, mcfg) -> dict:
    """Time the same-box NCCL fp32 arm and the hook-on-reference-model arm."""
    import gc

    from mini_nangila_b200.models import GPT2, Llama
    from mini_nangila_b200.train import DDPTrainer

    out = {}
    tokens = world * mb * seq * args.steps
    # plain NCCL fp32: same model class, optimizer and DDP settings as the product arm
    with torch.device(device):
        model = GPT2(mcfg) if args.model == "gpt2" else Llama(mcfg).to(torch.bfloat16)
    tr = DDPTrainer(model, lr=6e-4, hook="nccl", bucket_cap_mb=args.bucket_mb,
                    autocast_dtype=torch.bfloat16 if args.model == "gpt2" else None, device=device)
    ms = time_steps(tr.step, batches, args.warmup, args.steps, device)
    out["nccl_fp32"] = {"value": tokens / (ms / 1000.0), "ms_per_step": ms / args.steps,
                        "hook": "DDP built-in NCCL fp32 all-reduce, AdamW (fused) after backward"}
    del tr, model
    gc.collect()
    torch.cuda.empty_cache()
    try:
        step, hs, name = build_hook_on_reference_model(args, device)
    except ImportError as e:  # transformers missing
        out["hook_on_reference_model"] = {"unavailable": str(e)}
        return out
    ms = time_steps(step, batches, args.warmup, args.steps, device)
    if hs is not None and getattr(hs, "comm", None) is not None:
        hs.comm.check()
    out["hook_on_reference_model"] = {
        "value": tokens / (ms / 1000.0), "ms_per_step": ms / args.steps, "hook": name,
        "model": "transformers " + ("GPT2LMHeadModel" if args.model == "gpt2" else "LlamaForCausalLM"),
        "optimizer": "AdamW (foreach) after backward", "ddp": f"default arguments, bucket_cap_mb {args.bucket_mb:g}"}
    if hs is not None and getattr(hs, "comm", None) is not None:
        hs.comm.close()
    del step, hs
    gc.collect()
    torch.cuda.empty_cache()
    return out


def main():
    args = parse()
    from mini_nangila_b200.train import DDPTrainer, init_distributed
    from mini_nangila_b200.utils import ClockSampler, barrier_sync, max_over_ranks
    from mini_nangila_b200.workloads import GPT2SmallDDP, Llama1BTopK

    rank, world, local = init_distributed("nccl", timeout_s=300)
    device = torch.device("cuda", local)
    torch.manual_seed(1234)
    torch.backends.cuda.matmul.allow_tf32 = True
    if args.model == "gpt2":
        from mini_nangila_b200.models import GPT2, GPT2Config

        w = GPT2SmallDDP()
        mcfg = GPT2Config.small()
        vocab, mb, seq = mcfg.vocab_size, args.micro_batch or w.micro_batch, args.seq or w.seq
        model_name = "gpt2-small-124M"
    else:
        from mini_nangila_b200.models import Llama, LlamaConfig

        w = Llama1BTopK()
        mcfg = LlamaConfig.b1_1()
        vocab, mb, seq = mcfg.vocab_size, args.micro_batch or w.micro_batch, args.seq or w.seq
        model_name = "llama-1.1B"

    quiet = contextlib.redirect_stdout(open(os.devnull, "w")) if args.impl == "reference" else contextlib.nullcontext()
    trainer = None
    if args.impl == "reference":
        step_fn, why, hook_name = build_reference(args, device)
        if step_fn is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": why}))
            dist.destroy_process_group()
            return
    else:
        with torch.device(device):  # initialised on the device (fast for the 1.1B model)
            model = GPT2(mcfg) if args.model == "gpt2" else Llama(mcfg)
        if args.model == "llama":
            model = model.to(torch.bfloat16)
        hk = None
        if args.hook in ("fused", "compat"):
            momentum = args.momentum == "on" or (args.momentum == "auto" and args.mode != "topk")
            hk = dict(beta=0.9, bits=8 if args.mode == "int8" else 4, stochastic=True, use_momentum=momentum,
                      topk_percent=args.topk if args.mode == "topk" else 0.0, seed=12345,
                      error_feedback=True, variant=args.variant, max_ctas=args.max_ctas)
            if args.hook == "fused":
                hk.update(inflight_ctas=args.inflight_ctas, stream_priority=args.stream_priority,
                          l2_keep_mb=args.l2_keep_mb)
        overlap = args.hook == "fused" and args.overlap_opt == "on"
        trainer = DDPTrainer(model, lr=6e-4, hook=args.hook, hook_kwargs=hk, bucket_cap_mb=args.bucket_mb,
                             autocast_dtype=torch.bfloat16 if args.model == "gpt2" else None, device=device,
                             overlap_optimizer=overlap, optimizer_in_kernel=args.opt_in_kernel == "on")
        step_fn = trainer.step
        hook_name = {"fused": f"fused-{args.mode}", "nccl": "nccl-fp32-allreduce", "compat": f"compat-{args.mode}"}[args.hook]
        if args.hook != "nccl":
            hook_name += ("-ema" if momentum else "") + "-ef"
            if args.mode == "topk":
                hook_name += f"-keep{args.topk:g}"

    batches = make_batches(vocab, mb, seq, 4, 1000 + rank, device)
    with quiet:
        # nvidia-smi runs from before the warm-up, so that it is already
        # printing samples when the timed region starts; only the samples
        # of the timed region (begin / end) enter the clock record
        sampler = (ClockSampler(visible_gpu_indices(world), period_ms=args.clock_period_ms).start()
                   if (rank == 0 and not args.no_clocks) else None)
        for i in range(args.warmup):
            step_fn(*batches[i % len(batches)])
        barrier_sync(device)
        launches0 = trainer.kernel_launches() if trainer else 0
        barrier_sync(device)
        if sampler:
            sampler.begin()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for i in range(args.steps):
            step_fn(*batches[i % len(batches)])
        e.record()
        barrier_sync(device)
        if sampler:
            sampler.end()
        ms_local = s.elapsed_time(e)
        launches = (trainer.kernel_launches() - launches0) if trainer else 0
        clocks = sampler.stop() if sampler else None
        ms = max_over_ranks(ms_local, device)
        e2e = None
        if not args.no_e2e:
            host_batches = [(x.cpu().pin_memory(), y.cpu().pin_memory()) for x, y in batches]
            barrier_sync(device)
            import time

            t0 = time.perf_counter()
            seq_batches = [host_batches[i % len(host_batches)] for i in range(args.steps)]
            if trainer is not None:
                # every step: pinned H2D copy of its batch and a D2H read of its
                # loss, read one step late so the host does not wait in between
                losses = trainer.train_steps(seq_batches)
            else:
                losses, pending = [], None
                for x, y in seq_batches:
                    loss = step_fn(x.to(device, non_blocking=True), y.to(device, non_blocking=True))
                    out = torch.empty((), dtype=loss.dtype, pin_memory=True)
                    out.copy_(loss, non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record()
                    if pending is not None:
                        pending[1].synchronize()
                        losses.append(float(pending[0]))
                    pending = (out, ev)
                pending[1].synchronize()
                losses.append(float(pending[0]))
            assert len(losses) == args.steps
            barrier_sync(device)
            e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1000.0, device)
            xb, yb = host_batches[0]
            e2e = {
                "value": world * mb * seq * args.steps / (e2e_ms / 1000.0),
                "unit": "tokens/s",
                "ms_per_step": e2e_ms / args.steps,
                "h2d_bytes_per_step": int(xb.numel() * xb.element_size() + yb.numel() * yb.element_size()),
                "d2h_bytes_per_step": 4,
            }
    timeline = None
    if args.timeline and trainer is not None:
        from mini_nangila_b200.utils.timeline import summarize

        step_fn(*batches[0])
        trainer.timeline_next_step()
        step_fn(*batches[1])
        tl = trainer.timeline.collect()
        per_rank = [None] * world
        dist.all_gather_object(per_rank, {"rank": rank, "summary": summarize(tl), "timeline": tl})
        timeline = per_rank
    hs = trainer.hook_state if trainer else None
    if trainer is not None and hs is not None and getattr(hs, "comm", None) is not None:
        hs.comm.check()
    tokens = world * mb * seq * args.steps
    value = tokens / (ms / 1000.0)
    arms = None
    if trainer is not None and not args.no_arms:
        ratio_fields = (hs.compression_ratio() if hs is not None and hs.raw_bytes else None,
                        hs.last_variant if hs is not None else None,
                        (hs.comm.twoshot_min_bytes if hs is not None and getattr(hs, "comm", None) is not None
                         and hs.comm.world > 1 else None))
        if hs is not None and getattr(hs, "comm", None) is not None:
            hs.comm.close()
        trainer = None
        import gc

        gc.collect()
        torch.cuda.empty_cache()
        arms = comparison_arms(args, device, world, mb, seq, batches, mcfg)
    else:
        ratio_fields = (hs.compression_ratio() if hs is not None and hs.raw_bytes else None,
                        hs.last_variant if hs is not None else None,
                        (hs.comm.twoshot_min_bytes if hs is not None and getattr(hs, "comm", None) is not None
                         and hs.comm.world > 1 else None))
    if rank == 0:
        out = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (uniform random tokens from a seed; random-init weights)",
            "config": {
                "model": model_name,
                "global_batch": world * mb,
                "micro_batch": mb,
                "seq_len": seq,
                "parallelism": f"dp{world}",
                "hook": hook_name,
                "bucket_mb": args.bucket_mb,
                "optimizer": "AdamW lr 6e-4",
                "precision": "fp32 master weights, bf16 autocast" if args.model == "gpt2" else "bf16",
                "l2": "no flush: each step reads/writes ~2 GB of weights, grads and optimizer state (> 126 MB L2)",
            },
            "gpu_launches": launches,
        }
        if args.impl == "reference":
            out["impl"] = "reference"
        ratio, variant, twoshot_from = ratio_fields
        if ratio is not None:
            out["compression_ratio"] = ratio
            out["config"]["variant"] = variant
            if twoshot_from is not None:
                out["config"]["twoshot_from_mb"] = None if twoshot_from >= (1 << 60) else twoshot_from / 2 ** 20
        if trainer is not None or arms is not None:
            out["config"]["optimizer_overlap"] = bool(args.hook == "fused" and args.overlap_opt == "on")
            out["config"]["optimizer_in_kernel"] = bool(out["config"]["optimizer_overlap"]
                                                        and args.opt_in_kernel == "on" and args.model == "gpt2")
        if clocks is not None:
            out["clocks"] = clocks
        if e2e is not None:
            out["e2e"] = e2e
        if arms is not None:
            out.update(arms)
            if "value" in arms.get("nccl_fp32", {}):
                out["vs_nccl_fp32_same_box"] = value / arms["nccl_fp32"]["value"]
        if timeline is not None:
            with open(args.timeline, "w") as fh:
                json.dump(timeline, fh)
            out["timeline"] = {"file": args.timeline, "rank0": timeline[0]["summary"]}
        print(json.dumps(out), flush=True)
    if trainer is not None and hs is not None and getattr(hs, "comm", None) is not None:
        hs.comm.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
