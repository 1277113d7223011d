"""AdamW applied per bucket from the gradient hook (``DDPTrainer(
overlap_optimizer=True)``) against the usual AdamW step after backward, on
two gloo ranks (CPU, host hook): the parameters and the optimizer state must
be bit-identical after several steps, on every rank."""
import os
import socket

import pytest
import torch


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, errfile, outdir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mini_nangila_b200.models import GPT2, GPT2Config
        from mini_nangila_b200.train import DDPTrainer

        torch.set_num_threads(1)
        cfg = GPT2Config.tiny()
        res = {}
        for overlap in (False, True):
            torch.manual_seed(0)
            tr = DDPTrainer(GPT2(cfg), hook="host", device=torch.device("cpu"), bucket_cap_mb=0.05, lr=1e-3,
                            hook_kwargs=dict(use_momentum=True, seed=3), overlap_optimizer=overlap)
            if not overlap:
                # the same fused AdamW kernel, applied once after backward
                tr.opt = torch.optim.AdamW(tr.ddp.parameters(), lr=1e-3, fused=True)
            g = torch.Generator().manual_seed(10 + rank)
            for _ in range(4):
                t = torch.randint(0, cfg.vocab_size, (2, 17), generator=g)
                tr.step(t[:, :-1].contiguous(), t[:, 1:].contiguous())
            params = [p.detach().clone() for p in tr.model.parameters()]
            states = [{k: v.clone() for k, v in tr.opt.state[p].items()} for p in tr.model.parameters()]
            res[overlap] = (params, states)
        for a, b in zip(res[False][0], res[True][0]):
            assert torch.equal(a, b), "parameters differ"
        for sa, sb in zip(res[False][1], res[True][1]):
            assert sa.keys() == sb.keys()
            for k in sa:
                assert torch.equal(sa[k].float(), sb[k].float()), f"optimizer state {k} differs"
        torch.save(res[True][0], os.path.join(outdir, f"p{rank}.pt"))
    except Exception as e:
        with open(errfile, "a") as fh:
            fh.write(f"rank {rank}: {type(e).__name__}: {e}\n")
        raise
    finally:
        dist.destroy_process_group()


def test_bucket_adamw_matches_step_after_backward(tmp_path):
    import torch.multiprocessing as mp

    if not hasattr(torch, "_fused_adamw_"):
        pytest.skip("no fused AdamW op")
    err = str(tmp_path / "err.txt")
    mp.start_processes(_worker, args=(2, _port(), err, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert not os.path.exists(err) or open(err).read() == "", open(err).read()
    p0 = torch.load(tmp_path / "p0.pt")
    p1 = torch.load(tmp_path / "p1.pt")
    assert all(torch.equal(a, b) for a, b in zip(p0, p1)), "ranks disagree"


@pytest.mark.gpu
def test_bucket_adamw_fused_hook_matches_step_after_backward():
    """World 1 on a GPU: the fused hook with AdamW applied per bucket on the
    hook stream gives the parameters of AdamW after backward, bit for bit,
    and a recorded timeline names every bucket."""
    import torch.distributed as dist

    from mini_nangila_b200.models import GPT2, GPT2Config
    from mini_nangila_b200.train import DDPTrainer, init_distributed
    from mini_nangila_b200.utils.timeline import summarize

    init_distributed("nccl")
    try:
        dev = torch.device("cuda", 0)
        cfg = GPT2Config(vocab_size=1024, n_positions=128, n_layer=2, n_head=4, n_embd=128, n_inner=512)
        res = {}
        for overlap in (False, True):
            torch.manual_seed(0)
            tr = DDPTrainer(GPT2(cfg), hook="fused", device=dev, bucket_cap_mb=0.25,
                            hook_kwargs=dict(use_momentum=True), overlap_optimizer=overlap,
                            optimizer_in_kernel=False)
            g = torch.Generator(device=dev).manual_seed(1)
            for i in range(4):
                t = torch.randint(0, cfg.vocab_size, (2, 65), generator=g, device=dev)
                if overlap and i == 3:
                    tr.timeline_next_step()
                tr.step(t[:, :-1].contiguous(), t[:, 1:].contiguous())
            torch.cuda.synchronize()
            tr.hook_state.comm.check()
            res[overlap] = [p.detach().clone() for p in tr.model.parameters()]
            if overlap:
                tl = tr.timeline.collect()
                s = summarize(tl)
                assert s["buckets"] >= 2 and all("opt_end" in b for b in tl["buckets"])
                assert s["exposed_tail_ms"] >= 0.0
            tr.hook_state.comm.close()
        for a, b in zip(res[False], res[True]):
            assert torch.equal(a, b)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["int4", "topk"])
def test_adamw_inside_the_exchange_kernel_tracks_adamw_after_backward(mode):
    """World 1 on a GPU: AdamW applied by the fused kernel as it writes each
    averaged gradient.  Every step is checked on its own: from the weights
    and moments before the step and the step's averaged gradient (left in
    ``p.grad``), a float64 AdamW gives the weights and moments after it, and
    the kernel's are within fp32 rounding of those.  (Runs that differ only
    in the optimizer's rounding are not compared over several steps: the
    stochastic INT4 codes of the next step turn a one-ulp weight difference
    into a different rounding draw.)  Step counters stay in the optimizer's
    own state.  Top-k buckets have no in-kernel optimizer: with
    ``optimizer_in_kernel`` they take the per-bucket update instead."""
    import math

    import numpy as np
    import torch.distributed as dist

    from mini_nangila_b200.models import GPT2, GPT2Config
    from mini_nangila_b200.parallel.emulate import adamw_reference
    from mini_nangila_b200.train import DDPTrainer, init_distributed

    init_distributed("nccl")
    try:
        dev = torch.device("cuda", 0)
        cfg = GPT2Config(vocab_size=1024, n_positions=128, n_layer=2, n_head=4, n_embd=128, n_inner=512)
        torch.manual_seed(0)
        hk = dict(use_momentum=True) if mode == "int4" else dict(use_momentum=False, topk_percent=0.05)
        tr = DDPTrainer(GPT2(cfg), hook="fused", device=dev, bucket_cap_mb=0.25, hook_kwargs=hk,
                        overlap_optimizer=True, optimizer_in_kernel=True)
        params = list(tr.model.parameters())
        grp = tr.opt.param_groups[0]
        b1, b2 = grp["betas"]
        lr, wd, eps = grp["lr"], grp["weight_decay"], grp["eps"]
        ulp = 2.0 ** -24
        g = torch.Generator(device=dev).manual_seed(1)
        for t in range(1, 5):
            before = []
            for p in params:
                st = tr.opt.state[p]
                m0 = st["exp_avg"].double().cpu().numpy() if "exp_avg" in st else np.zeros(p.numel())
                v0 = st["exp_avg_sq"].double().cpu().numpy() if "exp_avg_sq" in st else np.zeros(p.numel())
                before.append((p.detach().double().cpu().numpy().ravel(), m0.ravel(), v0.ravel()))
            x = torch.randint(0, cfg.vocab_size, (2, 65), generator=g, device=dev)
            tr.step(x[:, :-1].contiguous(), x[:, 1:].contiguous())
            torch.cuda.synchronize()
            tr.hook_state.comm.check()
            hyper = [b1, b2, eps, 1.0 - lr * wd, lr / (1.0 - b1 ** t), 1.0 / math.sqrt(1.0 - b2 ** t)]
            moved = 0.0
            for p, (p0, m0, v0) in zip(params, before):
                st = tr.opt.state[p]
                assert st["step"].item() == float(t)
                gg = p.grad.detach().double().cpu().numpy().ravel()
                rp, rm, rv = adamw_reference(p0, m0, v0, gg, hyper)
                kp = p.detach().double().cpu().numpy().ravel()
                km = st["exp_avg"].double().cpu().numpy().ravel()
                kv = st["exp_avg_sq"].double().cpu().numpy().ravel()
                assert np.all(np.abs(km - rm) <= 8 * ulp * (b1 * np.abs(m0) + (1 - b1) * np.abs(gg)) + 1e-30)
                assert np.all(np.abs(kv - rv) <= 8 * ulp * (b2 * v0 + (1 - b2) * gg * gg) + 1e-36)
                if mode == "int4":
                    # the weight, from the kernel's own moments: a few ulps of
                    # the weight and of the update (top-k buckets take
                    # PyTorch's fused AdamW, whose rounding differs; its bit
                    # identity is checked above)
                    upd = hyper[4] * km / (np.sqrt(kv) * hyper[5] + eps)
                    rp2 = p0 * hyper[3] - upd
                    assert np.all(np.abs(kp - rp2) <= 4 * ulp * np.abs(p0) + 8 * ulp * np.abs(upd) + 1e-12), \
                        float(np.abs(kp - rp2).max())
                assert np.allclose(kp, rp, rtol=0, atol=lr)  # and near the float64 recursion
                moved = max(moved, float(np.abs(kp - p0).max()))
            assert moved > 1e-4
        tr.hook_state.comm.close()
    finally:
        dist.destroy_process_group()
