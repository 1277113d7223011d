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
def test_adamw_inside_the_exchange_kernel_tracks_adamw_after_backward():
    """World 1 on a GPU: AdamW applied by the fused kernel as it writes each
    averaged gradient stays within rounding of PyTorch's AdamW after
    backward over several steps, moves the weights, and keeps the step
    counters and moments in the optimizer's own state."""
    import torch.distributed as dist

    from mini_nangila_b200.models import GPT2, GPT2Config
    from mini_nangila_b200.train import DDPTrainer, init_distributed

    init_distributed("nccl")
    try:
        dev = torch.device("cuda", 0)
        cfg = GPT2Config(vocab_size=1024, n_positions=128, n_layer=2, n_head=4, n_embd=128, n_inner=512)
        res, init = {}, None
        for in_kernel in (False, True):
            torch.manual_seed(0)
            tr = DDPTrainer(GPT2(cfg), hook="fused", device=dev, bucket_cap_mb=0.25,
                            hook_kwargs=dict(use_momentum=True), overlap_optimizer=in_kernel,
                            optimizer_in_kernel=in_kernel)
            init = [p.detach().clone() for p in tr.model.parameters()]
            g = torch.Generator(device=dev).manual_seed(1)
            for _ in range(4):
                t = torch.randint(0, cfg.vocab_size, (2, 65), generator=g, device=dev)
                tr.step(t[:, :-1].contiguous(), t[:, 1:].contiguous())
            torch.cuda.synchronize()
            tr.hook_state.comm.check()
            res[in_kernel] = ([p.detach().clone() for p in tr.model.parameters()],
                              [tr.opt.state[p]["step"].item() for p in tr.model.parameters()])
            tr.hook_state.comm.close()
        for a, b, p0 in zip(res[False][0], res[True][0], init):
            assert torch.allclose(a, b, rtol=0, atol=2e-6), float((a - b).abs().max())
            assert float((b - p0).abs().max()) > 1e-5
        assert res[True][1] == res[False][1] == [4.0] * len(res[True][1])
    finally:
        dist.destroy_process_group()
