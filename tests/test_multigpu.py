"""Fused all-reduce across real ranks (one process per GPU over NCCL):
every rank's output must equal the C++ oracle bit for bit, which also makes
the predictor state identical on all ranks."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _data(n, seed, scale=1e-3):
    g = np.random.default_rng(seed)
    x = (g.standard_normal(n) * scale).astype(np.float32)
    x[g.random(n) < 0.3] *= 0.01
    return x


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cases, errfile):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from mini_nangila_b200 import _ext
        from mini_nangila_b200.parallel.fused import FusedAllReduce, topology

        h = _ext.host()
        nmax = max(c[0] for c in cases)
        comm = FusedAllReduce(nmax, device=dev, topk_k=26, timeout_s=20.0)
        inv = float(np.float32(1.0) / np.float32(world))
        for (n, mode, variant, drop) in cases:
            k = 26
            topo = topology(n, drop, 8, 3)
            bits = 8 if mode == "int8" else 4
            pred = _data(n, 5)
            efs = [_data(n, 900 + r, 1e-4) for r in range(world)]
            pred_d = torch.from_numpy(pred.copy()).to(dev)
            ef_d = torch.from_numpy(efs[rank].copy()).to(dev)
            for step in range(3):
                gs = [_data(n, 100 * step + r) for r in range(world)]
                gd = torch.from_numpy(gs[rank].copy()).to(dev)
                comm.allreduce_(gd, pred_d, ef_d, mode=mode, k=k, variant=variant, seed=11, bucket=3, step=step,
                                beta=0.9, first=(step == 0), topo_drop=drop, topo_seed=8,
                                max_ctas=7 if step == 1 else None)
                if mode == "topk":
                    encs = [h.product_topk_encode(gs[r], pred, efs[r], k, True, topo) for r in range(world)]
                    avg = h.product_topk_reduce([e[0] for e in encs], n, k, pred, inv)
                else:
                    encs = [h.product_encode(gs[r], pred, efs[r], bits, True, True, 11, r, 3, step, topo)
                            for r in range(world)]
                    fn = h.product_reduce_twoshot if variant == "twoshot" else h.product_reduce
                    avg = fn([e[0] for e in encs], n, bits, pred, inv)
                efs = [e[1] for e in encs]
                pred = h.product_ema(pred, avg, 0.9, step == 0)
                got = gd.cpu().numpy()
                if not np.array_equal(got.view(np.uint32), np.asarray(avg, np.float32).view(np.uint32)):
                    bad = int(np.sum(got.view(np.uint32) != np.asarray(avg, np.float32).view(np.uint32)))
                    raise AssertionError(f"rank {rank} {mode}/{variant} n={n} step {step}: {bad} elements differ")
                assert np.array_equal(pred_d.cpu().numpy().view(np.uint32), pred.view(np.uint32))
                assert np.array_equal(ef_d.cpu().numpy().view(np.uint32), efs[rank].view(np.uint32))
        comm.check()
        comm.close()
    except Exception as e:  # report to the parent
        with open(errfile, "a") as fh:
            fh.write(f"{type(e).__name__}: {e}\n")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_allreduce_matches_oracle_across_ranks(world, tmp_path):
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cases = []
    for n in (1000, 70001):
        for mode in ("int4", "int8", "topk"):
            for variant in (("oneshot", "twoshot") if mode != "topk" else ("oneshot",)):
                cases.append((n, mode, variant, 0.0))
                if n > 1000:
                    cases.append((n, mode, variant, 0.3))
    err = str(tmp_path / "err.txt")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_worker, args=(world, _port(), cases, err), nprocs=world, join=True, start_method="spawn")
    assert not os.path.exists(err) or open(err).read() == ""


def _leave_worker(rank, world, port, errfile, outdir):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from mini_nangila_b200.models import GPT2, GPT2Config
        from mini_nangila_b200.parallel.fused import CommError
        from mini_nangila_b200.train import DDPTrainer

        torch.manual_seed(0)
        cfg = GPT2Config.tiny()
        tr = DDPTrainer(GPT2(cfg), hook="fused", hook_kwargs=dict(use_momentum=True, seed=5, timeout_s=5.0),
                        device=dev, bucket_cap_mb=0.05, monitor=True)
        tr.monitor.timeout_s = 10.0
        g = torch.Generator().manual_seed(100 + rank)
        msg = "none"
        for step in range(3):
            if rank == 1 and step == 2:
                torch.cuda.synchronize()  # none of this rank's kernels in flight
                ok = tr.monitor.leave("test leave")
                open(os.path.join(outdir, "f1.txt"), "w").write(f"left ack={ok}")
                return
            t = torch.randint(0, cfg.vocab_size, (2, 17), generator=g).to(dev)
            try:
                tr.step(t[:, :-1], t[:, 1:])
                torch.cuda.synchronize()
            except CommError as e:
                msg = str(e)
                break
        tr.hook_state.comm.check()  # no launch gave up
        open(os.path.join(outdir, f"f{rank}.txt"), "w").write(msg)
    except Exception as e:
        with open(errfile, "a") as fh:
            fh.write(f"{type(e).__name__}: {e}\n")
        raise
    finally:
        dist.destroy_process_group()


def test_rank_leaving_between_steps_fused(tmp_path):
    """Two ranks with the fused hook: rank 1 leaves between steps; rank 0
    notices in the store before launching, unmaps rank 1's region and
    acknowledges, rank 1 then frees it.  NVLS is off; nothing waits on the
    departed rank on the device."""
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    err = str(tmp_path / "err.txt")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.start_processes(_leave_worker, args=(2, _port(), err, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    assert not os.path.exists(err) or open(err).read() == ""
    assert "rank 1 left (test leave)" in (tmp_path / "f0.txt").read_text()
    assert (tmp_path / "f1.txt").read_text() == "left ack=True"
