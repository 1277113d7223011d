"""DDP comm hooks on CPU gloo process groups (world 2): the host
implementation of the product format gives bit-identical averages and
predictor states on every rank and matches the oracle; the compat hook
reproduces the reference's algorithm; a rank that fails is detected by the
others through the process-group timeout (no GPU involved)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=60):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _train_worker(rank, world, port, impl, mode, outdir):
    dist = _init(rank, world, port)
    try:
        from mini_nangila_b200.models import GPT2, GPT2Config
        from mini_nangila_b200.train import DDPTrainer

        torch.manual_seed(0)
        cfg = GPT2Config.tiny()
        topo = mode.endswith("+topo")
        mode = mode.split("+")[0]
        kw = dict(use_momentum=True, bits=8 if mode == "int8" else 4,
                  topk_percent=0.1 if mode == "topk" else 0.0, seed=5, topo_drop_percent=0.3 if topo else 0.0)
        if impl == "host":
            kw["error_feedback"] = True
        tr = DDPTrainer(GPT2(cfg), hook=impl, hook_kwargs=kw, device=torch.device("cpu"), bucket_cap_mb=0.05)
        g = torch.Generator().manual_seed(100 + rank)
        losses, grads = [], []
        for _ in range(3):
            t = torch.randint(0, cfg.vocab_size, (2, 17), generator=g)
            losses.append(float(tr.step(t[:, :-1], t[:, 1:])))
            # the gradients are views of the buckets: the hook's averages
            grads.append(torch.cat([p.grad.reshape(-1) for p in tr.model.parameters()]).clone())
        params = torch.cat([p.detach().reshape(-1) for p in tr.model.parameters()])
        hs = tr.hook_state
        preds = [st.pred.clone() for _, st in sorted(hs.buckets.items())] if impl == "host" else \
            [v.clone() for _, v in sorted(hs.compat_states.items())]
        torch.save({"params": params, "grads": grads, "preds": preds, "losses": losses, "ratio": hs.compression_ratio()},
                   os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("impl,mode", [("host", "int4"), ("host", "int8"), ("host", "topk"), ("host", "int4+topo"),
                                       ("host", "topk+topo"), ("compat", "int4"), ("compat", "topk"),
                                       ("compat", "int4+topo")])
def test_ddp_hook_ranks_stay_identical(impl, mode, tmp_path):
    mp.start_processes(_train_worker, args=(2, _port(), impl, mode, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    r0, r1 = torch.load(tmp_path / "r0.pt"), torch.load(tmp_path / "r1.pt")
    # Every rank gets the same averaged gradients and keeps the same
    # predictor state, bit for bit, and (with the trainer's fused AdamW) the
    # same parameters.
    for a, b in zip(r0["grads"], r1["grads"]):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    for a, b in zip(r0["preds"], r1["preds"]):
        assert torch.equal(a, b)
    assert torch.equal(r0["params"].view(torch.int32), r1["params"].view(torch.int32))
    assert r0["ratio"] > 3.0
    assert all(np.isfinite(r0["losses"]))


def _oracle_worker(rank, world, port, outdir):
    dist = _init(rank, world, port)
    try:
        from mini_nangila_b200 import _ext
        from mini_nangila_b200.parallel.hook import HookConfig, NangilaHookState, _host_hook

        class Bucket:
            def __init__(self, t):
                self.t = t

            def buffer(self):
                return self.t

            def index(self):
                return 0

            def parameters(self):
                return []

        hs = NangilaHookState(HookConfig(impl="host", use_momentum=True, seed=9))
        n = 5000
        gs = [np.random.default_rng(50 + r).standard_normal(n).astype(np.float32) * np.float32(1e-3)
              for r in range(world)]
        buf = torch.from_numpy(gs[rank].copy())
        _host_hook(hs, Bucket(buf)).wait()
        h = _ext.host()
        wires = [h.product_encode(gs[r], np.zeros(n, np.float32), np.zeros(n, np.float32), 4, True, True, 9, r, 0,
                                  1)[0] for r in range(world)]
        ref = h.product_reduce(wires, n, 4, np.zeros(n, np.float32), float(np.float32(1) / np.float32(world)))
        np.save(os.path.join(outdir, f"o{rank}.npy"), np.stack([buf.numpy(), ref]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
def test_host_hook_matches_oracle(world, tmp_path):
    mp.start_processes(_oracle_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        got, ref = np.load(tmp_path / f"o{r}.npy")
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("mode", ["int4", "topk+topo"])
def test_ddp_hook_ranks_stay_identical_world3(mode, tmp_path):
    """An odd world size: rank-ordered sums and per-rank noise keys still give
    every rank the same averaged gradients, predictor states and parameters."""
    mp.start_processes(_train_worker, args=(3, _port(), "host", mode, str(tmp_path)), nprocs=3, join=True,
                       start_method="spawn")
    rs = [torch.load(tmp_path / f"r{r}.pt") for r in range(3)]
    for r in rs[1:]:
        assert all(torch.equal(a.view(torch.int32), b.view(torch.int32)) for a, b in zip(rs[0]["grads"], r["grads"]))
        assert all(torch.equal(a, b) for a, b in zip(rs[0]["preds"], r["preds"]))
        assert torch.equal(rs[0]["params"].view(torch.int32), r["params"].view(torch.int32))
    assert all(np.isfinite(rs[0]["losses"]))


def _metrics_worker(rank, world, port, outdir):
    dist = _init(rank, world, port)
    try:
        from mini_nangila_b200.parallel.hook import HookConfig, NangilaHookState, _host_hook

        class Bucket:
            def __init__(self, t):
                self.t = t

            def buffer(self):
                return self.t

            def index(self):
                return 0

            def parameters(self):
                return []

        path = os.path.join(outdir, "metrics.csv")
        hs = NangilaHookState(HookConfig(impl="host", use_momentum=True, seed=9, metrics_path=path))
        n = 3000
        for call in range(2):
            g = np.random.default_rng(10 * call + rank).standard_normal(n).astype(np.float32) * np.float32(1e-3)
            pred = None if call == 0 else hs.buckets[0].pred.numpy().copy()
            _host_hook(hs, Bucket(torch.from_numpy(g.copy()))).wait()
            want = np.abs(g.astype(np.float64) if pred is None else (g - pred).astype(np.float64)).mean()
            np.save(os.path.join(outdir, f"m{rank}_{call}.npy"), np.array([want]))
    finally:
        dist.destroy_process_group()


def test_host_hook_metrics_log_residual_mean_abs(tmp_path):
    """rank 0 writes one reference-layout line per hook call with
    res_mean_abs = mean |g - pred| of its own bucket (comm_hook.py:178)."""
    mp.start_processes(_metrics_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    lines = (tmp_path / "metrics.csv").read_text().splitlines()
    assert len(lines) == 2  # rank 0 only
    for call, line in enumerate(lines):
        kv = line.split(",")
        d = dict(zip(kv[0::2], kv[1::2]))
        assert kv[0::2] == ["ts", "hook_idx", "bucket_elems", "raw_bytes", "comp_bytes", "ratio", "res_mean_abs"]
        assert int(d["hook_idx"]) == call + 1 and int(d["bucket_elems"]) == 3000
        want = float(np.load(tmp_path / f"m0_{call}.npy")[0])
        assert float(d["res_mean_abs"]) == pytest.approx(want, rel=1e-5)


def _dying_worker(rank, world, port, outdir):
    """Rank 1 raises between steps without joining the next collective; rank 0
    must get an error from its next collective (short process-group timeout)
    instead of hanging."""
    import time

    dist = _init(rank, world, port, timeout_s=5)
    if rank == 1:
        dist.barrier()
        raise SystemExit(3)
    dist.barrier()
    t0 = time.time()
    err = ""
    try:
        x = torch.ones(4)
        dist.all_reduce(x)
    except Exception as e:  # noqa: BLE001
        err = type(e).__name__
    with open(os.path.join(outdir, "rank0.txt"), "w") as fh:
        fh.write(f"{err}:{time.time() - t0:.1f}")


def test_dead_rank_detected_by_timeout(tmp_path):
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=_dying_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    for p in ps:
        if p.is_alive():
            p.kill()
    txt = (tmp_path / "rank0.txt").read_text()
    err, dt = txt.split(":")
    assert err != "" and float(dt) < 30.0


def _fault_worker(rank, world, port, outdir, spec):
    os.environ["NGL_FAULT"] = spec
    dist = _init(rank, world, port)
    try:
        from mini_nangila_b200.models import GPT2, GPT2Config
        from mini_nangila_b200.parallel.fused import CommError
        from mini_nangila_b200.train import DDPTrainer

        torch.manual_seed(0)
        cfg = GPT2Config.tiny()
        tr = DDPTrainer(GPT2(cfg), hook="host", hook_kwargs=dict(use_momentum=True, seed=5),
                        device=torch.device("cpu"), bucket_cap_mb=0.05)
        g = torch.Generator().manual_seed(100 + rank)
        msg = "none"
        try:
            for _ in range(3):
                t = torch.randint(0, cfg.vocab_size, (2, 17), generator=g)
                tr.step(t[:, :-1], t[:, 1:])
        except CommError as e:
            msg = str(e)
        except RuntimeError as e:  # DDP wraps exceptions raised inside the hook
            msg = str(e) if "rank 1" in str(e) else "other: " + str(e)[:200]
        (open(os.path.join(outdir, f"f{rank}.txt"), "w")).write(msg)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind,needle", [("corrupt", "checksum"), ("mismatch", "disagree")])
def test_injected_payload_fault_is_detected_on_every_rank(kind, needle, tmp_path):
    """A rank's payload is corrupted (or claims another bucket) on its 3rd
    hook call: every rank detects it from the checksummed header and raises,
    naming the rank; none proceeds with a wrong average."""
    mp.start_processes(_fault_worker, args=(2, _port(), str(tmp_path), f"{kind}:1:3"), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        msg = (tmp_path / f"f{r}.txt").read_text()
        assert "rank 1" in msg and needle in msg, msg


def _plain_worker(rank, world, port, outdir):
    dist = _init(rank, world, port)
    try:
        from mini_nangila_b200.models import GPT2, GPT2Config
        from mini_nangila_b200.train import DDPTrainer

        res = {}
        for variant in ("nccl", None):
            torch.manual_seed(0)
            cfg = GPT2Config.tiny()
            kw = dict(variant="nccl") if variant else None
            tr = DDPTrainer(GPT2(cfg), hook="fused" if variant else "nccl", hook_kwargs=kw,
                            device=torch.device("cpu"), bucket_cap_mb=0.05)
            g = torch.Generator().manual_seed(100 + rank)
            for _ in range(2):
                t = torch.randint(0, cfg.vocab_size, (2, 17), generator=g)
                tr.step(t[:, :-1], t[:, 1:])
            res[str(variant)] = torch.cat([p.detach().reshape(-1) for p in tr.model.parameters()])
        torch.save(res, os.path.join(outdir, f"p{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_nccl_variant_is_the_plain_allreduce(tmp_path):
    """variant="nccl" routes buckets through the uncompressed averaged
    all-reduce: parameters match stock DDP on every rank."""
    mp.start_processes(_plain_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    p0, p1 = torch.load(tmp_path / "p0.pt"), torch.load(tmp_path / "p1.pt")
    assert torch.equal(p0["nccl"], p1["nccl"])
    assert torch.allclose(p0["nccl"], p0["None"], atol=1e-6)


def _leave_worker(rank, world, port, outdir, crash):
    dist = _init(rank, world, port, timeout_s=30)
    try:
        from mini_nangila_b200.models import GPT2, GPT2Config
        from mini_nangila_b200.parallel.fused import CommError
        from mini_nangila_b200.train import DDPTrainer

        torch.manual_seed(0)
        cfg = GPT2Config.tiny()
        tr = DDPTrainer(GPT2(cfg), hook="host", hook_kwargs=dict(use_momentum=True, seed=5),
                        device=torch.device("cpu"), bucket_cap_mb=0.05, monitor=True)
        tr.monitor.timeout_s = 5.0
        g = torch.Generator().manual_seed(100 + rank)
        msg = "none"
        for step in range(3):
            if rank == 1 and step == 1:
                if crash:
                    os._exit(0)  # no announcement: the others see silence
                ok = tr.monitor.leave("test leave")
                open(os.path.join(outdir, "f1.txt"), "w").write(f"left ack={ok}")
                return
            t = torch.randint(0, cfg.vocab_size, (2, 17), generator=g)
            try:
                tr.step(t[:, :-1], t[:, 1:])
            except CommError as e:
                msg = str(e)
                break
        open(os.path.join(outdir, f"f{rank}.txt"), "w").write(msg)
    finally:
        if not (crash and rank == 1):
            dist.destroy_process_group()


@pytest.mark.parametrize("crash", [False, True])
def test_rank_leaving_between_steps_is_noticed_before_the_next_launch(crash, tmp_path):
    """A rank that leaves between steps announces it in the store (or crashes
    and stays silent); the survivor raises CommError naming it before the
    next step's collectives, instead of waiting in one."""
    import time as _t

    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=_leave_worker, args=(r, 2, port, str(tmp_path), crash)) for r in range(2)]
    t0 = _t.time()
    for p in ps:
        p.start()
    for p in ps:
        p.join(120)
    for p in ps:
        if p.is_alive():
            p.kill()
    msg = (tmp_path / "f0.txt").read_text()
    assert "rank 1" in msg and ("left (test leave)" in msg if not crash else "silent" in msg), msg
    if not crash:
        assert (tmp_path / "f1.txt").read_text() == "left ack=True"
    assert _t.time() - t0 < 100
