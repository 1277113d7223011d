"""Resumable hook state (checkpoint / resume of the predictor, error
feedback and step keys).

* Same bucket layout: a hook state restored from ``state_dict`` continues
  bit-identically to an uninterrupted one.
* Another layout: each parameter's predictor / EF values follow it into the
  new buckets (DDP's first iteration after a restart, or its bucket rebuild
  after the first iteration, regroups parameters).
* DDP's own rebuild inside a run keeps every parameter's state (the new
  buckets continue at the old call count instead of restarting).
"""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _Bucket:
    """A DDP GradBucket stand-in whose gradients are views of one buffer."""

    def __init__(self, idx, params, order, rng):
        self.idx = idx
        self.params = [params[i] for i in order]
        sizes = [p.numel() for p in self.params]
        self.buf = torch.from_numpy((rng.standard_normal(sum(sizes)) * 1e-3).astype(np.float32))
        offs = np.concatenate([[0], np.cumsum(sizes)])
        self.grads = [self.buf[offs[i]:offs[i + 1]] for i in range(len(sizes))]

    def buffer(self):
        return self.buf

    def index(self):
        return self.idx

    def parameters(self):
        return self.params

    def gradients(self):
        return self.grads


def _single_rank():
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_port()))
    dist.init_process_group("gloo", rank=0, world_size=1)


def _hook_state(params, **kw):
    from mini_nangila_b200.parallel.hook import HookConfig, NangilaHookState

    hs = NangilaHookState(HookConfig(impl="host", use_momentum=True, seed=11, **kw))
    hs.param_index = {p.data_ptr(): i for i, p in enumerate(params)}
    return hs


def _run(hs, layouts, calls, seed0, params):
    """calls x (every bucket of `layouts`), returns the averaged buffers."""
    from mini_nangila_b200.parallel.hook import _host_hook

    out = []
    for c in range(calls):
        rng = np.random.default_rng(seed0 + c)
        for b, order in enumerate(layouts):
            bk = _Bucket(b, params, order, rng)
            _host_hook(hs, bk).wait()
            out.append(bk.buf.clone())
    return out


def test_same_layout_resume_is_bit_identical():
    _single_rank()
    try:
        params = [torch.zeros(n) for n in (700, 300, 1200, 5)]
        layout = [[3, 2], [1, 0]]
        for kw in ({}, {"topk_percent": 0.1}):
            a = _hook_state(params, **kw)
            full = _run(a, layout, 5, 0, params)
            b = _hook_state(params, **kw)
            _run(b, layout, 3, 0, params)
            c = _hook_state(params, **kw)
            c.load_state_dict(b.state_dict())
            tail = _run(c, layout, 2, 3, params)
            for x, y in zip(full[6:], tail):
                assert torch.equal(x.view(torch.int32), y.view(torch.int32))
            assert {k: v.calls for k, v in c.buckets.items()} == {0: 5, 1: 5}
    finally:
        dist.destroy_process_group()


def test_state_follows_its_parameters_into_another_layout():
    _single_rank()
    try:
        params = [torch.zeros(n) for n in (700, 300, 1200, 5)]
        a = _hook_state(params)
        _run(a, [[3, 2], [1, 0]], 2, 0, params)
        sd = a.state_dict()
        per_param = {}
        for bst in a.buckets.values():
            for pi, off, n in bst.layout:
                per_param[pi] = (bst.pred[off:off + n].clone(), bst.ef[off:off + n].clone())
        # restore into one bucket holding the parameters in another order
        from mini_nangila_b200.parallel.hook import _get_state

        c = _hook_state(params)
        c.load_state_dict(sd)
        bk = _Bucket(0, params, [0, 2, 1, 3], np.random.default_rng(9))
        st, first = _get_state(c, 0, bk.buf, bk, True, True)
        assert not first and st.calls == 3
        for pi, off, n in st.layout:
            assert torch.equal(st.pred[off:off + n], per_param[pi][0])
            assert torch.equal(st.ef[off:off + n], per_param[pi][1])
    finally:
        dist.destroy_process_group()


class _MLP(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.net = torch.nn.Sequential(torch.nn.Linear(32, 128), torch.nn.ReLU(), torch.nn.Linear(128, 10))

    def forward(self, x, y):
        return torch.nn.functional.cross_entropy(self.net(x), y)


def _ddp_worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mini_nangila_b200.train import DDPTrainer

        kw = dict(use_momentum=True, bits=4, seed=5, error_feedback=True)
        g = torch.Generator().manual_seed(100 + rank)
        data = [(torch.randn(16, 32, generator=g), torch.randint(0, 10, (16,), generator=g)) for _ in range(6)]
        torch.manual_seed(0)
        a = DDPTrainer(_MLP(), hook="host", hook_kwargs=kw, device=torch.device("cpu"))
        for x, y in data[:3]:
            a.step(x, y)
        # DDP rebuilt its buckets after the first iteration: the states moved
        # with their parameters, so every bucket has seen all three steps
        calls = sorted(st.calls for st in a.hook_state.buckets.values())
        sd = a.state_dict()
        saved_layouts = sorted(tuple(tuple(x) for x in d["layout"]) for d in sd["hook"]["buckets"].values())
        torch.manual_seed(7)
        c = DDPTrainer(_MLP(), hook="host", hook_kwargs=kw, device=torch.device("cpu"))
        c.load_state_dict(sd)
        losses = [float(c.step(x, y)) for x, y in data[3:]]
        layouts = sorted(st.layout for st in c.hook_state.buckets.values())
        torch.save({"calls": calls, "c_calls": sorted(st.calls for st in c.hook_state.buckets.values()),
                    "same_layout": layouts == saved_layouts, "losses": losses, "steps": c.steps_done},
                   os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_ddp_trainer_resume_and_rebuild(tmp_path):
    mp.start_processes(_ddp_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        d = torch.load(tmp_path / f"r{r}.pt")
        assert d["calls"] and all(c == 3 for c in d["calls"])
        assert all(c == 6 for c in d["c_calls"]) and d["steps"] == 6
        assert d["same_layout"] and all(np.isfinite(d["losses"]))
