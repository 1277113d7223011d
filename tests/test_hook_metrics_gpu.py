"""The fused hook's metrics (reference layout, comm_hook.py:307-319): the
residual statistic res_mean_abs = mean |g - pred| is computed on the device
and its line written once the value has landed; logging leaves the reduced
gradients bit-identical to a run without it."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


class _Bucket:
    def __init__(self, t):
        self.t = t

    def buffer(self):
        return self.t

    def index(self):
        return 0

    def parameters(self):
        return []


def test_fused_hook_metrics_are_device_side_and_leave_the_bucket_alone(tmp_path):
    from mini_nangila_b200.parallel.fused import FusedAllReduce
    from mini_nangila_b200.parallel.hook import HookConfig, NangilaHookState, _fused_hook

    dev = torch.device("cuda", 0)
    n = 300_000
    runs = {}
    for path in (None, str(tmp_path / "m.csv")):
        hs = NangilaHookState(HookConfig(impl="fused", use_momentum=True, seed=3, metrics_path=path))
        hs.comm = FusedAllReduce(n, device=dev, modes=(hs.config.mode,))
        hs.stream = torch.cuda.Stream(device=dev)
        outs, wants = [], []
        for call in range(3):
            g = torch.randn(n, generator=torch.Generator(device=dev).manual_seed(call), device=dev) * 1e-3
            pred = hs.buckets[0].pred.clone() if call else None
            wants.append(float(((g.double() - pred.double()) if call else g.double()).abs().mean()))
            buf = g.clone()
            _fused_hook(hs, _Bucket(buf)).wait()
            torch.cuda.current_stream().wait_stream(hs.stream)
            outs.append(buf.clone())
        torch.cuda.synchronize()
        hs.comm.check()
        if path:
            assert hs.flush_metrics(wait=True) >= 0 and not hs.pending_metrics
            lines = open(path).read().splitlines()
            assert len(lines) == 3
            for call, line in enumerate(lines):
                d = dict(zip(line.split(",")[0::2], line.split(",")[1::2]))
                assert int(d["hook_idx"]) == call + 1 and int(d["bucket_elems"]) == n
                assert float(d["res_mean_abs"]) == pytest.approx(wants[call], rel=1e-4)
        runs[path is not None] = outs
    for a, b in zip(runs[False], runs[True]):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    assert np.isfinite([float(x.abs().mean()) for x in runs[True]]).all()
