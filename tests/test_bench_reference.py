"""bench.py's reference arm (the unmodified nangila_ddp hook from
baseline/_ref on stock transformers models of the benchmark families),
built tiny and stepped on CPU: GPT-2 with the INT4 + EMA hook and the
Llama family with the hook in top-k mode."""
import os
import socket
import sys
import types

import pytest
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "nangila_ddp")),
                    reason="reference not installed in baseline/_ref")
@pytest.mark.parametrize("model,mode,name", [("gpt2", "int4", "reference-nangila_ddp-int4-ema"),
                                             ("llama", "topk", "reference-nangila_ddp-int4-topk0.05")])
def test_reference_arm_steps(model, mode, name):
    import bench

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(s.getsockname()[1]))
    s.close()
    dist.init_process_group("gloo", rank=0, world_size=1)
    saved_path = list(sys.path)
    try:
        args = types.SimpleNamespace(model=model, mode=mode, topk=0.05, momentum="auto", bucket_mb=25.0)
        step, why, hook_name = bench.build_reference(args, torch.device("cpu"), tiny=True)
        assert why is None and hook_name == name
        g = torch.Generator().manual_seed(0)
        x, y = torch.randint(0, 512, (2, 16), generator=g), torch.randint(0, 512, (2, 16), generator=g)
        losses = [float(step(x, y)) for _ in range(2)]
        assert all(torch.isfinite(torch.tensor(losses)))
    finally:
        dist.destroy_process_group()
        # build_reference puts baseline/_ref first on sys.path and imports the
        # reference's nangila_ddp; later tests in this process must get the shim
        sys.path[:] = saved_path
        for name in [m for m in sys.modules if m == "nangila_ddp" or m.startswith("nangila_ddp.")]:
            if "_ref" in (getattr(sys.modules[name], "__file__", "") or ""):
                del sys.modules[name]


def test_hook_on_reference_model_arm_steps():
    """bench.py's same-model arm: this framework's hook on the stock
    transformers GPT-2 with foreach AdamW and default DDP (tiny, CPU host hook)."""
    import bench

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(s.getsockname()[1]))
    s.close()
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        args = types.SimpleNamespace(model="gpt2", mode="int4", topk=0.05, momentum="auto", variant="auto", bucket_mb=25.0)
        step, hs, name = bench.build_hook_on_reference_model(args, torch.device("cpu"), tiny=True)
        assert name == "fused-int4-ema-ef"
        g = torch.Generator().manual_seed(0)
        x, y = torch.randint(0, 512, (2, 16), generator=g), torch.randint(0, 512, (2, 16), generator=g)
        losses = [float(step(x, y)) for _ in range(2)]
        assert all(torch.isfinite(torch.tensor(losses))) and hs.raw_bytes > 0
    finally:
        dist.destroy_process_group()
