"""bench.py's one JSON line (rank 0) on one GPU: the keys and types the
benchmark contract names, a value consistent with the timed steps, clocks
sampled during the timed region, and the end-to-end figure with its
host-to-device and device-to-host bytes (a short run of the real workload)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.gpu
def test_bench_prints_one_contract_line():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    # a single rank of its own: no rendezvous variables left by earlier tests
    env = {k: v for k, v in os.environ.items()
           if k not in ("MASTER_PORT", "RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE")}
    env["MASTER_ADDR"] = "127.0.0.1"
    r = subprocess.run([sys.executable, "bench.py", "--steps", "10", "--warmup", "3", "--no-arms"], cwd=ROOT,
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for key, typ in [("metric", str), ("value", float), ("unit", str), ("n_gpus", int), ("steps", int),
                     ("warmup", int), ("ms_per_step", float), ("higher_is_better", bool), ("scaling", str),
                     ("dtype", str), ("data", str), ("config", dict), ("gpu_launches", int), ("e2e", dict)]:
        assert isinstance(d[key], typ), key
    assert "vs_baseline" in d
    assert d["n_gpus"] == 1 and d["steps"] == 10 and d["warmup"] == 3
    assert d["higher_is_better"] is True and d["scaling"] == "weak" and d["dtype"] == "bf16"
    cfg = d["config"]
    assert cfg["model"] == "gpt2-small-124M" and cfg["seq_len"] == 1024 and cfg["parallelism"] == "dp1"
    assert cfg["global_batch"] == 8
    # tokens/s of the whole job from the timed steps
    assert abs(d["value"] - 8 * 1024 / (d["ms_per_step"] / 1000.0)) <= 1e-6 * d["value"]
    assert d["gpu_launches"] == 13 * 10  # one fused kernel per bucket and step
    e2e = d["e2e"]
    assert e2e["unit"] == "tokens/s" and e2e["value"] > 0
    assert e2e["h2d_bytes_per_step"] == 2 * 8 * 1024 * 8  # int64 inputs and targets
    assert e2e["d2h_bytes_per_step"] == 4  # the fp32 loss
    clocks = d.get("clocks")
    assert clocks is not None and clocks["sm_max_mhz"] and isinstance(clocks["reasons"], list)
