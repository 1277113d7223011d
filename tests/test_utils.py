"""Measurement helpers: clock sampling (against a fake nvidia-smi that
prints the queried fields), max over ranks on gloo, NVTX ranges without
CUDA."""
import os
import socket
import time

import torch
import torch.multiprocessing as mp

from mini_nangila_b200.utils.clocks import FIELDS, ClockSampler
from mini_nangila_b200.utils.nvtx import enabled, nvtx_range
from mini_nangila_b200.utils.timing import WallTimer


def test_clock_sampler_parses_samples_and_reasons(tmp_path, monkeypatch):
    fake = tmp_path / "nvidia-smi"
    loaded = "0, 1965, 1965, 700.5, 0x4, Not Active, Not Active, Not Active, Active"
    idle = "0, 345, 1965, 95.0, 0x0, Not Active, Not Active, Not Active, Not Active"
    fake.write_text("#!/bin/sh\n" + "".join(f"echo '{r}'\n" for r in (idle, loaded, loaded, loaded, idle))
                    + "exec sleep 30\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}:{os.environ['PATH']}")
    s = ClockSampler([0], period_ms=50).start()
    time.sleep(0.5)
    out = s.stop()
    assert len(loaded.split(",")) == len(FIELDS)
    assert out["samples"] == 5 and out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"] and out["power_w_max"] == 700.5


def test_clock_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))
    out = ClockSampler().start().stop()
    assert out["samples"] == 0 and out["sm_mhz"] is None


def _max_worker(rank, world, port, outdir):
    import torch.distributed as dist

    from mini_nangila_b200.utils.timing import barrier_sync, max_over_ranks

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        barrier_sync()
        v = max_over_ranks(10.0 + rank)
        torch.save(v, os.path.join(outdir, f"m{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks(tmp_path):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.start_processes(_max_worker, args=(3, port, str(tmp_path)), nprocs=3, join=True, start_method="spawn")
    assert [torch.load(tmp_path / f"m{r}.pt") for r in range(3)] == [12.0, 12.0, 12.0]


def test_nvtx_range_and_wall_timer():
    if not torch.cuda.is_available():
        assert not enabled()
    with nvtx_range("x"):
        t = WallTimer().start()
    assert t.stop() >= 0.0


def test_nvlink_counter_falls_back_to_byte_counters(monkeypatch):
    """utils.nvlink against a fake NVML: a driver that does not serve the
    THROUGHPUT_DATA fields (138/139) but does serve the NVLink 5 byte
    counters (202/204) on links 0-3 is read through the latter, in bytes."""
    import sys
    import types

    import torch

    from mini_nangila_b200.utils import nvlink

    class V:
        def __init__(self, ret, val=0):
            self.nvmlReturn = ret
            self.value = types.SimpleNamespace(ullVal=val)

    counts = {202: 1000, 204: 3000}

    def field_values(_h, ids):
        out = []
        for fid, link in ids:
            if fid in counts and link < 4:
                out.append(V(0, counts[fid] + link))
            else:
                out.append(V(3))  # NVML_ERROR_NOT_SUPPORTED
        return out

    fake = types.SimpleNamespace(nvmlInit=lambda: None, nvmlDeviceGetHandleByPciBusId=lambda bus: bus,
                                 nvmlDeviceGetFieldValues=field_values)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda i: types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1b, pci_device_id=0))
    c = nvlink.NvlinkCounter(0)
    assert c.available and c.source == "COUNT_BYTES"
    assert c.read() == (4 * 1000 + 6, 4 * 3000 + 6)
    counts[202] += 500
    tx, rx = c.read()
    assert tx == 4 * 1500 + 6 and rx == 4 * 3000 + 6


def test_clock_sampler_keeps_the_marked_region(tmp_path, monkeypatch):
    """Samples written before begin() and after end() are left out; a region
    that saw no sample of its own takes the samples on either side."""
    fake = tmp_path / "nvidia-smi"
    warm = "0, 900, 1965, 300.0, 0x0, Not Active, Not Active, Not Active, Not Active"
    hot = "0, 1800, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active"
    cool = "0, 345, 1965, 95.0, 0x0, Not Active, Not Active, Not Active, Not Active"
    gate = tmp_path / "go"
    # two samples at once, then one per file that appears under tmp_path
    script = "#!/bin/sh\n" + f"echo '{warm}'\necho '{warm}'\n"
    script += f"while [ ! -e {gate}1 ]; do sleep 0.02; done\necho '{hot}'\necho '{hot}'\n"
    script += f"while [ ! -e {gate}2 ]; do sleep 0.02; done\necho '{cool}'\nexec sleep 30\n"
    fake.write_text(script)
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}:{os.environ['PATH']}")

    def wait_lines(s, n):
        t0 = time.time()
        while s._lines() < n and time.time() - t0 < 10:
            time.sleep(0.02)

    s = ClockSampler([0], period_ms=50).start()
    wait_lines(s, 2)
    s.begin()
    (tmp_path / "go1").write_text("")
    wait_lines(s, 4)
    s.end()
    (tmp_path / "go2").write_text("")
    wait_lines(s, 5)
    out = s.stop()
    assert out["samples"] == 2 and out["sm_mhz"] == 1800.0 and out["reasons"] == ["sw_power_cap"]

    (tmp_path / "go1").unlink()
    (tmp_path / "go2").unlink()
    s = ClockSampler([0], period_ms=50).start()
    wait_lines(s, 2)
    s.begin()
    s.end()  # nothing written in between
    out = s.stop()
    assert out["samples"] == 1 and out["sm_mhz"] == 900.0
