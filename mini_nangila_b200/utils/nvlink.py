"""NVLink traffic of this process's GPU from NVML's per-link data counters.

``NvlinkCounter(device).read()`` returns the cumulative payload bytes sent
and received over all NVLinks of the GPU (NVML field values
``NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX`` / ``_RX`` per link, which count
KiB of data, protocol overhead excluded).  The difference of two reads
around a run of kernels is their NVLink traffic, measured by the hardware:
no profiler, and nothing is changed on the GPU (the counters are only
read, never cleared).  The GPU is found by its PCI bus id, so CUDA and NVML
device numbering need not agree.  Without NVML (or on a GPU without
NVLink) ``available`` is False and reads return (0, 0).
"""
from __future__ import annotations

import torch

_TX, _RX = 138, 139  # NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX / _RX
_MAX_LINKS = 18


class NvlinkCounter:
    def __init__(self, device: torch.device | int):
        self.available = False
        self._h = None
        self._links: list[int] = []
        try:
            import pynvml

            pynvml.nvmlInit()
            idx = device.index if isinstance(device, torch.device) else int(device)
            p = torch.cuda.get_device_properties(idx)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            vals = pynvml.nvmlDeviceGetFieldValues(self._h, [(_TX, link) for link in range(_MAX_LINKS)])
            self._links = [link for link, v in enumerate(vals) if v.nvmlReturn == 0]
            self.available = bool(self._links)
        except Exception:  # no NVML, no such field on this GPU, no NVLink
            self.available = False

    def read(self) -> tuple[int, int]:
        """(bytes sent, bytes received) over all links since the counters' origin."""
        if not self.available:
            return (0, 0)
        ids = [(_TX, link) for link in self._links] + [(_RX, link) for link in self._links]
        vals = self._nvml.nvmlDeviceGetFieldValues(self._h, ids)
        tot = [0, 0]
        for i, v in enumerate(vals):
            if v.nvmlReturn != 0:
                continue
            x = v.value
            num = x.ullVal if hasattr(x, "ullVal") else int(x)
            tot[0 if i < len(self._links) else 1] += int(num) * 1024  # the counters count KiB
        return tot[0], tot[1]
