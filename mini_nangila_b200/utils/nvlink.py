"""NVLink traffic of this process's GPU from NVML's per-link data counters.

``NvlinkCounter(device).read()`` returns the cumulative bytes sent and
received over all NVLinks of the GPU, from NVML's per-link field values:
``NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX`` / ``_RX`` (KiB of data, protocol
overhead excluded) where the driver serves them, else the NVLink 5
counters ``NVML_FI_DEV_NVLINK_COUNT_XMIT_BYTES`` / ``_RCV_BYTES`` (bytes;
``source`` names the pair in use).  The difference of two reads
around a run of kernels is their NVLink traffic, measured by the hardware:
no profiler, and nothing is changed on the GPU (the counters are only
read, never cleared).  The GPU is found by its PCI bus id, so CUDA and NVML
device numbering need not agree.  Without NVML (or on a GPU without
NVLink) ``available`` is False and reads return (0, 0).
"""
from __future__ import annotations

import torch

# (tx field, rx field, bytes per count, name), in order of preference
_FIELDS = (
    (138, 139, 1024, "THROUGHPUT_DATA"),  # NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX / _RX (KiB)
    (202, 204, 1, "COUNT_BYTES"),  # NVML_FI_DEV_NVLINK_COUNT_XMIT_BYTES / _RCV_BYTES (bytes)
)
_MAX_LINKS = 18


class NvlinkCounter:
    def __init__(self, device: torch.device | int):
        self.available = False
        self.source = ""
        self._h = None
        self._links: list[int] = []
        self._tx = self._rx = self._unit = 0
        try:
            import pynvml

            pynvml.nvmlInit()
            idx = device.index if isinstance(device, torch.device) else int(device)
            p = torch.cuda.get_device_properties(idx)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            for tx, rx, unit, name in _FIELDS:
                vals = pynvml.nvmlDeviceGetFieldValues(self._h, [(tx, link) for link in range(_MAX_LINKS)])
                links = [link for link, v in enumerate(vals) if v.nvmlReturn == 0]
                if links:
                    self._links, self._tx, self._rx, self._unit, self.source = links, tx, rx, unit, name
                    self.available = True
                    break
        except Exception:  # no NVML, no such field on this GPU, no NVLink
            self.available = False

    def read(self) -> tuple[int, int]:
        """(bytes sent, bytes received) over all links since the counters' origin."""
        if not self.available:
            return (0, 0)
        ids = [(self._tx, link) for link in self._links] + [(self._rx, link) for link in self._links]
        vals = self._nvml.nvmlDeviceGetFieldValues(self._h, ids)
        tot = [0, 0]
        for i, v in enumerate(vals):
            if v.nvmlReturn != 0:
                continue
            x = v.value
            num = x.ullVal if hasattr(x, "ullVal") else int(x)
            tot[0 if i < len(self._links) else 1] += int(num) * self._unit
        return tot[0], tot[1]
