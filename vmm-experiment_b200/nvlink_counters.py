"""NVLink traffic of one GPU from its hardware counters, read through NVML.

Used by the multicast sweep and the benchmark to show the exchange's bytes on
the wire next to the event-timed bandwidth: bytes transmitted and received over
all of the GPU's active NVLinks, summed over links, read before and after a
timed region.  Reading the counters changes nothing on the GPU.

NVML fields, in order of preference:
  NVML_FI_DEV_NVLINK_COUNT_XMIT_BYTES / _RCV_BYTES   (202 / 204, bytes)
  NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX / _RX         (138 / 139, KiB of data)
each per link (scopeId = link index).
"""
from __future__ import annotations

MAX_LINKS = 18
_FIELDS = [("count_bytes", 202, 204, 1), ("throughput_data_kib", 138, 139, 1024)]


class NvlinkCounters:
    """Cumulative NVLink tx/rx bytes of the GPU that is `torch_device` in this
    process.  `available` is False (with `why`) when NVML or the fields are
    missing; `read()` then returns None."""

    def __init__(self, torch_device: int):
        self.available = False
        self.why = ""
        self.links = []
        self.kind = None
        self.last = None  # (tx, rx) bytes of the last region a caller measured
        try:
            import pynvml
            import torch

            self._nv = pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(torch_device).uuid)
            if not uuid.startswith("GPU-"):
                uuid = "GPU-" + uuid
            self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            for link in range(MAX_LINKS):
                try:
                    if pynvml.nvmlDeviceGetNvLinkState(self._h, link) == pynvml.NVML_FEATURE_ENABLED:
                        self.links.append(link)
                except pynvml.NVMLError:
                    continue
            if not self.links:
                self.why = "no active NVLink"
                return
            for kind, tx, rx, scale in _FIELDS:
                if self._sample(tx, rx, scale) is not None:
                    self.kind, self._tx, self._rx, self._scale = kind, tx, rx, scale
                    self.available = True
                    return
            self.why = "NVML returned no NVLink byte counters"
        except Exception as e:  # no NVML library, no permission, unknown device
            self.why = f"{type(e).__name__}: {e}"[:200]

    def _sample(self, tx, rx, scale):
        nv = self._nv
        ids = [(tx, link) for link in self.links] + [(rx, link) for link in self.links]
        try:
            vals = nv.nvmlDeviceGetFieldValues(self._h, ids)
        except nv.NVMLError:
            return None
        out = [0, 0]
        for i, v in enumerate(vals):
            if v.nvmlReturn != nv.NVML_SUCCESS:
                return None
            out[0 if i < len(self.links) else 1] += int(v.value.ullVal) * scale
        return out

    def read(self):
        """(tx_bytes, rx_bytes) summed over the active links, or None."""
        if not self.available:
            return None
        return self._sample(self._tx, self._rx, self._scale)

    def describe(self):
        if not self.available:
            return {"unavailable": self.why}
        return {"source": f"NVML {self.kind} counters, summed over {len(self.links)} active links"}


def delta(before, after):
    if before is None or after is None:
        return None
    return after[0] - before[0], after[1] - before[1]
