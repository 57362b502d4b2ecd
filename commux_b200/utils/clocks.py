"""Sample GPU clocks and throttle reasons while a benchmark runs (read-only).

A native thread (``commux_b200._C.ClockSampler``, C++, no GIL) polls NVML
every ``interval_ms`` (default 1 ms) for the SM clock, the maximum SM clock,
power and the active clock-event reasons; every sample falls inside the timed
region, so all of them count as "under load". Without the native module a
Python thread polls through pynvml instead and uses utilisation >= 50 % to mark
samples under load. The summary gives the median SM clock, the maximum SM
clock and every throttle reason that was active. Nothing here changes a GPU
setting; only query functions are called.
"""

from __future__ import annotations

import statistics
import threading
import time

_REASONS = {  # NVML clock-event reason bits
    "sw_power_cap": 0x4,
    "hw_slowdown": 0x8,
    "sw_thermal_slowdown": 0x20,
    "hw_thermal_slowdown": 0x40,
    "hw_power_brake_slowdown": 0x80,
}


class ClockSampler:
    def __init__(self, gpu_ids: list[str], interval_ms: float = 1.0, raw_path: str | None = None):
        self.gpu_ids = gpu_ids
        self.interval = interval_ms / 1e3
        self.raw_path = raw_path
        self._rows: list[tuple] = []
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self._handles = []
        self.error = None

    def start(self) -> "ClockSampler":
        # native sampler (C++ thread, no GIL): a sample per interval even when
        # the Python thread is busy launching work
        try:
            from commux_b200 import _C

            self._native = [_C.ClockSampler(g, int(self.interval * 1e6)) for g in self.gpu_ids]
            if self._native and not any(n.error for n in self._native):
                for n in self._native:
                    n.start()
                return self
        except Exception:
            pass
        self._native = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            for g in self.gpu_ids:
                if ":" in g:
                    self._handles.append(pynvml.nvmlDeviceGetHandleByPciBusId(g))
                else:
                    self._handles.append(pynvml.nvmlDeviceGetHandleByIndex(int(g)))
        except Exception as e:  # no NVML on this machine
            self.error = str(e)
            return self
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def _sample(self):
        n = self._nvml
        for h in self._handles:
            try:
                sm = n.nvmlDeviceGetClockInfo(h, n.NVML_CLOCK_SM)
                smax = n.nvmlDeviceGetMaxClockInfo(h, n.NVML_CLOCK_SM)
                util = n.nvmlDeviceGetUtilizationRates(h).gpu
                try:
                    reasons = n.nvmlDeviceGetCurrentClocksEventReasons(h)
                except AttributeError:
                    reasons = n.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                power = n.nvmlDeviceGetPowerUsage(h) / 1000.0
                self._rows.append((time.time(), sm, smax, util, reasons, power))
            except Exception as e:
                self.error = str(e)

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.interval)

    def stop(self) -> dict | None:
        if getattr(self, "_native", None):
            rows = []
            for n in self._native:
                for t_us, sm, smax, reasons, mw in n.stop():
                    # every native sample falls inside the timed region:
                    # utilisation 100 marks it "under load"
                    rows.append((t_us / 1e6, sm, smax, 100, reasons, mw / 1000.0))
            self._rows = rows
            if self.raw_path:
                with open(self.raw_path, "w") as f:
                    f.write("t,sm_mhz,sm_max_mhz,util,reasons_mask,power_w\n")
                    for r in rows:
                        f.write(",".join(str(x) for x in r) + "\n")
            return summarize(rows)
        if self._thread is None:
            return None
        self._sample()  # at least one sample at the end of the region
        self._stop.set()
        self._thread.join(timeout=2)
        if self.raw_path:
            with open(self.raw_path, "w") as f:
                f.write("t,sm_mhz,sm_max_mhz,util,reasons_mask,power_w\n")
                for r in self._rows:
                    f.write(",".join(str(x) for x in r) + "\n")
        return summarize(self._rows)


def summarize(rows) -> dict | None:
    if not rows:
        return None
    sms = [r[1] for r in rows]
    loaded = [r[1] for r in rows if r[3] >= 50]
    mask = 0
    for r in rows:
        mask |= int(r[4])
    reasons = sorted(k for k, bit in _REASONS.items() if mask & bit)
    return {"sm_mhz": statistics.median(loaded or sms), "sm_max_mhz": max(r[2] for r in rows),
            "reasons": reasons, "samples": len(rows), "samples_under_load": len(loaded),
            "power_w_max": round(max(r[5] for r in rows), 1)}


def gpu_uuid(device_index: int) -> str | None:
    """NVML id of a torch CUDA device: its PCI bus id (the CUDA UUID that torch
    reports need not equal NVML's), else the index."""
    try:
        import torch

        p = torch.cuda.get_device_properties(device_index)
        return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except Exception:
        return str(device_index)
