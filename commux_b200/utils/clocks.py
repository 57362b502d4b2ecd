"""Sample GPU clocks and throttle reasons while a benchmark runs (read-only).

Runs ``nvidia-smi --query-gpu=... -lms <interval>`` for the given GPUs in a
subprocess and summarises the samples taken under load: median SM clock, the
maximum SM clock and every throttle reason that was active. Nothing here
changes a GPU setting.
"""

from __future__ import annotations

import shutil
import statistics
import subprocess
import tempfile

_FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_ids: list[str], interval_ms: int = 200, raw_path: str | None = None):
        self.gpu_ids = gpu_ids
        self.interval_ms = interval_ms
        self.raw_path = raw_path
        self.proc = None
        self.out = None

    def start(self) -> "ClockSampler":
        exe = shutil.which("nvidia-smi")
        if exe is None or not self.gpu_ids:
            return self
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        cmd = [exe, f"--query-gpu={_FIELDS}", "--format=csv,noheader,nounits",
               "-lms", str(self.interval_ms), "-i", ",".join(self.gpu_ids)]
        self.proc = subprocess.Popen(cmd, stdout=self.out, stderr=subprocess.DEVNULL)
        return self

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        self.out.seek(0)
        text = self.out.read()
        if self.raw_path:
            with open(self.raw_path, "w") as f:
                f.write(text)
        rows = [[c.strip() for c in r.split(",")] for r in text.strip().splitlines() if r.strip()]
        return summarize(rows)


def summarize(rows: list[list[str]]) -> dict | None:
    samples, loaded, reasons, maxes = [], [], set(), []
    for r in rows:
        if len(r) < 10:
            continue
        try:
            sm, smax, util = float(r[2]), float(r[3]), float(r[5])
        except ValueError:
            continue
        samples.append(sm)
        maxes.append(smax)
        if util >= 50:
            loaded.append(sm)
        for name, val in zip(_REASONS, r[6:10]):
            if val.strip().lower() == "active":
                reasons.add(name)
    if not samples:
        return None
    use = loaded or samples
    return {"sm_mhz": statistics.median(use), "sm_max_mhz": max(maxes),
            "reasons": sorted(reasons), "samples": len(samples), "samples_under_load": len(loaded)}


def gpu_uuid(device_index: int) -> str | None:
    """nvidia-smi id of a torch CUDA device: its PCI bus id (the CUDA UUID that
    torch reports need not equal NVML's), else the index."""
    try:
        import torch
        p = torch.cuda.get_device_properties(device_index)
        return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except Exception:
        return str(device_index)
