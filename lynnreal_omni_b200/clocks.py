"""SM clock / power / clock-event-reason sampling of one GPU (NVML reads only).

``ClockSampler(device)`` starts a separate Python process that polls NVML every
``period_ms`` and writes one line per sample; ``stop()`` ends it and summarises
the samples taken while the GPU was under load. A process (not a thread) keeps
the sampling period independent of the launching thread's GIL. Nothing is ever
set on the GPU.
"""
from __future__ import annotations

import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
           "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}


def _poll(uuid: str, out: str, period_ms: float) -> None:
    import pynvml as n
    n.nvmlInit()
    h = n.nvmlDeviceGetHandleByUUID(uuid)
    with open(out, "w", buffering=1) as f:
        f.write(f"max {n.nvmlDeviceGetMaxClockInfo(h, n.NVML_CLOCK_SM)}\n")
        while True:
            try:
                f.write(f"{n.nvmlDeviceGetClockInfo(h, n.NVML_CLOCK_SM)} "
                        f"{n.nvmlDeviceGetPowerUsage(h) / 1000.0:.1f} "
                        f"{n.nvmlDeviceGetCurrentClocksEventReasons(h)}\n")
            except n.NVMLError:
                pass
            time.sleep(period_ms / 1000.0)


class ClockSampler:
    def __init__(self, uuid: str, period_ms: float = 5.0):
        self.uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        self.period_ms = period_ms
        fd, self.path = tempfile.mkstemp(prefix="lr_clocks", suffix=".txt")
        os.close(fd)
        self.proc = None

    def start(self) -> None:
        self.proc = subprocess.Popen([sys.executable, "-m", "lynnreal_omni_b200.clocks", self.uuid, self.path,
                                      str(self.period_ms)], cwd=str(Path(__file__).resolve().parents[1]),
                                     stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        deadline = time.time() + 20
        while time.time() < deadline:  # wait for the first sample line
            if self.proc.poll() is not None:
                break
            try:
                if len(Path(self.path).read_text().splitlines()) >= 2:
                    break
            except OSError:
                pass
            time.sleep(0.01)

    def stop(self) -> dict:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        lines = Path(self.path).read_text().splitlines() if Path(self.path).exists() else []
        Path(self.path).unlink(missing_ok=True)
        max_sm = None
        samples = []
        for line in lines:
            parts = line.split()
            if parts[:1] == ["max"]:
                max_sm = float(parts[1])
            elif len(parts) == 3:
                samples.append((float(parts[0]), float(parts[1]), int(parts[2])))
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": max_sm, "reasons": ["no samples"], "source": "nvml"}
        hi = max(p for _, p, _ in samples)
        loaded = [s for s in samples if s[1] >= 0.5 * hi] or samples
        reasons = sorted({k for _, _, r in loaded for k, bit in REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(c for c, _, _ in loaded), "sm_max_mhz": max_sm, "reasons": reasons,
                "samples": len(samples), "samples_under_load": len(loaded), "power_w_max": hi,
                "source": f"nvml in a separate process, {self.period_ms:g} ms"}


if __name__ == "__main__":
    _poll(sys.argv[1], sys.argv[2], float(sys.argv[3]))
