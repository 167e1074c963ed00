"""Background sampler of GPU utilisation, SM clock and memory through NVML
(nvidia-ml-py), with throttle reasons.  Read-only: it never changes a GPU
setting.  The reference's monitor (utils/gpu_monitor.py:6-75) samples
utilisation only and is never started; this one feeds the bench's clock
record."""
from __future__ import annotations

import statistics
import threading
import time
from typing import Dict, List, Optional


class GPUMonitor:
    def __init__(self, device_index: int = 0, interval_s: float = 0.05, nvml=None):
        self.device_index = device_index
        self.interval_s = interval_s
        self._nvml = nvml
        self.samples: List[Dict[str, float]] = []
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None

    def _lib(self):
        if self._nvml is None:
            import pynvml

            self._nvml = pynvml
        return self._nvml

    def start(self) -> "GPUMonitor":
        nv = self._lib()
        nv.nvmlInit()
        self._handle = nv.nvmlDeviceGetHandleByIndex(self.device_index)
        self._stop.clear()
        self._thread = threading.Thread(target=self._run, name="t1-gpumon", daemon=True)
        self._thread.start()
        return self

    def _run(self) -> None:
        nv = self._nvml
        while not self._stop.is_set():
            try:
                util = nv.nvmlDeviceGetUtilizationRates(self._handle)
                clk = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
                mem = nv.nvmlDeviceGetMemoryInfo(self._handle)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle) \
                    if hasattr(nv, "nvmlDeviceGetCurrentClocksEventReasons") else 0
                self.samples.append({"t": time.time(), "gpu_util": float(util.gpu),
                                     "mem_util": float(util.memory), "sm_mhz": float(clk),
                                     "mem_used_gb": mem.used / 1e9, "reasons": int(reasons)})
            except Exception:
                pass
            self._stop.wait(self.interval_s)

    def stop(self) -> Dict[str, float]:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        try:
            self._nvml.nvmlShutdown()
        except Exception:
            pass
        return self.summary()

    def summary(self) -> Dict[str, float]:
        if not self.samples:
            return {}
        return {
            "samples": len(self.samples),
            "gpu_util_mean": statistics.mean(s["gpu_util"] for s in self.samples),
            "sm_mhz_median": statistics.median(s["sm_mhz"] for s in self.samples),
            "mem_used_gb_max": max(s["mem_used_gb"] for s in self.samples),
        }
