"""Timing and environment helpers shared by the harnesses.

Timing follows the reference's methodology (profiling/gate/bench_capacity_gate.py:88-109,
profiling/portable/measure_params.py:36-54): a CUDA graph of ``inner`` launches,
replayed ``reps`` times after warm-up, CUDA events around each replay, median
per launch. Clocks are sampled through NVML while the timed work runs (read
only; nothing here changes a GPU setting).
"""

from __future__ import annotations

import json
import os
import statistics
import sys
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
if PKG not in sys.path:
    sys.path.insert(0, PKG)
DROPIN = os.path.join(PKG, "dropin")
if DROPIN not in sys.path:
    sys.path.insert(0, DROPIN)

import torch  # noqa: E402


def graph_time_us(fn, inner: int = 10, reps: int = 30, warm: int = 3) -> float:
    """Median microseconds per launch of ``fn`` under a CUDA graph of ``inner`` launches."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(inner):
            fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        g.replay()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e) * 1e3 / inner)
    del g
    return statistics.median(ts)


def graph_time_us_indexed(make_fn, inner: int = 10, reps: int = 30, warm: int = 3) -> float:
    """As graph_time_us, for ``make_fn(i)`` returning the i-th launch of the graph
    (rotating weight copies: launch i uses copy i % R, so consecutive launches
    never re-read the same weights from L2)."""
    for i in range(warm):
        make_fn(i)()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(inner):
            make_fn(i)()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        g.replay()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e) * 1e3 / inner)
    del g
    return statistics.median(ts)


class ClockSampler:
    """Samples SM clock and throttle reasons every 200 ms through NVML (read-only)."""

    def __init__(self, index: int = 0):
        self.index = index
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._ok = False

    def __enter__(self):
        self.start()
        return self

    def __exit__(self, *exc):
        self.info = self.stop()

    def start(self):
        try:
            import pynvml as N

            N.nvmlInit()
            self._N = N
            self._h = N.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self._h, N.NVML_CLOCK_SM)
            self._ok = True
        except Exception:  # noqa: BLE001
            return

        def loop():
            while not self._stop.is_set():
                try:
                    mhz = self._N.nvmlDeviceGetClockInfo(self._h, self._N.NVML_CLOCK_SM)
                    rs = self._N.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                    self.samples.append((mhz, rs))
                except Exception:  # noqa: BLE001
                    pass
                time.sleep(0.2)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()

    def stop(self) -> dict:
        if not self._ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        self._stop.set()
        self._thread.join(timeout=2)
        N = self._N
        names = {
            "hw_slowdown": getattr(N, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sw_thermal_slowdown": getattr(N, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(N, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_power_cap": getattr(N, "nvmlClocksEventReasonSwPowerCap", 0x4),
        }
        seen = sorted({k for _, r in self.samples for k, bit in names.items() if r & bit})
        mhz = [m for m, _ in self.samples]
        return {"sm_mhz": int(statistics.median(mhz)) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": seen, "samples": len(mhz)}


def gpu_info() -> dict:
    p = torch.cuda.get_device_properties(0)
    return {"gpu": p.name, "sms": p.multi_processor_count, "l2_mb": round(p.L2_cache_size / 2**20, 1),
            "hbm_gb": round(p.total_memory / 1e9, 1), "torch": torch.__version__}


def save_json(path: str, obj) -> None:
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "w") as f:
        json.dump(obj, f, indent=1)
    print(f"saved {path}", flush=True)
