"""GPU clock and throttle-reason sampling during a timed region.

Where NVML answers (``pynvml``), a thread reads the SM clock, the maximum
clock and the active clock-event reasons every 5 ms, so a timed region of a
hundred milliseconds carries about twenty samples.  Otherwise ``nvidia-smi``
polls the GPU in a child process and a reader thread stamps each line with
the host clock.  Entering the context waits (up to a few seconds)
for the first sample, so the poller is running before the timed region
starts, and leaving it waits for one more sample, so a region shorter than
the polling interval still has one.  The summary keeps only samples stamped
inside the region (or the first one after it ends when none is): median SM
clock under load, max clock, active throttle reasons.  Reading clocks
changes no GPU setting.
"""
from __future__ import annotations

import subprocess
import threading
import time


class _NvmlPoller:
    """Read-only NVML polling of one GPU in a thread; lines in nvidia-smi's CSV layout."""

    PERIOD_S = 0.005

    def __init__(self, gpu: int, sink) -> None:
        import pynvml

        self.nv = pynvml
        pynvml.nvmlInit()
        self.h = pynvml.nvmlDeviceGetHandleByIndex(gpu)
        self.gpu, self.sink = gpu, sink
        self.stop = threading.Event()
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _line(self) -> str:
        nv, h = self.nv, self.h
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        try:
            power = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
        except nv.NVMLError:
            power = 0.0
        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        # hw_slowdown, hw_thermal_slowdown, sw_thermal_slowdown, sw_power_cap
        order = (nv.nvmlClocksThrottleReasonHwSlowdown, nv.nvmlClocksThrottleReasonHwThermalSlowdown,
                 nv.nvmlClocksThrottleReasonSwThermalSlowdown, nv.nvmlClocksThrottleReasonSwPowerCap)
        flags = ["Active" if bits & b else "Not Active" for b in order]
        return f"{self.gpu}, {sm}, {mx}, {power:.1f}, {bits:#x}, " + ", ".join(flags)

    def _run(self) -> None:
        while not self.stop.is_set():
            try:
                self.sink(self._line())
            except Exception:
                return
            self.stop.wait(self.PERIOD_S)

    def start(self) -> None:
        self.thread.start()

    def terminate(self) -> None:
        self.stop.set()
        self.thread.join(timeout=5)
        try:
            self.nv.nvmlShutdown()
        except Exception:
            pass


class ClockSampler:
    """Clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    INTERVAL_MS = 50
    START_WAIT_S = 5.0

    def __init__(self, gpu: int) -> None:
        self.gpu = gpu
        self.proc = None
        self.nvml = None
        self.samples: list[tuple[float, str]] = []
        self.t0 = self.t1 = 0.0
        self._cv = threading.Condition()
        self._reader = None

    def _read(self) -> None:
        for line in self.proc.stdout:
            if line.strip():
                with self._cv:
                    self.samples.append((time.monotonic(), line))
                    self._cv.notify_all()

    def _wait_for(self, count: int, timeout: float) -> None:
        with self._cv:
            self._cv.wait_for(lambda: len(self.samples) >= count, timeout=timeout)

    def _push(self, line: str) -> None:
        with self._cv:
            self.samples.append((time.monotonic(), line))
            self._cv.notify_all()

    def __enter__(self):
        self.nvml = None
        try:
            self.nvml = _NvmlPoller(self.gpu, self._push)
            self.nvml.start()
            self._wait_for(1, self.START_WAIT_S)
            self.t0 = time.monotonic()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.INTERVAL_MS)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except (FileNotFoundError, OSError):
            self.proc = None
        if self.proc is not None:
            self._reader = threading.Thread(target=self._read, daemon=True)
            self._reader.start()
            self._wait_for(1, self.START_WAIT_S)
        self.t0 = time.monotonic()
        return self

    def __exit__(self, *exc):
        self.t1 = time.monotonic()
        if self.nvml is not None:
            self.nvml.terminate()
            return
        if self.proc is None:
            return
        with self._cv:
            after = len(self.samples) + 1
        self._wait_for(after, 1.0)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        if self._reader is not None:
            self._reader.join(timeout=5)

    def region_lines(self) -> list[str]:
        inside = [line for t, line in self.samples if self.t0 <= t <= self.t1]
        if not inside:
            inside = [line for t, line in self.samples if t > self.t1][:1]
        return inside

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.region_lines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        sm.sort()
        return {
            "sm_mhz": sm[len(sm) // 2] if sm else None,
            "sm_max_mhz": mx,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }
