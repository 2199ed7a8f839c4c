"""Host-side watchdog for GPU steps: a daemon thread polls the completion of
the last armed CUDA event (``event.query()``, never a blocking sync) and
trips when it is still pending past a deadline. The engine arms it after
every prefill chunk / decode burst (``VLLM_B200_WATCHDOG_S`` > 0) and raises
on its next step once tripped, so a wedged step surfaces as an error with the
device status word instead of a silent stall. Kernels already bound every
on-chip wait; this covers what they cannot see (a peer process that died, a
stream blocked on the host).

Reference parity: the failure-detection plan in the reference's notes
(cudaStreamQuery polling with a deadline); the reference relies on service
restarts and has no watchdog.
"""
from __future__ import annotations

import logging
import threading
import time

logger = logging.getLogger("vllm.b200.watchdog")


class StreamWatchdog:
    def __init__(self, deadline_s: float, poll_s: float = 0.05, on_trip=None, clock=time.monotonic):
        self.deadline_s = float(deadline_s)
        self.poll_s = float(poll_s)
        self.on_trip = on_trip
        self.clock = clock
        self.tripped = False
        self.trip_info: str | None = None
        self._armed = None  # (event, t0, what)
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name="b200-watchdog", daemon=True)
        self._thread.start()

    def arm(self, event, what: str = "step") -> None:
        """Watch ``event`` (anything with ``query() -> bool``) from now on."""
        with self._lock:
            self._armed = (event, self.clock(), what)

    def disarm(self) -> None:
        with self._lock:
            self._armed = None

    def check(self) -> None:
        """Raise if the watchdog has tripped (call before issuing more work)."""
        if self.tripped:
            raise RuntimeError(f"GPU watchdog: {self.trip_info}")

    def poll_once(self) -> None:
        with self._lock:
            armed = self._armed
        if armed is None or self.tripped:
            return
        ev, t0, what = armed
        if ev.query():
            with self._lock:
                if self._armed is armed:
                    self._armed = None
            return
        waited = self.clock() - t0
        if waited > self.deadline_s:
            self.tripped = True
            self.trip_info = f"{what} still running after {waited:.1f} s (deadline {self.deadline_s} s)"
            logger.error("%s", self.trip_info)
            if self.on_trip is not None:
                self.on_trip(self.trip_info)

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self.poll_once()
            except Exception as e:  # noqa: BLE001 - a dead context must not kill the thread silently
                self.tripped = True
                self.trip_info = f"event query failed: {e}"
                logger.error("%s", self.trip_info)
            self._stop.wait(self.poll_s)

    def close(self) -> None:
        self._stop.set()
        self._thread.join(timeout=1.0)
