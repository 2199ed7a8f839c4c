"""Host watchdog (deadline on a pending GPU event, polled, never blocking)
and NVTX range helpers. CPU only: the events are fakes."""
import pytest

from vllm_sm70_b200.utils import tracing
from vllm_sm70_b200.utils.watchdog import StreamWatchdog


class FakeEvent:
    def __init__(self, done=False):
        self.done = done

    def query(self):
        return self.done


class Clock:
    def __init__(self):
        self.t = 0.0

    def __call__(self):
        return self.t


def _wd(deadline=1.0):
    clock = Clock()
    trips = []
    wd = StreamWatchdog(deadline, poll_s=3600, on_trip=trips.append, clock=clock)
    return wd, clock, trips


def test_completed_event_never_trips():
    wd, clock, trips = _wd()
    ev = FakeEvent(done=False)
    wd.arm(ev, "decode")
    clock.t = 0.5
    wd.poll_once()
    ev.done = True
    clock.t = 5.0
    wd.poll_once()  # completed -> disarmed
    clock.t = 50.0
    wd.poll_once()
    assert not wd.tripped and trips == []
    wd.check()
    wd.close()


def test_pending_event_trips_after_deadline():
    wd, clock, trips = _wd(deadline=2.0)
    wd.arm(FakeEvent(done=False), "prefill chunk")
    clock.t = 1.9
    wd.poll_once()
    assert not wd.tripped
    clock.t = 2.5
    wd.poll_once()
    assert wd.tripped and len(trips) == 1 and "prefill chunk" in trips[0]
    with pytest.raises(RuntimeError, match="watchdog"):
        wd.check()
    wd.poll_once()  # trips once
    assert len(trips) == 1
    wd.close()


def test_rearm_resets_deadline():
    wd, clock, _ = _wd(deadline=1.0)
    wd.arm(FakeEvent(done=False), "a")
    clock.t = 0.9
    wd.arm(FakeEvent(done=False), "b")  # new step armed at t=0.9
    clock.t = 1.5
    wd.poll_once()
    assert not wd.tripped
    clock.t = 2.0
    wd.poll_once()
    assert wd.tripped and "b" in wd.trip_info
    wd.close()


def test_query_error_trips():
    class Bad:
        def query(self):
            raise RuntimeError("context lost")

    wd = StreamWatchdog(10.0, poll_s=0.01)
    wd.arm(Bad(), "x")
    import time

    for _ in range(200):
        if wd.tripped:
            break
        time.sleep(0.01)
    assert wd.tripped and "context lost" in wd.trip_info
    wd.close()


def test_nvtx_ranges(monkeypatch):
    import torch

    calls = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda n: calls.append(("push", n)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append(("pop",)))
    tracing.set_enabled(False)
    with tracing.nvtx("off"):
        pass
    assert calls == []
    tracing.set_enabled(True)
    try:
        with tracing.nvtx("layer0"):
            tracing.push("attn")
            tracing.pop()
    finally:
        tracing.set_enabled(None)
    assert calls == [("push", "layer0"), ("push", "attn"), ("pop",), ("pop",)]
