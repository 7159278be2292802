"""bench.py's timed region on CPU: what runs between the two CUDA events.

The events bracket exactly the K timed calls. The clock sampler's NVML queries run on its
own thread, started before the warm-up; inside the timed region the caller's thread only
flips its tag. A device-side lead (a short GPU spin) is enqueued before the start event so
that the host's launch of the first call is not timed either.
"""
import contextlib
import inspect

import pytest

import bench


class _Log(list):
    pass


@pytest.fixture
def fake_cuda(monkeypatch):
    import torch
    log = _Log()

    class FakeEvent:
        count = 0

        def __init__(self, enable_timing=False):
            FakeEvent.count += 1
            self.name = f"e{FakeEvent.count - 1}"

        def record(self, stream=None):
            log.append(f"record {self.name}")

        def synchronize(self):
            log.append(f"sync {self.name}")

        def elapsed_time(self, other):
            return 12.0

    monkeypatch.setattr(torch.cuda, "Event", FakeEvent)
    monkeypatch.setattr(torch.cuda, "_sleep", lambda cycles: log.append("lead"))
    monkeypatch.setattr(torch.cuda, "stream", lambda s: contextlib.nullcontext())
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda msg: None)
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: None)
    return log


class _FakeSampler:
    def __init__(self, log):
        self.log = log

    def start(self):
        self.log.append("sampler start")

    def enter(self, label="timed"):
        self.log.append("enter")

    def leave(self):
        self.log.append("leave")


def test_start_event_directly_precedes_the_timed_calls(fake_cuda):
    log = fake_cuda
    steps, warmup = 4, 3
    ms = bench.timed(lambda: log.append("call"), steps, warmup, stream=None,
                     barrier=lambda: log.append("barrier"), sampler=_FakeSampler(log))
    assert ms == 12.0 / steps
    expect = (["call"] * warmup + ["barrier", "enter", "lead", "record e0"] + ["call"] * steps
              + ["record e1", "sync e1", "leave", "barrier"])
    assert log == expect


def test_sampler_tagging_makes_no_nvml_query():
    calls = []

    class FakeNV:
        NVML_CLOCK_SM = 0

        def nvmlDeviceGetClockInfo(self, h, which):
            calls.append("clock")
            return 1965

        def nvmlDeviceGetCurrentClocksEventReasons(self, h):
            calls.append("reasons")
            return 0x4

    s = bench.ClockSampler.__new__(bench.ClockSampler)
    s.samples, s.max_mhz, s.period, s.region = [], 1965, 0.001, None
    s.nv, s.h = FakeNV(), object()
    import threading
    s._stop, s._thread = threading.Event(), None
    s.enter()
    s.leave()
    assert calls == []  # the timed region's own thread never talks to NVML
    s.enter("b200")
    s.start()
    import time
    t0 = time.time()
    while not any(x[2] for x in s.samples) and time.time() - t0 < 5:
        time.sleep(0.005)
    s.leave()
    s.stop()
    summ = s.summary("b200")
    assert summ["sm_mhz"] == 1965 and summ["reasons"] == ["sw_power_cap"]
    assert summ["window"] == "timed region 'b200'"


def test_run_b200_starts_the_sampler_before_its_first_timed_block():
    src = inspect.getsource(bench.run_b200)
    assert src.index("sampler.start()") < src.index("run_timed(step")
    assert "sampler.start()" not in inspect.getsource(bench.timed)
