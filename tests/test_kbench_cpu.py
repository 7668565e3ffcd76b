"""Host logic of the kernel sweep (yalm_b200/kbench.py) without a GPU: the timing bookkeeping runs
against a stand-in CUDA clock in which every launch advances the device time by a planted
duration, so the mean and the per-launch percentiles it reports can be checked exactly."""
import numpy as np
import pytest


@pytest.fixture
def fake_cuda(monkeypatch):
    import torch
    clock = {"t": 0.0, "spins": []}

    class Event:
        def __init__(self, enable_timing=True):
            self.t = None

        def record(self, stream=None):
            self.t = clock["t"]

        def synchronize(self):
            pass

        def elapsed_time(self, other):
            return other.t - self.t

    def sleep(cycles):
        clock["spins"].append(cycles)
        clock["t"] += 7.0  # the spin's own time lies before the first event of a pass

    monkeypatch.setattr(torch.cuda, "Event", Event)
    monkeypatch.setattr(torch.cuda, "_sleep", sleep)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    return clock


def test_mean_and_percentiles_from_planted_durations(fake_cuda):
    from yalm_b200 import kbench
    planted = np.tile([0.010, 0.012, 0.020, 0.011], 50)  # ms per launch, cycled
    it = iter(planted)
    calls = []

    def launch(i):
        calls.append(i)
        fake_cuda["t"] += next(it)

    ms = kbench._time(launch, 40, warm=2)
    # 2 warm-up launches, then two timed passes of 40
    assert calls == [0, 1] + list(range(40)) + list(range(40))
    # the mean pass covers planted[2:42]; the percentile pass planted[42:82]
    assert ms == pytest.approx(planted[2:42].mean(), abs=1e-12)
    per = planted[42:82] * 1000.0
    for q in (10, 50, 90):
        assert kbench._LAST_SPREAD[f"p{q}_us"] == pytest.approx(round(float(np.percentile(per, q)), 2))
    # each pass is queued behind one spin sized for its launches
    assert fake_cuda["spins"] == [60_000 * 40, 60_000 * 40]


def test_warm_up_count_follows_the_command_line(fake_cuda):
    from yalm_b200 import kbench
    calls = []

    def launch(i):
        calls.append(i)
        fake_cuda["t"] += 0.005

    saved = kbench._WARM
    try:
        kbench._WARM = 0
        kbench._time(launch, 1)
        assert calls == [0]  # no warm-up, and one timed pass below 3 launches (no percentiles)
        assert kbench._LAST_SPREAD == {}
        calls.clear()
        kbench._WARM = 3
        kbench._time(launch, 3)
        assert calls == [0, 1, 2, 0, 1, 2, 0, 1, 2]
        assert set(kbench._LAST_SPREAD) == {"p10_us", "p50_us", "p90_us"}
    finally:
        kbench._WARM = saved
