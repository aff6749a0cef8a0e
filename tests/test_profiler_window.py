"""The CUDA profiler step window (MINISGL_CUDA_PROFILER_STEPS=a:b): parsing,
and start / stop placement over scheduler steps, with recording fakes in
place of cudaProfilerStart / Stop."""

import pytest

from minisgl.scheduler.profile import CudaProfilerWindow, parse_step_window


def test_parse_step_window():
    assert parse_step_window("") is None and parse_step_window("  ") is None
    assert parse_step_window("3:7") == (3, 7)
    for bad in ("5", "7:3", "2:2", "-1:4", "a:b", "1:2:3"):
        with pytest.raises(ValueError):
            parse_step_window(bad)


def test_window_brackets_steps():
    calls = []
    w = CudaProfilerWindow((2, 5), start=lambda: calls.append("start"), stop=lambda: calls.append("stop"),
                           sync=lambda: calls.append("sync"))
    seen = []
    for step in range(8):
        w.on_step(step)
        seen.append((step, w.active))
        calls.append(step)
    # started before the forward of step 2, stopped (after a sync) before step 5
    assert calls == [0, 1, "start", 2, 3, 4, "sync", "stop", 5, 6, 7]
    assert [s for s, active in seen if active] == [2, 3, 4]


def test_window_never_reached():
    calls = []
    w = CudaProfilerWindow((10, 12), start=lambda: calls.append("start"), stop=lambda: calls.append("stop"),
                           sync=lambda: None)
    for step in range(5):
        w.on_step(step)
    assert calls == [] and not w.active
