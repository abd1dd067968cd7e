"""Host side of the step graphs' capture guard (pagedcore_b200.graph._capturing).

A CUDA graph dropped in a reference cycle is destroyed whenever Python's
cycle collector runs; during a capture that destroy would invalidate the
capture.  The guard collects first, keeps automatic collection off for the
capture and restores the caller's setting afterwards, also when the capture
raises.  CUDA's capture itself is replaced by a recording stand-in here; the
GPU test of the same guard is tests/test_graph_gpu.py.
"""

from __future__ import annotations

import contextlib
import gc

import pytest

from pagedcore_b200 import graph


@pytest.fixture
def capture_log(monkeypatch):
    log = []

    @contextlib.contextmanager
    def fake_graph(cuda_graph, stream=None, capture_error_mode="global"):
        log.append(("begin", capture_error_mode, gc.isenabled()))
        yield
        log.append(("end", gc.isenabled()))

    monkeypatch.setattr(graph.torch.cuda, "graph", fake_graph)
    return log


def test_capture_runs_thread_local_with_the_collector_off_then_restores_it(capture_log) -> None:
    assert gc.isenabled()
    with graph._capturing(object(), object()):
        assert not gc.isenabled()
    assert gc.isenabled()
    assert capture_log == [("begin", "thread_local", False), ("end", False)]


def test_collector_is_restored_when_the_capture_raises(capture_log) -> None:
    with pytest.raises(RuntimeError, match="launch failed"):
        with graph._capturing(object(), object()):
            raise RuntimeError("launch failed")
    assert gc.isenabled()


def test_a_caller_that_disabled_the_collector_keeps_it_disabled(capture_log) -> None:
    gc.disable()
    try:
        with graph._capturing(object(), object()):
            pass
        assert not gc.isenabled()
    finally:
        gc.enable()


def test_dead_cycles_are_collected_before_the_capture_begins(capture_log) -> None:
    import weakref

    class Holder:
        pass

    holder = Holder()
    ref = weakref.ref(holder)
    cycle = [holder]
    cycle.append(cycle)
    del holder, cycle
    threshold = gc.get_threshold()
    gc.set_threshold(0)  # no automatic collection: only the guard's own collects
    try:
        assert ref() is not None
        with graph._capturing(object(), object()):
            assert ref() is None
    finally:
        gc.set_threshold(*threshold)
