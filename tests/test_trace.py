"""Per-request stage timeline helper (OMNI_TRACE)."""
import time

from sglang_omni_b200.utils import trace


def test_trace_marks_first_event_and_medians(monkeypatch):
    monkeypatch.setattr(trace, "ENABLED", True)
    trace.clear()
    for i in range(3):
        rid = f"s-0-{i}"
        trace.mark(rid, "a")
        time.sleep(0.002)
        trace.mark(rid, "b")
        trace.mark(rid, "b")          # only the first occurrence counts
    trace.mark("other-1", "a")
    s = trace.summary("s-0-")
    assert list(s) == ["a", "b"] and s["a"] == 0.0 and s["b"] >= 2.0
    trace.batch("enc", 4, 0.01)
    assert trace.batches()[-1] == ("enc", 4, 0.01)
    trace.clear()


def test_trace_disabled_is_noop(monkeypatch):
    monkeypatch.setattr(trace, "ENABLED", False)
    trace.clear()
    trace.mark("x", "a")
    assert trace.summary() == {}
