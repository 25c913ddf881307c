"""CPU: the bench's NVML clock record (bench.ClockSampler), fed a poller log
written by the test instead of a live NVML poller.  The bench line's `clocks`
object is how a run shows that no throttling (hw_slowdown, thermal) and no
leftover clock lock affected the timed region."""
from __future__ import annotations

import ast
import importlib.util
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    if "bench" in sys.modules:
        return sys.modules["bench"]
    spec = importlib.util.spec_from_file_location("bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["bench"] = mod
    spec.loader.exec_module(mod)
    return mod


class _Done:
    """Stands in for the poller process: already finished."""

    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def _sampler(tmp_path, lines, t0, max_mhz=1965):
    cs = _bench().ClockSampler.__new__(_bench().ClockSampler)
    path = tmp_path / "poll.clocks"
    path.write_text("ready %d\n" % max_mhz + "".join(f"{t} {mhz} {reasons} {mw}\n" for t, mhz, reasons, mw in lines))
    cs.path = str(path)
    cs.fh = open(path, "a")
    cs.proc = _Done()
    cs.error = None
    cs.max_mhz = max_mhz
    cs.t0 = t0
    return cs


def test_poller_script_parses():
    ast.parse(_bench()._CLOCK_POLLER)


def test_samples_inside_the_region(tmp_path, monkeypatch):
    import time
    now = time.time_ns()
    lines = [(now - 5_000_000, 1500, 0, 200000)] + [(now + i * 200_000, 1965, 0x4, 300000) for i in range(5)]
    cs = _sampler(tmp_path, lines, now)
    monkeypatch.setattr(_bench().time, "time_ns", lambda: now + 1_000_000)
    out = cs.stop()
    assert out["samples"] == 5 and out["sm_mhz"] == 1965 and out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"] and out["power_w_max"] == 300.0
    assert "inside the timed region" in out["source"]


def test_short_region_takes_the_bracketing_polls(tmp_path, monkeypatch):
    now = 10_000_000_000
    lines = [(now - 300_000_000, 1965, 0, 250000), (now + 2_000_000 + 400_000_000, 1950, 0x8, 260000)]
    cs = _sampler(tmp_path, lines, now)
    monkeypatch.setattr(_bench().time, "time_ns", lambda: now + 2_000_000)
    out = cs.stop()
    assert out["samples"] == 2 and out["reasons"] == ["hw_slowdown"]
    assert "bracketing" in out["source"] and "400.0 ms away" in out["source"]


def test_no_polls_at_all_says_unavailable(tmp_path, monkeypatch):
    now = 10_000_000_000
    cs = _sampler(tmp_path, [], now)
    monkeypatch.setattr(_bench().time, "time_ns", lambda: now + 2_000_000)
    assert "unavailable" in cs.stop()
