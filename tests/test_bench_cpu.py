"""bench.py host logic that needs no GPU: the clock sampler that records SM clocks and throttle reasons
during the timed region, driven here by a stand-in `nvidia-smi` on PATH."""

from __future__ import annotations

import os
import stat
import sys
import textwrap

FAKE_SMI = textwrap.dedent(
    """\
    #!{python}
    import sys, time
    time.sleep({delay})  # a slow start, as nvidia-smi has while it loads NVML
    while True:
        print("0, 1965, 1965, 612.5, 0x0000000000000004, Not Active, Not Active, Not Active, {cap}", flush=True)
        time.sleep(0.05)
    """
)


def _fake_smi(tmp_path, monkeypatch, delay: float, cap: str) -> None:
    path = tmp_path / "nvidia-smi"
    path.write_text(FAKE_SMI.format(python=sys.executable, delay=delay, cap=cap))
    path.chmod(path.stat().st_mode | stat.S_IXUSR)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")


def test_short_timed_region_still_gets_a_sample(tmp_path, monkeypatch) -> None:
    """A timed region shorter than the sampling period (and than nvidia-smi's start-up) still reports
    the clock: entering waits for the first sample, leaving waits for one more."""
    import bench

    _fake_smi(tmp_path, monkeypatch, delay=0.3, cap="Not Active")
    with bench.ClockSampler(0) as clk:
        pass  # an empty timed region
    s = clk.summary()
    assert s["samples"] >= 1
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == []


def test_throttle_reasons_are_reported(tmp_path, monkeypatch) -> None:
    import bench

    _fake_smi(tmp_path, monkeypatch, delay=0.0, cap="Active")
    with bench.ClockSampler(0) as clk:
        import time

        time.sleep(0.2)
    s = clk.summary()
    assert s["samples"] >= 2
    assert s["reasons"] == ["sw_power_cap"]


def test_missing_nvidia_smi_gives_an_empty_summary(tmp_path, monkeypatch) -> None:
    import bench

    monkeypatch.setenv("PATH", str(tmp_path))
    with bench.ClockSampler(0) as clk:
        pass
    assert clk.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
