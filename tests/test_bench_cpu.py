"""bench.py host logic that needs no GPU: the reference arm's JSON line, and the clock sampler that
records SM clocks and throttle reasons during the timed region, driven here by a stand-in `nvidia-smi`
on PATH."""

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


def test_reference_arm_prints_the_contract_line(monkeypatch, capsys) -> None:
    """`bench.py --impl reference` on a stand-in config small enough for a CPU test (the real ones take
    seconds per pair): one JSON line with the keys and units the bench contract asks of the reference arm,
    its `config` object identical to the GPU arm's, and the CPU work actually timed."""
    import argparse
    import json

    import bench

    monkeypatch.setitem(bench.CONFIGS, "tiny", (1, 4, 48, 16, True))
    monkeypatch.setattr(bench.os, "cpu_count", lambda: 2)
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    bench.run_reference(argparse.Namespace(config="tiny", steps=2, warmup=1))
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "impl", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):  # fmt: skip
        assert key in line, key
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == "TFLOP/s" and line["higher_is_better"] is True
    assert line["n_gpus"] == 1 and line["steps"] == 2 and line["warmup"] == 1
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert line["config"] == bench.config_dict("tiny", 1)
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["unit"] == "TFLOP/s" and cb["cores"] == 2 and cb["kind"] == "port"
    assert cb["sample"]
    e2e = line["e2e"]
    assert e2e == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_is_rank_zero_only(monkeypatch, capsys) -> None:
    """Under torchrun every rank but 0 exits without work or output."""
    import argparse

    import bench

    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    bench.run_reference(argparse.Namespace(config="cfg5", steps=20, warmup=5))
    assert capsys.readouterr().out == ""
