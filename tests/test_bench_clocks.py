"""bench.py's clock sampler, against a fake nvidia-smi on PATH (no GPU needed).

The sampler must be running before a timed region starts, keep only the samples
written after `region_start()`, and report the throttle reasons it saw."""
import importlib.util
import os
import stat
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FAKE = """#!/bin/sh
# prints one sample every 20 ms: the first three at 1000 MHz (before the region), then 1900 MHz
n=0
while true; do
  if [ $n -lt 3 ]; then mhz=1000; else mhz=1900; fi
  echo "0, $mhz, 1965, 700.0, 0x4, Not Active, Not Active, Not Active, Active"
  n=$((n+1))
  sleep 0.02
done
"""


def _load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_sampler_keeps_region_samples(tmp_path, monkeypatch):
    fake = tmp_path / "nvidia-smi"
    fake.write_text(FAKE)
    fake.chmod(fake.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    bench = _load_bench()
    s = bench.ClockSampler("0")
    s.start()
    assert s._rows(), "start() returns only after the first sample"
    time.sleep(0.1)                       # past the three 1000 MHz samples
    s.region_start()
    time.sleep(0.15)                      # the timed region
    clk = s.stop()
    assert clk["samples"] >= 2
    assert clk["sm_mhz"] == 1900.0
    assert clk["sm_max_mhz"] == 1965.0
    assert clk["reasons"] == ["sw_power_cap"]


def test_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))
    bench = _load_bench()
    s = bench.ClockSampler("0")
    s.start()
    s.region_start()
    assert s.stop()["reasons"] == ["nvidia-smi unavailable"]
