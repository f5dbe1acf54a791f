"""bench.py's clock sampler against a fake nvidia-smi (no GPU needed): samples
are host-stamped on arrival and only those inside the timed region count."""

import importlib.util
import os
import stat
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FAKE = """#!/bin/sh
i=0
while [ $i -lt 200 ]; do
  if [ $i -lt 8 ]; then
    echo "0, 1900, 1965, 300.0, 0x0, Not Active, Not Active, Not Active, Not Active"
  else
    echo "0, 1350, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active"
  fi
  echo "1, 1200, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, Not Active"
  i=$((i+1))
  sleep 0.05
done
"""


def _load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_sampler_keeps_timed_region_samples(tmp_path, monkeypatch):
    exe = tmp_path / "nvidia-smi"
    exe.write_text(FAKE)
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    bench = _load_bench()
    sampler = bench.ClockSampler([0])
    sampler.start()
    time.sleep(0.6)           # "warm-up": the idle samples at 1900 MHz arrive now
    sampler.mark_start()
    time.sleep(0.5)           # timed region
    sampler.mark_end()
    out = sampler.stop()
    assert out["samples"] >= 3
    assert out["sm_mhz"] == 1350.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]


def test_visible_gpu_indices(monkeypatch):
    bench = _load_bench()
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3,5")
    assert bench.visible_gpu_indices(2) == [3, 5]
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-abc")
    assert bench.visible_gpu_indices(2) == [0, 1]
