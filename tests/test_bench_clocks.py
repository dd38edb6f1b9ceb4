"""The bench's clock sampler on the CPU, against a fake `nvidia-smi` that prints the
queried fields after a start-up delay longer than the timed regions below."""
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FAKE = """#!/bin/bash
sleep 0.4
while true; do
  echo "0, 1890, 1965, 612.5, 0x4, Not Active, Not Active, Not Active, Active"
  sleep 0.05
done
"""


def _sampler(tmp_path, monkeypatch):
    exe = tmp_path / 'nvidia-smi'
    exe.write_text(FAKE)
    exe.chmod(0o755)
    monkeypatch.setenv('PATH', f'{tmp_path}{os.pathsep}{os.environ["PATH"]}')
    sys.path.insert(0, ROOT)
    import bench
    return bench.ClockSampler


def test_region_shorter_than_start_up_still_gets_a_sample(tmp_path, monkeypatch):
    sampler = _sampler(tmp_path, monkeypatch)
    with sampler(0) as clocks:
        time.sleep(0.01)
    s = clocks.summary()
    assert s['samples'] >= 1
    assert s['sm_mhz'] == 1890.0 and s['sm_max_mhz'] == 1965.0
    assert s['reasons'] == ['sw_power_cap']


def test_longer_region_keeps_only_its_own_samples(tmp_path, monkeypatch):
    sampler = _sampler(tmp_path, monkeypatch)
    with sampler(0) as clocks:
        time.sleep(0.3)
    s = clocks.summary()
    # about one sample per 50 ms inside the region plus the one after it
    assert 3 <= s['samples'] <= 9


def test_missing_tool_reports_no_samples(tmp_path, monkeypatch):
    sys.path.insert(0, ROOT)
    import bench
    monkeypatch.setenv('PATH', str(tmp_path))
    with bench.ClockSampler(0) as clocks:
        pass
    assert clocks.summary() == dict(sm_mhz=None, sm_max_mhz=None, reasons=[], samples=0)
