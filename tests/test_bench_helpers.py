"""Host-side helpers of ``bench.py``: clock sampling (against a fake ``nvidia-smi``) and the per-phase binning."""
import importlib.util
import os
import stat
import time
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_module", str(ROOT / "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_sampler_reads_a_query_loop(tmp_path, monkeypatch, bench):
    fake = tmp_path / "nvidia-smi"
    fake.write_text(
        "#!/usr/bin/env bash\n"
        "echo '2026/01/02 03:04:05.250, 1400, 1965, 990.5, Not Active, Not Active, Not Active, Active'\n"
        "echo '2026/01/02 03:04:05.450, 1500, 1965, 1001.0, Not Active, Not Active, Not Active, Active'\n"
        "echo 'garbage line'\n"
        "echo '2026/01/02 03:04:05.650, 1450, 1965, 998.0, Not Active, Not Active, Not Active, Not Active'\n"
        "sleep 30\n"
    )
    fake.chmod(fake.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    sampler = bench.ClockSampler(0)
    sampler.start()
    time.sleep(1.0)
    got = sampler.stop()
    assert got == {"sm_mhz": 1450.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    assert [round(b[0] - sampler.samples[0][0], 3) for b in sampler.samples] == [0.0, 0.2, 0.4] and sampler.samples[1][1:] == (1500.0, 1001.0)


def test_samples_are_binned_by_device_phase(bench):
    t0 = 1000.0
    samples = [(t0 + 0.1, 1500.0, 900.0), (t0 + 0.3, 1480.0, 950.0), (t0 + 0.5, 1400.0, 1000.0), (t0 + 0.7, 1380.0, 1000.0),
               (t0 + 0.9, 1390.0, 1000.0), (t0 + 1.1, 1490.0, 940.0), (t0 + 5.0, 1000.0, 100.0), (t0 - 1.0, 900.0, 90.0)]
    # forward 0-400 ms, backward 400-1000 ms, forward again 1000-1200 ms; samples outside every phase are dropped
    bounds = [("forward", 0.0, 400.0), ("backward", 400.0, 1000.0), ("forward", 1000.0, 1200.0)]
    got = bench.clocks_by_phase(samples, t0, bounds)
    assert got["forward"] == {"sm_mhz": 1490.0, "power_w": 940.0, "samples": 3}
    assert got["backward"] == {"sm_mhz": 1390.0, "power_w": 1000.0, "samples": 3}
    assert bench.clocks_by_phase([], t0, bounds) == {}
