"""bench.py's clock record, on the CPU with a stand-in nvidia-smi on PATH:
the sampler returns only once the first sample is written (nvidia-smi is
slow to start), keeps the samples from the timed region on, and reports the
throttle reasons that are active in them."""
import importlib.util
import os
import time

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROW = "0, {mhz}, 1965, 700.0, 0x0, {hw}, Not Active, Not Active, {cap}"


def load_bench():
    spec = importlib.util.spec_from_file_location("f5_bench", os.path.join(os.path.dirname(HERE), "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture
def fake_smi(tmp_path, monkeypatch):
    """Writes a stand-in nvidia-smi that starts after 0.3 s, prints one idle
    row, then busy rows every 20 ms (rows given by the test)."""
    def make(first, busy):
        p = tmp_path / "nvidia-smi"
        p.write_text("#!/bin/bash\nsleep 0.3\n"
                     f"echo '{first}'\n"
                     f"while true; do echo '{busy}'; sleep 0.02; done\n")
        p.chmod(0o755)
        monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    return make


def test_sampler_waits_for_nvidia_smi_and_drops_the_idle_row(fake_smi):
    b = load_bench()
    fake_smi(ROW.format(mhz=345, hw="Not Active", cap="Not Active"),
             ROW.format(mhz=1965, hw="Not Active", cap="Active"))
    c = b.ClockSampler(0)
    c.start()                      # returns after the idle row is written
    time.sleep(0.03)               # a timed region shorter than 2 samples
    r = c.stop()
    assert r["samples"] >= 2
    assert r["sm_mhz"] == 1965.0 and r["sm_max_mhz"] == 1965.0
    assert r["reasons"] == ["sw_power_cap"]


def test_sampler_reports_a_slowdown(fake_smi):
    b = load_bench()
    fake_smi(ROW.format(mhz=1965, hw="Not Active", cap="Not Active"),
             ROW.format(mhz=1200, hw="Active", cap="Not Active"))
    c = b.ClockSampler(0)
    c.start()
    r = c.stop()
    assert r["sm_mhz"] == 1200.0 and r["reasons"] == ["hw_slowdown"]


def test_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    b = load_bench()
    monkeypatch.setenv("PATH", str(tmp_path))   # no nvidia-smi anywhere
    c = b.ClockSampler(0)
    c.start()
    assert c.stop()["reasons"] == ["nvidia-smi unavailable"]
