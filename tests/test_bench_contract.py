"""The benchmark's JSON contract on the CPU: the reference arm's line (run as
the driver runs it, without the product library), the rank-sum choice of
``--reduce auto`` and the clock sampler's timed-region window (against a
fake NVML)."""
import json
import os
import subprocess
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402

REQUIRED = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
            "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config")

# Runs the reference arm in a fresh interpreter, then reports whether the
# product library was ever mapped into that process.
_DRIVER = r"""
import json, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"]
sys.path.insert(0, {root!r})
import bench
bench.main()
maps = open("/proc/self/maps").read()
print(json.dumps({{"product_mapped": "libgdn_b200" in maps}}))
"""


def test_reference_arm_line_and_no_product_library():
    r = subprocess.run([sys.executable, "-c", _DRIVER.format(root=ROOT)], cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
    line, probe = lines[0], lines[-1]
    assert not probe["product_mapped"]
    for key in REQUIRED:
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["unit"] == bench.UNIT and line["metric"] == bench.METRIC
    assert line["value"] > 0 and line["higher_is_better"] is True
    # Same configuration keys as the product arm on one GPU.
    assert line["config"] == bench.prefill_config(1, bench.resolve_reduce("auto", 1))
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["e2e"]["value"] == line["value"]


@pytest.mark.parametrize("gpus,want", [(1, "ce"), (2, "ce"), (4, "ce"), (8, "rs")])
def test_reduce_auto_choice(gpus, want):
    assert bench.resolve_reduce("auto", gpus) == want
    for explicit in ("ce", "fused", "nccl", "rs"):
        assert bench.resolve_reduce(explicit, gpus) == explicit


class _FakeNvml:
    NVML_CLOCK_SM = 0

    def __init__(self, mhz, reasons):
        self.mhz, self.reasons = mhz, reasons

    def nvmlDeviceGetMaxClockInfo(self, h, kind):
        return 1965

    def nvmlDeviceGetClockInfo(self, h, kind):
        return self.mhz

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return self.reasons


def test_clock_sampler_keeps_samples_of_the_timed_region(monkeypatch):
    fake = _FakeNvml(1900, 0x4)
    monkeypatch.setattr(bench.ClockSampler, "_nvml_handle", lambda self: (fake, object()))
    with bench.ClockSampler(0) as c:
        time.sleep(0.05)
    out = c.summary()
    assert out["source"] == "nvml, 2 ms"
    assert out["samples"] >= 3
    assert out["sm_mhz"] == 1900 and out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"]


def test_clock_sampler_samples_a_region_shorter_than_its_period(monkeypatch):
    fake = _FakeNvml(1965, 0)
    monkeypatch.setattr(bench.ClockSampler, "_nvml_handle", lambda self: (fake, object()))
    c = bench.ClockSampler(0)
    c.__enter__()
    c.samples.clear()          # as if the poller had not run inside the region
    c.stop.set()
    c.__exit__(None, None, None)
    out = c.summary()
    assert out["samples"] == 1 and out["sm_mhz"] == 1965 and out["reasons"] == []
