"""The bench's clock record on CPU: a stand-in for nvidia-smi prints one
sample every 50 ms after a start-up delay; the sampler keeps only the samples
that arrive inside the timed block and reports the throttle reasons seen."""
import sys
import time

import bench

LINE = "0, {mhz}, 1965, 700.0, 0x0, {hw}, Not Active, Not Active, {cap}"


def fake(delay, n, hw="Not Active", cap="Not Active", start=1900):
    code = ("import time\n"
            f"time.sleep({delay})\n"
            f"for i in range({n}):\n"
            f"    print({LINE!r}.format(mhz={start} + i, hw={hw!r}, cap={cap!r}), flush=True)\n"
            "    time.sleep(0.05)\n")
    return [sys.executable, "-c", code]


def test_samples_only_inside_the_timed_block():
    with bench.ClockSampler(0, cmd=fake(0.3, 100)) as c:
        time.sleep(0.25)
    summ = c.summary()
    # the first sample (1900) arrives before the block starts and is not counted
    assert 3 <= summ["samples"] <= 8
    assert summ["sm_mhz"] > 1900 and summ["sm_max_mhz"] == 1965
    assert summ["reasons"] == []


def test_reports_throttle_reasons():
    with bench.ClockSampler(0, cmd=fake(0.0, 100, hw="Active", cap="Active")) as c:
        time.sleep(0.15)
    assert c.summary()["reasons"] == ["hw_slowdown", "sw_power_cap"]


def test_no_sampler_available():
    with bench.ClockSampler(0, cmd=["/nonexistent/nvidia-smi"]) as c:
        pass
    assert c.summary()["sm_mhz"] is None and c.summary()["samples"] == 0
