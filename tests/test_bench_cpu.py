"""Host logic of bench.py without a GPU: the clock record taken during the timed region (median SM
clock, throttle reasons that make a run invalid) and the workload both arms name."""
import bench


def _line(sm, mx, hw="Not Active", hw_th="Not Active", sw_th="Not Active", cap="Not Active"):
    active = "0x0000000000000004" if cap == "Active" else "0x0000000000000000"
    return f"0, {sm}, {mx}, 812.40, {active}, {hw}, {hw_th}, {sw_th}, {cap}"


def _summary(lines):
    s = bench.ClockSampler(0)
    s.lines = lines
    return s.summary()


def test_clock_summary_median_and_reasons():
    lines = [_line(1965, 1965), _line(1777, 1965, cap="Active"), _line(1800, 1965, cap="Active"),
             "garbage line", _line("[N/A]", 1965)]
    s = _summary(lines)
    assert s["samples"] == 3 and s["sm_mhz"] == 1800.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]


def test_clock_summary_reports_every_slowdown_reason():
    s = _summary([_line(1200, 1965, hw="Active", hw_th="Active", sw_th="Active")])
    assert s["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]


def test_clock_summary_without_samples():
    s = _summary([])
    assert s["sm_mhz"] is None and s["samples"] == 0 and s["reasons"] == []


def test_both_arms_name_the_same_workload_and_context():
    for cfg, ctx in (("mistral-7b", 4096), ("llama-70b", 8192), ("tiny", 1024)):
        bench.PROMPT_LEN, bench.DECODE_LEN = bench.WORKLOADS[cfg]
        name = bench.workload_name(cfg)
        assert name.startswith(cfg) and f"{bench.PROMPT_LEN}-token prompt" in name
        assert bench.context_of(cfg) == ctx
    bench.PROMPT_LEN, bench.DECODE_LEN = bench.WORKLOADS["mistral-7b"]
    assert bench.workload_name("mistral-7b") == "mistral-7b batch-1 decode: 16-token prompt, decode positions 16..135"


def test_yalm_generation_stats_definition():
    """yalm's throughput (src/main.cpp:195-206): all tokens of the sequence over hydrate + decode."""
    s = bench.yalm_generation_stats(16, 120, 0.5, 0.01)
    assert s == {"tokens": 136, "hydrate_s": 0.5, "total_s": 1.7, "throughput_tok_s": 80.0}


def test_clock_sampler_waits_for_its_first_sample_and_keeps_one_for_short_regions(tmp_path, monkeypatch):
    """A fake nvidia-smi that starts slowly and prints a sample every 50 ms: the timed region opens
    only after the first sample, and a region shorter than the sampling period still records the
    first sample after it."""
    import os
    import time
    fake = tmp_path / "nvidia-smi"
    fake.write_text("#!/bin/sh\nsleep 0.3\nwhile true; do echo '0, 1965, 1965, 700.0, 0x0, Not Active, "
                    "Not Active, Not Active, Not Active'; sleep 0.05; done\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    t = time.monotonic()
    with bench.ClockSampler(0) as c:
        assert time.monotonic() - t >= 0.25  # waited for the sampler to start
    s = c.summary()
    assert s["samples"] >= 1 and s["sm_mhz"] == 1965.0 and s["reasons"] == []
    with bench.ClockSampler(0) as c:
        time.sleep(0.3)
    assert c.summary()["samples"] >= 3
