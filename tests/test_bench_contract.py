"""Host-side pieces of bench.py that decide what its JSON line says (no GPU needed):
the throttle-reason decoding of the clock sampler, the roofline denominators, and
the fixed keys of a result line."""

import json

import bench


def _sampler_with(samples):
    s = bench.ClockSampler.__new__(bench.ClockSampler)  # no NVML, no thread
    s.samples = samples
    s.max_mhz = 1965
    s._t = None
    s._stop = bench.threading.Event()
    return s


def test_clock_reasons_are_decoded_and_idle_is_dropped():
    sw_power_cap, hw_slowdown, idle = 0x4, 0x8, 0x1
    out = _sampler_with([(0.0, 1900, sw_power_cap | idle), (0.1, 1950, 0), (0.2, 1800, hw_slowdown)]).stop()
    assert out == {"sm_mhz": 1900, "sm_max_mhz": 1965, "reasons": ["hw_slowdown", "sw_power_cap"], "samples": 3}


def test_thermal_reasons_have_their_nvml_bits():
    names = bench.ClockSampler.REASONS
    assert names[0x20] == "sw_thermal_slowdown" and names[0x40] == "hw_thermal_slowdown"
    out = _sampler_with([(0.0, 1965, 0x20 | 0x40)]).stop()
    assert out["reasons"] == ["hw_thermal_slowdown", "sw_thermal_slowdown"]


def test_no_samples_reports_none():
    assert _sampler_with([]).stop()["sm_mhz"] is None


def test_peaks_have_the_denominators_the_roofline_uses():
    peaks = bench.load_peaks()
    assert peaks["source"] in ("measured", "fallback")
    for key in ("hbm_gbs", "bf16_tflops"):
        assert float(peaks[key]) > 0


def test_result_line_carries_the_contract_keys(capsys):
    bench._line("m", 1.0, "tokens/s", 5, 3, 2.0, True, "bf16", {"workload": "w"}, gpu_launches=7)
    d = json.loads(capsys.readouterr().out.strip())
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d
    assert d["gpu_launches"] == 7 and d["config"] == {"workload": "w"}


def test_peak_choice_follows_the_sampled_clocks():
    peaks = {"bf16_tflops": 1649.3, "bf16_tflops_sustained": 1394.0}
    short_at_max = bench.choose_peak(peaks, {"sm_mhz": 1965, "sm_max_mhz": 1965}, 0.17)
    assert short_at_max["kind"] == "burst" and short_at_max["value"] == 1649.3
    long_region = bench.choose_peak(peaks, {"sm_mhz": 1965, "sm_max_mhz": 1965}, 4.0)
    assert long_region["kind"] == "sustained" and long_region["value"] == 1394.0
    capped = bench.choose_peak(peaks, {"sm_mhz": 1400, "sm_max_mhz": 1965}, 0.2)
    assert capped["kind"] == "sustained"
    unknown = bench.choose_peak(peaks, {"sm_mhz": None, "sm_max_mhz": None}, 0.2)
    assert unknown["kind"] == "sustained" and unknown["burst"] == 1649.3


def test_gate_up_traffic_names_the_capture_it_came_from():
    for cap in bench.GATE_UP_DRAM_CAPTURE.values():
        assert cap["bytes"] > 0 and "commit" in cap["source"] and "profiles/" in cap["source"]
