"""bench.py's host-side helpers (no GPU): the roofline denominator choice."""
import bench

PEAKS = {"burst": 1700.0, "sustained": 1400.0}


def test_burst_without_power_cap():
    c = {"reasons": [], "sm_mhz": 1965, "sm_max_mhz": 1965}
    assert bench.choose_peak(PEAKS, 5.0, c)[1] == "burst"
    assert bench.choose_peak(PEAKS, 0.01, None)[1] == "burst"


def test_sustained_when_the_cap_holds_the_clock_down():
    # a short region whose samples show the cap at a low median clock
    c = {"reasons": ["sw_power_cap"], "sm_mhz": 1440, "sm_max_mhz": 1965}
    peak, kind, why = bench.choose_peak(PEAKS, 0.585, c)
    assert (peak, kind) == (1400.0, "sustained") and "1440" in why
    # a long capped region
    c = {"reasons": ["sw_power_cap"], "sm_mhz": 1900, "sm_max_mhz": 1965}
    assert bench.choose_peak(PEAKS, 2.0, c)[1] == "sustained"


def test_burst_when_the_cap_flickers_at_full_clock():
    c = {"reasons": ["sw_power_cap"], "sm_mhz": 1950, "sm_max_mhz": 1965}
    assert bench.choose_peak(PEAKS, 0.01, c)[1] == "burst"
