"""bench.py's pure-Python decisions, on the CPU: which bf16 peak the GEMM
roofline is measured against, and which reassembly path value_with_gather
reports."""
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

import bench  # noqa: E402

PEAKS = {"hbm_gbs": 6455.6, "bf16_tflops": 1708.2, "bf16_tflops_sustained": 1414.4}


def test_roofline_peak_burst_at_full_clock():
    clk = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []}
    assert bench.roofline_peak(PEAKS, clk) == (1708.2, False)


def test_roofline_peak_sustained_under_power_cap():
    clk = {"sm_mhz": 1432.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}
    assert bench.roofline_peak(PEAKS, clk) == (1414.4, True)


def test_roofline_peak_needs_both_low_clock_and_power_cap():
    # cap flagged but clock at maximum; low clock without the cap (a lock,
    # rejected by the timing rules rather than re-based)
    assert bench.roofline_peak(PEAKS, {"sm_mhz": 1960.0, "sm_max_mhz": 1965.0,
                                       "reasons": ["sw_power_cap"]})[1] is False
    assert bench.roofline_peak(PEAKS, {"sm_mhz": 1200.0, "sm_max_mhz": 1965.0, "reasons": []})[1] is False


def test_roofline_peak_without_clock_samples_or_sustained_figure():
    assert bench.roofline_peak(PEAKS, None) == (1708.2, False)
    assert bench.roofline_peak(PEAKS, {"sm_mhz": None, "sm_max_mhz": None,
                                       "reasons": ["nvidia-smi unavailable"]}) == (1708.2, False)
    only_burst = {"bf16_tflops": 1590.0}
    clk = {"sm_mhz": 1300.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}
    assert bench.roofline_peak(only_burst, clk) == (1590.0, True)


def test_best_path_ignores_paths_that_did_not_run():
    paths = {"ncclAllGather": 2.27, "fused": 1.68, "multicast": None, "copy_engines": 2.65}
    assert bench.best_path(paths) == "fused"
    assert bench.best_path({"ncclAllGather": 1.1, "fused": None}) == "ncclAllGather"
