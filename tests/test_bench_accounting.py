"""CPU checks of bench.py's accounting: the algorithmic FLOPs per chunk that the
roofline divides by, for every workload, against per-config figures worked out
independently from the model shapes (PR1 0.23, Std 3.11, two-stem 6.21, Large
18.6, R0 7.05 TFLOP per chunk), and
the clock sampler's reading of nvidia-smi's CSV (the throttle reasons decide
whether a bench line is kept)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "mbr-cuda-tile_b200"))


@pytest.mark.parametrize("workload,tflop,frames", [("pr1", 0.23, 801), ("std", 3.11, 801), ("two_stem", 6.21, 801),
                                                   ("large", 18.6, 1101), ("r0", 7.05, 1301)])
def test_flops_per_chunk(workload, tflop, frames):
    import bench
    import csm_tool

    wl = bench.WORKLOADS[workload]
    cfg = csm_tool.base_config(**csm_tool.PRESETS[wl["preset"]])
    T = cfg["chunk_size"] // cfg["stft_hop_length"] + 1
    assert T == frames
    f = bench.model_flops(cfg, T, 1, bench.band_dims(cfg))
    assert abs(sum(f.values()) / 1e12 - tflop) <= 0.01 * tflop
    # the time attention term alone: 4 T^2 dh H per sequence, one sequence per band and chunk
    Lt = cfg["depth"] * cfg["time_transformer_depth"]
    assert f["attn_time"] == Lt * 4.0 * T * T * cfg["dim_head"] * cfg["heads"] * cfg["num_bands"]


def test_clock_sampler_reasons():
    import bench

    cs = bench.ClockSampler(0)
    cs.lines = [
        "0, 1717, 1965, 990.1, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1740, 1965, 995.0, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1700, 1965, 1000.2, 0x4, Not Active, Not Active, Not Active, Not Active",
    ]
    s = cs.summary()
    assert s["sm_mhz"] == 1717.0 and s["sm_max_mhz"] == 1965.0 and s["reasons"] == ["sw_power_cap"]
    cs.lines = ["0, 1200, 1965, 700.0, 0x40, Not Active, Active, Not Active, Not Active"]
    assert cs.summary()["reasons"] == ["hw_thermal_slowdown"]
    cs.lines = []
    assert cs.summary()["reasons"] == ["unsampled"]
