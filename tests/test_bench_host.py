"""bench.py host logic on CPU: the clock record summary (median SM clock,
throttle reasons from the event-reason bit mask), the roofline's choice of
bound, and the per-call kernel counts it claims for the topology entry
points."""
import os
import sys

import pytest
import torch

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _sampler(tmp_path, lines):
    s = bench.ClockSampler(0)
    s.proc = object()  # as if nvidia-smi ran
    s.path = str(tmp_path / "clocks.csv")
    with open(s.path, "w") as f:
        f.write("\n".join(lines) + "\n")
    return s


def test_clock_summary_median_and_reasons(tmp_path):
    s = _sampler(tmp_path, ["1965, 1965, 700.1, 0x0000000000000000",
                            "1950, 1965, 990.0, 0x0000000000000004",
                            "1965, 1965, 800.0, 0x0000000000000001",
                            "not a sample line"])
    out = s.summary()
    assert out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0 and out["samples"] == 3
    assert out["reasons"] == ["sw_power_cap"]          # gpu_idle is not a throttle reason


def test_clock_summary_reports_thermal_and_hw_slowdown(tmp_path):
    s = _sampler(tmp_path, ["1200, 1965, 1000.0, 0x0000000000000048"])
    assert s.summary()["reasons"] == ["hw_slowdown", "hw_thermal_slowdown"]


def test_clock_summary_without_samples(tmp_path):
    out = _sampler(tmp_path, []).summary()
    assert out["sm_mhz"] is None and out["samples"] == 0


def test_conv_roofline_picks_the_slower_bound():
    n, cin, cout = 1000, 64, 64
    nbr = torch.full((n, 27), n, dtype=torch.int32)
    nbr[:, 13] = torch.arange(n, dtype=torch.int32)          # centre tap only: E = n
    state = {"nbr": nbr}
    prof = {"conv": (2, 0.02)}                               # 10 us per launch
    # a huge tensor peak: the compulsory bytes bound the launch
    r = bench.conv_roofline(prof, "conv", cin, cout, state, n, 108, 0, "f32", 1e9, 1000.0, "measured", 3)
    alg = n * (cin * 4 + cout * 4 + 108) + 27 * cin * cout * 4
    assert r["bound"] == "hbm" and r["algorithmic_bytes_per_launch"] == alg
    assert r["achieved"] == pytest.approx(alg / 10e-6 / 1e9)
    assert r["frac"] == pytest.approx(r["achieved"] / 1000.0)
    # a tiny tensor peak: the flops bound it, against the peak per issued MMA
    r = bench.conv_roofline(prof, "conv", cin, cout, state, n, 108, 0, "f32", 1e-3, 1e9, "measured", 3)
    assert r["bound"] == "tensor" and r["flops_per_launch"] == 2.0 * cin * cout * n
    assert r["peak"] == pytest.approx(1e-3 / 3)
    # no launches recorded: no roofline
    assert bench.conv_roofline({}, "conv", cin, cout, state, n, 108, 0, "f32", 1.0, 1.0, "m", 1)["bound"] is None


def test_topology_kernel_counts_match_the_launch_code():
    """Kernels per call as launched by csrc/topology.cu: voxel table 4, the
    neighbour map 1 + 3 per-voxel fallbacks, the stride-2 maps 10 (9 when the
    neighbour kernel has done the first-child scan)."""
    src = open(os.path.join(ROOT, "mogecpp_b200", "csrc", "topology.cu")).read()

    def launches(fn):
        body = src[src.index(fn):]
        body = body[:body.index("\n}\n")]
        return body.count("<<<")
    build, mp, s2 = launches("cudaError_t launch_brick_build("), launches("cudaError_t launch_map("), \
        launches("cudaError_t launch_stride2(")
    # launch_map holds both instantiations of the brick kernel, one of which runs
    assert (build, mp - 1, s2) == (4, 4, 10)
    assert bench.TOPO_KERNELS == {"make_level": build + mp - 1, "downsample": build + s2,
                                  "make_level_downsample": build + mp - 1 + s2 - 1}


def test_plan_kernel_counts():
    """A plan build launches header, mask keys, the 27-bit row sort, tile
    lists and the 8-bit tile sort; cub sorts up to 256 x 19 items in one
    kernel, else histogram + exclusive sum + one onesweep pass per 8 bits.
    The launch lists agree: 5 onesweep launches per shell_4m step (24,576
    tiles), 4 per res4_c128 step (2,851 tiles, single-tile schedule sort)."""
    assert bench.plan_kernels(3145728) == 1 + 1 + 6 + 1 + 3
    assert bench.plan_kernels(364846) == 1 + 1 + 6 + 1 + 1
    assert bench.plan_kernels(4864) == 5 and bench.plan_kernels(4865) == 10
    assert bench.plan_kernels(0) == 1
    assert bench.radix_sort_kernels(24576, 8) - 2 == 1 and bench.radix_sort_kernels(3145728, 27) - 2 == 4
