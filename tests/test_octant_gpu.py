"""Octant-weighted stride-2 conv and its transpose on the tensor cores
(msc_octant_maps, msc_conv_plan_build_rect, msc_octant_conv) against the
oracle (tests/test_octant_oracle.py pins it to the reference's pool_down /
nearest_up).  Maps bit-exact; features fp32 rel-L2 1e-4, bf16 / Q8_0
rel-L2 1e-3 and max-abs 1e-2."""
import numpy as np
import pytest
import torch

from conftest import max_abs, rel_l2
from gpu_util import TOL_FP16, TOL_FP32, dev, host, weight_tensor
from mogecpp_b200 import synth
from oracle.oracle import W_F32, W_Q8_0

pytestmark = pytest.mark.gpu


def _octant_weight(seed, cin, cout):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((cout, 8 * cin)) / np.sqrt(8.0 * cin)).astype(np.float32)


def _tol(y, ref, fp32):
    if fp32:
        assert rel_l2(y, ref) < TOL_FP32, rel_l2(y, ref)
    else:
        assert rel_l2(y, ref) < TOL_FP16[0], rel_l2(y, ref)
        assert max_abs(y, ref) < TOL_FP16[1], max_abs(y, ref)


@pytest.fixture(scope="module")
def level(ex, oracle):
    c = synth.small_coords(71, extent=22, grid=32)
    cd = dev(c)
    tr = ex.downsample(cd)
    down, up = ex.octant_maps(cd, tr)
    ex.check()
    return dict(c=c, cd=cd, tr=tr, down=down, up=up, ref=oracle.downsample(c))


def test_octant_maps_match_oracle(ex, oracle, level):
    parent, pool, inv, up = level["ref"]
    down_ref, up_ref = oracle.octant_maps(level["c"], pool, up)
    np.testing.assert_array_equal(host(level["down"]), down_ref)
    np.testing.assert_array_equal(host(level["up"]), up_ref)


def test_octant_maps_on_the_u_level_set(ex, oracle):
    c = synth.unet_coords()
    cd = dev(c)
    tr = ex.downsample(cd)
    down, up = ex.octant_maps(cd, tr)
    ex.check()
    _, pool, _, upr = oracle.downsample(c)
    d_ref, u_ref = oracle.octant_maps(c, pool, upr)
    np.testing.assert_array_equal(host(down), d_ref)
    np.testing.assert_array_equal(host(up), u_ref)


@pytest.mark.parametrize("tag,cin,cout,xdt", [("f32", 64, 128, torch.float32), ("f32", 64, 128, torch.bfloat16),
                                              ("q8_0", 128, 128, torch.float16), ("f16", 128, 64, torch.float16)])
@pytest.mark.parametrize("planned", [False, True])
def test_strided_conv_matches_oracle(ex, oracle, level, tag, cin, cout, xdt, planned):
    nfine, np_ = level["c"].shape[0], level["tr"].np
    w = _octant_weight(72, cin, cout)
    b = np.linspace(-0.2, 0.2, cout).astype(np.float32)
    x = synth.features(73, nfine, cin)
    xd = dev(x).to(xdt)
    pw = ex.prepare_weight(weight_tensor(oracle, w, tag), tag, cin, cout, 8)
    plan = ex.conv_plan_rect(level["down"], nfine) if planned else None
    y = ex.octant_conv(xd, level["down"], pw, dev(b), plan=plan)
    ex.check()
    wt = {"f32": W_F32, "f16": 1, "q8_0": W_Q8_0}[tag]
    ref = oracle.conv_rect(xd.float().cpu().numpy(), host(level["down"]), np_, 8, w, wt, b)
    _tol(host(y), ref, fp32=(tag == "f32" and xdt == torch.float32))


@pytest.mark.parametrize("tag,cin,cout", [("f32", 128, 64), ("q8_0", 128, 128)])
@pytest.mark.parametrize("planned", [False, True])
def test_transposed_conv_matches_oracle(ex, oracle, level, tag, cin, cout, planned):
    nfine, np_ = level["c"].shape[0], level["tr"].np
    w = _octant_weight(74, cin, cout)
    b = np.linspace(-0.1, 0.3, cout).astype(np.float32)
    x = synth.features(75, np_, cin)
    pw = ex.prepare_weight(weight_tensor(oracle, w, tag), tag, cin, cout, 8)
    plan = ex.conv_plan_rect(level["up"], np_) if planned else None
    y = ex.octant_conv(dev(x), level["up"], pw, dev(b), plan=plan)
    ex.check()
    ref = oracle.conv_rect(x, host(level["up"]), nfine, 8, w, {"f32": W_F32, "q8_0": W_Q8_0}[tag], b)
    _tol(host(y), ref, fp32=(tag == "f32"))


def test_planned_and_unplanned_strided_conv_agree_bit_for_bit(ex, oracle, level):
    nfine = level["c"].shape[0]
    w = _octant_weight(76, 128, 128)
    pw = ex.prepare_weight(weight_tensor(oracle, w, "q8_0"), "q8_0", 128, 128, 8)
    xd = dev(synth.features(77, nfine, 128)).to(torch.float16)
    a = ex.octant_conv(xd, level["down"], pw)
    b = ex.octant_conv(xd, level["down"], pw, plan=ex.conv_plan_rect(level["down"], nfine))
    ex.check()
    assert bool((a == b).all())


def test_plan_for_another_input_count_is_rejected(ex, level):
    from mogecpp_b200.lib import MscError
    nfine, np_ = level["c"].shape[0], level["tr"].np
    w = ex.prepare_weight(dev(_octant_weight(78, 64, 64)), "f32", 64, 64, 8)
    plan = ex.conv_plan_rect(level["down"], nfine + 1)
    with pytest.raises(MscError):
        ex.octant_conv(dev(synth.features(79, nfine, 64)), level["down"], w, plan=plan)
    ex.check()


@pytest.mark.parametrize("ydt", [torch.float32, torch.bfloat16])
def test_transposed_conv_with_decoder_skip(ex, oracle, level, ydt):
    """The U-level's upsample: transposed conv back onto the fine rows plus
    the encoder's skip rows, fused into the conv epilogue."""
    nfine, np_ = level["c"].shape[0], level["tr"].np
    w = _octant_weight(80, 128, 64)
    x = synth.features(81, np_, 128)
    skip = synth.features(82, nfine, 64)
    skip_d = dev(skip).to(ydt)
    pw = ex.prepare_weight(dev(w), "f32", 128, 64, 8)
    y = ex.octant_conv(dev(x), level["up"], pw, None, out_dtype=ydt, plan=ex.conv_plan_rect(level["up"], np_),
                       skip=skip_d)
    ex.check()
    ref = oracle.conv_rect(x, host(level["up"]), nfine, 8, w, W_F32) + skip_d.float().cpu().numpy()
    # bf16 rows: compare with the reference rounded to bf16 (the output
    # format's own rounding is 2^-9 relative)
    ref = torch.from_numpy(ref).to(ydt).float().numpy()
    _tol(host(y.float()), ref, fp32=(ydt == torch.float32))
