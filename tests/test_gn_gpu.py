"""GroupNorm residual block (conv1 -> GroupNorm(32) -> SiLU -> conv2 -> +x)
against the oracle's restatement of ggml's group_norm_f32 composition."""
import numpy as np
import pytest
import torch

from conftest import max_abs, rel_l2
from gpu_util import TOL_FP16, TOL_FP32, dev, host, weight_tensor
from mogecpp_b200 import synth
from mogecpp_b200.lib import MscError
from oracle.oracle import W_F32, W_Q8_0

pytestmark = pytest.mark.gpu
WT = {"f32": W_F32, "q8_0": W_Q8_0}


def two_sample_coords(seed):
    a = synth.small_coords(seed, extent=20, grid=28, b=0)
    b = synth.small_coords(seed + 1, extent=16, grid=24, b=1)
    return np.concatenate([a, b]).astype(np.int32)


def raw_gn_block(seed, c):
    rng = np.random.default_rng(seed)
    return dict(gn_w=(1 + 0.1 * rng.standard_normal(c)).astype(np.float32),
                gn_b=(0.1 * rng.standard_normal(c)).astype(np.float32),
                w1=synth.conv_weight(seed + 1, c, c), b1=(0.05 * rng.standard_normal(c)).astype(np.float32),
                w2=synth.conv_weight(seed + 2, c, c), b2=(0.05 * rng.standard_normal(c)).astype(np.float32))


def make_gn_block(ex, oracle, raw, tag, c):
    return dict(gn_w=dev(raw["gn_w"]), gn_b=dev(raw["gn_b"]), b1=dev(raw["b1"]), b2=dev(raw["b2"]),
                w1=ex.prepare_weight(weight_tensor(oracle, raw["w1"], tag), tag, c, c, 27),
                w2=ex.prepare_weight(weight_tensor(oracle, raw["w2"], tag), tag, c, c, 27))


def check_tol(y, ref, exact_fp32):
    if exact_fp32:
        assert rel_l2(y, ref) < TOL_FP32
    else:
        assert rel_l2(y, ref) < TOL_FP16[0] and max_abs(y, ref) < TOL_FP16[1]


@pytest.mark.parametrize("tag", ["f32", "q8_0"])
@pytest.mark.parametrize("c", [64, 128])
def test_gn_block_matches_oracle(ex, oracle, tag, c):
    coords = two_sample_coords(300)
    nbr = oracle.make_level(coords)
    x = dev(synth.features(301, coords.shape[0], c))
    xin = host(x)
    raw = raw_gn_block(302, c)
    ref = oracle.res_block_gn(xin, nbr, coords[:, 3], raw, WT[tag])
    ex.res_block_gn(x, dev(nbr), dev(coords), 2, make_gn_block(ex, oracle, raw, tag, c))
    ex.check()
    check_tol(host(x), ref, tag == "f32")


@pytest.mark.parametrize("tag", ["f32", "q8_0"])
def test_gn_block_fp16_state_and_plan(ex, oracle, tag):
    """fp16 features, no affine, tap-ordered plan."""
    coords = two_sample_coords(310)
    nbr = oracle.make_level(coords)
    x = dev(synth.features(311, coords.shape[0], 128)).to(torch.float16)
    xin = host(x)
    raw = raw_gn_block(312, 128)
    raw["gn_w"] = raw["gn_b"] = None
    ref = oracle.res_block_gn(xin, nbr, coords[:, 3], raw, WT[tag])
    blk = make_gn_block(ex, oracle, {**raw, "gn_w": np.ones(128, np.float32), "gn_b": np.zeros(128, np.float32)},
                        tag, 128)
    blk["gn_w"] = blk["gn_b"] = None
    coords_d, nbr_d = dev(coords), dev(nbr)
    plan = ex.conv_plan(coords_d, nbr_d, kind="tap_order")
    ex.res_block_gn(x, nbr_d, coords_d, 2, blk, plan=plan)
    ex.check()
    check_tol(host(x), ref, False)


def test_gn_block_allreduce_callback(ex, oracle):
    """The all-reduce hook is called once per block with the whole statistics
    buffer; an identity reduction leaves the result bit-identical."""
    coords = two_sample_coords(320)
    nbr = dev(oracle.make_level(coords))
    cd = dev(coords)
    x0 = dev(synth.features(321, coords.shape[0], 64))
    blk = make_gn_block(ex, oracle, raw_gn_block(322, 64), "q8_0", 64)
    a = x0.clone()
    ex.res_block_gn(a, nbr, cd, 2, blk)
    seen = []

    def ident(t):
        seen.append(t.numel())
        t.mul_(1.0)
    b = x0.clone()
    ex.res_block_gn(b, nbr, cd, 2, blk, allreduce=ident)
    ex.check()
    assert seen == [2 * 65]
    assert torch.equal(a, b)

    def broken(t):
        raise RuntimeError("peer lost")
    with pytest.raises(MscError, match="all-reduce failed"):
        ex.res_block_gn(x0.clone(), nbr, cd, 2, blk, allreduce=broken)


def test_gn_block_statistics_over_owned_rows(ex, oracle):
    """Rows past n_stat (halo rows) are normalised with the owned rows'
    statistics but do not enter them: a second copy of the level with other
    features, appended as rows [n, 2n), leaves the first copy's result equal
    to the single-copy oracle."""
    coords = two_sample_coords(330)
    n = coords.shape[0]
    nbr = oracle.make_level(coords)
    raw = raw_gn_block(332, 64)
    xin = synth.features(331, n, 64)
    ref = oracle.res_block_gn(xin, nbr, coords[:, 3], raw, W_F32)
    blk = make_gn_block(ex, oracle, raw, "f32", 64)
    nbr2 = np.concatenate([np.where(nbr >= n, 2 * n, nbr), np.where(nbr >= n, 2 * n, nbr + n)]).astype(np.int32)
    x = dev(np.concatenate([xin, 3.0 * xin + 1.0]).astype(np.float32))
    ex.res_block_gn(x, dev(nbr2), dev(np.concatenate([coords, coords])), 2, blk, n_stat=n)
    ex.check()
    check_tol(host(x)[:n], ref, True)


def test_gn_block_bad_sample_index(ex, oracle):
    """A sample index outside [0, nsamples), in an owned or a halo row, is a
    device failure reported by msc_check."""
    coords = two_sample_coords(340)
    nbr = dev(oracle.make_level(coords))
    blk = make_gn_block(ex, oracle, raw_gn_block(342, 64), "f32", 64)
    for row in (0, coords.shape[0] - 1):
        bad = coords.copy()
        bad[row, 3] = 2   # nsamples = 2
        x = dev(synth.features(341, coords.shape[0], 64))
        ex.res_block_gn(x, nbr, dev(bad), 2, blk, n_stat=coords.shape[0] - 1)
        with pytest.raises(MscError, match="coordinate-out-of-range"):
            ex.check()
