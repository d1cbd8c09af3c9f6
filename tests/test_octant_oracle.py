"""The octant-weighted stride-2 conv and its transpose have no counterpart in
the reference (its stride-2 operators are pool + linear and linear +
nearest up), so their oracle is pinned through identities with operators
that are pinned to the reference:
  * the octant maps hold each fine voxel exactly once, at its own octant,
    under the parent downsample gave it;
  * the rectangular conv over the 27-tap map of a level equals the level's
    sparse_conv;
  * with one weight W for all eight octants the strided conv is count x the
    mean-pool linear of pool_down (bias removed), and the transpose is
    nearest_up's linear + parent gather."""
import numpy as np
import pytest

from conftest import rel_l2
from mogecpp_b200 import synth
from oracle.oracle import W_F32


def _level(seed):
    coords = synth.small_coords(seed, extent=18, grid=32)
    return coords


def test_octant_maps_place_every_child_once(oracle):
    c = _level(61)
    parent, pool, inv, up = oracle.downsample(c)
    down, upm = oracle.octant_maps(c, pool, up)
    nfine, np_ = c.shape[0], parent.shape[0]
    oct_ = (c[:, 0] & 1) * 4 + (c[:, 1] & 1) * 2 + (c[:, 2] & 1)
    assert (down[:, 8:] == nfine).all() and (upm[:, 8:] == np_).all()
    present = down[:, :8][down[:, :8] < nfine]
    np.testing.assert_array_equal(np.sort(present), np.arange(nfine))
    p_of, o_of = np.nonzero(down[:, :8] < nfine)
    child = down[p_of, o_of]
    np.testing.assert_array_equal(up[child], p_of)
    np.testing.assert_array_equal(oct_[child], o_of)
    np.testing.assert_array_equal(upm[np.arange(nfine), oct_], up)
    mask = np.ones_like(upm, dtype=bool)
    mask[np.arange(nfine), oct_] = False
    assert (upm[mask] == np_).all()


def test_rect_conv_over_a_level_map_is_the_sparse_conv(oracle):
    c = _level(62)
    nbr = oracle.make_level(c)
    x = synth.features(63, c.shape[0], 64)
    w = synth.conv_weight(64, 64, 64)
    b = np.linspace(-0.1, 0.1, 64).astype(np.float32)
    np.testing.assert_array_equal(oracle.conv_rect(x, nbr, c.shape[0], 27, w, W_F32, b),
                                  oracle.sparse_conv(x, nbr, w, W_F32, b))


@pytest.mark.parametrize("cin,cout", [(64, 128), (128, 64)])
def test_equal_octant_weights_reduce_to_pool_and_up(oracle, cin, cout):
    c = _level(65)
    parent, pool, inv, up = oracle.downsample(c)
    down, upm = oracle.octant_maps(c, pool, up)
    nfine, np_ = c.shape[0], parent.shape[0]
    rng = np.random.default_rng(66)
    W = (rng.standard_normal((cout, cin)) / np.sqrt(cin)).astype(np.float32)
    W8 = np.tile(W, (1, 8))                         # the same W at every octant
    xf = synth.features(67, nfine, cin)
    count = np.round(1.0 / inv).astype(np.float64)
    strided = oracle.conv_rect(xf, down, np_, 8, W8, W_F32)
    pooled = oracle.pool_down(xf, pool, inv, W, W_F32)
    assert rel_l2(strided, pooled * count[:, None]) < 1e-5
    xc = synth.features(68, np_, cin)
    assert rel_l2(oracle.conv_rect(xc, upm, nfine, 8, W8, W_F32), oracle.nearest_up(xc, up, W, W_F32)) < 1e-6
