"""The oracle against the reference's own CPU code run live (mogecpp
src/sparse.cpp + ggml CPU, compiled from the reference sources into
oracle/_ref/), on seeded random inputs beyond the golden fixtures: random
extents, densities and voxel orders (shuffled, so first-occurrence numbering
is exercised), duplicated coordinates in make_level, and sparse_conv with
each weight type.  Skipped where the reference build is absent."""
import os

import numpy as np
import pytest

from conftest import ROOT, max_abs, rel_l2
from mogecpp_b200 import synth
from oracle.oracle import W_F16, W_F32, W_Q8_0

REF_SO = os.path.join(ROOT, "oracle", "_ref", "libmoge_ref.so")
pytestmark = pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference CPU build not present")


@pytest.fixture(scope="module")
def ref():
    from oracle.oracle import Reference
    return Reference(n_threads=4)


def random_voxels(seed, dup=False):
    """A random blob set: extent 6..40 per axis, density 5..60 %, shuffled."""
    rng = np.random.default_rng(seed)
    ext = rng.integers(6, 41, size=3)
    dens = rng.uniform(0.05, 0.6)
    n = max(1, int(dens * np.prod(ext)))
    pts = np.stack([rng.integers(0, e, size=n) for e in ext], 1)
    pts += rng.integers(0, 3000, size=3)  # away from the origin, still in 19 bits
    c = np.zeros((n, 4), np.int32)
    c[:, :3] = pts
    c = synth.dedup_sorted(c)
    c = c[rng.permutation(len(c))]
    if dup:
        extra = c[rng.integers(0, len(c), size=max(1, len(c) // 20))]
        c = np.concatenate([c, extra])[rng.permutation(len(c) + len(extra))]
    return np.ascontiguousarray(c)


@pytest.mark.parametrize("seed", range(8))
def test_make_level_equals_the_reference(oracle, ref, seed):
    c = random_voxels(100 + seed, dup=seed % 2 == 1)
    np.testing.assert_array_equal(oracle.make_level(c), ref.make_level(c))


@pytest.mark.parametrize("seed", range(8))
def test_downsample_equals_the_reference(oracle, ref, seed):
    c = random_voxels(200 + seed)
    parent, pool, inv, up = oracle.downsample(c)
    rp, rpool, rinv, rup = ref.downsample(c)
    np.testing.assert_array_equal(parent[:, :3], rp)
    np.testing.assert_array_equal(pool, rpool)
    np.testing.assert_array_equal(inv, rinv)
    np.testing.assert_array_equal(up, rup)


@pytest.mark.parametrize("wtype,cin,cout,tol", [(W_F32, 32, 64, 1e-6), (W_F16, 64, 32, 1e-6),
                                                (W_Q8_0, 64, 64, 1e-6), (W_Q8_0, 128, 128, 1e-6)])
def test_sparse_conv_equals_the_reference(oracle, ref, wtype, cin, cout, tol):
    c = synth.small_coords(300 + cin + cout, extent=20, grid=24)
    c = c[np.random.default_rng(cin).permutation(len(c))]
    nbr = oracle.make_level(c)
    x = synth.features(cin, len(c), cin)
    w = synth.conv_weight(cout, cin, cout)
    if wtype == W_F16:
        w = w.astype(np.float16).astype(np.float32)
    b = np.random.default_rng(cout).standard_normal(cout).astype(np.float32)
    y = oracle.sparse_conv(x, nbr, w, wtype, b)
    yr = ref.sparse_conv(x, nbr, w, wtype, b)
    assert rel_l2(y, yr) < tol
    assert max_abs(y, yr) < 1e-4
