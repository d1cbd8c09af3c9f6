"""The packed sparse27 weight layout and the neighbour-tap order, on the
oracle (CPU), as the reference's converter tests pin them
(tests/test_converter.py:167-205 in mogecpp): a packed weight is
[cout][27 * cin] with cin fastest inside tap t = (dx+1)*9 + (dy+1)*3 + (dz+1)
(dz fastest), the neighbour map's column order; and the conv is the sum over
taps of W_t @ gather_t(x), the packed gather-GEMM contraction."""
import numpy as np

from oracle.oracle import W_F32


def _tap(dx, dy, dz):
    return (dx + 1) * 9 + (dy + 1) * 3 + (dz + 1)


def test_neighbour_columns_follow_the_tap_order(oracle):
    g = np.arange(3)
    x, y, z = np.meshgrid(g, g, g, indexing="ij")
    coords = np.stack([x.ravel() + 10, y.ravel() + 20, z.ravel() + 30, 0 * x.ravel()], 1).astype(np.int32)
    order = np.random.default_rng(4).permutation(len(coords))
    coords = np.ascontiguousarray(coords[order])
    nbr = oracle.make_level(coords)
    centre = int(np.flatnonzero((coords[:, :3] == (11, 21, 31)).all(1))[0])
    for dx in (-1, 0, 1):
        for dy in (-1, 0, 1):
            for dz in (-1, 0, 1):
                j = nbr[centre, _tap(dx, dy, dz)]
                assert tuple(coords[j, :3]) == (11 + dx, 21 + dy, 31 + dz)


def test_packed_weight_is_tap_major_with_cin_fastest(oracle):
    """A voxel whose only neighbour sits at tap t, with the one-hot input
    channel k there, outputs column t * cin + k of the packed weight."""
    cin, cout = 32, 32
    w = np.random.default_rng(5).standard_normal((cout, 27 * cin)).astype(np.float32)
    for (dx, dy, dz), k in (((1, -1, 0), 3), ((-1, -1, -1), 0), ((0, 0, 1), 31), ((1, 1, 1), 17)):
        coords = np.array([[50, 50, 50, 0], [50 + dx, 50 + dy, 50 + dz, 0]], np.int32)
        nbr = oracle.make_level(coords)
        nbr[0, 13] = 2  # drop the centre tap (the voxel itself): row 0 sees only its neighbour
        x = np.zeros((2, cin), np.float32)
        x[1, k] = 1.0
        y = oracle.sparse_conv(x, nbr, w, W_F32)
        np.testing.assert_array_equal(y[0], w[:, _tap(dx, dy, dz) * cin + k])


def test_tapwise_sum_is_the_packed_gather_gemm(oracle):
    rng = np.random.default_rng(23)
    cin, cout, n = 32, 64, 300
    x = rng.standard_normal((n, cin)).astype(np.float32)
    nbr = rng.integers(0, n + 1, size=(n, 27)).astype(np.int32)  # n = missing
    w = rng.standard_normal((cout, 27 * cin)).astype(np.float32)
    xs = np.concatenate([x, np.zeros((1, cin), np.float32)])     # zero sentinel row
    full = np.concatenate([xs[nbr[:, t]] for t in range(27)], 1).astype(np.float64) @ w.T.astype(np.float64)
    tapwise = sum(xs[nbr[:, t]].astype(np.float64) @ w[:, t * cin:(t + 1) * cin].T.astype(np.float64)
                  for t in range(27))
    np.testing.assert_allclose(tapwise, full, rtol=1e-12, atol=1e-12)
    y = oracle.sparse_conv(x, nbr, w, W_F32)
    np.testing.assert_allclose(y, full, rtol=2e-5, atol=2e-5)
