"""GPU topology (hash build, 27-tap neighbour map, stride-2 maps) against the
reference's golden outputs and the oracle: bit-exact."""
import numpy as np
import pytest

from gpu_util import dev, host, numpy_neighbor_map
from mogecpp_b200 import synth
from mogecpp_b200.lib import MscError

pytestmark = pytest.mark.gpu

TOPO = ["surface", "surface_z1", "cube", "single", "odd_line", "shuffled"]


@pytest.mark.parametrize("name", TOPO)
def test_make_level_matches_reference(ex, golden_topology, name):
    c = golden_topology[f"topo_{name}_coords"]
    nbr = ex.make_level(dev(c))
    ex.check()
    np.testing.assert_array_equal(host(nbr), golden_topology[f"topo_{name}_nbr"])


@pytest.mark.parametrize("name", TOPO)
def test_downsample_matches_reference(ex, golden_topology, name):
    g = golden_topology
    tr = ex.downsample(dev(g[f"topo_{name}_coords"]))
    np.testing.assert_array_equal(host(tr.parent)[:, :3], g[f"topo_{name}_parent"])
    np.testing.assert_array_equal(host(tr.pool_rows), g[f"topo_{name}_pool"])
    np.testing.assert_array_equal(host(tr.inv_count), g[f"topo_{name}_inv"])
    np.testing.assert_array_equal(host(tr.up_rows), g[f"topo_{name}_up"])


@pytest.mark.parametrize("gen", ["conv_c64", "res4_c128", "unet"])
def test_workload_topology_matches_oracle(ex, oracle, gen):
    c = {"conv_c64": synth.conv_c64_coords, "res4_c128": synth.res4_c128_coords, "unet": synth.unet_coords}[gen]()
    cd = dev(c)
    nbr = ex.make_level(cd)
    ex.check()
    np.testing.assert_array_equal(host(nbr), oracle.make_level(c))
    tr = ex.downsample(cd)
    parent, pool, inv, up = oracle.downsample(c)
    np.testing.assert_array_equal(host(tr.parent), parent)
    np.testing.assert_array_equal(host(tr.pool_rows), pool)
    np.testing.assert_array_equal(host(tr.inv_count), inv)
    np.testing.assert_array_equal(host(tr.up_rows), up)


def test_four_million_voxel_topology_properties(ex):
    """Full-size topology: the map equals an independent sorted-key search, is
    symmetric (j = nbr[i][t] <=> i = nbr[j][26-t]), and the stride-2 maps are
    consistent (every fine voxel sits in exactly one slot of its parent)."""
    c = synth.topo_4m_coords()
    n = c.shape[0]
    cd = dev(c)
    nbr = host(ex.make_level(cd))
    ex.check()
    np.testing.assert_array_equal(nbr, numpy_neighbor_map(c))
    i = np.repeat(np.arange(n), 27)
    t = np.tile(np.arange(27), n)
    j = nbr.ravel()
    ok = j < n
    assert np.array_equal(nbr[j[ok], 26 - t[ok]], i[ok])
    tr = ex.downsample(cd)
    pool = host(tr.pool_rows)
    up = host(tr.up_rows)
    filled = pool[pool < n]
    assert filled.size == n and np.array_equal(np.sort(filled), np.arange(n))
    slot_of = np.full(n, -1)
    for s in range(8):
        m = pool[s] < n
        slot_of[pool[s][m]] = s
        assert np.array_equal(up[pool[s][m]], np.nonzero(m)[0])
    parent = host(tr.parent)
    np.testing.assert_array_equal(parent[up][:, :3], c[:, :3] // 2)
    # parents are numbered in first-occurrence order
    first = np.full(tr.np, n)
    np.minimum.at(first, up, np.arange(n))
    assert np.all(np.diff(first) > 0)
    # slots follow arrival (index) order among siblings
    for s in range(1, 8):
        m = pool[s] < n
        assert np.all(pool[s][m] > pool[s - 1][m])


def test_batch_field_separates_samples(ex, oracle):
    a = synth.small_coords(3, extent=10, grid=16, b=0)
    b = synth.small_coords(3, extent=10, grid=16, b=1)
    c = np.concatenate([a, b])
    nbr = host(ex.make_level(dev(c)))
    np.testing.assert_array_equal(nbr, oracle.make_level(c))
    na = a.shape[0]
    assert np.all((nbr[:na] < na) | (nbr[:na] == c.shape[0]))
    assert np.all(nbr[na:] >= na)


def test_empty_level(ex):
    c = np.zeros((0, 4), dtype=np.int32)
    nbr = ex.make_level(dev(c))
    assert tuple(nbr.shape) == (0, 27)
    tr = ex.downsample(dev(c))
    assert tr.np == 0


def test_duplicates_resolve_to_first_index_in_make_level(ex, oracle):
    c = synth.small_coords(4, extent=8, grid=16)
    c = np.concatenate([c, c[:5]])
    nbr = host(ex.make_level(dev(c)))
    bits = ex.check()
    assert bits & 8  # duplicate flag is informational
    np.testing.assert_array_equal(nbr, oracle.make_level(c))


def test_duplicates_are_rejected_by_downsample(ex):
    c = synth.small_coords(4, extent=8, grid=16)
    c = np.concatenate([c, c[:1]])
    with pytest.raises(MscError):
        ex.downsample(dev(c))


def test_out_of_range_coordinate_is_reported(ex):
    c = synth.small_coords(4, extent=8, grid=16).copy()
    c[3, 2] = -1
    ex.make_level(dev(c))
    with pytest.raises(MscError, match="coordinate"):
        ex.check()
    ex.check()  # status was cleared


@pytest.mark.parametrize("spacing", [4, 5])
def test_sparse_input_takes_the_per_voxel_hash(ex, oracle, spacing):
    """Voxels on a lattice of spacing >= 4 fill one 4x4x4 brick each: more
    bricks than the record budget (n / 4 + 1024), so make_level switches to
    the per-voxel hash on the device; plus a few dense clusters so that some
    taps are present.  Bit-exact against the oracle either way."""
    g = np.arange(0, 22 * spacing, spacing)
    x, y, z = np.meshgrid(g, g, g[:12], indexing="ij")
    lat = np.stack([x.ravel(), y.ravel(), z.ravel(), np.zeros(x.size, np.int64)], 1)
    blob = np.array([(200 + a, 200 + b, 10 + c, 0) for a in range(3) for b in range(3) for c in range(3)])
    coords = synth.dedup_sorted(np.concatenate([lat, blob]).astype(np.int32))
    nbr = host(ex.make_level(dev(coords)))
    ex.check()
    np.testing.assert_array_equal(nbr, oracle.make_level(coords))


@pytest.mark.parametrize("gen", ["golden", "topo_4m", "res4_c128", "sparse"])
def test_make_level_downsample_equals_the_two_calls(ex, oracle, golden_topology, gen):
    """msc_make_level_downsample (one voxel table for both maps; the
    neighbour kernel also runs the first-child pass) gives the neighbour map
    of msc_make_level and the stride-2 maps of msc_downsample, bit for bit,
    and both equal the oracle: the reference's shuffled golden set, the
    4M-voxel stress set (against the two calls only), the 364,846-voxel
    res4_c128 set (more than 1024 first-child scan blocks), and a lattice
    sparse enough for the per-voxel hash."""
    if gen == "golden":
        c = golden_topology["topo_shuffled_coords"]
    elif gen == "topo_4m":
        c = synth.topo_4m_coords()
    elif gen == "res4_c128":
        c = synth.res4_c128_coords()
    else:
        g = np.arange(0, 22 * 5, 5)
        x, y, z = np.meshgrid(g, g, g[:12], indexing="ij")
        c = np.stack([x.ravel(), y.ravel(), z.ravel(), np.zeros(x.size, np.int64)], 1).astype(np.int32)
    cd = dev(c)
    nbr_f, tr_f = ex.make_level_downsample(cd)
    ex.check()
    nbr = ex.make_level(cd)
    tr = ex.downsample(cd)
    ex.check()
    assert tr_f.np == tr.np
    assert bool((nbr_f == nbr).all())
    for a, b in ((tr_f.parent, tr.parent), (tr_f.pool_rows, tr.pool_rows), (tr_f.inv_count, tr.inv_count),
                 (tr_f.up_rows, tr.up_rows)):
        assert bool((a == b).all())
    if gen != "topo_4m":
        np.testing.assert_array_equal(host(nbr_f), oracle.make_level(c))
        parent, pool, inv, up = oracle.downsample(c)
        np.testing.assert_array_equal(host(tr_f.parent), parent)
        np.testing.assert_array_equal(host(tr_f.pool_rows), pool)
        np.testing.assert_array_equal(host(tr_f.inv_count), inv)
        np.testing.assert_array_equal(host(tr_f.up_rows), up)
