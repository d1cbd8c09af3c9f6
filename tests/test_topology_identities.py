"""Identities the device topology relies on, checked on the oracle (CPU).

make_level_downsample's neighbour kernel derives the stride-2 maps' first
children from the neighbour row it has just built: the 2 x 2 x 2 cell of a
voxel (the voxels with the same parent, c >> 1) is the set of its taps at
offsets {0, s} per axis, s = +1 on an even coordinate and -1 on an odd one.
From those 8 taps: first child = smallest index, the voxel's slot = the
number of siblings with a smaller index, count = their number; parent ids
are the first children's ranks in index order (an exclusive scan of the
first-child flags, computed in blocks of 256 voxels plus a scan of the block
sums).  This restates that derivation in numpy and checks it against the
oracle's downsample (the reference's serial loop, src/sparse.cpp:312-357)."""
import numpy as np
import pytest

from mogecpp_b200 import synth

BLOCK = 256


def stride2_from_rows(coords, nbr):
    n = len(coords)
    idx = np.arange(n)
    s = [np.where(coords[:, a] & 1, 0, 2) for a in range(3)]  # tap digit of the sibling offset
    first = np.full(n, np.iinfo(np.int64).max)
    count = np.zeros(n, np.int64)
    rank = np.zeros(n, np.int64)
    for o in range(8):
        dx = np.where(o & 4, s[0], 1)
        dy = np.where(o & 2, s[1], 1)
        dz = np.where(o & 1, s[2], 1)
        j = nbr[idx, dx * 9 + dy * 3 + dz].astype(np.int64)
        ok = j < n
        count += ok
        rank += ok & (j < idx)
        first = np.where(ok, np.minimum(first, j), first)
    flag = (first == idx).astype(np.int64)
    nblk = (n + BLOCK - 1) // BLOCK
    padded = np.zeros(nblk * BLOCK, np.int64)
    padded[:n] = flag
    blocks = padded.reshape(nblk, BLOCK)
    excl = (np.cumsum(blocks, 1) - blocks).reshape(-1)[:n]
    bsum = blocks.sum(1)
    bsum_excl = np.cumsum(bsum) - bsum
    np_ = int(bsum.sum())
    up = excl[first] + bsum_excl[first // BLOCK]
    parent = np.zeros((np_, 4), np.int64)
    parent[up[flag == 1]] = np.concatenate([coords[flag == 1, :3] >> 1, coords[flag == 1, 3:]], 1)
    pool = np.full((8, np_), n, np.int64)
    pool[rank, up] = idx
    inv = np.zeros(np_, np.float32)
    inv[up[rank == 0]] = (np.float32(1) / count[rank == 0].astype(np.float32)).astype(np.float32)
    return parent, pool, inv, up


def _sets():
    rng = np.random.default_rng(11)
    out = {"small": synth.small_coords(3), "conv_c64": synth.conv_c64_coords()}
    c = rng.integers(0, 90, size=(400000, 4)).astype(np.int32)
    c[:, 3] = rng.integers(0, 3, size=len(c))
    c = synth.dedup_sorted(c)
    out["random_3_samples_shuffled"] = c[rng.permutation(len(c))]   # > 1024 scan blocks
    return out


SETS = _sets()


@pytest.mark.parametrize("name", sorted(SETS))
def test_stride2_maps_follow_from_the_neighbour_rows(oracle, name):
    c = np.ascontiguousarray(SETS[name])
    parent, pool, inv, up = stride2_from_rows(c, oracle.make_level(c))
    rp, rpool, rinv, rup = oracle.downsample(c)
    np.testing.assert_array_equal(parent, rp)
    np.testing.assert_array_equal(pool, rpool)
    np.testing.assert_array_equal(inv, rinv)
    np.testing.assert_array_equal(up, rup)


def test_golden_sets(oracle, golden_topology):
    for name in ["surface", "surface_z1", "cube", "single", "odd_line", "shuffled"]:
        c = golden_topology[f"topo_{name}_coords"]
        parent, pool, inv, up = stride2_from_rows(c, golden_topology[f"topo_{name}_nbr"])
        np.testing.assert_array_equal(parent[:, :3], golden_topology[f"topo_{name}_parent"])
        np.testing.assert_array_equal(pool, golden_topology[f"topo_{name}_pool"])
        np.testing.assert_array_equal(inv, golden_topology[f"topo_{name}_inv"])
        np.testing.assert_array_equal(up, golden_topology[f"topo_{name}_up"])
