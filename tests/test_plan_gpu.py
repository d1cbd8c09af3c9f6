"""Conv plans (msc_conv_plan_build) and the convs that run over them
(msc_sparse_conv_planned / msc_res_block_planned): the tap order for the
neighbour-map conv and the row-cache plan for the row-cached Q8_0 conv.

The tap order must be a permutation sorted, stably, by the class-ordered
tap-mask key.  The row-cache plan's integer content is checked exactly
against the neighbour map:
every voxel appears once, in Morton order; every subtile's U list holds
exactly the distinct neighbours of its rows; every (row, tap) slot points at
the neighbour the map names, or is 0xFFFF where the map says missing.  The
conv over the plan is checked against the oracle at the features tolerance
(rel-L2 1e-3, max-abs 1e-2) and against the unplanned conv, which computes the
same exact per-block sums in another tap order (rel-L2 1e-5)."""
import numpy as np
import pytest
import torch

from conftest import max_abs, rel_l2
from gpu_util import TOL_FP16, dev, host, weight_tensor
from mogecpp_b200 import synth
from mogecpp_b200.lib import MscError
from oracle.oracle import W_Q8_0

pytestmark = pytest.mark.gpu

PLAN_CAP = 384
NO_SLOT = 0xFFFF


def _align(v):
    return (v + 255) // 256 * 256


def parse_plan(buf, n):
    """Sections of a plan buffer (layout of mogecpp_b200/csrc/plan.h)."""
    b = buf.cpu().numpy()
    hdr = b[:48]
    magic = int(hdr[:4].view(np.uint32)[0])
    overflow = int(hdr[4:8].view(np.int32)[0])
    hn, max_desc, pool_cap = (int(v) for v in hdr[8:32].view(np.int64))
    ndesc, pool_used = (int(v) for v in hdr[32:48].view(np.uint64))
    off = _align(48)
    perm = b[off:off + 4 * n].view(np.int32)
    off += _align(4 * n)
    desc = b[off:off + 16 * max_desc].view(np.int32).reshape(max_desc, 4)
    off += _align(16 * max_desc)
    slots = b[off:off + 2 * 27 * n].view(np.uint16).reshape(n, 27)
    off += _align(2 * 27 * n)
    order = b[off:off + 4 * n].view(np.int32)
    off += _align(4 * n)
    pool = b[off:off + 4 * pool_cap].view(np.int32)
    return dict(magic=magic, overflow=overflow, n=hn, max_desc=max_desc, ndesc=ndesc, pool_used=pool_used,
                perm=perm, desc=desc[:ndesc], slots=slots, order=order, pool=pool)


def _spread3(v):
    v = v.astype(np.uint64) & np.uint64(0xFFFF)
    r = np.zeros_like(v)
    for i in range(16):
        r |= ((v >> np.uint64(i)) & np.uint64(1)) << np.uint64(3 * i)
    return r


def morton_keys(coords):
    c = coords.astype(np.int64)
    return ((c[:, 3].astype(np.uint64) & np.uint64(0x7F)) << np.uint64(48)) | _spread3(c[:, 0]) | \
        (_spread3(c[:, 1]) << np.uint64(1)) | (_spread3(c[:, 2]) << np.uint64(2))


def check_plan(p, coords, nbr):
    n = coords.shape[0]
    assert p["magic"] == 0x4E4C5053 and p["overflow"] == 0 and p["n"] == n
    perm = p["perm"]
    np.testing.assert_array_equal(np.sort(perm), np.arange(n))
    keys = morton_keys(coords)[perm]
    assert np.all(keys[1:] >= keys[:-1]), "plan rows are not in Morton order"
    raw = p["desc"]
    # descriptor {row_begin, u_off, rows | u_cnt << 8, tap mask}
    desc = np.stack([raw[:, 0], raw[:, 2] & 0xFF, raw[:, 1], raw[:, 2] >> 8, raw[:, 3]], 1)
    desc = desc[np.argsort(desc[:, 0], kind="stable")]
    # subtiles tile [0, n) exactly, in 128-row blocks cut into equal power-of-two pieces
    assert desc[0, 0] == 0
    np.testing.assert_array_equal(desc[1:, 0], desc[:-1, 0] + desc[:-1, 1])
    assert desc[-1, 0] + desc[-1, 1] == n
    assert np.all((desc[:, 1] >= 1) & (desc[:, 1] <= 128))
    assert np.all(desc[:, 0] % 8 == 0), "subtiles start at multiples of 8 rows"
    assert np.all(desc[:, 0] // 128 == (desc[:, 0] + desc[:, 1] - 1) // 128), "subtile crosses a 128-row block"
    assert np.all(desc[:, 2] % 4 == 0), "U lists start at multiples of 4 entries"
    assert np.all(desc[:, 3] <= PLAN_CAP)
    assert int(((desc[:, 3] + 3) // 4 * 4).sum()) == p["pool_used"]
    for r0, rows, uoff, ucnt, mask in desc:
        ul = p["pool"][uoff:uoff + ucnt]
        assert len(np.unique(ul)) == ucnt, "duplicate U-list entry"
        want = nbr[perm[r0:r0 + rows]]
        sl = p["slots"][r0:r0 + rows].astype(np.int64)
        miss = want >= n
        np.testing.assert_array_equal(sl == NO_SLOT, miss)
        np.testing.assert_array_equal(ul[np.where(miss, 0, sl)][~miss], want[~miss])
        assert set(ul.tolist()) == set(want[~miss].tolist()), "U list holds rows no tap reads"
        present = np.any(~miss, axis=0)
        assert int(mask) == int(sum(1 << t for t in range(27) if present[t])), "tap mask"
    return desc


def dense_offset_cube(side=20, offset=(5, 3, 6)):
    """A solid block whose Morton blocks straddle curve boundaries, so that many
    128-row blocks reference more than 384 distinct rows and split."""
    g = np.arange(side)
    x, y, z = np.meshgrid(g + offset[0], g + offset[1], g + offset[2], indexing="ij")
    c = np.stack([x.ravel(), y.ravel(), z.ravel(), np.zeros(side ** 3, np.int64)], 1).astype(np.int32)
    keys = synth.pack_keys(c)
    return c[np.argsort(keys, kind="stable")]


def _level(ex, oracle, coords, kind="row_cache"):
    nbr = oracle.make_level(coords)
    cd = dev(coords)
    plan = ex.conv_plan(cd, dev(nbr), kind)
    ex.check()
    return nbr, plan


def tap_order_keys(nbr):
    """Sort key of the tap order: the tap mask with corners in the high bits,
    then edges, faces, centre (tap index order within a class), taken to its
    position in the reflected Gray-code sequence (prefix xor)."""
    n = nbr.shape[0]
    bits = np.zeros(27, dtype=np.int64)
    nxt = 26
    for cls in (3, 2, 1, 0):
        for t in range(27):
            d = (t // 9 - 1, (t // 3) % 3 - 1, t % 3 - 1)
            if sum(abs(v) for v in d) == cls:
                bits[t] = nxt
                nxt -= 1
    k = ((nbr < n).astype(np.int64) << bits[None, :]).sum(1)
    for sh in (1, 2, 4, 8, 16):
        k ^= k >> sh
    return k


@pytest.mark.parametrize("case", ["surface", "split", "ragged"])
def test_tap_order_is_a_stable_sort_by_mask(ex, oracle, case):
    coords = {"surface": synth.small_coords(205, extent=28, grid=32), "split": dense_offset_cube(),
              "ragged": synth.small_coords(31, extent=30, grid=32)[:129]}[case]
    nbr, plan = _level(ex, oracle, coords, "tap_order")
    order = parse_plan(plan, coords.shape[0])["order"]
    np.testing.assert_array_equal(order, np.argsort(tap_order_keys(nbr), kind="stable"))


def test_tap_order_tile_lists(ex, oracle):
    """A tap-order plan also stores, per 128-row tile, the rows (-1 past n),
    their neighbour lists in tap order (-1 = missing) and the tile's tap
    mask, after the other sections (plan.h PlanTiles)."""
    coords = synth.small_coords(31, extent=30, grid=32)[:1000]   # ragged last tile
    n = coords.shape[0]
    nbr, plan = _level(ex, oracle, coords, "tap_order")
    order = parse_plan(plan, n)["order"]
    b = plan.cpu().numpy()
    ntiles = (n + 127) // 128
    npad = ntiles * 128
    base = len(b) - _align(4 * ntiles) - _align(4 * 27 * npad) - _align(4 * npad)
    rows = b[base:base + 4 * npad].view(np.int32)
    off = base + _align(4 * npad)
    tnbr = b[off:off + 4 * 27 * npad].view(np.int32).reshape(npad, 27)
    off += _align(4 * 27 * npad)
    mask = b[off:off + 4 * ntiles].view(np.uint32)
    exp_rows = np.full(npad, -1, np.int32)
    exp_rows[:n] = order
    np.testing.assert_array_equal(rows, exp_rows)
    exp_nbr = np.full((npad, 27), -1, np.int32)
    sel = nbr[order]
    exp_nbr[:n] = np.where(sel < n, sel, -1)
    np.testing.assert_array_equal(tnbr, exp_nbr)
    bits = (exp_nbr >= 0).reshape(ntiles, 128, 27).any(1)
    np.testing.assert_array_equal(mask, (bits * (1 << np.arange(27))).sum(1).astype(np.uint32))


@pytest.mark.parametrize("tag", ["f32", "f16", "q8_0"])
@pytest.mark.parametrize("cin,cout", [(64, 64), (128, 128)])
def test_tap_ordered_conv_matches_oracle(ex, oracle, tag, cin, cout):
    from oracle.oracle import W_F16, W_F32
    coords = synth.small_coords(240 + cin, extent=24, grid=32, dilation="z1")
    n = coords.shape[0]
    nbr, plan = _level(ex, oracle, coords, "tap_order")
    x = synth.features(241, n, cin)
    w = synth.conv_weight(242, cin, cout)
    b = (0.1 * np.random.default_rng(243).standard_normal(cout)).astype(np.float32)
    ref = oracle.sparse_conv(x, nbr, w, {"f32": W_F32, "f16": W_F16, "q8_0": W_Q8_0}[tag], b)
    pw = ex.prepare_weight(weight_tensor(oracle, w, tag), tag, cin, cout, 27)
    y = host(ex.sparse_conv(dev(x), dev(nbr), pw, dev(b), plan=plan))
    yu = host(ex.sparse_conv(dev(x), dev(nbr), pw, dev(b)))
    ex.check()
    if tag == "f32":
        assert rel_l2(y, ref) < 1e-4
    else:
        assert rel_l2(y, ref) < TOL_FP16[0] and max_abs(y, ref) < TOL_FP16[1]
    assert rel_l2(y, yu) < 1e-5, rel_l2(y, yu)


def test_tap_ordered_res_block_matches_oracle(ex, oracle):
    from test_blocks_gpu import make_block, raw_block
    coords = synth.small_coords(250, extent=28, grid=32)
    nbr, plan = _level(ex, oracle, coords, "tap_order")
    x = dev(synth.features(251, coords.shape[0], 128)).to(torch.float16)
    raw = raw_block(252, 128)
    xin = host(x)
    ex.res_block(x, dev(nbr), make_block(ex, oracle, raw, "q8_0", 128), plan=plan)
    ex.check()
    ref = oracle.res_block(xin, nbr, raw, W_Q8_0)
    y = host(x)
    assert rel_l2(y, ref) < TOL_FP16[0] and max_abs(y, ref) < TOL_FP16[1]


@pytest.mark.parametrize("case", ["surface", "two_samples", "split"])
def test_plan_is_consistent_with_the_neighbour_map(ex, oracle, case):
    if case == "surface":
        coords = synth.small_coords(200, extent=28, grid=32)
    elif case == "two_samples":
        a = synth.small_coords(201, extent=20, grid=32)
        b = synth.small_coords(202, extent=20, grid=32)
        b[:, 3] = 1
        coords = np.concatenate([a, b])
    else:
        coords = dense_offset_cube()
    nbr, plan = _level(ex, oracle, coords)
    desc = check_plan(parse_plan(plan, coords.shape[0]), coords, nbr)
    if case == "split":
        assert np.any(desc[:, 1] < 128), "expected split subtiles"


@pytest.mark.parametrize("n", [1, 5, 127, 128, 129, 300])
def test_plan_ragged_sizes(ex, oracle, n):
    coords = synth.small_coords(31, extent=30, grid=32)[:n]
    nbr, plan = _level(ex, oracle, coords)
    check_plan(parse_plan(plan, n), coords, nbr)


def _q8_conv_case(ex, oracle, coords, cin, cout, xdt, seed):
    n = coords.shape[0]
    nbr, plan = _level(ex, oracle, coords)
    x = synth.features(seed, n, cin)
    w = synth.conv_weight(seed + 1, cin, cout)
    b = (0.1 * np.random.default_rng(seed + 2).standard_normal(cout)).astype(np.float32)
    xd = dev(x).to(xdt)
    ref = oracle.sparse_conv(host(xd), nbr, w, W_Q8_0, b)
    pw = ex.prepare_weight(weight_tensor(oracle, w, "q8_0"), "q8_0", cin, cout, 27)
    # the plan replaces the neighbour map for cin = 128; other widths ignore it
    y = ex.sparse_conv(xd, None if cin == 128 else dev(nbr), pw, dev(b), plan=plan)
    ex.check()
    y_unplanned = ex.sparse_conv(xd, dev(nbr), pw, dev(b))
    ex.check()
    return host(y), ref, host(y_unplanned)


@pytest.mark.parametrize("xdt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("cin,cout", [(64, 64), (64, 128), (128, 64), (128, 128)])
def test_planned_q8_conv_matches_oracle(ex, oracle, xdt, cin, cout):
    coords = synth.small_coords(210 + cin + cout, extent=24, grid=32)
    y, ref, yu = _q8_conv_case(ex, oracle, coords, cin, cout, xdt, 220)
    assert rel_l2(y, ref) < TOL_FP16[0] and max_abs(y, ref) < TOL_FP16[1], (rel_l2(y, ref), max_abs(y, ref))
    assert rel_l2(y, yu) < 1e-5, rel_l2(y, yu)


@pytest.mark.parametrize("cin,cout", [(64, 64), (128, 128)])
def test_planned_q8_conv_split_subtiles(ex, oracle, cin, cout):
    y, ref, yu = _q8_conv_case(ex, oracle, dense_offset_cube(), cin, cout, torch.float32, 230)
    assert rel_l2(y, ref) < TOL_FP16[0] and max_abs(y, ref) < TOL_FP16[1], (rel_l2(y, ref), max_abs(y, ref))
    assert rel_l2(y, yu) < 1e-5, rel_l2(y, yu)


@pytest.mark.parametrize("n", [1, 5, 127, 128, 129, 300])
def test_planned_q8_conv_ragged(ex, oracle, n):
    coords = synth.small_coords(31, extent=30, grid=32)[:n]
    y, ref, yu = _q8_conv_case(ex, oracle, coords, 128, 128, torch.float32, 240)
    assert rel_l2(y, ref) < TOL_FP16[0] and max_abs(y, ref) < TOL_FP16[1]
    assert rel_l2(y, yu) < 1e-5


def test_planned_conv_with_isolated_voxels_gives_bias(ex, oracle):
    """Voxels 3 apart have only their own centre tap; with zero features every
    output row is the bias (a missing tap contributes exactly 0)."""
    g = np.arange(0, 30, 3)
    x, y, z = np.meshgrid(g, g, g, indexing="ij")
    coords = np.stack([x.ravel(), y.ravel(), z.ravel(), np.zeros(x.size, np.int64)], 1).astype(np.int32)
    n = coords.shape[0]
    nbr, plan = _level(ex, oracle, coords)
    b = np.arange(128, dtype=np.float32)
    pw = ex.prepare_weight(weight_tensor(oracle, synth.conv_weight(250, 128, 128), "q8_0"), "q8_0", 128, 128, 27)
    out = host(ex.sparse_conv(torch.zeros((n, 128), device="cuda"), None, pw, dev(b), plan=plan))
    ex.check()
    np.testing.assert_array_equal(out, np.broadcast_to(b, (n, 128)))


def test_planned_res_block_and_chain(ex, oracle):
    """Two Q8_0 residual blocks at C=128 with fp16 state over one plan: each
    block within the features tolerance of the oracle on its actual input."""
    from test_blocks_gpu import make_block, raw_block
    coords = synth.small_coords(260, extent=28, grid=32)
    nbr, plan = _level(ex, oracle, coords)
    x = dev(synth.features(261, coords.shape[0], 128)).to(torch.float16)
    for blk in range(2):
        raw = raw_block(270 + 10 * blk, 128)
        xin = host(x)
        ex.res_block(x, None, make_block(ex, oracle, raw, "q8_0", 128), plan=plan)
        ex.check()
        y = host(x)
        ref = oracle.res_block(xin, nbr, raw, W_Q8_0)
        assert rel_l2(y, ref) < TOL_FP16[0] and max_abs(y, ref) < TOL_FP16[1], (blk, rel_l2(y, ref))


def test_plan_ignored_for_float_weights(ex, oracle):
    """F32 weights take the neighbour-map conv even when a plan is given."""
    coords = synth.small_coords(280, extent=20, grid=32)
    nbr, plan = _level(ex, oracle, coords)
    x = dev(synth.features(281, coords.shape[0], 64))
    pw = ex.prepare_weight(weight_tensor(oracle, synth.conv_weight(282, 64, 64), "f32"), "f32", 64, 64, 27)
    a = host(ex.sparse_conv(x, dev(nbr), pw, None, plan=plan))
    b = host(ex.sparse_conv(x, dev(nbr), pw, None))
    ex.check()
    np.testing.assert_array_equal(a, b)


def test_plan_of_another_level_is_rejected(ex, oracle):
    coords = synth.small_coords(290, extent=20, grid=32)
    nbr, plan = _level(ex, oracle, coords)
    n2 = coords.shape[0] - 1
    pw = ex.prepare_weight(weight_tensor(oracle, synth.conv_weight(291, 64, 64), "q8_0"), "q8_0", 64, 64, 27)
    with pytest.raises(MscError, match="plan covers"):
        ex.sparse_conv(dev(synth.features(292, n2, 64)), dev(nbr[:n2]), pw, None, plan=plan)
    with pytest.raises(MscError, match="not built by this context"):
        ex.sparse_conv(dev(synth.features(292, n2, 64)), dev(nbr[:n2]), pw, None,
                       plan=torch.empty(256, dtype=torch.uint8, device="cuda"))
