"""Conv plans (msc_conv_plan_build) and the convs that run over them
(msc_sparse_conv_planned / msc_res_block_planned).

A plan is the voxels of one level sorted, stably, by a class-ordered
tap-mask key, plus per 128-row tile the rows, their neighbour lists and the
tile's tap mask.  Its integer content is checked exactly against the
neighbour map; the conv over the plan is checked against the oracle at the
features tolerance (rel-L2 1e-3, max-abs 1e-2) and against the unplanned
conv, bit for bit: the conv visits a row's taps in ascending order in any
tile."""
import numpy as np
import pytest
import torch

from conftest import max_abs, rel_l2
from gpu_util import TOL_FP16, dev, host, weight_tensor
from mogecpp_b200 import synth
from mogecpp_b200.lib import MscError
from oracle.oracle import W_Q8_0

pytestmark = pytest.mark.gpu


def _align(v):
    return (v + 255) // 256 * 256


def parse_plan(buf, n):
    """Sections of a plan buffer (layout of mogecpp_b200/csrc/plan.h):
    header {magic, reserved, n}, order [n], tile rows [n_pad], tile
    neighbour lists [n_pad][27], tile masks [n_pad / 128], tile schedule
    [n_pad / 128]."""
    b = buf.cpu().numpy()
    magic = int(b[:4].view(np.uint32)[0])
    hn = int(b[8:16].view(np.int64)[0])
    ntiles = (n + 127) // 128
    npad = ntiles * 128
    off = _align(16)
    order = b[off:off + 4 * n].view(np.int32)
    off += _align(4 * n)
    rows = b[off:off + 4 * npad].view(np.int32)
    off += _align(4 * npad)
    tnbr = b[off:off + 4 * 27 * npad].view(np.int32).reshape(npad, 27)
    off += _align(4 * 27 * npad)
    mask = b[off:off + 4 * ntiles].view(np.uint32)
    off += _align(4 * ntiles)
    sched = b[off:off + 4 * ntiles].view(np.int32)
    return dict(magic=magic, n=hn, order=order, rows=rows, nbr=tnbr, mask=mask, sched=sched)


def dense_offset_cube(side=20, offset=(5, 3, 6)):
    """A solid block of voxels (every interior voxel has all 27 taps)."""
    g = np.arange(side)
    x, y, z = np.meshgrid(g + offset[0], g + offset[1], g + offset[2], indexing="ij")
    c = np.stack([x.ravel(), y.ravel(), z.ravel(), np.zeros(side ** 3, np.int64)], 1).astype(np.int32)
    keys = synth.pack_keys(c)
    return c[np.argsort(keys, kind="stable")]


def _level(ex, oracle, coords):
    nbr = oracle.make_level(coords)
    cd = dev(coords)
    plan = ex.conv_plan(cd, dev(nbr))
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
    nbr, plan = _level(ex, oracle, coords)
    order = parse_plan(plan, coords.shape[0])["order"]
    np.testing.assert_array_equal(order, np.argsort(tap_order_keys(nbr), kind="stable"))


def check_tiles(p, nbr):
    """Tile rows = the order padded with -1; tile neighbour lists = the map's
    rows in that order with -1 for missing taps; masks = the OR over rows."""
    n = nbr.shape[0]
    ntiles = (n + 127) // 128
    npad = ntiles * 128
    order = p["order"]
    exp_rows = np.full(npad, -1, np.int32)
    exp_rows[:n] = order
    np.testing.assert_array_equal(p["rows"], exp_rows)
    exp_nbr = np.full((npad, 27), -1, np.int32)
    sel = nbr[order]
    exp_nbr[:n] = np.where(sel < n, sel, -1)
    np.testing.assert_array_equal(p["nbr"], exp_nbr)
    bits = (exp_nbr >= 0).reshape(ntiles, 128, 27).any(1)
    np.testing.assert_array_equal(p["mask"], (bits * (1 << np.arange(27))).sum(1).astype(np.uint32))


def test_tap_order_tile_lists(ex, oracle):
    coords = synth.small_coords(31, extent=30, grid=32)[:1000]   # ragged last tile
    nbr, plan = _level(ex, oracle, coords)
    p = parse_plan(plan, coords.shape[0])
    assert p["magic"] == 0x4E4C5053 and p["n"] == coords.shape[0]
    check_tiles(p, nbr)


def test_tile_schedule_sorts_tiles_by_cost(ex, oracle):
    """The schedule lists every tile once, by descending cost (4 x the tile's
    taps + the taps of each 32-row quarter, summed), ties in tile order."""
    coords = synth.small_coords(33, extent=34, grid=48)
    nbr, plan = _level(ex, oracle, coords)
    p = parse_plan(plan, coords.shape[0])
    ntiles = p["mask"].shape[0]
    v = (p["nbr"] >= 0).reshape(ntiles, 4, 32, 27)
    cost = 4 * v.any((1, 2)).sum(1) + v.any(2).sum((1, 2))
    np.testing.assert_array_equal(p["sched"], np.argsort(-cost, kind="stable"))


@pytest.mark.parametrize("tag", ["f32", "f16", "q8_0"])
@pytest.mark.parametrize("cin,cout", [(64, 64), (128, 128)])
def test_tap_ordered_conv_matches_oracle(ex, oracle, tag, cin, cout):
    from oracle.oracle import W_F16, W_F32
    coords = synth.small_coords(240 + cin, extent=24, grid=32, dilation="z1")
    n = coords.shape[0]
    nbr, plan = _level(ex, oracle, coords)
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
    np.testing.assert_array_equal(y, yu)  # one tap order per row, any tiling


def test_tap_ordered_res_block_matches_oracle(ex, oracle):
    from test_blocks_gpu import make_block, raw_block
    coords = synth.small_coords(250, extent=28, grid=32)
    nbr, plan = _level(ex, oracle, coords)
    x = dev(synth.features(251, coords.shape[0], 128)).to(torch.float16)
    raw = raw_block(252, 128)
    xin = host(x)
    ex.res_block(x, dev(nbr), make_block(ex, oracle, raw, "q8_0", 128), plan=plan)
    ex.check()
    ref = oracle.res_block(xin, nbr, raw, W_Q8_0)
    y = host(x)
    assert rel_l2(y, ref) < TOL_FP16[0] and max_abs(y, ref) < TOL_FP16[1]


@pytest.mark.parametrize("n", [1, 5, 127, 128, 129, 300])
def test_plan_ragged_sizes(ex, oracle, n):
    coords = synth.small_coords(31, extent=30, grid=32)[:n]
    nbr, plan = _level(ex, oracle, coords)
    p = parse_plan(plan, n)
    np.testing.assert_array_equal(p["order"], np.argsort(tap_order_keys(nbr), kind="stable"))
    check_tiles(p, nbr)


def _q8_conv_case(ex, oracle, coords, cin, cout, xdt, seed):
    n = coords.shape[0]
    nbr, plan = _level(ex, oracle, coords)
    x = synth.features(seed, n, cin)
    w = synth.conv_weight(seed + 1, cin, cout)
    b = (0.1 * np.random.default_rng(seed + 2).standard_normal(cout)).astype(np.float32)
    xd = dev(x).to(xdt)
    ref = oracle.sparse_conv(host(xd), nbr, w, W_Q8_0, b)
    pw = ex.prepare_weight(weight_tensor(oracle, w, "q8_0"), "q8_0", cin, cout, 27)
    y = ex.sparse_conv(xd, dev(nbr), pw, dev(b), plan=plan)
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
    np.testing.assert_array_equal(y, yu)  # one tap order per row, any tiling


@pytest.mark.parametrize("cin,cout", [(64, 64), (128, 128)])
def test_planned_q8_conv_solid_block(ex, oracle, cin, cout):
    y, ref, yu = _q8_conv_case(ex, oracle, dense_offset_cube(), cin, cout, torch.float32, 230)
    assert rel_l2(y, ref) < TOL_FP16[0] and max_abs(y, ref) < TOL_FP16[1], (rel_l2(y, ref), max_abs(y, ref))
    np.testing.assert_array_equal(y, yu)  # one tap order per row, any tiling


@pytest.mark.parametrize("n", [1, 5, 127, 128, 129, 300])
def test_planned_q8_conv_ragged(ex, oracle, n):
    coords = synth.small_coords(31, extent=30, grid=32)[:n]
    y, ref, yu = _q8_conv_case(ex, oracle, coords, 128, 128, torch.float32, 240)
    assert rel_l2(y, ref) < TOL_FP16[0] and max_abs(y, ref) < TOL_FP16[1]
    np.testing.assert_array_equal(y, yu)


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
    out = host(ex.sparse_conv(torch.zeros((n, 128), device="cuda"), dev(nbr), pw, dev(b), plan=plan))
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
        ex.res_block(x, dev(nbr), make_block(ex, oracle, raw, "q8_0", 128), plan=plan)
        ex.check()
        y = host(x)
        ref = oracle.res_block(xin, nbr, raw, W_Q8_0)
        assert rel_l2(y, ref) < TOL_FP16[0] and max_abs(y, ref) < TOL_FP16[1], (blk, rel_l2(y, ref))


def test_plan_with_float_weights(ex, oracle):
    """F32 weights over a plan: each row's taps are summed in the same order
    in any tile, so the result is the unplanned one bit for bit."""
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
