"""Seeded synthetic workloads: the voxel sets the benchmark and the full-size
parity tests run on are pinned (count, bounds, digest), ordered and free of
duplicates, and the slab-wise feature draw equals the full draw."""
import hashlib

import numpy as np
import pytest

from mogecpp_b200 import synth

# name -> (voxels, min (x, y, z, b), max (x, y, z, b), sha256 prefix of the int32 rows)
WORKLOADS = {
    "conv_c64_coords": (77507, (0, 0, 39, 0), (127, 127, 89, 0), "fa47453595f4a0ef"),
    "res4_c128_coords": (364846, (0, 0, 77, 0), (255, 255, 178, 0), "19eb9dc8813edb38"),
    "unet_coords": (730717, (0, 0, 78, 0), (255, 255, 179, 1), "4f1177b95ecc05d6"),
    "topo_4m_coords": (4026477, (103, 67, 137, 0), (1014, 964, 860, 0), "44a30ffdade1eb10"),
    "shell_4m_coords": (3145728, (0, 0, 327, 0), (1023, 1023, 696, 0), "0ff66ad2d8eb05dd"),
}


@pytest.mark.parametrize("name", sorted(WORKLOADS))
def test_workload_voxel_sets_are_pinned(name):
    n, lo, hi, digest = WORKLOADS[name]
    c = getattr(synth, name)()
    assert c.dtype == np.int32 and c.shape == (n, 4)
    assert tuple(c.min(0)) == lo and tuple(c.max(0)) == hi
    assert hashlib.sha256(np.ascontiguousarray(c).tobytes()).hexdigest()[:16] == digest
    keys = synth.pack_keys(c)
    assert bool(np.all(keys[1:] > keys[:-1])), "rows must be unique and in (b, z, y, x) order"
    np.testing.assert_array_equal(synth.unpack_keys(keys), c)


def test_feature_rows_of_a_slab_equal_the_full_draw():
    n, c = 3 * 65536 + 1234, 8
    full = synth.features(7, n, c)
    rng = np.random.default_rng(0)
    rows = np.sort(rng.choice(n, size=5000, replace=False))
    np.testing.assert_array_equal(synth.features_rows(7, rows, c), full[rows])
    # a contiguous slab crossing a chunk boundary
    slab = np.arange(65536 - 100, 2 * 65536 + 100)
    np.testing.assert_array_equal(synth.features_rows(7, slab, c), full[slab])
    assert synth.features_rows(7, np.empty(0, np.int64), c).shape == (0, c)


def test_weight_quantiser_rounds_half_away_from_zero():
    """Model-file Q8_0 (ggml quantize_row_q8_0_ref): d = amax / 127 as fp16,
    q = round half away from zero of x / d."""
    w = np.zeros(32, np.float32)
    w[0] = 127.0                  # d = 1
    w[1], w[2] = 2.5, -2.5        # ties: away from zero
    w[3], w[4] = 0.49, -126.6
    q = synth.quantize_q8_0(w)
    assert q.shape == (34,)
    assert q[:2].view(np.float16)[0] == np.float16(1.0)
    codes = q[2:].view(np.int8)
    assert list(codes[:5]) == [127, 3, -3, 0, -127]
    assert not codes[5:].any()
