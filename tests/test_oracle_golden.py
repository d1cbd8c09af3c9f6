"""The oracle port against the reference's own outputs (golden fixtures made
by tests/golden/make_golden.py from mogecpp's src/sparse.cpp + ggml CPU)."""
import numpy as np
import pytest

from conftest import max_abs, rel_l2
from oracle.oracle import W_F16, W_F32, W_Q8_0

TOPO = ["surface", "surface_z1", "cube", "single", "odd_line", "shuffled"]
WT = {"f32": W_F32, "f16": W_F16, "q8_0": W_Q8_0}


@pytest.mark.parametrize("name", TOPO)
def test_make_level_bit_exact(oracle, golden_topology, name):
    c = golden_topology[f"topo_{name}_coords"]
    np.testing.assert_array_equal(oracle.make_level(c), golden_topology[f"topo_{name}_nbr"])


@pytest.mark.parametrize("name", TOPO)
def test_downsample_bit_exact(oracle, golden_topology, name):
    g = golden_topology
    c = g[f"topo_{name}_coords"]
    parent, pool, inv, up = oracle.downsample(c)
    np.testing.assert_array_equal(parent[:, :3], g[f"topo_{name}_parent"])
    np.testing.assert_array_equal(pool, g[f"topo_{name}_pool"])
    np.testing.assert_array_equal(inv, g[f"topo_{name}_inv"])
    np.testing.assert_array_equal(up, g[f"topo_{name}_up"])


@pytest.mark.parametrize("tag", ["f32", "f16", "q8_0"])
def test_sparse_conv_matches_reference(oracle, golden_features, tag):
    f = golden_features
    y = oracle.sparse_conv(f["x"].astype(np.float32), f["nbr"], f[f"conv_{tag}_w"].astype(np.float32), WT[tag],
                           f[f"conv_{tag}_b"].astype(np.float32))
    assert rel_l2(y, f[f"conv_{tag}_y"]) < 1e-6
    assert max_abs(y, f[f"conv_{tag}_y"]) < 1e-5


@pytest.mark.parametrize("tag,tol", [("f32", 1e-6), ("q8_0", 1e-3)])
def test_res_block_matches_reference(oracle, golden_features, tag, tol):
    # Q8_0: the activation quantiser turns ~1e-7 summation-order differences
    # into occasional one-step flips, hence the fp16-path tolerance.
    f = golden_features
    blk = {k: f[f"res_{tag}_{k}"].astype(np.float32) for k in ("norm_w", "norm_b", "w1", "b1", "w2", "b2")}
    y = oracle.res_block(f["x"].astype(np.float32), f["nbr"], blk, WT[tag])
    assert rel_l2(y, f[f"res_{tag}_y"]) < tol


def test_pool_down_matches_reference(oracle, golden_features):
    f = golden_features
    y = oracle.pool_down(f["x"].astype(np.float32), f["pool_rows"], f["inv"], f["pool_w"].astype(np.float32), W_F32,
                         f["pool_b"].astype(np.float32))
    assert rel_l2(y, f["pool_y"]) < 1e-6


def test_nearest_up_matches_reference(oracle, golden_features):
    f = golden_features
    y = oracle.nearest_up(f["up_x"].astype(np.float32), f["up_rows"], f["up_w"].astype(np.float32), W_F32,
                          f["up_b"].astype(np.float32))
    assert rel_l2(y, f["up_y"]) < 1e-6


def test_q8_0_activation_quantiser_rounds_half_to_even(oracle):
    # x86 ggml quantize_row_q8_0: id = 127/amax, round-half-even; amax = 127
    # makes x*id exact so the ties are visible.
    x = np.zeros(32, dtype=np.float32)
    x[0] = 127.0
    x[1], x[2], x[3], x[4] = 0.5, 1.5, 2.5, -2.5
    q = oracle.quantize_q8_0_act(x)[0]["qs"]
    assert list(q[:5]) == [127, 0, 2, 2, -2]
    # weights use ggml's reference quantiser: round half away from zero
    qw = oracle.quantize_q8_0(x)[0]["qs"]
    assert list(qw[:5]) == [127, 1, 2, 3, -3]


def test_fp16_conversion_matches_numpy(oracle):
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.standard_normal(10000) * 10.0 ** rng.integers(-9, 6, 10000),
                        [0.0, -0.0, 65504.0, 65520.0, 6.1e-5, 5.96e-8, 2.98e-8, 1e-30, np.inf, -np.inf]]).astype(np.float32)
    got = np.array([oracle.lib.orc_fp32_to_fp16(float(a)) for a in v], dtype=np.uint16)
    np.testing.assert_array_equal(got, v.astype(np.float16).view(np.uint16))


def test_synthetic_q8_0_quantiser_matches_oracle(oracle):
    from mogecpp_b200 import synth
    w = synth.conv_weight(3, 64, 64)
    w[0, :32] = np.linspace(-1, 1, 32) * 127 / 127  # includes exact .5 ties after scaling
    mine = synth.quantize_q8_0(w)
    ref = np.frombuffer(oracle.quantize_q8_0(w).tobytes(), dtype=np.uint8)
    np.testing.assert_array_equal(mine, ref)
