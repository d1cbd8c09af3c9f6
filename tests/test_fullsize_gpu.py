"""Feature parity at the benchmark workloads' full sizes, against the
reference's own CPU build (oracle/_ref: mogecpp src/sparse.cpp + ggml 0.25.3,
all host threads).

* conv_c64 (77,507 voxels): one fp32 submanifold conv, C = 64, rel-L2 1e-4.
* res4_c128 (364,846 voxels): four GroupNorm(32) residual blocks at C = 128,
  fp16 state, Q8_0 weights; each block against the reference on the block's
  actual input (rel-L2 1e-3, max-abs 1e-2), and the chain against the
  reference's own chain with the same fp16 state rounding.
* unet_c64 (two surfaces, 2 x ~350k voxels): conv 64 -> pool + linear ->
  conv 128 -> linear + nearest up + skip with bf16 activations and fp32
  weights; each stage against the reference on the stage's bf16 input (the
  reference has no batch field: one call per sample), fp32 outputs at 1e-4.
* shell_4m (the 8-block LayerNorm stack the benchmark times): on a z-slab of
  131,072 voxels (the first in (b, z, y, x) order, a self-contained set),
  each block against the reference res_block on its actual input, and the
  chain against the reference chain.

Blocks: the state is fp16, so a block's output differs from the
reference's fp32 output by the fp16 rounding (rel-L2 2.1e-4 measured on both
stacks); against the reference output rounded to fp16 the same rows agree to
rel-L2 < 1e-4 (only last-bit summation-order differences remain).

Chains: ggml re-quantises every conv input to Q8_0, which turns last-bit
differences of fp32 summation order into one-step code flips that compound
over blocks; the reference and the oracle (both exact up to summation
order) already differ by rel-L2 1.3e-3 after four blocks on the small test
surface, and this build's four-block GroupNorm chain measured 3.1e-3 against
the reference's chain on res4_c128.  The chain bounds (5e-3 for four blocks,
8e-3 for eight) only catch gross drift; every block is held to the full
tolerance on identical inputs."""
import os

import numpy as np
import pytest
import torch

from conftest import ROOT, max_abs, rel_l2
from gpu_util import TOL_FP16, TOL_FP32, dev, host
from mogecpp_b200 import synth

pytestmark = pytest.mark.gpu

REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libmoge_ref.so")


@pytest.fixture(scope="module")
def ref():
    from oracle.oracle import Reference
    if not os.path.exists(REF_LIB):
        pytest.skip("the reference CPU build (oracle/_ref) is not built")
    return Reference(n_threads=os.cpu_count() or 1)


def _blocks(nblocks, c):
    import bench
    return bench.block_params(nblocks, c)


def _dev_block(ex, raw, c):
    q = lambda k: ex.prepare_weight(dev(np.frombuffer(synth.quantize_q8_0(raw[k]).tobytes(), np.uint8).copy()),
                                    "q8_0", c, c, 27)
    return dict(norm_w=dev(raw["norm_w"]), norm_b=dev(raw["norm_b"]), gn_w=dev(raw["gn_w"]), gn_b=dev(raw["gn_b"]),
                b1=dev(raw["b1"]), b2=dev(raw["b2"]), w1=q("w1"), w2=q("w2"))


def test_conv_c64_full_matches_reference(ex, ref):
    from oracle.oracle import W_F32
    coords = synth.conv_c64_coords()
    n = coords.shape[0]
    cd = dev(coords)
    nbr_d = ex.make_level(cd)
    plan = ex.conv_plan(cd, nbr_d)
    nbr = host(nbr_d)
    np.testing.assert_array_equal(nbr, ref.make_level(coords))
    x = synth.features(2, n, 64)
    w = synth.conv_weight(2100, 64, 64)
    b = (0.05 * np.random.default_rng(2101).standard_normal(64)).astype(np.float32)
    pw = ex.prepare_weight(dev(w), "f32", 64, 64, 27)
    y = host(ex.sparse_conv(dev(x), nbr_d, pw, dev(b), plan=plan))
    ex.check()
    r = ref.sparse_conv(x, nbr, w, W_F32, b)
    assert rel_l2(y, r) < TOL_FP32, rel_l2(y, r)


def test_res4_c128_groupnorm_blocks_match_reference(ex, ref):
    from oracle.oracle import W_Q8_0
    coords = synth.res4_c128_coords()
    n = coords.shape[0]
    cd = dev(coords)
    nbr_d = ex.make_level(cd)
    plan = ex.conv_plan(cd, nbr_d)
    nbr = host(nbr_d)
    x = dev(synth.features(2, n, 128, np.float16))
    chain = host(x)
    errs = []
    for raw in _blocks(4, 128):
        xin = host(x)
        ex.res_block_gn(x, nbr_d, cd, 1, _dev_block(ex, raw, 128), eps=1e-5, plan=plan)
        ex.check()
        y = host(x)
        r = ref.res_block_gn(xin, nbr, raw, W_Q8_0, 32, 1e-5)
        r16 = r.astype(np.float16).astype(np.float32)
        errs.append((rel_l2(y, r), max_abs(y, r), rel_l2(y, r16)))
        assert rel_l2(y, r) < TOL_FP16[0] and max_abs(y, r) < TOL_FP16[1], errs
        assert rel_l2(y, r16) < 1e-4, errs
        chain = ref.res_block_gn(chain, nbr, raw, W_Q8_0, 32, 1e-5).astype(np.float16).astype(np.float32)
    assert rel_l2(host(x), chain) < 5e-3, (rel_l2(host(x), chain), errs)


def test_unet_level_full_bf16_matches_reference(ex, ref):
    import bench
    from oracle.oracle import W_F32
    coords = synth.unet_coords()
    p = bench.unet_params()
    cd = dev(coords)
    nbr_d = ex.make_level(cd)
    tr = ex.downsample(cd)
    nbr_c_d = ex.make_level(tr.parent.contiguous())
    x = dev(synth.features(2, coords.shape[0], 64)).to(torch.bfloat16)
    P = lambda k, ci, co, t: ex.prepare_weight(dev(p[k]), "f32", ci, co, t)
    pw0, pwl, pw1, pwu = P("w0", 64, 64, 27), P("wl", 64, 128, 1), P("w1", 128, 128, 27), P("wu", 128, 64, 1)
    # each stage in fp32, then rounded to bf16 as the next stage's input
    h0 = ex.sparse_conv(x, nbr_d, pw0, None, out_dtype=torch.float32)
    h0b = h0.to(torch.bfloat16)
    h1 = ex.pool_down(h0b, tr, pwl, None, out_dtype=torch.float32)
    h1b = h1.to(torch.bfloat16)
    h2 = ex.sparse_conv(h1b, nbr_c_d, pw1, None, out_dtype=torch.float32)
    h2b = h2.to(torch.bfloat16)
    y = ex.nearest_up(h2b, tr, pwu, None, skip=h0b, out_dtype=torch.float32)
    ex.check()
    nbr, nbr_c = host(nbr_d), host(nbr_c_d)
    pool, inv, up, parent = host(tr.pool_rows), host(tr.inv_count), host(tr.up_rows), host(tr.parent)
    fine_b, par_b = coords[:, 3], parent[:, 3]
    for b in (0, 1):
        f = np.flatnonzero(fine_b == b)
        q = np.flatnonzero(par_b == b)
        # the sample's own maps: indices renumbered into the sample
        fmap = np.full(coords.shape[0] + 1, f.size, np.int64)
        fmap[f] = np.arange(f.size)
        pmap = np.full(parent.shape[0] + 1, q.size, np.int64)
        pmap[q] = np.arange(q.size)
        c_f, c_q = coords[f].copy(), parent[q].copy()
        c_f[:, 3] = 0
        c_q[:, 3] = 0
        nb = ref.make_level(c_f)
        np.testing.assert_array_equal(nb, fmap[np.minimum(nbr[f], coords.shape[0])].astype(np.int32))
        rp, rpool, rinv, rup = ref.downsample(c_f)
        np.testing.assert_array_equal(rp, c_q[:, :3])
        np.testing.assert_array_equal(rpool, fmap[np.minimum(pool[:, q], coords.shape[0])].astype(np.int32))
        np.testing.assert_array_equal(rup, pmap[up[f]].astype(np.int32))
        np.testing.assert_array_equal(rinv, inv[q])
        nbc = ref.make_level(c_q)
        np.testing.assert_array_equal(nbc, pmap[np.minimum(nbr_c[q], parent.shape[0])].astype(np.int32))
        r0 = ref.sparse_conv(host(x)[f], nb, p["w0"], W_F32, None)
        assert rel_l2(host(h0)[f], r0) < TOL_FP32, rel_l2(host(h0)[f], r0)
        r1 = ref.pool_down(host(h0b)[f], rpool, rinv, p["wl"], W_F32, None)
        assert rel_l2(host(h1)[q], r1) < TOL_FP32, rel_l2(host(h1)[q], r1)
        r2 = ref.sparse_conv(host(h1b)[q], nbc, p["w1"], W_F32, None)
        assert rel_l2(host(h2)[q], r2) < TOL_FP32, rel_l2(host(h2)[q], r2)
        ry = ref.nearest_up(host(h2b)[q], rup, p["wu"], W_F32, None) + host(h0b)[f]
        assert rel_l2(host(y)[f], ry) < TOL_FP32, rel_l2(host(y)[f], ry)


def test_shell_4m_slab_sample_blocks_match_reference(ex, ref):
    from oracle.oracle import W_Q8_0
    ns = 131072
    coords = synth.shell_4m_coords()[:ns]
    cd = dev(coords)
    nbr_d = ex.make_level(cd)
    plan = ex.conv_plan(cd, nbr_d)
    nbr = host(nbr_d)
    np.testing.assert_array_equal(nbr, ref.make_level(coords))
    x = dev(synth.features_rows(2, np.arange(ns), 128, np.float16))
    chain = host(x)
    errs = []
    for raw in _blocks(8, 128):
        xin = host(x)
        ex.res_block(x, nbr_d, _dev_block(ex, raw, 128), plan=plan)
        ex.check()
        y = host(x)
        r = ref.res_stack(xin, nbr, [raw], W_Q8_0)[0]
        r16 = r.astype(np.float16).astype(np.float32)
        errs.append((rel_l2(y, r), max_abs(y, r), rel_l2(y, r16)))
        assert rel_l2(y, r) < TOL_FP16[0] and max_abs(y, r) < TOL_FP16[1], errs
        assert rel_l2(y, r16) < 1e-4, errs
        chain = ref.res_stack(chain, nbr, [raw], W_Q8_0)[0].astype(np.float16).astype(np.float32)
    assert rel_l2(host(x), chain) < 8e-3, (rel_l2(host(x), chain), errs)
