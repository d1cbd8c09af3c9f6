"""Tensor-core sparse conv / linear against the reference goldens and the
oracle (tolerances: fp32 rel-L2 1e-4; fp16/bf16/Q8_0 rel-L2 1e-3, max-abs 1e-2)."""
import numpy as np
import pytest
import torch

from conftest import max_abs, rel_l2
from gpu_util import TOL_FP16, TOL_FP32, dev, host, weight_tensor
from mogecpp_b200 import synth
from mogecpp_b200.lib import MscError
from oracle.oracle import W_F16, W_F32, W_Q8_0

pytestmark = pytest.mark.gpu
WT = {"f32": W_F32, "f16": W_F16, "q8_0": W_Q8_0}


def tol_ok(y, ref, fp32):
    if fp32:
        assert rel_l2(y, ref) < TOL_FP32, rel_l2(y, ref)
    else:
        assert rel_l2(y, ref) < TOL_FP16[0], rel_l2(y, ref)
        assert max_abs(y, ref) < TOL_FP16[1], max_abs(y, ref)


@pytest.mark.parametrize("tag", ["f32", "f16", "q8_0"])
def test_sparse_conv_matches_reference_golden(ex, oracle, golden_features, tag):
    f = golden_features
    x = dev(f["x"].astype(np.float32))
    w = ex.prepare_weight(weight_tensor(oracle, f[f"conv_{tag}_w"].astype(np.float32), tag), tag, 64, 64, 27)
    y = ex.sparse_conv(x, dev(f["nbr"]), w, dev(f[f"conv_{tag}_b"].astype(np.float32)))
    ex.check()
    tol_ok(host(y), f[f"conv_{tag}_y"], fp32=(tag == "f32"))


def _case(seed, n_extent=20, c=128):
    coords = synth.small_coords(seed, extent=n_extent, grid=32)
    return coords, synth.features(seed + 1, coords.shape[0], c)


@pytest.mark.parametrize("tag", ["f32", "f16", "q8_0"])
@pytest.mark.parametrize("xdt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("cin,cout", [(64, 64), (64, 128), (128, 64), (128, 128)])
def test_sparse_conv_matches_oracle(ex, oracle, tag, xdt, cin, cout):
    coords, x = _case(100 + cin + cout, c=cin)
    n = coords.shape[0]
    nbr = oracle.make_level(coords)
    w = synth.conv_weight(7, cin, cout)
    b = (0.1 * np.random.default_rng(8).standard_normal(cout)).astype(np.float32)
    xd = dev(x).to(xdt)
    xr = host(xd)  # the oracle sees the same rounded inputs
    ref = oracle.sparse_conv(xr, nbr, w, WT[tag], b)
    pw = ex.prepare_weight(weight_tensor(oracle, w, tag), tag, cin, cout, 27)
    y = ex.sparse_conv(xd, dev(nbr), pw, dev(b))
    ex.check()
    tol_ok(host(y), ref, fp32=(tag == "f32" and xdt == torch.float32))
    assert n > 128


@pytest.mark.parametrize("n", [1, 5, 127, 128, 129, 300])
def test_sparse_conv_ragged_tiles(ex, oracle, n):
    coords = synth.small_coords(31, extent=30, grid=32)[:n]
    nbr = oracle.make_level(coords)
    x = synth.features(32, n, 64)
    w = synth.conv_weight(33, 64, 64)
    ref = oracle.sparse_conv(x, nbr, w, W_F32, None)
    pw = ex.prepare_weight(weight_tensor(oracle, w, "f32"), "f32", 64, 64, 27)
    y = ex.sparse_conv(dev(x), dev(nbr), pw, None)
    ex.check()
    tol_ok(host(y), ref, fp32=True)


def test_sparse_conv_output_dtypes(ex, oracle):
    coords, x = _case(41, c=64)
    nbr = oracle.make_level(coords)
    w = synth.conv_weight(42, 64, 64)
    ref = oracle.sparse_conv(x, nbr, w, W_F32, None)
    pw = ex.prepare_weight(weight_tensor(oracle, w, "f32"), "f32", 64, 64, 27)
    for dt in (torch.float16, torch.bfloat16):
        y = ex.sparse_conv(dev(x), dev(nbr), pw, None, out_dtype=dt)
        ex.check()
        assert y.dtype == dt
        assert rel_l2(host(y), ref) < (2e-3 if dt == torch.float16 else 8e-3)


@pytest.mark.parametrize("tag", ["f32", "f16", "q8_0"])
@pytest.mark.parametrize("cin,cout", [(64, 128), (128, 64)])
def test_linear_matches_oracle(ex, oracle, tag, cin, cout):
    n = 1000
    x = synth.features(50, n, cin)
    w = (np.random.default_rng(51).standard_normal((cout, cin)) / np.sqrt(cin)).astype(np.float32)
    b = (0.1 * np.random.default_rng(52).standard_normal(cout)).astype(np.float32)
    ref = oracle.linear(x, w, WT[tag], b)
    pw = ex.prepare_weight(weight_tensor(oracle, w, tag), tag, cin, cout, 1)
    y = ex.linear(dev(x), pw, dev(b))
    ex.check()
    tol_ok(host(y), ref, fp32=(tag == "f32"))


def test_all_sentinel_rows_give_bias(ex, oracle):
    n = 200
    nbr = np.full((n, 27), n, dtype=np.int32)
    x = synth.features(60, n, 64)
    b = np.arange(64, dtype=np.float32)
    pw = ex.prepare_weight(weight_tensor(oracle, synth.conv_weight(61, 64, 64), "f32"), "f32", 64, 64, 27)
    y = host(ex.sparse_conv(dev(x), dev(nbr), pw, dev(b)))
    ex.check()
    np.testing.assert_array_equal(y, np.broadcast_to(b, (n, 64)))


def test_unsupported_channels_rejected(ex, oracle):
    w = weight_tensor(oracle, synth.conv_weight(1, 32, 32), "f32")
    with pytest.raises(MscError):
        ex.prepare_weight(w, "f32", 32, 32, 27)


def test_workspace_too_small_rejected(ex, oracle):
    import ctypes as C
    coords, x = _case(70, c=64)
    nbr = dev(oracle.make_level(coords))
    pw = ex.prepare_weight(weight_tensor(oracle, synth.conv_weight(71, 64, 64), "f32"), "f32", 64, 64, 27)
    xd = dev(x)
    y = torch.empty_like(xd)
    ws = torch.empty(1024, dtype=torch.uint8, device="cuda")
    rc = ex.lib.msc_sparse_conv(ex.ctx, C.c_void_p(xd.data_ptr()), 0, x.shape[0], 64, C.c_void_p(nbr.data_ptr()),
                                C.c_void_p(pw.blob.data_ptr()), None, C.c_void_p(y.data_ptr()), 0,
                                C.c_void_p(ws.data_ptr()), 1024, None)
    assert rc == -5 and "workspace" in ex.lib.msc_last_error().decode()


@pytest.mark.parametrize("tag,xdt", [("q8_0", torch.float16), ("f32", torch.float32)])
@pytest.mark.parametrize("flags", [(True, True, True, True), (False, True, False, False), (True, False, True, False),
                                   (False, False, False, True)])
def test_fused_conv_matches_oracle_composition(ex, oracle, tag, xdt, flags):
    """msc_sparse_conv_fused: [SiLU](W * gather([SiLU]([LayerNorm](x))) + b)
    [+ residual] against the oracle's layer_norm, silu and sparse_conv run
    one after the other."""
    ln, silu_in, silu_out, res = flags
    coords = synth.small_coords(200, extent=22, grid=32)
    n = coords.shape[0]
    nbr = oracle.make_level(coords)
    rng = np.random.default_rng(201)
    x = synth.features(202, n, 128)
    gamma = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(128)).astype(np.float32)
    w = synth.conv_weight(203, 128, 128)
    b = (0.05 * rng.standard_normal(128)).astype(np.float32)
    r = synth.features(204, n, 128)
    xd = dev(x).to(xdt)
    xin = xd.float().cpu().numpy()
    pw = ex.prepare_weight(weight_tensor(oracle, w, tag), tag, 128, 128, 27)
    rd = dev(r).to(xdt) if res else None
    y = ex.sparse_conv_fused(xd, dev(nbr), pw, dev(b), plan=ex.conv_plan(dev(coords), dev(nbr)),
                             norm_w=dev(gamma), norm_b=dev(beta), layer_norm=ln, silu_in=silu_in,
                             silu_out=silu_out, residual=rd)
    ex.check()
    h = oracle.layer_norm(xin, gamma, beta, 1e-6) if ln else xin
    if silu_in:
        h = oracle.silu(h)
    ref = oracle.sparse_conv(h, nbr, w, WT[tag], b)
    if silu_out:
        ref = oracle.silu(ref)
    if res:
        ref = ref + rd.float().cpu().numpy()
    tol_ok(host(y), ref, fp32=(tag == "f32" and xdt == torch.float32))
