"""Level-0 image topology, log-depth quantisation and the device refiner
(msc_refiner_*) against the reference.

* quantize_topology_z and make_dense_image_level: bit-exact against the
  reference's outputs (tests/golden/image_topology.npz: half-way ties,
  negative log depths, a flat image, single pixels).
* refine_once of the small synthetic refiner (three levels, C = 64 / 128,
  tests/golden/refiner.npz made by the reference's SparseRefiner): the
  log-depth update within rel-L2 1e-4 of the reference for F32 weights and
  1e-3 for F16 weights (activations rounded to fp16 as ggml does), the level
  sizes of the cached topology equal to the oracle's stride-2 chain, a repeated
  pass served by the topology cache, and the host-buffer entry point equal to
  the device one."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ROOT, rel_l2
from gpu_util import dev, host
from mogecpp_b200 import synth
from mogecpp_b200.lib import MscError

pytestmark = pytest.mark.gpu
IMG = ["surface", "ties", "negative", "flat", "single", "row"]


@pytest.fixture(scope="module")
def golden_image():
    return np.load(os.path.join(GOLDEN, "image_topology.npz"))


@pytest.fixture(scope="module")
def golden_refiner():
    return np.load(os.path.join(GOLDEN, "refiner.npz"))


@pytest.mark.parametrize("name", IMG)
def test_image_topology_matches_reference(ex, golden_image, name):
    g = golden_image
    w, h = (int(v) for v in g[f"img_{name}_shape"])
    z = ex.quantize_topology_z(dev(g[f"img_{name}_fc"]), float(g[f"img_{name}_res"][0]))
    np.testing.assert_array_equal(host(z), g[f"img_{name}_zbin"])
    coords, nbr = ex.make_dense_image_level(z, w, h)
    ex.check()
    np.testing.assert_array_equal(host(nbr), g[f"img_{name}_nbr"])
    yy, xx = np.divmod(np.arange(w * h), w)
    np.testing.assert_array_equal(host(coords), np.stack([yy, xx, g[f"img_{name}_zbin"], 0 * xx], 1))


def test_image_topology_large_matches_oracle(ex, oracle):
    fc, _, _, _ = synth.refiner_inputs(31, 640, 480, 16, 8)
    z = ex.quantize_topology_z(dev(fc), 256.0)
    zo = oracle.quantize_topology_z(fc, 256.0)
    np.testing.assert_array_equal(host(z), zo)
    _, nbr = ex.make_dense_image_level(z, 640, 480)
    np.testing.assert_array_equal(host(nbr), oracle.dense_image_level(zo, 640, 480))


def test_quantize_rejects_non_finite_depth(ex):
    fc = np.zeros((16, 3), np.float32)
    fc[5, 2] = np.nan
    with pytest.raises(MscError, match="out of range"):
        ex.quantize_topology_z(dev(fc), 256.0)


def _refiner(ex, tag):
    from mogecpp_b200.sparse import SparseRefiner
    seed, wd = {"f32": (7, "f32"), "f16": (9, "f16")}[tag]
    return SparseRefiner(ex, synth.refiner_mogg(seed, synth.SMALL_REFINER, wd))


@pytest.mark.parametrize("tag,tol", [("f32", 1e-4), ("f16", 1e-3)])
def test_refine_once_matches_reference(ex, golden_refiner, tag, tol):
    g = golden_refiner
    w, h, ew, eh = (int(v) for v in g["shape"])
    R = _refiner(ex, tag)
    fc = dev(g["fc"])
    R.refine_once(fc, w, h, dev(g["enc"]), ew, eh)
    got = host(fc)
    np.testing.assert_array_equal(got[:, :2], g["fc"][:, :2])   # only log z changes
    d_got, d_ref = got[:, 2] - g["fc"][:, 2], g[f"{tag}_logz"] - g["fc"][:, 2]
    assert rel_l2(d_got, d_ref) < tol, rel_l2(d_got, d_ref)


def test_refiner_topology_cache_and_levels(ex, oracle, golden_refiner):
    g = golden_refiner
    w, h, ew, eh = (int(v) for v in g["shape"])
    R = _refiner(ex, "f32")
    enc = dev(g["enc"])
    a, b = dev(g["fc"]), dev(g["fc"])
    R.refine_once(a, w, h, enc, ew, eh)
    R.refine_once(b, w, h, enc, ew, eh)      # same log z: the cached topology serves it
    assert R.cache_stats() == (1, 1)
    np.testing.assert_array_equal(host(a), host(b))
    # level sizes: the oracle's stride-2 chain from the level-0 voxels
    z = oracle.quantize_topology_z(g["fc"], 256.0)
    yy, xx = np.divmod(np.arange(w * h), w)
    c = np.stack([yy, xx, z, 0 * z], 1).astype(np.int32)
    sizes = [c.shape[0]]
    for _ in range(len(synth.SMALL_REFINER["model_channels"]) - 1):
        c = oracle.downsample(c)[0]
        sizes.append(c.shape[0])
    assert R.level_sizes() == sizes
    R.refine_once(a, w, h, enc, ew, eh)      # log z moved: a new topology
    assert R.cache_stats() == (1, 2)


def test_refiner_host_buffers_match_device(ex, golden_refiner):
    g = golden_refiner
    w, h, ew, eh = (int(v) for v in g["shape"])
    R = _refiner(ex, "f16")
    d = dev(g["fc"])
    R.refine_once(d, w, h, dev(g["enc"]), ew, eh)
    hfc = torch.from_numpy(g["fc"].copy())
    R.refine_once(hfc, w, h, torch.from_numpy(g["enc"].copy()), ew, eh)
    np.testing.assert_array_equal(hfc.numpy(), host(d))


def test_refiner_rejects_a_grid_that_does_not_match_the_encoder(ex, golden_refiner):
    g = golden_refiner
    R = _refiner(ex, "f32")
    with pytest.raises(MscError, match="does not match encoder"):
        R.refine_once(dev(g["fc"]), 64, 48, dev(g["enc"]), 15, 12)


def test_refiner_config_from_mogg_metadata(ex):
    R = _refiner(ex, "f32")
    c = R.config
    assert c.num_levels == 3 and list(c.model_channels[:3]) == [64, 128, 128]
    assert c.encoder_downsample == 4 and c.encoder_channels == 64 and abs(c.depth_resolution - 256.0) < 1e-6


def test_refine_once_live_reference_five_levels(ex):
    """A five-level refiner (encoder_downsample 16) on a 256 x 192 point map
    with F16 weights, against the reference's refine_once run now."""
    if not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libmoge_ref.so")):
        pytest.skip("reference CPU build not present")
    from mogecpp_b200.sparse import SparseRefiner
    from oracle.oracle import Reference
    img = synth.refiner_mogg(11, synth.REFINER_5L, "f16")
    fc, enc, ew, eh = synth.refiner_inputs(12, 256, 192, 16, synth.REFINER_5L["encoder_channels"])
    ref, _ = Reference(n_threads=os.cpu_count() or 1).refine_once(img, fc, 256, 192, enc, ew, eh)
    R = SparseRefiner(ex, img)
    d = dev(fc)
    R.refine_once(d, 256, 192, dev(enc), ew, eh)
    assert rel_l2(host(d)[:, 2] - fc[:, 2], ref[:, 2] - fc[:, 2]) < 1e-3
