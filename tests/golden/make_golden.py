"""Generates the golden fixtures of tests/golden/ by running the reference.

The reference here is mogecpp's own CPU code (src/sparse.cpp + vendored
ggml 0.25.3), compiled from the read-only reference tree by
oracle/ref/Makefile into oracle/_ref/libmoge_ref.so.  Run from the repo root
in a checkout that has the reference tree next to it:

    make -f oracle/ref/Makefile REF=<path to mogecpp>
    python tests/golden/make_golden.py             # every fixture
    python tests/golden/make_golden.py groupnorm   # groupnorm.npz only
    python tests/golden/make_golden.py image       # image_topology.npz only
    python tests/golden/make_golden.py refiner     # refiner.npz only

Fixtures are seeded synthetic inputs and the reference's outputs; the tests
use them to pin the oracle port and the GPU path.  Inputs are rounded to
fp16-representable values so the files stay small (f16 storage) while the
computation itself still runs in the precision under test.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from mogecpp_b200 import synth  # noqa: E402
from oracle.oracle import Reference, W_F16, W_F32, W_Q8_0  # noqa: E402


def f16r(a):
    return np.asarray(a, dtype=np.float32).astype(np.float16)


def topology_cases():
    cases = {
        "surface": synth.small_coords(5, extent=24, grid=32),
        "surface_z1": synth.small_coords(6, extent=20, grid=32, dilation="z1"),
        "cube": synth.dedup_sorted(np.array([(x, y, z, 0) for x in range(4) for y in range(4) for z in range(4)],
                                            dtype=np.int32)),
        "single": np.array([[3, 5, 7, 0]], dtype=np.int32),
        "odd_line": np.array([[1, 1, z, 0] for z in range(1, 12, 3)], dtype=np.int32),
        # input order is not sorted: indices follow the given list order
        "shuffled": synth.small_coords(7, extent=12, grid=16)[np.random.default_rng(7).permutation(
            synth.small_coords(7, extent=12, grid=16).shape[0])],
    }
    return cases


def groupnorm_fixture(R):
    """ggml_group_norm (32 groups, eps 1e-5) of two samples' features, each
    normalised over its own voxels (the reference has no GroupNorm block;
    this pins the oracle's restatement of ggml's kernel)."""
    rng = np.random.default_rng(80)
    out = {}
    for s, n in enumerate((300, 200)):
        x = f16r(rng.standard_normal((n, 128)) * (1.5 + s) + 0.3 * s)
        out[f"gn{s}_x"] = x
        out[f"gn{s}_y"] = R.group_norm(x.astype(np.float32), 32, 1e-5)
    np.savez_compressed(os.path.join(HERE, "groupnorm.npz"), **out)
    print("groupnorm.npz", os.path.getsize(os.path.join(HERE, "groupnorm.npz")), "bytes")


def image_cases():
    """Point maps [h*w][3] for quantize_topology_z + make_dense_image_level."""
    cases = {}
    fc, _, _, _ = synth.refiner_inputs(5, 40, 32, 4, 8)
    cases["surface"] = (fc, 40, 32, 256.0)
    # log z exactly half-way between bins (z * 256 = k + 0.5): round half to even
    w, h = 12, 10
    k = np.arange(w * h) % 7 - 3
    t = np.zeros((w * h, 3), np.float32)
    t[:, 2] = (k + 0.5) / 256.0
    cases["ties"] = (t, w, h, 256.0)
    # negative log depths (z < 1) and a coarser resolution
    fc2, _, _, _ = synth.refiner_inputs(6, 24, 20, 4, 8)
    fc2[:, 2] -= 1.7
    cases["negative"] = (fc2, 24, 20, 96.0)
    flat = np.zeros((9 * 7, 3), np.float32)
    flat[:, 2] = 0.25
    cases["flat"] = (flat, 9, 7, 256.0)
    one = np.array([[0.1, 0.2, 0.7]], np.float32)
    cases["single"] = (one, 1, 1, 256.0)
    line = np.zeros((5, 3), np.float32)
    line[:, 2] = np.array([0.0, 1, 2, 4, 5], np.float32) / 256.0
    cases["row"] = (line, 5, 1, 256.0)
    return cases


def image_fixture(R):
    out = {}
    for name, (fc, w, h, r) in image_cases().items():
        z = R.quantize_topology_z(fc, w, h, r)
        out[f"img_{name}_fc"] = fc
        out[f"img_{name}_shape"] = np.array([w, h], np.int32)
        out[f"img_{name}_res"] = np.array([r], np.float32)
        out[f"img_{name}_zbin"] = z
        out[f"img_{name}_nbr"] = R.make_dense_image_level(z, w, h)
    np.savez_compressed(os.path.join(HERE, "image_topology.npz"), **out)
    print("image_topology.npz", os.path.getsize(os.path.join(HERE, "image_topology.npz")), "bytes")


REFINER_CASES = {"f32": (7, "f32"), "f16": (9, "f16")}   # model seed, weight storage


def refiner_fixture(R):
    """SparseRefiner::refine_once of the small synthetic refiner
    (synth.SMALL_REFINER, weights regenerated from the seed) on a 64 x 48
    point map: the updated log z of one pass."""
    out = {}
    fc, enc, ew, eh = synth.refiner_inputs(8, 64, 48, 4, synth.SMALL_REFINER["encoder_channels"])
    out["fc"] = fc
    out["enc"] = enc
    out["shape"] = np.array([64, 48, ew, eh], np.int32)
    for tag, (seed, wd) in REFINER_CASES.items():
        img = synth.refiner_mogg(seed, synth.SMALL_REFINER, wd)
        y, _ = R.refine_once(img, fc, 64, 48, enc, ew, eh)
        out[f"{tag}_logz"] = y[:, 2]
    np.savez_compressed(os.path.join(HERE, "refiner.npz"), **out)
    print("refiner.npz", os.path.getsize(os.path.join(HERE, "refiner.npz")), "bytes")


def main():
    R = Reference(n_threads=os.cpu_count() or 1)
    only = {"groupnorm": groupnorm_fixture, "image": image_fixture, "refiner": refiner_fixture}
    if sys.argv[1:] and sys.argv[1] in only:
        only[sys.argv[1]](R)
        return
    groupnorm_fixture(R)
    image_fixture(R)
    refiner_fixture(R)
    out = {}
    for name, c in topology_cases().items():
        c = np.ascontiguousarray(c, dtype=np.int32)
        nbr = R.make_level(c)
        parent, pool, inv, up = R.downsample(c)
        out[f"topo_{name}_coords"] = c
        out[f"topo_{name}_nbr"] = nbr
        out[f"topo_{name}_parent"] = parent
        out[f"topo_{name}_pool"] = pool
        out[f"topo_{name}_inv"] = inv
        out[f"topo_{name}_up"] = up
    np.savez_compressed(os.path.join(HERE, "topology.npz"), **out)

    # ---- features: sparse conv, res block, pool / up at C=64 -------------
    c = synth.small_coords(11, extent=14, grid=16)
    n = c.shape[0]
    nbr = R.make_level(c)
    C = 64
    x = f16r(synth.features(12, n, C))
    feats = {"coords": c, "nbr": nbr, "x": x}
    for tag, wt in (("f32", W_F32), ("f16", W_F16), ("q8_0", W_Q8_0)):
        w = f16r(synth.conv_weight(20 + wt, C, C))
        b = f16r(np.random.default_rng(30 + wt).standard_normal(C) * 0.1)
        y = R.sparse_conv(x.astype(np.float32), nbr, w.astype(np.float32), wt, b.astype(np.float32))
        feats[f"conv_{tag}_w"] = w
        feats[f"conv_{tag}_b"] = b
        feats[f"conv_{tag}_y"] = y
    for tag, wt in (("f32", W_F32), ("q8_0", W_Q8_0)):
        rng = np.random.default_rng(40 + wt)
        blk = dict(norm_w=f16r(1 + 0.1 * rng.standard_normal(C)), norm_b=f16r(0.1 * rng.standard_normal(C)),
                   w1=f16r(synth.conv_weight(50 + wt, C, C)), b1=f16r(0.05 * rng.standard_normal(C)),
                   w2=f16r(synth.conv_weight(60 + wt, C, C)), b2=f16r(0.05 * rng.standard_normal(C)))
        y, _ = R.res_stack(x.astype(np.float32), nbr, [{k: v.astype(np.float32) for k, v in blk.items()}], wt)
        for k, v in blk.items():
            feats[f"res_{tag}_{k}"] = v
        feats[f"res_{tag}_y"] = y
    parent, pool, inv, up = R.downsample(c)
    wl = f16r(np.random.default_rng(70).standard_normal((2 * C, C)) / np.sqrt(C))
    bl = f16r(0.1 * np.random.default_rng(71).standard_normal(2 * C))
    yp = R.pool_down(x.astype(np.float32), pool, inv, wl.astype(np.float32), W_F32, bl.astype(np.float32))
    wu = f16r(np.random.default_rng(72).standard_normal((C, 2 * C)) / np.sqrt(2 * C))
    bu = f16r(0.1 * np.random.default_rng(73).standard_normal(C))
    xu = f16r(yp)
    yu = R.nearest_up(xu.astype(np.float32), up, wu.astype(np.float32), W_F32, bu.astype(np.float32))
    feats.update(pool_rows=pool, inv=inv, up_rows=up, pool_w=wl, pool_b=bl, pool_y=yp, up_x=xu, up_w=wu, up_b=bu,
                 up_y=yu)
    np.savez_compressed(os.path.join(HERE, "features.npz"), **feats)
    for f in ("topology.npz", "features.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    main()
