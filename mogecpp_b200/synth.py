"""Seeded synthetic sparse-voxel workloads.

The refiner in mogecpp voxelises a predicted depth surface
(``src/sparse.cpp:363-431``: one voxel per pixel at a quantised log-depth
bin).  These generators stand in for that input with seeded height-field
surfaces of the same character: a thin, slowly varying 2.5-D shell in a cubic
grid, optionally dilated, deduplicated, and ordered by the packed
``(b, z, y, x)`` key so that every z-slab is a contiguous index range.

Coordinates are int32 ``[N, 4]`` rows ``(x, y, z, b)``: ``x`` is the image
row, ``y`` the image column and ``z`` the depth bin, as in the reference's
``Coord3`` (``src/sparse.cpp:69-74``); ``b`` is the sample index.  The voxel
index used by every map is the row position in this array.

Workloads (sizes recorded by ``describe()``):

* ``conv_c64``   seed 0, 128^3, z = 64 + 20 sin(x/9) cos(y/13) + N(0, 1.5),
  one-voxel (6-connected) dilation; C=64 fp32 single submanifold conv.
* ``res4_c128``  seed 1, 256^3, the same surface with amplitude, periods and
  noise doubled; four residual blocks at C=128, fp16 state, Q8_0 weights.
* ``unet_c64``   seeds 2 and 3, 256^3, batch 2; C=64 -> pool -> C=128 -> up.
* ``topo_4m``    union of 8 surfaces (seeds 10-17), each on a 300^2 patch at a
  seeded random offset inside 1024^3; topology only.
* ``shell_4m``   seed 20, full 1024^2 surface, 3-voxel-thick shell along z.
"""

from __future__ import annotations

import numpy as np

_OFFS = np.array([(dx, dy, dz) for dx in (-1, 0, 1) for dy in (-1, 0, 1) for dz in (-1, 0, 1)],
                 dtype=np.int64)
_CROSS = np.array([(0, 0, 0), (1, 0, 0), (-1, 0, 0), (0, 1, 0), (0, -1, 0), (0, 0, 1), (0, 0, -1)], dtype=np.int64)


def pack_keys(coords: np.ndarray) -> np.ndarray:
    """Packs (x, y, z, b) rows into uint64 keys ordered (b, z, y, x).

    Layout: b in bits 57..63 (7 bits), z in 38..56, y in 19..37, x in 0..18
    (19 bits each).  Sorting keys sorts voxels by (b, z, y, x).
    """
    c = coords.astype(np.uint64)
    return (c[:, 3] << np.uint64(57)) | (c[:, 2] << np.uint64(38)) | (c[:, 1] << np.uint64(19)) | c[:, 0]


def unpack_keys(keys: np.ndarray) -> np.ndarray:
    m = np.uint64((1 << 19) - 1)
    out = np.empty((keys.shape[0], 4), dtype=np.int32)
    out[:, 0] = (keys & m).astype(np.int32)
    out[:, 1] = ((keys >> np.uint64(19)) & m).astype(np.int32)
    out[:, 2] = ((keys >> np.uint64(38)) & m).astype(np.int32)
    out[:, 3] = (keys >> np.uint64(57)).astype(np.int32)
    return out


def height_surface(seed: int, extent: int, grid: int, z0: float, amp: float, px: float, py: float,
                   noise: float, dilation: str, offset=(0, 0, 0), b: int = 0) -> np.ndarray:
    """Voxelised height field z(x, y) over an extent x extent patch.

    ``dilation``: "none"; "z1" (z +-1, a 3-voxel-thick shell); "cross" (the
    one-voxel dilation by the 6-connected unit ball: the voxel and its face
    neighbours); or "xyz1" (full 3x3x3 cube).  Voxels outside [0, grid) are
    dropped.
    """
    rng = np.random.default_rng(seed)
    x, y = np.meshgrid(np.arange(extent, dtype=np.float64), np.arange(extent, dtype=np.float64), indexing="ij")
    z = z0 + amp * np.sin(x / px) * np.cos(y / py) + rng.normal(0.0, noise, size=x.shape)
    base = np.stack([x.ravel(), y.ravel(), np.rint(z).ravel()], axis=1).astype(np.int64)
    base += np.asarray(offset, dtype=np.int64)[None, :]
    if dilation == "none":
        pts = base
    elif dilation == "z1":
        pts = np.concatenate([base + np.array([0, 0, d]) for d in (-1, 0, 1)])
    elif dilation == "cross":
        pts = (base[:, None, :] + _CROSS[None, :, :]).reshape(-1, 3)
    elif dilation == "xyz1":
        pts = (base[:, None, :] + _OFFS[None, :, :]).reshape(-1, 3)
    else:
        raise ValueError(dilation)
    ok = np.all((pts >= 0) & (pts < grid), axis=1)
    pts = pts[ok]
    out = np.empty((pts.shape[0], 4), dtype=np.int32)
    out[:, :3] = pts
    out[:, 3] = b
    return out


def dedup_sorted(coords: np.ndarray) -> np.ndarray:
    """Deduplicates voxels and orders them by the packed (b, z, y, x) key."""
    return unpack_keys(np.unique(pack_keys(coords)))


def conv_c64_coords(seed: int = 0) -> np.ndarray:
    return dedup_sorted(height_surface(seed, 128, 128, 64.0, 20.0, 9.0, 13.0, 1.5, "cross"))


def res4_c128_coords(seed: int = 1) -> np.ndarray:
    return dedup_sorted(height_surface(seed, 256, 256, 128.0, 40.0, 18.0, 26.0, 3.0, "cross"))


def unet_coords(seeds=(2, 3)) -> np.ndarray:
    parts = [height_surface(s, 256, 256, 128.0, 40.0, 18.0, 26.0, 3.0, "cross", b=i) for i, s in enumerate(seeds)]
    return dedup_sorted(np.concatenate(parts))


def topo_4m_coords(seeds=tuple(range(10, 18))) -> np.ndarray:
    parts = []
    for s in seeds:
        rng = np.random.default_rng(1000 + s)
        off = (int(rng.integers(0, 1024 - 300)), int(rng.integers(0, 1024 - 300)), int(rng.integers(0, 1024 - 300)))
        parts.append(height_surface(s, 300, 1024, 150.0, 60.0, 27.0, 39.0, 3.0, "cross", offset=off))
    return dedup_sorted(np.concatenate(parts))


def shell_4m_coords(seed: int = 20) -> np.ndarray:
    return dedup_sorted(height_surface(seed, 1024, 1024, 512.0, 160.0, 72.0, 104.0, 6.0, "z1"))


def small_coords(seed: int, extent: int = 24, grid: int = 32, dilation: str = "cross", b: int = 0) -> np.ndarray:
    """A small surface for fast parity cases."""
    return dedup_sorted(height_surface(seed, extent, grid, grid / 2, grid / 6, 3.0, 4.0, 1.0, dilation, b=b))


_FEATURE_CHUNK = 65536


def features_rows(seed: int, rows: np.ndarray, c: int, dtype=np.float32) -> np.ndarray:
    """N(0, 1) features of the given rows of a seeded [n, c] array, drawn in
    float32 chunks of 65536 rows with their own streams, so that a rank can
    draw only its slab's rows and get the same values as a full draw."""
    rows = np.asarray(rows, dtype=np.int64)
    out = np.empty((rows.shape[0], c), dtype=dtype)
    if rows.size == 0:
        return out
    chunk = rows // _FEATURE_CHUNK
    for ch in np.unique(chunk):
        sel = np.flatnonzero(chunk == ch)
        block = np.random.default_rng([seed, int(ch)]).standard_normal((_FEATURE_CHUNK, c), dtype=np.float32)
        out[sel] = block[rows[sel] - ch * _FEATURE_CHUNK]
    return out


def features(seed: int, n: int, c: int, dtype=np.float32) -> np.ndarray:
    """N(0, 1) features for rows 0..n-1 (see features_rows)."""
    return features_rows(seed, np.arange(n), c, dtype)


def conv_weight(seed: int, cin: int, cout: int) -> np.ndarray:
    """Packed sparse27 weight [cout, 27*cin] (cin fastest, tap order of the
    neighbour map), drawn from N(0, (1/sqrt(27*cin))^2)."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((cout, 27 * cin)) / np.sqrt(27.0 * cin)).astype(np.float32)


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """ggml block_q8_0 rows of w (row length % 32 == 0) as raw uint8 bytes.

    The model-file quantiser ggml uses for weights (ggml-quants.c:274-296
    quantize_row_q8_0_ref): per 32 values d = amax/127 stored as fp16,
    q = round-half-away-from-zero(x / d)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    blk = w.reshape(-1, 32)
    amax = np.abs(blk).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    x = (blk * idv[:, None]).astype(np.float32)
    q = (np.sign(x) * np.floor(np.abs(x).astype(np.float64) + 0.5)).astype(np.int8)
    out = np.empty((blk.shape[0], 34), dtype=np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def describe(coords: np.ndarray) -> dict:
    return {"n": int(coords.shape[0]),
            "extent": [int(coords[:, i].max()) + 1 if coords.shape[0] else 0 for i in range(3)],
            "batch": int(coords[:, 3].max()) + 1 if coords.shape[0] else 0}


# ------------------------------------------------------------ refiner models

SMALL_REFINER = dict(model_channels=[64, 128, 128], encoder_blocks=[1, 1, 1], decoder_blocks=[1, 1],
                     bottleneck_blocks=1, encoder_channels=64, fuse_channels=64, fuse_hidden=128)
# A five-level refiner (four stride-2 levels, encoder_downsample 16) at the
# channel widths the tensor-core convs run (64 / 128).
REFINER_5L = dict(model_channels=[64, 64, 128, 128, 128], encoder_blocks=[1, 1, 1, 1, 1],
                  decoder_blocks=[1, 1, 1, 1], bottleneck_blocks=1, encoder_channels=128, fuse_channels=128,
                  fuse_hidden=128)


def refiner_mogg(seed: int, cfg: dict, wdtype: str = "f32", depth_resolution: float = 256.0) -> bytes:
    """A MOGG image of a MoGe-3 sparse refiner with seeded random weights:
    the refiner.* metadata of SparseConfig (src/sparse.cpp:985-1007) and the
    tensors SparseRefiner reads (sparse conv weights packed [cout][27 cin],
    linear weights [cout][cin]).  wdtype: "f32" or "f16" weight storage
    (biases and norm affines stay F32)."""
    from . import mogg
    rng = np.random.default_rng(seed)
    wt = mogg.T_F32 if wdtype == "f32" else mogg.T_F16
    mc = list(cfg["model_channels"])
    L = len(mc)
    t = []

    def lin(name, cin, cout):
        t.append(mogg.tensor(name + ".weight", rng.standard_normal((cout, cin)) / np.sqrt(cin), wt))
        t.append(mogg.tensor(name + ".bias", 0.05 * rng.standard_normal(cout), mogg.T_F32))

    def block(pfx, c):
        t.append(mogg.tensor(pfx + ".norm1.weight", 1 + 0.1 * rng.standard_normal(c), mogg.T_F32))
        t.append(mogg.tensor(pfx + ".norm1.bias", 0.1 * rng.standard_normal(c), mogg.T_F32))
        for k in ("conv1", "conv2"):
            t.append(mogg.tensor(f"{pfx}.{k}.weight.mogg_sparse27",
                                 rng.standard_normal((c, 27 * c)) / np.sqrt(27.0 * c), wt))
            t.append(mogg.tensor(f"{pfx}.{k}.bias", 0.05 * rng.standard_normal(c), mogg.T_F32))

    lin("refiner.input_proj", 3, mc[0])
    for lv in range(L):
        for b in range(cfg["encoder_blocks"][lv]):
            block(f"refiner.down_stages.{lv}.{b}", mc[lv])
        if lv + 1 < L:
            lin(f"refiner.downsample_blocks.{lv}.linear", mc[lv], mc[lv + 1])
    lin("refiner.encoder_fuse", cfg["encoder_channels"], cfg["fuse_channels"])
    lin("refiner.fuse_proj.0", mc[-1] + cfg["fuse_channels"], cfg["fuse_hidden"])
    lin("refiner.fuse_proj.2", cfg["fuse_hidden"], mc[-1])
    for b in range(cfg["bottleneck_blocks"]):
        block(f"refiner.bottleneck_stage.{b}", mc[-1])
    for u in range(L - 1):
        tgt = L - 2 - u
        lin(f"refiner.upsample_blocks.{u}.linear", mc[tgt + 1], mc[tgt])
        for b in range(cfg["decoder_blocks"][u]):
            block(f"refiner.up_stages.{u}.{b}", mc[tgt])
    lin("refiner.out_proj", mc[0], 1)
    meta = {"refiner.present": True, "refiner.in_channels": 3, "refiner.out_channels": 1,
            "refiner.encoder_channels": cfg["encoder_channels"], "refiner.model_channels": mc,
            "refiner.encoder_blocks_per_level": list(cfg["encoder_blocks"]),
            "refiner.decoder_blocks_per_level": list(cfg["decoder_blocks"]),
            "refiner.bottleneck_blocks": cfg["bottleneck_blocks"], "refiner.downsample_factors": [2] * (L - 1),
            "refiner.encoder_downsample": 2 ** (L - 1), "refiner.depth_resolution": float(depth_resolution)}
    return mogg.build(meta, t)


def refiner_inputs(seed: int, width: int, height: int, encoder_downsample: int, encoder_channels: int):
    """A predicted point map (factor_coord [h*w][3] = x/z, y/z, log z) of a
    smooth depth surface with two depth steps (so that some neighbouring
    pixels fall more than one bin apart), and a dense encoder feature matrix
    [eh*ew][encoder_channels] ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    v, u = np.meshgrid(np.arange(height, dtype=np.float64), np.arange(width, dtype=np.float64), indexing="ij")
    z = 2.0 + 0.5 * np.sin(u / 97.0) * np.cos(v / 71.0) + 0.3 * (u > width * 0.6) - 0.2 * (v > height * 0.7)
    z += rng.normal(0.0, 0.002, size=z.shape)
    fx = (u - width / 2) / (0.8 * width)
    fy = (v - height / 2) / (0.8 * width)
    fc = np.stack([fx, fy, np.log(z)], axis=-1).reshape(-1, 3).astype(np.float32)
    ew, eh = width // encoder_downsample, height // encoder_downsample
    enc = rng.standard_normal((eh * ew, encoder_channels)).astype(np.float32)
    return fc, enc, ew, eh
