"""Host-side mirror of the reference's sparse operator surface, on the B200 path.

``SparseCudaExecutor`` plays the role of the reference's backend executor
seam (``SparseMetalExecutor``, src/sparse_metal.hpp:21-52): ``create()`` binds
a CUDA device and fails on anything but sm_100, and its methods are the
refiner's operators with the reference's names and argument meaning
(src/sparse.cpp):

    make_level(coords)                    -> nbr [n, 27]          (:238-272)
    conv_plan(coords, nbr)                -> plan (no counterpart: tap-ordered conv tiles)
    downsample(coords)                    -> Transition           (:312-357)
    sparse_conv(x, nbr, w, bias)          -> y [n, cout]          (:579-627)
    res_block(x, nbr, block)              -> x (in place)         (:629-642)
    res_block_gn(x, nbr, coords, ...)     -> x (in place)         (GroupNorm variant; ggml group_norm)
    pool_down(x, tr, w, bias)             -> y [np, cout]         (:646-668)
    nearest_up(x, tr, w, bias, skip)      -> y [nfine, cout]      (:670-674)
    linear(x, w, bias)                    -> y [n, cout]          (:515-518)
    quantize_topology_z(factor_coord, r)  -> zbin [h*w]           (:363-406)
    make_dense_image_level(zbin, w, h)    -> coords, nbr          (:274-310)

``SparseRefiner`` is the refiner itself (SparseRefiner, src/sparse.hpp:41-66):
built from a MOGG image, ``refine_once`` updates log z of a point map in
place with every step on the GPU.

Every call goes through the C ABI of ``libmoge_sparse_cuda.so``; tensors are
torch CUDA tensors used only as device memory.  Errors raise ``MscError``
with the library's message, as the reference throws ``std::runtime_error``.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import lib as L

_DT = {torch.float32: L.MSC_F32, torch.float16: L.MSC_F16, torch.bfloat16: L.MSC_BF16}
_WT = {"f32": L.MSC_W_F32, "f16": L.MSC_W_F16, "q8_0": L.MSC_W_Q8_0}


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


@dataclass
class Transition:
    """Stride-2 maps (reference ``Transition``, src/sparse.cpp:139-147)."""
    parent: torch.Tensor      # [np, 4] int32 parent coordinates
    pool_rows: torch.Tensor   # [8, np] int32, slot-major, sentinel nfine
    inv_count: torch.Tensor   # [np] float32
    up_rows: torch.Tensor     # [nfine] int32
    np: int
    nfine: int
    np_dev: torch.Tensor | None = None  # [1] int32 parent count on the device


@dataclass
class PreparedWeight:
    """Weights converted once into the tensor-core blob (``msc_weight_prepare``)."""
    blob: torch.Tensor
    wtype: str
    cin: int
    cout: int
    ntaps: int


class SparseCudaExecutor:
    def __init__(self, device: int = 0):
        self.lib = L.load()
        self.device = device
        torch.cuda.set_device(device)
        h = C.c_void_p()
        L.check(self.lib.msc_create(device, C.byref(h)))
        self.ctx = h
        self._ws = None

    @classmethod
    def create(cls, device: int = 0) -> "SparseCudaExecutor | None":
        """Returns None when no sm_100 device is available (as the reference's
        stub executor does, src/sparse_metal_stub.cpp:18-20)."""
        try:
            if not torch.cuda.is_available():
                return None
            return cls(device)
        except (L.MscError, RuntimeError):
            return None

    def close(self):
        if self.ctx:
            self.lib.msc_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------- plumbing
    def workspace(self, nbytes: int) -> torch.Tensor:
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=f"cuda:{self.device}")
        return self._ws

    def check(self) -> int:
        """Syncs the current stream and raises on any device-side failure."""
        bits = C.c_uint32(0)
        L.check(self.lib.msc_check(self.ctx, _stream(), C.byref(bits)))
        return bits.value

    def profile(self, enable: bool = True) -> None:
        """Starts / stops per-launch CUDA-event timing of this executor's kernels."""
        L.check(self.lib.msc_profile_enable(self.ctx, int(enable)))

    def profile_read(self) -> dict:
        """{kernel family: (launches, total ms)} since the last read; syncs."""
        buf = (L.ProfileEntry * 32)()
        cnt = C.c_int(0)
        L.check(self.lib.msc_profile_read(self.ctx, buf, 32, C.byref(cnt)))
        return {buf[i].name.decode(): (buf[i].launches, buf[i].total_ms) for i in range(min(cnt.value, 32))}

    # ---------------------------------------------------------- topology
    def make_level(self, coords: torch.Tensor) -> torch.Tensor:
        n = coords.shape[0]
        nbr = torch.empty((n, 27), dtype=torch.int32, device=coords.device)
        wsb = self.lib.msc_topology_workspace_bytes(n)
        ws = self.workspace(wsb)
        L.check(self.lib.msc_make_level(self.ctx, _p(coords), n, _p(nbr), _p(ws), wsb, _stream()))
        return nbr

    def downsample(self, coords: torch.Tensor, sync: bool = True) -> Transition:
        """Stride-2 maps.  With sync=False the parent count stays on the
        device (no stream sync): the returned tensors are then sized for the
        worst case (np = nfine) and ``np`` is -1; read ``np_dev``."""
        n = coords.shape[0]
        dev = coords.device
        parent = torch.empty((max(n, 1), 4), dtype=torch.int32, device=dev)
        np_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        pool = torch.empty(8 * max(n, 1), dtype=torch.int32, device=dev)
        inv = torch.empty(max(n, 1), dtype=torch.float32, device=dev)
        up = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        wsb = self.lib.msc_topology_workspace_bytes(n)
        ws = self.workspace(wsb)
        np_host = C.c_int64(0)
        L.check(self.lib.msc_downsample(self.ctx, _p(coords), n, _p(parent), _p(np_dev), _p(pool), _p(inv), _p(up),
                                        C.byref(np_host) if sync else None, _p(ws), wsb, _stream()))
        if not sync:
            return Transition(parent, pool, inv, up[:n], -1, n, np_dev)
        m = np_host.value
        return Transition(parent[:m], pool[:8 * m].view(8, m), inv[:m], up[:n], m, n, np_dev)

    def make_level_downsample(self, coords: torch.Tensor, sync: bool = True):
        """make_level and downsample of the same voxels in one call (one
        voxel table): returns (nbr, Transition), as the two calls would."""
        n = coords.shape[0]
        dev = coords.device
        nbr = torch.empty((n, 27), dtype=torch.int32, device=dev)
        parent = torch.empty((max(n, 1), 4), dtype=torch.int32, device=dev)
        np_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        pool = torch.empty(8 * max(n, 1), dtype=torch.int32, device=dev)
        inv = torch.empty(max(n, 1), dtype=torch.float32, device=dev)
        up = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        wsb = self.lib.msc_topology_workspace_bytes(n)
        ws = self.workspace(wsb)
        np_host = C.c_int64(0)
        L.check(self.lib.msc_make_level_downsample(self.ctx, _p(coords), n, _p(nbr), _p(parent), _p(np_dev), _p(pool),
                                                   _p(inv), _p(up), C.byref(np_host) if sync else None, _p(ws), wsb,
                                                   _stream()))
        if not sync:
            return nbr, Transition(parent, pool, inv, up[:n], -1, n, np_dev)
        m = np_host.value
        return nbr, Transition(parent[:m], pool[:8 * m].view(8, m), inv[:m], up[:n], m, n, np_dev)

    def conv_plan(self, coords: torch.Tensor, nbr: torch.Tensor, kind: str = "tap_order") -> torch.Tensor:
        """Conv plan of a level (``msc_conv_plan_build``) for sparse_conv /
        res_block on the same level: the voxels in tiles of rows with similar
        neighbourhoods (any weights)."""
        n = coords.shape[0]
        pb = self.lib.msc_conv_plan_bytes(n)
        plan = torch.empty(pb, dtype=torch.uint8, device=coords.device)
        wsb = self.lib.msc_conv_plan_workspace_bytes(n)
        ws = self.workspace(wsb)
        code = {"tap_order": L.MSC_PLAN_TAP_ORDER}[kind]
        L.check(self.lib.msc_conv_plan_build(self.ctx, _p(coords), n, _p(nbr), code, _p(plan), pb, _p(ws), wsb,
                                             _stream()))
        return plan

    def quantize_topology_z(self, factor_coord: torch.Tensor, depth_resolution: float) -> torch.Tensor:
        """Log-depth voxel bins of an image: factor_coord [h*w, 3] float32 on
        the device -> zbin [h*w] int32 (syncs)."""
        n = factor_coord.shape[0]
        z = torch.empty(n, dtype=torch.int32, device=factor_coord.device)
        L.check(self.lib.msc_quantize_topology_z(self.ctx, _p(factor_coord), n, depth_resolution, _p(z), _stream()))
        return z

    def make_dense_image_level(self, zbin: torch.Tensor, width: int, height: int):
        """Level 0 of the refiner's pyramid: coords [n, 4] (row, column, zbin,
        0) and the neighbour map [n, 27] from the pixel grid."""
        n = width * height
        coords = torch.empty((n, 4), dtype=torch.int32, device=zbin.device)
        nbr = torch.empty((n, 27), dtype=torch.int32, device=zbin.device)
        L.check(self.lib.msc_make_dense_image_level(self.ctx, _p(zbin), width, height, _p(coords), _p(nbr),
                                                    _stream()))
        return coords, nbr

    # ---------------------------------------------------------- weights
    def prepare_weight(self, w: torch.Tensor, wtype: str, cin: int, cout: int, ntaps: int) -> PreparedWeight:
        """w: packed [cout, ntaps*cin] float32 / float16, or uint8 block_q8_0 rows."""
        code = _WT[wtype]
        nb = self.lib.msc_weight_blob_bytes(code, cin, cout, ntaps)
        blob = torch.empty(nb, dtype=torch.uint8, device=w.device)
        L.check(self.lib.msc_weight_prepare(self.ctx, code, _p(w), cin, cout, ntaps, _p(blob), nb, _stream()))
        return PreparedWeight(blob, wtype, cin, cout, ntaps)

    # ---------------------------------------------------------- operators
    def sparse_conv(self, x, nbr, w: PreparedWeight, bias=None, out_dtype=torch.float32, plan=None):
        n, cin = x.shape
        y = torch.empty((n, w.cout), dtype=out_dtype, device=x.device)
        wsb = self.lib.msc_op_workspace_bytes(n, max(cin, w.cout))
        ws = self.workspace(wsb)
        L.check(self.lib.msc_sparse_conv_planned(self.ctx, _p(x), _DT[x.dtype], n, cin, _p(nbr), _p(plan),
                                                 _p(w.blob), _p(bias), _p(y), _DT[out_dtype], _p(ws), wsb,
                                                 _stream()))
        return y

    def sparse_conv_fused(self, x, nbr, w: PreparedWeight, bias=None, out_dtype=torch.float32, plan=None,
                          norm_w=None, norm_b=None, layer_norm=False, eps=1e-6, silu_in=False, silu_out=False,
                          residual=None):
        """y = [SiLU](W * gather([SiLU]([LayerNorm](x))) + bias) [+ residual]
        in one conv (msc_sparse_conv_fused)."""
        n, cin = x.shape
        y = torch.empty((n, w.cout), dtype=out_dtype, device=x.device)
        wsb = self.lib.msc_op_workspace_bytes(n, max(cin, w.cout))
        ws = self.workspace(wsb)
        f = L.ConvFusion(1 if layer_norm else 0, _p(norm_w), _p(norm_b), eps, 1 if silu_in else 0,
                         1 if silu_out else 0, _p(residual), _DT[residual.dtype] if residual is not None else 0)
        L.check(self.lib.msc_sparse_conv_fused(self.ctx, _p(x), _DT[x.dtype], n, cin, _p(nbr), _p(plan), C.byref(f),
                                               _p(w.blob), _p(bias), _p(y), _DT[out_dtype], _p(ws), wsb, _stream()))
        return y

    def octant_maps(self, coords: torch.Tensor, tr: "Transition"):
        """(down_nbr [np][27], up_nbr [nfine][27]) of a synced stride-2
        transition: the maps of the octant-weighted strided conv and of its
        transpose (an extension; the reference's stride-2 operators are pool
        + linear and linear + nearest up)."""
        nfine, np_ = coords.shape[0], tr.np
        down = torch.empty((max(np_, 1), 27), dtype=torch.int32, device=coords.device)
        up = torch.empty((max(nfine, 1), 27), dtype=torch.int32, device=coords.device)
        L.check(self.lib.msc_octant_maps(self.ctx, _p(coords), nfine, _p(tr.pool_rows), _p(tr.up_rows), np_,
                                         _p(down), _p(up), _stream()))
        return down[:np_], up[:nfine]

    def conv_plan_rect(self, nbr: torch.Tensor, n_in: int) -> torch.Tensor:
        """Tap-order plan of a map whose entries index n_in rows of another
        level (msc_conv_plan_build_rect)."""
        n = nbr.shape[0]
        pb = self.lib.msc_conv_plan_bytes(n)
        plan = torch.empty(pb, dtype=torch.uint8, device=nbr.device)
        wsb = self.lib.msc_conv_plan_workspace_bytes(n)
        ws = self.workspace(wsb)
        L.check(self.lib.msc_conv_plan_build_rect(self.ctx, n, n_in, _p(nbr), _p(plan), pb, _p(ws), wsb,
                                                  _stream()))
        return plan

    def octant_conv(self, x, nbr, w: PreparedWeight, bias=None, out_dtype=torch.float32, plan=None, skip=None):
        """y [nbr rows][cout] = sum_o W_o x[nbr[i][o]] + bias (+ skip) (w
        prepared with ntaps = 8): the strided conv over down_nbr, the
        transpose over up_nbr."""
        n_in, cin = x.shape
        n_out = nbr.shape[0]
        y = torch.empty((n_out, w.cout), dtype=out_dtype, device=x.device)
        wsb = self.lib.msc_op_workspace_bytes(max(n_in, 1), max(cin, w.cout))
        ws = self.workspace(wsb)
        L.check(self.lib.msc_octant_conv(self.ctx, _p(x), _DT[x.dtype], n_in, cin, _p(nbr), n_out, _p(plan),
                                         _p(w.blob), _p(bias), _p(skip), _DT[skip.dtype] if skip is not None else 0,
                                         _p(y), _DT[out_dtype], _p(ws), wsb, _stream()))
        return y

    def linear(self, x, w: PreparedWeight, bias=None, out_dtype=torch.float32):
        n, cin = x.shape
        y = torch.empty((n, w.cout), dtype=out_dtype, device=x.device)
        wsb = self.lib.msc_op_workspace_bytes(n, max(cin, w.cout))
        ws = self.workspace(wsb)
        L.check(self.lib.msc_linear(self.ctx, _p(x), _DT[x.dtype], n, cin, _p(w.blob), _p(bias), _p(y),
                                    _DT[out_dtype], _p(ws), wsb, _stream()))
        return y

    def res_block(self, x, nbr, blk: dict, plan=None):
        """In place on x.  blk: norm_w, norm_b, w1 (PreparedWeight), b1, w2, b2."""
        n, c = x.shape
        wsb = self.lib.msc_op_workspace_bytes(n, c)
        ws = self.workspace(wsb)
        L.check(self.lib.msc_res_block_planned(self.ctx, _p(x), _DT[x.dtype], n, c, _p(nbr), _p(plan),
                                               _p(blk.get("norm_w")), _p(blk.get("norm_b")), _p(blk["w1"].blob),
                                               _p(blk.get("b1")), _p(blk["w2"].blob), _p(blk.get("b2")), _p(ws),
                                               wsb, _stream()))
        return x

    def res_stack(self, x, nbr, blocks: list, plan=None):
        """In place on x: len(blocks) residual blocks in a row (``msc_res_stack``)."""
        n, c = x.shape
        k = len(blocks)
        wsb = self.lib.msc_op_workspace_bytes(n, c)
        ws = self.workspace(wsb)

        def arr(key, attr=None):
            vals = [b.get(key) for b in blocks]
            if all(v is None for v in vals):
                return None
            ptrs = [None if v is None else (getattr(v, attr) if attr else v).data_ptr() for v in vals]
            return (C.c_void_p * k)(*ptrs)
        L.check(self.lib.msc_res_stack(self.ctx, _p(x), _DT[x.dtype], n, c, _p(nbr), _p(plan), k, arr("norm_w"),
                                       arr("norm_b"), arr("w1", "blob"), arr("b1"), arr("w2", "blob"), arr("b2"),
                                       _p(ws), wsb, _stream()))
        return x

    def level_stack_host(self, coords_host, x_host, blocks: list, y_host, ws=None, stream=None, copy_in=None,
                         copy_out=None):
        """A level's LayerNorm residual stack from host tensors to host
        tensors (``msc_level_stack_host``): coords [n, 4] int32 and x [n, c]
        in, the result into y_host (may be x_host).  Asynchronous on
        ``stream`` (default: the current stream), copies on copy_in /
        copy_out when given; ws is a device uint8 workspace of
        ``level_stack_host_workspace(n, c)`` bytes (one per call in flight).
        Returns ws."""
        n, c = x_host.shape
        k = len(blocks)
        wsb = self.lib.msc_level_stack_host_workspace_bytes(n, c)
        if ws is None:
            ws = torch.empty(wsb, dtype=torch.uint8, device=torch.device("cuda", self.device))

        def arr(key, attr=None):
            vals = [b.get(key) for b in blocks]
            if all(v is None for v in vals):
                return None
            ptrs = [None if v is None else (getattr(v, attr) if attr else v).data_ptr() for v in vals]
            return (C.c_void_p * k)(*ptrs)
        st = stream.cuda_stream if stream is not None else _stream()
        L.check(self.lib.msc_level_stack_host(self.ctx, _p(coords_host), _p(x_host), _DT[x_host.dtype], n, c, k,
                                              arr("norm_w"), arr("norm_b"), arr("w1", "blob"), arr("b1"),
                                              arr("w2", "blob"), arr("b2"), _p(y_host), _p(ws), ws.numel(), st,
                                              copy_in.cuda_stream if copy_in is not None else None,
                                              copy_out.cuda_stream if copy_out is not None else None))
        return ws

    def level_stack_host_workspace(self, n: int, c: int) -> int:
        return self.lib.msc_level_stack_host_workspace_bytes(n, c)

    def res_block_gn(self, x, nbr, coords, nsamples: int, blk: dict, eps: float = 1e-5, plan=None,
                     n_stat: int | None = None, allreduce=None):
        """In place on x: x + conv2(SiLU(GroupNorm_32(conv1(x) + b1))) + b2.

        blk: w1, b1, w2, b2 as for res_block, gn_w / gn_b the GroupNorm
        affine.  coords [n, 4] int32 give each row's sample (field 3).  Rows
        [0, n_stat) enter the sample-wide statistics (default: all rows);
        ``allreduce(t)``, when given, sums the float64 tensor t over all
        ranks in place on the current stream (one call per block)."""
        n, c = x.shape
        n_stat = n if n_stat is None else n_stat
        wsb = self.lib.msc_res_block_gn_workspace_bytes(n, c, nsamples)
        ws = self.workspace(wsb)
        stats = torch.empty(self.lib.msc_gn_stats_doubles(nsamples), dtype=torch.float64, device=x.device)
        cb = None
        if allreduce is not None:
            base = stats.data_ptr()

            def _cb(buf, count, _stream, _user):
                try:
                    off = (buf - base) // 8
                    allreduce(stats[off:off + count])
                    return 0
                except Exception:  # noqa: BLE001 - reported through the return code
                    return 1
            cb = L.ALLREDUCE_FN(_cb)
        L.check(self.lib.msc_res_block_gn(self.ctx, _p(x), _DT[x.dtype], n, n_stat, c, _p(coords), nsamples,
                                          _p(nbr), _p(plan), _p(blk.get("gn_w")), _p(blk.get("gn_b")), eps,
                                          _p(blk["w1"].blob), _p(blk.get("b1")), _p(blk["w2"].blob),
                                          _p(blk.get("b2")), _p(stats), cb, None, _p(ws), wsb, _stream()))
        return x

    def pool_down(self, x, tr: Transition, w: PreparedWeight, bias=None, out_dtype=torch.float32):
        nfine, c = x.shape
        y = torch.empty((tr.np, w.cout), dtype=out_dtype, device=x.device)
        wsb = self.lib.msc_op_workspace_bytes(max(tr.np, 1), max(c, w.cout))
        ws = self.workspace(wsb)
        L.check(self.lib.msc_pool_down(self.ctx, _p(x), _DT[x.dtype], nfine, c, _p(tr.pool_rows), _p(tr.inv_count),
                                       tr.np, _p(w.blob), _p(bias), _p(y), _DT[out_dtype], _p(ws), wsb, _stream()))
        return y

    def nearest_up(self, x, tr: Transition, w: PreparedWeight, bias=None, skip=None, out_dtype=torch.float32):
        np_, c = x.shape
        y = torch.empty((tr.nfine, w.cout), dtype=out_dtype, device=x.device)
        wsb = self.lib.msc_op_workspace_bytes(max(np_, 1), max(c, w.cout))
        ws = self.workspace(wsb)
        L.check(self.lib.msc_nearest_up(self.ctx, _p(x), _DT[x.dtype], np_, c, _p(tr.up_rows), tr.nfine,
                                        _p(w.blob), _p(bias), _p(skip),
                                        _DT[skip.dtype] if skip is not None else 0, _p(y), _DT[out_dtype], _p(ws),
                                        wsb, _stream()))
        return y


class SparseRefiner:
    """The MoGe-3 sparse refiner on the device (the reference's SparseRefiner,
    src/sparse.hpp:41-66, and refine_once, src/sparse.cpp:1014-1296).

    Built from a MOGG image held in memory (its refiner.* metadata and
    tensors); the topology of the last pass is cached and reused when the
    quantised log-depth bins are unchanged (get_topology_cached,
    src/sparse.cpp:443-472)."""

    def __init__(self, ex: SparseCudaExecutor, mogg: bytes):
        self.ex = ex
        self.lib = ex.lib
        h = C.c_void_p()
        L.check(self.lib.msc_refiner_create(ex.ctx, mogg, len(mogg), _stream(), C.byref(h)))
        self.h = h
        cfg = L.SparseConfig()
        L.check(self.lib.msc_refiner_config(self.h, C.byref(cfg)))
        self.config = cfg

    def close(self):
        if self.h:
            self.lib.msc_refiner_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def refine_once(self, factor_coord: torch.Tensor, width: int, height: int, encoder_feature: torch.Tensor,
                    encoder_width: int, encoder_height: int) -> torch.Tensor:
        """factor_coord [h*w, 3] float32 (device: updated in place; host:
        through the host-buffer entry point); encoder_feature [eh*ew, C]."""
        fn = self.lib.msc_refiner_refine_once if factor_coord.is_cuda else self.lib.msc_refiner_refine_once_host
        L.check(fn(self.h, _p(factor_coord), width, height, _p(encoder_feature), encoder_width, encoder_height,
                   _stream()))
        return factor_coord

    def cache_stats(self) -> tuple[int, int]:
        hits, misses = C.c_uint64(0), C.c_uint64(0)
        L.check(self.lib.msc_refiner_cache_stats(self.h, C.byref(hits), C.byref(misses)))
        return hits.value, misses.value

    def level_sizes(self) -> list[int]:
        buf = (C.c_int64 * L.MAX_LEVELS)()
        cnt = C.c_int(0)
        L.check(self.lib.msc_refiner_level_sizes(self.h, buf, L.MAX_LEVELS, C.byref(cnt)))
        return [buf[i] for i in range(cnt.value)]
