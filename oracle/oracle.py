"""Python bindings for the CPU oracle and for the compiled reference.

TEST INFRASTRUCTURE ONLY: tests/, the smoke check and bench.py's CPU-baseline
leg import this module as the checker.  The product never does.

* ``Oracle`` wraps ``oracle/liboracle.so``: the plain-C restatement of the
  reference's sparse path (``oracle/oracle.c``).
* ``Reference`` wraps ``oracle/_ref/libmoge_ref.so``: the reference's own
  ``src/sparse.cpp`` + ggml 0.25.3 CPU backend, compiled by
  ``oracle/ref/Makefile``.  It exists only where that library was built.
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
W_F32, W_F16, W_Q8_0 = 0, 1, 8

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i64 = C.c_int64

Q8_BLOCK = np.dtype([("d", "<u2"), ("qs", "i1", (32,))])


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def _opt(a):
    return None if a is None else _c(a, np.float32).ctypes.data_as(C.c_void_p)


class Oracle:
    def __init__(self, path: str | None = None):
        path = path or os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run make -f oracle/Makefile")
        L = self.lib = C.CDLL(path)
        L.orc_make_level.argtypes = [_i32p, C.c_int32, _i32p]
        L.orc_downsample.argtypes = [_i32p, C.c_int32, _i32p, C.POINTER(C.c_int32), _i32p, _f32p, _i32p]
        L.orc_sparse_conv.argtypes = [_f32p, _i64, C.c_int, _i32p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, _f32p]
        L.orc_linear.argtypes = [_f32p, _i64, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, _f32p]
        L.orc_conv_rect.argtypes = [_f32p, _i64, C.c_int, _i32p, _i64, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                    C.c_void_p, _f32p]
        L.orc_octant_maps.argtypes = [_i32p, _i64, _i32p, _i32p, _i64, _i32p, _i32p]
        L.orc_layer_norm.argtypes = [_f32p, _i64, C.c_int, C.c_void_p, C.c_void_p, C.c_float, _f32p]
        L.orc_silu.argtypes = [_f32p, _i64]
        L.orc_res_block.argtypes = [_f32p, _i64, C.c_int, _i32p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p, C.c_void_p, C.c_void_p, _f32p]
        L.orc_pool_down.argtypes = [_f32p, _i64, C.c_int, _i32p, _f32p, _i64, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                    C.c_void_p, _f32p]
        L.orc_nearest_up.argtypes = [_f32p, _i64, C.c_int, _i32p, _i64, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                     _f32p]
        L.orc_group_norm.argtypes = [_f32p, _i64, C.c_int, _i32p, C.c_int, C.c_int, C.c_float, C.c_void_p,
                                     C.c_void_p, _f32p]
        L.orc_res_block_gn.argtypes = [_f32p, _i64, C.c_int, _i32p, _i32p, C.c_int, C.c_int, C.c_float, C.c_int,
                                       C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, _f32p]
        L.orc_quantize_q8_0_ref.argtypes = [_f32p, C.c_void_p, _i64]
        L.orc_quantize_q8_0_act.argtypes = [_f32p, C.c_void_p, _i64]
        L.orc_fp32_to_fp16.argtypes = [C.c_float]
        L.orc_fp32_to_fp16.restype = C.c_uint16
        L.orc_quantize_topology_z.argtypes = [_f32p, _i64, C.c_float, _i32p]
        L.orc_dense_image_level.argtypes = [_i32p, C.c_int32, C.c_int32, _i32p]

    # -- weights --------------------------------------------------------
    def quantize_q8_0(self, w: np.ndarray) -> np.ndarray:
        """ggml quantize_row_q8_0_ref over rows of w (row length % 32 == 0)."""
        w = _c(w, np.float32)
        out = np.zeros(w.size // 32, dtype=Q8_BLOCK)
        self.lib.orc_quantize_q8_0_ref(w.ravel(), out.ctypes.data_as(C.c_void_p), w.size)
        return out.reshape(w.shape[:-1] + (w.shape[-1] // 32,))

    def quantize_q8_0_act(self, x: np.ndarray) -> np.ndarray:
        x = _c(x, np.float32)
        out = np.zeros(x.size // 32, dtype=Q8_BLOCK)
        self.lib.orc_quantize_q8_0_act(x.ravel(), out.ctypes.data_as(C.c_void_p), x.size)
        return out.reshape(x.shape[:-1] + (x.shape[-1] // 32,))

    @staticmethod
    def weight_payload(w: np.ndarray, wtype: int, q: "Oracle"):
        if wtype == W_F32:
            return _c(w, np.float32)
        if wtype == W_F16:
            return _c(w, np.float32).astype(np.float16)
        if wtype == W_Q8_0:
            return q.quantize_q8_0(w)
        raise ValueError(wtype)

    # -- topology -------------------------------------------------------
    def make_level(self, coords: np.ndarray) -> np.ndarray:
        coords = _c(coords, np.int32)
        n = coords.shape[0]
        nbr = np.empty(27 * n, dtype=np.int32)
        rc = self.lib.orc_make_level(coords.ravel(), n, nbr)
        if rc != 0:
            raise ValueError(f"orc_make_level failed ({rc})")
        return nbr.reshape(n, 27)

    def downsample(self, coords: np.ndarray):
        coords = _c(coords, np.int32)
        n = coords.shape[0]
        parent = np.empty(4 * max(n, 1), dtype=np.int32)
        npo = C.c_int32(0)
        pool = np.empty(8 * max(n, 1), dtype=np.int32)
        inv = np.empty(max(n, 1), dtype=np.float32)
        up = np.empty(max(n, 1), dtype=np.int32)
        rc = self.lib.orc_downsample(coords.ravel(), n, parent, C.byref(npo), pool, inv, up)
        if rc != 0:
            raise ValueError(f"orc_downsample failed ({rc})")
        np_ = npo.value
        return (parent[:4 * np_].reshape(np_, 4), pool[:8 * np_].reshape(8, np_), inv[:np_], up[:n])

    def quantize_topology_z(self, factor_coord: np.ndarray, depth_resolution: float) -> np.ndarray:
        fc = _c(factor_coord, np.float32).reshape(-1, 3)
        z = np.empty(fc.shape[0], dtype=np.int32)
        if self.lib.orc_quantize_topology_z(fc.ravel(), fc.shape[0], depth_resolution, z) != 0:
            raise ValueError("z-bin extent overflow")
        return z

    def dense_image_level(self, zbin: np.ndarray, width: int, height: int) -> np.ndarray:
        nbr = np.empty(27 * width * height, dtype=np.int32)
        self.lib.orc_dense_image_level(_c(zbin, np.int32), width, height, nbr)
        return nbr.reshape(-1, 27)

    # -- features -------------------------------------------------------
    def sparse_conv(self, x, nbr, w, wtype, bias=None):
        x = _c(x, np.float32)
        n, cin = x.shape
        payload = self.weight_payload(w, wtype, self)
        cout = w.shape[0]
        y = np.empty((n, cout), dtype=np.float32)
        self.lib.orc_sparse_conv(x, n, cin, _c(nbr, np.int32), wtype, payload.ctypes.data_as(C.c_void_p), cout,
                                 _opt(bias), y)
        return y

    def conv_rect(self, x, nbr, n_out, ntaps, w, wtype, bias=None):
        """Conv from x's rows to n_out rows over nbr [n_out][27] (first ntaps
        columns): the octant-weighted stride-2 conv and its transpose."""
        x = _c(x, np.float32)
        n_in, cin = x.shape
        payload = self.weight_payload(w, wtype, self)
        cout = w.shape[0]
        y = np.empty((n_out, cout), dtype=np.float32)
        self.lib.orc_conv_rect(x, n_in, cin, _c(nbr, np.int32), n_out, ntaps, wtype,
                               payload.ctypes.data_as(C.c_void_p), cout, _opt(bias), y)
        return y

    def octant_maps(self, coords, pool_rows, up_rows):
        """(down [np][27], up [nfine][27]) of a stride-2 transition."""
        coords = _c(coords, np.int32)
        pool_rows = _c(pool_rows, np.int32)
        nfine, np_ = coords.shape[0], pool_rows.size // 8
        down = np.empty(np_ * 27, dtype=np.int32)
        up = np.empty(nfine * 27, dtype=np.int32)
        self.lib.orc_octant_maps(coords.ravel(), nfine, pool_rows.ravel(), _c(up_rows, np.int32), np_, down, up)
        return down.reshape(np_, 27), up.reshape(nfine, 27)

    def linear(self, x, w, wtype, bias=None):
        x = _c(x, np.float32)
        n, cin = x.shape
        payload = self.weight_payload(w, wtype, self)
        y = np.empty((n, w.shape[0]), dtype=np.float32)
        self.lib.orc_linear(x, n, cin, wtype, payload.ctypes.data_as(C.c_void_p), w.shape[0], _opt(bias), y)
        return y

    def layer_norm(self, x, gamma=None, beta=None, eps=1e-6):
        x = _c(x, np.float32)
        y = np.empty_like(x)
        self.lib.orc_layer_norm(x, x.shape[0], x.shape[1], _opt(gamma), _opt(beta), eps, y)
        return y

    def silu(self, x):
        y = _c(x, np.float32).copy()
        self.lib.orc_silu(y.ravel(), y.size)
        return y

    def res_block(self, x, nbr, p: dict, wtype):
        x = _c(x, np.float32)
        n, c = x.shape
        w1 = self.weight_payload(p["w1"], wtype, self)
        w2 = self.weight_payload(p["w2"], wtype, self)
        y = np.empty_like(x)
        self.lib.orc_res_block(x, n, c, _c(nbr, np.int32), wtype, _opt(p["norm_w"]), _opt(p["norm_b"]),
                               w1.ctypes.data_as(C.c_void_p), _opt(p["b1"]), w2.ctypes.data_as(C.c_void_p),
                               _opt(p["b2"]), y)
        return y

    def group_norm(self, x, sample, groups=32, eps=1e-5, gamma=None, beta=None):
        """Sample-wide GroupNorm (ggml group_norm_f32 per sample, then affine)."""
        x = _c(x, np.float32)
        sample = _c(sample, np.int32)
        y = np.empty_like(x)
        ns = int(sample.max()) + 1 if sample.size else 1
        self.lib.orc_group_norm(x, x.shape[0], x.shape[1], sample, ns, groups, eps, _opt(gamma), _opt(beta), y)
        return y

    def res_block_gn(self, x, nbr, sample, p: dict, wtype, groups=32, eps=1e-5):
        """conv1 -> GroupNorm -> SiLU -> conv2 -> +x; p: gn_w, gn_b, w1, b1, w2, b2."""
        x = _c(x, np.float32)
        n, c = x.shape
        sample = _c(sample, np.int32)
        ns = int(sample.max()) + 1 if sample.size else 1
        w1 = self.weight_payload(p["w1"], wtype, self)
        w2 = self.weight_payload(p["w2"], wtype, self)
        y = np.empty_like(x)
        self.lib.orc_res_block_gn(x, n, c, _c(nbr, np.int32), sample, ns, groups, eps, wtype, _opt(p.get("gn_w")),
                                  _opt(p.get("gn_b")), w1.ctypes.data_as(C.c_void_p), _opt(p["b1"]),
                                  w2.ctypes.data_as(C.c_void_p), _opt(p["b2"]), y)
        return y

    def pool_down(self, x, pool_rows, inv_count, w, wtype, bias=None):
        x = _c(x, np.float32)
        nfine, c = x.shape
        slots, np_ = pool_rows.shape
        payload = self.weight_payload(w, wtype, self)
        y = np.empty((np_, w.shape[0]), dtype=np.float32)
        self.lib.orc_pool_down(x, nfine, c, _c(pool_rows, np.int32).ravel(), _c(inv_count, np.float32), np_, slots,
                               wtype, payload.ctypes.data_as(C.c_void_p), w.shape[0], _opt(bias), y)
        return y

    def nearest_up(self, x, up_rows, w, wtype, bias=None):
        x = _c(x, np.float32)
        np_, c = x.shape
        nfine = up_rows.shape[0]
        payload = self.weight_payload(w, wtype, self)
        y = np.empty((nfine, w.shape[0]), dtype=np.float32)
        self.lib.orc_nearest_up(x, np_, c, _c(up_rows, np.int32), nfine, wtype, payload.ctypes.data_as(C.c_void_p),
                                w.shape[0], _opt(bias), y)
        return y


class Reference:
    """The reference's own CPU implementation (src/sparse.cpp + ggml CPU)."""

    def __init__(self, path: str | None = None, n_threads: int | None = None):
        path = path or os.path.join(HERE, "_ref", "libmoge_ref.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run make -f oracle/ref/Makefile")
        L = self.lib = C.CDLL(path)
        self.n_threads = n_threads or os.cpu_count() or 1
        L.ref_last_error.restype = C.c_char_p
        L.ref_make_level.argtypes = [_i32p, C.c_int32, _i32p]
        L.ref_downsample.argtypes = [_i32p, C.c_int32, C.c_int32, _i32p, C.POINTER(C.c_int32), _i32p, _f32p, _i32p]
        L.ref_sparse_conv.argtypes = [C.c_int, _f32p, _i64, _i64, _i32p, C.c_int, _f32p, _i64, C.c_void_p, _f32p]
        L.ref_res_stack.argtypes = [C.c_int, _f32p, _i64, _i64, _i32p, C.c_int, C.c_int, _f32p, _f32p, _f32p, _f32p,
                                    _f32p, _f32p, _f32p, C.c_int, C.POINTER(C.c_double)]
        L.ref_pool_down.argtypes = [C.c_int, _f32p, _i64, _i64, _i32p, _f32p, _i64, C.c_int, C.c_int, _f32p, _i64,
                                    C.c_void_p, _f32p]
        L.ref_nearest_up.argtypes = [C.c_int, _f32p, _i64, _i64, _i32p, _i64, C.c_int, _f32p, _i64, C.c_void_p, _f32p]
        L.ref_topology_timed.argtypes = [_i32p, C.c_int32, C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_double)]
        L.ref_group_norm.argtypes = [C.c_int, _f32p, _i64, _i64, C.c_int, C.c_float, _f32p]
        L.ref_quantize_topology_z.argtypes = [_f32p, C.c_int32, C.c_int32, C.c_float, _i32p]
        L.ref_make_dense_image_level.argtypes = [_i32p, C.c_int32, C.c_int32, _i32p]
        L.ref_refine_once.argtypes = [C.c_int, C.c_char_p, C.c_size_t, _f32p, C.c_int32, C.c_int32, _f32p,
                                      C.c_int32, C.c_int32, C.c_int, C.POINTER(C.c_double)]

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError("reference: " + self.lib.ref_last_error().decode())

    @staticmethod
    def _xyz(coords):
        coords = np.asarray(coords)
        if coords.shape[1] == 4 and coords.shape[0] and coords[:, 3].max() > 0:
            raise ValueError("the reference has no batch field; call it once per sample")
        return _c(coords[:, :3], np.int32)

    def group_norm(self, x, groups=32, eps=1e-5):
        """ggml_group_norm of one sample's [n, c] features (no affine)."""
        x = _c(x, np.float32)
        y = np.empty_like(x)
        self._check(self.lib.ref_group_norm(self.n_threads, x, x.shape[0], x.shape[1], groups, eps, y))
        return y

    def quantize_topology_z(self, factor_coord, width, height, depth_resolution):
        fc = _c(factor_coord, np.float32).reshape(-1)
        z = np.empty(width * height, dtype=np.int32)
        self._check(self.lib.ref_quantize_topology_z(fc, width, height, depth_resolution, z))
        return z

    def make_dense_image_level(self, zbin, width, height):
        nbr = np.empty(27 * width * height, dtype=np.int32)
        self._check(self.lib.ref_make_dense_image_level(_c(zbin, np.int32), width, height, nbr))
        return nbr.reshape(-1, 27)

    def refine_once(self, mogg: bytes, factor_coord, width, height, encoder_feature, ew, eh, passes=1):
        """SparseRefiner::refine_once, `passes` times on one refiner; returns
        (updated factor_coord [h*w][3], median seconds per pass)."""
        fc = _c(factor_coord, np.float32).reshape(-1).copy()
        enc = _c(encoder_feature, np.float32).reshape(-1)
        sec = C.c_double(0.0)
        self._check(self.lib.ref_refine_once(self.n_threads, mogg, len(mogg), fc, width, height, enc, ew, eh, passes,
                                             C.byref(sec)))
        return fc.reshape(-1, 3), sec.value

    def make_level(self, coords):
        c3 = self._xyz(coords)
        n = c3.shape[0]
        nbr = np.empty(27 * n, dtype=np.int32)
        self._check(self.lib.ref_make_level(c3.ravel(), n, nbr))
        return nbr.reshape(n, 27)

    def downsample(self, coords):
        c3 = self._xyz(coords)
        n = c3.shape[0]
        parent = np.empty(3 * max(n, 1), dtype=np.int32)
        npo = C.c_int32(0)
        pool = np.empty(8 * max(n, 1), dtype=np.int32)
        inv = np.empty(max(n, 1), dtype=np.float32)
        up = np.empty(max(n, 1), dtype=np.int32)
        self._check(self.lib.ref_downsample(c3.ravel(), n, 2, parent, C.byref(npo), pool, inv, up))
        np_ = npo.value
        return parent[:3 * np_].reshape(np_, 3), pool[:8 * np_].reshape(8, np_), inv[:np_], up[:n]

    def sparse_conv(self, x, nbr, w, wtype, bias=None):
        x = _c(x, np.float32)
        n, cin = x.shape
        y = np.empty((n, w.shape[0]), dtype=np.float32)
        self._check(self.lib.ref_sparse_conv(self.n_threads, x, n, cin, _c(nbr, np.int32).ravel(), wtype,
                                             _c(w, np.float32), w.shape[0], _opt(bias), y))
        return y

    def res_block_gn(self, x, nbr, p: dict, wtype, groups=32, eps=1e-5):
        """One sample's GroupNorm residual block composed from the reference's
        sparse conv and ggml_group_norm: x + conv2(SiLU(GN(conv1(x) + b1) *
        gn_w + gn_b)) + b2 (affine, SiLU and skip in float32 numpy)."""
        x = _c(x, np.float32)
        h = self.group_norm(self.sparse_conv(x, nbr, p["w1"], wtype, p["b1"]), groups, eps)
        if p.get("gn_w") is not None:
            h = h * p["gn_w"]
        if p.get("gn_b") is not None:
            h = h + p["gn_b"]
        h = h / (np.float32(1.0) + np.exp(-h))
        return self.sparse_conv(h, nbr, p["w2"], wtype, p["b2"]) + x

    def res_stack(self, x, nbr, blocks: list, wtype, iters=0):
        """Runs len(blocks) reference res_blocks; returns (y, median seconds)."""
        x = _c(x, np.float32)
        n, c = x.shape
        cat = lambda k: _c(np.stack([b[k] for b in blocks]), np.float32)
        y = np.empty_like(x)
        sec = C.c_double(0.0)
        self._check(self.lib.ref_res_stack(self.n_threads, x, n, c, _c(nbr, np.int32).ravel(), wtype, len(blocks),
                                           cat("norm_w"), cat("norm_b"), cat("w1"), cat("b1"), cat("w2"), cat("b2"),
                                           y, iters, C.byref(sec)))
        return y, sec.value

    def pool_down(self, x, pool_rows, inv_count, w, wtype, bias=None):
        x = _c(x, np.float32)
        nfine, c = x.shape
        slots, np_ = pool_rows.shape
        y = np.empty((np_, w.shape[0]), dtype=np.float32)
        self._check(self.lib.ref_pool_down(self.n_threads, x, nfine, c, _c(pool_rows, np.int32).ravel(),
                                           _c(inv_count, np.float32), np_, slots, wtype, _c(w, np.float32),
                                           w.shape[0], _opt(bias), y))
        return y

    def nearest_up(self, x, up_rows, w, wtype, bias=None):
        x = _c(x, np.float32)
        np_, c = x.shape
        nfine = up_rows.shape[0]
        y = np.empty((nfine, w.shape[0]), dtype=np.float32)
        self._check(self.lib.ref_nearest_up(self.n_threads, x, np_, c, _c(up_rows, np.int32), nfine, wtype,
                                            _c(w, np.float32), w.shape[0], _opt(bias), y))
        return y

    def topology_timed(self, coords, iters=5):
        c3 = self._xyz(coords)
        a, b = C.c_double(0), C.c_double(0)
        self._check(self.lib.ref_topology_timed(c3.ravel(), c3.shape[0], iters, C.byref(a), C.byref(b)))
        return a.value, b.value
