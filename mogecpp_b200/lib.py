"""ctypes binding of ``libmoge_sparse_cuda.so`` (C ABI: include/moge_sparse_cuda.h).

Loading fails loudly when the library has not been built: there is no CPU or
PyTorch fallback for any operator of this package.
"""

from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libmoge_sparse_cuda.so")

MSC_OK = 0
MSC_F32, MSC_F16, MSC_BF16 = 0, 1, 2
MSC_PLAN_TAP_ORDER = 0
MSC_W_F32, MSC_W_F16, MSC_W_Q8_0 = 0, 1, 8
DEV_TIMEOUT, DEV_HASH_FULL, DEV_BAD_COORD, DEV_DUP_COORD, DEV_POOL_OVERFLOW, DEV_BAD_INDEX = 1, 2, 4, 8, 16, 32

_vp, _i64, _sz, _i32 = C.c_void_p, C.c_int64, C.c_size_t, C.c_int

# name -> (restype, argtypes); the exported set of the C ABI
SIGNATURES = {
    "msc_abi_version": (C.c_int, []),
    "msc_last_error": (C.c_char_p, []),
    "msc_create": (C.c_int, [_i32, C.POINTER(_vp)]),
    "msc_destroy": (C.c_int, [_vp]),
    "msc_check": (C.c_int, [_vp, _vp, C.POINTER(C.c_uint32)]),
    "msc_topology_workspace_bytes": (_sz, [_i64]),
    "msc_make_level": (C.c_int, [_vp, _vp, _i64, _vp, _vp, _sz, _vp]),
    "msc_make_level_noalloc": (C.c_int, [_vp, _i64, _vp, _vp, _vp]),
    "msc_downsample": (C.c_int, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, C.POINTER(_i64), _vp, _sz, _vp]),
    "msc_make_level_downsample": (C.c_int, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, C.POINTER(_i64), _vp,
                                            _sz, _vp]),
    "msc_weight_blob_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "msc_weight_prepare": (C.c_int, [_vp, _i32, _vp, _i32, _i32, _i32, _vp, _sz, _vp]),
    "msc_op_workspace_bytes": (_sz, [_i64, _i32]),
    "msc_sparse_conv": (C.c_int, [_vp, _vp, _i32, _i64, _i32, _vp, _vp, _vp, _vp, _i32, _vp, _sz, _vp]),
    "msc_conv_plan_bytes": (_sz, [_i64]),
    "msc_conv_plan_workspace_bytes": (_sz, [_i64]),
    "msc_conv_plan_build": (C.c_int, [_vp, _vp, _i64, _vp, _i32, _vp, _sz, _vp, _sz, _vp]),
    "msc_conv_plan_build_rect": (C.c_int, [_vp, _i64, _i64, _vp, _vp, _sz, _vp, _sz, _vp]),
    "msc_octant_maps": (C.c_int, [_vp, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp]),
    "msc_octant_conv": (C.c_int, [_vp, _vp, _i32, _i64, _i32, _vp, _i64, _vp, _vp, _vp, _vp, _i32, _vp, _i32, _vp,
                                  _sz, _vp]),
    "msc_sparse_conv_planned": (C.c_int, [_vp, _vp, _i32, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _sz,
                                          _vp]),
    "msc_sparse_conv_fused": (C.c_int, [_vp, _vp, _i32, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _sz,
                                        _vp]),
    "msc_res_block_planned": (C.c_int, [_vp, _vp, _i32, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                        _sz, _vp]),
    "msc_level_stack_host_workspace_bytes": (_sz, [_i64, _i32]),
    "msc_level_stack_host": (C.c_int, [_vp, _vp, _vp, _i32, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                       _sz, _vp, _vp, _vp]),
    "msc_res_stack": (C.c_int, [_vp, _vp, _i32, _i64, _i32, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                                _vp]),
    "msc_gn_stats_doubles": (_i64, [_i32]),
    "msc_res_block_gn_workspace_bytes": (_sz, [_i64, _i32, _i32]),
    "msc_res_block_gn": (C.c_int, [_vp, _vp, _i32, _i64, _i64, _i32, _vp, _i32, _vp, _vp, _vp, _vp, C.c_float, _vp,
                                   _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "msc_linear": (C.c_int, [_vp, _vp, _i32, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _sz, _vp]),
    "msc_res_block": (C.c_int, [_vp, _vp, _i32, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "msc_pool_down": (C.c_int, [_vp, _vp, _i32, _i64, _i32, _vp, _vp, _i64, _vp, _vp, _vp, _i32, _vp, _sz, _vp]),
    "msc_nearest_up": (C.c_int, [_vp, _vp, _i32, _i64, _i32, _vp, _i64, _vp, _vp, _vp, _i32, _vp, _i32, _vp, _sz,
                                 _vp]),
    "msc_quantize_topology_z": (C.c_int, [_vp, _vp, _i64, C.c_float, _vp, _vp]),
    "msc_make_dense_image_level": (C.c_int, [_vp, _vp, _i32, _i32, _vp, _vp, _vp]),
    "msc_refiner_create": (C.c_int, [_vp, C.c_char_p, _sz, _vp, C.POINTER(_vp)]),
    "msc_refiner_destroy": (C.c_int, [_vp]),
    "msc_refiner_config": (C.c_int, [_vp, _vp]),
    "msc_refiner_cache_stats": (C.c_int, [_vp, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "msc_refiner_level_sizes": (C.c_int, [_vp, C.POINTER(_i64), _i32, C.POINTER(_i32)]),
    "msc_refiner_refine_once": (C.c_int, [_vp, _vp, _i32, _i32, _vp, _i32, _i32, _vp]),
    "msc_refiner_refine_once_host": (C.c_int, [_vp, _vp, _i32, _i32, _vp, _i32, _i32, _vp]),
    "msc_slab_create": (C.c_int, [_vp, _vp, C.POINTER(_vp)]),
    "msc_slab_destroy": (C.c_int, [_vp]),
    "msc_slab_get_handle": (C.c_int, [_vp, _vp]),
    "msc_slab_connect": (C.c_int, [_vp, _vp, _vp]),
    "msc_slab_set_level": (C.c_int, [_vp, _vp, _vp]),
    "msc_slab_put_features": (C.c_int, [_vp, _vp, _vp]),
    "msc_slab_get_features": (C.c_int, [_vp, _vp, _vp]),
    "msc_slab_features_ptr": (C.c_int, [_vp, C.POINTER(_vp)]),
    "msc_slab_res_block": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "msc_wait_probe": (C.c_int, [_vp, _i64, _vp]),
    "msc_profile_enable": (C.c_int, [_vp, _i32]),
    "msc_profile_read": (C.c_int, [_vp, _vp, _i32, C.POINTER(_i32)]),
}


# int (*)(double* buf, int64_t count, void* stream, void* user)
ALLREDUCE_FN = C.CFUNCTYPE(C.c_int, _vp, _i64, _vp, _vp)


MAX_LEVELS = 8


class SparseConfig(C.Structure):
    """msc_sparse_config (the reference's SparseConfig, src/sparse.hpp:21-33)."""
    _fields_ = [("in_channels", C.c_int), ("out_channels", C.c_int), ("encoder_channels", C.c_int),
                ("num_levels", C.c_int), ("model_channels", C.c_int * MAX_LEVELS),
                ("encoder_blocks", C.c_int * MAX_LEVELS), ("decoder_blocks", C.c_int * MAX_LEVELS),
                ("downsample_factors", C.c_int * MAX_LEVELS), ("bottleneck_blocks", C.c_int),
                ("encoder_downsample", C.c_int), ("depth_resolution", C.c_float)]


class ConvFusion(C.Structure):
    """msc_conv_fusion: prologue (LayerNorm, SiLU) and epilogue (SiLU, residual) of a fused conv."""
    _fields_ = [("layer_norm", C.c_int), ("norm_w", C.c_void_p), ("norm_b", C.c_void_p), ("eps", C.c_float),
                ("silu_in", C.c_int), ("silu_out", C.c_int), ("residual", C.c_void_p), ("residual_dtype", C.c_int)]


class SlabDesc(C.Structure):
    """msc_slab_desc: one rank's z-slab shard ([owned | halo below | halo above])."""
    _fields_ = [("rank", C.c_int), ("world", C.c_int), ("channels", C.c_int), ("n_local", C.c_int64),
                ("n_owned", C.c_int64), ("n_halo_lo", C.c_int64), ("n_halo_hi", C.c_int64), ("send_lo", C.c_int64),
                ("send_hi", C.c_int64)]


SLAB_HANDLE_BYTES = 512


class ProfileEntry(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("launches", C.c_int64), ("total_ms", C.c_double)]


class MscError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


_LIB = None


def load(path: str = LIB_PATH) -> C.CDLL:
    """Loads and types the library; raises if it is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise ImportError(f"{path} is not built: run `python -m mogecpp_b200.build` "
                          "(this package has no CPU fallback)")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def check(rc: int) -> None:
    if rc != MSC_OK:
        raise MscError(rc, load().msc_last_error().decode())
