"""msc_make_level_noalloc: the neighbour map for callers that cannot allocate
device memory (a runtime whose device memory belongs to another allocator, or
latency-critical code that must not call cudaMalloc).  Its hash table is a
fixed array inside the library, shared by every call; these checks run it
twice in a row on different voxel sets through the C ABI and compare each map
with msc_make_level's (integer maps: bit-exact).  Kept in its own file so that
it runs after every other test, and self-contained so it also passes alone in
a fresh process."""

import ctypes as C

import numpy as np
import pytest

from mogecpp_b200 import synth
from mogecpp_b200 import lib as L

pytestmark = pytest.mark.gpu


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def test_make_level_noalloc_matches_workspace_entry_point():
    import torch
    lib = L.load()
    ctx = C.c_void_p()
    L.check(lib.msc_create(0, C.byref(ctx)))
    try:
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        for seed, extent in ((11, 40), (12, 64)):  # two calls in a row, the second larger
            coords = torch.from_numpy(synth.small_coords(seed, extent=extent, grid=96)).cuda()
            n = coords.shape[0]
            got = torch.full((n, 27), -7, dtype=torch.int32, device="cuda")
            L.check(lib.msc_make_level_noalloc(_ptr(coords), n, _ptr(got), _ptr(status), stream))
            want = torch.empty((n, 27), dtype=torch.int32, device="cuda")
            wsb = lib.msc_topology_workspace_bytes(n)
            ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
            L.check(lib.msc_make_level(ctx, _ptr(coords), n, _ptr(want), _ptr(ws), wsb, stream))
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            np.testing.assert_array_equal(got.cpu().numpy(), want.cpu().numpy())
    finally:
        lib.msc_destroy(ctx)


def test_make_level_noalloc_rejects_more_than_its_table_holds():
    lib = L.load()
    rc = lib.msc_make_level_noalloc(None, 524289, None, None, None)
    assert rc == -1
    assert "524288" in lib.msc_last_error().decode()
