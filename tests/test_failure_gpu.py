"""Failure detection on the GPU without a fault: every cross-GPU wait in
this library is bounded, gives up with MSC_DEV_TIMEOUT in the context's
status word and returns, so the host learns of a neighbour that never
arrives and the context stays usable.  The probe runs the slab path's wait
on a flag that nothing sets."""
import ctypes as C

import numpy as np
import pytest
import torch

from gpu_util import dev, host
from mogecpp_b200 import lib as L
from mogecpp_b200 import synth

pytestmark = pytest.mark.gpu


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_wait_that_runs_out_is_reported_and_the_context_recovers(ex, oracle):
    ex.check()
    assert ex.lib.msc_wait_probe(ex.ctx, 20000, _stream()) == 0    # 20 ms budget
    bits = C.c_uint32(0)
    rc = ex.lib.msc_check(ex.ctx, _stream(), C.byref(bits))
    assert rc == -4 and bits.value & L.DEV_TIMEOUT, (rc, bits.value)
    assert "wait-timeout" in ex.lib.msc_last_error().decode()
    # the status word was cleared and the context runs the next call
    coords = synth.small_coords(3, extent=12, grid=16)
    np.testing.assert_array_equal(host(ex.make_level(dev(coords))), oracle.make_level(coords))
    assert ex.check() == 0


def test_probe_rejects_a_budget_beyond_two_seconds(ex):
    assert ex.lib.msc_wait_probe(ex.ctx, 3_000_000, _stream()) == -1
