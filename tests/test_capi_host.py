"""C-ABI library: loads without a GPU, exports every declared symbol, and its
host-side logic (size queries, argument checks) behaves."""
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "moge_sparse_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(msc_[a-z_0-9]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from mogecpp_b200 import lib as L
    lib = L.load()
    syms = declared_symbols()
    assert len(syms) >= 15
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    assert set(syms) == set(L.SIGNATURES), "ctypes signature table out of sync with the header"


def test_abi_version():
    from mogecpp_b200 import lib as L
    assert L.load().msc_abi_version() == 1


def test_size_queries_are_host_only():
    from mogecpp_b200 import lib as L
    lib = L.load()
    # Q8_0 with cin 128: int8 tiles + block scales; Q8_0 with cin 64: an
    # exact fp16 hi/lo pair
    def r256(v):
        return (v + 255) // 256 * 256
    assert lib.msc_weight_blob_bytes(L.MSC_W_Q8_0, 128, 128, 27) == 256 + 27 * 128 * 128 + 27 * 4 * 128 * 4
    assert lib.msc_weight_blob_bytes(L.MSC_W_Q8_0, 128, 64, 1) == 256 + 128 * 64 + 4 * 64 * 4
    assert lib.msc_weight_blob_bytes(L.MSC_W_Q8_0, 64, 64, 27) == 256 + 2 * 27 * 64 * 64 * 2
    assert lib.msc_weight_blob_bytes(L.MSC_W_F32, 64, 64, 27) == 256 + 2 * 27 * 64 * 64 * 2
    assert lib.msc_weight_blob_bytes(L.MSC_W_F16, 64, 64, 27) == 256 + 27 * 64 * 64 * 2
    assert lib.msc_weight_blob_bytes(99, 64, 64, 27) == 0
    assert lib.msc_topology_workspace_bytes(1000) > 2048 * 16
    assert lib.msc_op_workspace_bytes(1000, 128) >= 1000 * 128 * 8
    # conv plan: header + order + tile rows + tile neighbour lists + tile masks
    npad = 8 * 128
    # header | order | tile rows | tile neighbour lists | tile masks | tile schedule
    assert lib.msc_conv_plan_bytes(1000) == (r256(16) + r256(4000) + r256(4 * npad) + r256(4 * 27 * npad) +
                                             2 * r256(4 * 8))
    assert lib.msc_conv_plan_bytes(-1) == 0
    assert lib.msc_conv_plan_workspace_bytes(1000) >= 1000 * 12
    # GroupNorm statistics: 32 sums, 1 count, 32 squared deviations per sample
    assert lib.msc_gn_stats_doubles(3) == 3 * 65
    assert lib.msc_gn_stats_doubles(0) == 0
    assert lib.msc_res_block_gn_workspace_bytes(1000, 128, 2) == lib.msc_op_workspace_bytes(1000, 128) + 512
    assert lib.msc_res_block_gn_workspace_bytes(1000, 128, 0) == 0


def test_create_fails_cleanly_without_sm100():
    import ctypes as C
    import torch
    from mogecpp_b200 import lib as L
    if torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0):
        pytest.skip("an sm_100 device is present")
    lib = L.load()
    h = C.c_void_p()
    rc = lib.msc_create(0, C.byref(h))
    assert rc != 0
    assert lib.msc_last_error().decode()


def test_null_context_is_rejected():
    from mogecpp_b200 import lib as L
    lib = L.load()
    rc = lib.msc_make_level(None, None, 0, None, None, 0, None)
    assert rc == -1
    assert "context" in lib.msc_last_error().decode()


def _c_program(syms):
    """A C99 program that references every declared entry point (so the link
    resolves each one against the library) and calls the host-only ones."""
    table = ",\n    ".join(f"(msc_fn)&{s}" for s in syms)
    return f"""#include <stdio.h>
#include <string.h>
#include "moge_sparse_cuda.h"

typedef void (*msc_fn)(void);
static const msc_fn kEntryPoints[] = {{
    {table}
}};

int main(void) {{
    size_t k, present = 0;
    int rc;
    for (k = 0; k < sizeof(kEntryPoints) / sizeof(kEntryPoints[0]); ++k) present += kEntryPoints[k] != NULL;
    rc = msc_make_level(NULL, NULL, 0, NULL, NULL, 0, NULL);
    printf("entry_points %lu\\n", (unsigned long)present);
    printf("abi %d\\n", msc_abi_version());
    printf("topology_ws_1000 %lu\\n", (unsigned long)msc_topology_workspace_bytes(1000));
    printf("null_ctx_rc %d\\n", rc);
    printf("null_ctx_error_has_context %d\\n", strstr(msc_last_error(), "context") != NULL);
    return 0;
}}
"""


@pytest.mark.parametrize("compiler,std", [("gcc", "-std=c99"), ("g++", "-std=c++11")])
def test_header_compiles_links_and_runs_from_plain_c(tmp_path, compiler, std):
    """What a cgo / JNI / N-API binding sees: the header alone, compiled as
    strict C99 (and as C++ through its extern "C" guard), linked against the
    shared library, run on a host without a GPU."""
    import shutil
    import subprocess
    from mogecpp_b200 import lib as L
    if shutil.which(compiler) is None:
        pytest.skip(f"{compiler} is not installed")
    if not os.path.exists(L.LIB_PATH):
        pytest.skip("library not built")
    syms = declared_symbols()
    src = tmp_path / ("abi.c" if compiler == "gcc" else "abi.cpp")
    src.write_text(_c_program(syms))
    exe = tmp_path / "abi"
    libdir = os.path.dirname(L.LIB_PATH)
    cmd = [compiler, std, "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", os.path.join(ROOT, "include"),
           str(src), "-o", str(exe), "-L", libdir, "-l:" + os.path.basename(L.LIB_PATH), "-Wl,-rpath," + libdir]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True, timeout=60).stdout
    got = dict(line.split() for line in out.splitlines())
    assert int(got["entry_points"]) == len(syms)
    assert int(got["abi"]) == 1
    assert int(got["topology_ws_1000"]) == L.load().msc_topology_workspace_bytes(1000)
    assert int(got["null_ctx_rc"]) == -1
    assert got["null_ctx_error_has_context"] == "1"


def test_cxx_seam_compiles_and_reports_no_device(tmp_path):
    """include/moge_sparse_cuda.hpp, the C++17 seam mogecpp's refiner loop
    calls (moge_cuda::Device, SparseConfig, SparseRefiner), compiles warning
    free against the header alone and, without an sm_100 GPU, reports the
    device unavailable and turns C ABI failures into moge_cuda::Error."""
    import shutil
    import subprocess
    import torch
    from mogecpp_b200 import lib as L
    if shutil.which("g++") is None:
        pytest.skip("g++ is not installed")
    if not os.path.exists(L.LIB_PATH):
        pytest.skip("library not built")
    exe = tmp_path / "seam"
    libdir = os.path.dirname(L.LIB_PATH)
    cmd = ["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "cxx_seam_probe.cpp"), "-o", str(exe), "-L", libdir,
           "-l:" + os.path.basename(L.LIB_PATH), "-Wl,-rpath," + libdir]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True, timeout=60).stdout
    lines = {ln.split()[0]: ln.split()[1:] for ln in out.splitlines()}
    sm100 = torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    assert lines["device"] == ["sm100" if sm100 else "none"]
    assert lines["null_ctx_code"] == ["-1"]
    assert lines["null_ctx_message"] == ["1"]
    assert lines["default_config"] == ["0", "3", "16", "256.0"]
