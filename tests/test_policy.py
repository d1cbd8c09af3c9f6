"""Policy pinned by source inspection (the reference pins its runtime policy
the same way, tests/test_runtime_policy.py in mogecpp):

* the product (the package and its CUDA sources) never reaches the oracle or
  the reference build: those are test infrastructure;
* there is no CPU or PyTorch fallback: loading the library fails loudly when
  it is not built, and the package's operators only call the C ABI;
* every ncu command recorded under profiles/ leaves the GPU clocks alone."""
import glob
import os
import re

import pytest

from conftest import ROOT

PKG = os.path.join(ROOT, "mogecpp_b200")


def _sources(patterns):
    out = []
    for p in patterns:
        out += glob.glob(os.path.join(ROOT, p), recursive=True)
    return sorted(f for f in out if "/_work/" not in f and "/_build/" not in f and "/_ref/" not in f)


def test_product_never_reaches_the_oracle():
    for f in _sources(["mogecpp_b200/*.py", "mogecpp_b200/csrc/*"]):
        src = open(f).read()
        assert not re.search(r"^\s*(import|from)\s+oracle\b", src, re.M), f
        assert "liboracle" not in src and "libmoge_ref" not in src, f


def test_library_load_fails_loudly_without_the_build(tmp_path):
    from mogecpp_b200 import lib as L
    saved = L._LIB
    L._LIB = None
    try:
        with pytest.raises(ImportError, match="no CPU fallback"):
            L.load(str(tmp_path / "missing.so"))
    finally:
        L._LIB = saved


def test_package_has_no_torch_compute_fallback():
    """The operator module reaches results only through the C ABI: no torch
    math on features (matmul, conv, layer / group norm, silu) stands in."""
    src = open(os.path.join(PKG, "sparse.py")).read()
    for banned in ("torch.matmul", "torch.mm(", "@ w", "F.conv", "torch.nn.functional", "layer_norm(", "group_norm(",
                   "torch.sigmoid", ".silu("):
        assert banned not in src, banned


def test_profiles_ncu_commands_leave_clocks_alone():
    for f in glob.glob(os.path.join(ROOT, "profiles", "*.md")):
        for line in open(f):
            if re.search(r"^\s*ncu\s", line):
                assert "--clock-control none" in line, (f, line)
