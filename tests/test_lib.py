"""The C-ABI library loads and exports every symbol include/vtnk_b200.h
declares (CPU: no compute calls)."""

import ctypes
import re
from pathlib import Path

from conftest import ROOT


def test_library_exports_header_symbols():
    from rectokens_b200 import _lib

    header = (ROOT / "include" / "vtnk_b200.h").read_text()
    declared = set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]*?\b(vtnk_\w+)\s*\(", header, re.M))
    assert declared, "no declarations found"
    lib = _lib.lib()
    for name in sorted(declared):
        assert hasattr(lib, name), f"{name} not exported"
    assert set(_lib.EXPORTS) <= declared
    assert lib.vtnk_version() >= 100


def test_argument_errors_are_reported_without_gpu():
    import pytest
    import torch

    from rectokens_b200 import _lib

    lib = _lib.lib()
    # k > max_branches is rejected before any launch (torch.topk raises in the reference)
    a = torch.zeros(0, 4)
    lin = _lib.Linear(None, 0, 4, 4, None, 8, 8, 1, None, _lib.F32)
    csr = _lib.Csr(1, 1, 1, 1, 0)
    rc = lib.vtnk_fused_linear_constrained_node_transition_topk(
        lin, None, csr, 2, 3, None, None, None, None, None)
    assert rc == 1
    assert b"k (3)" in lib.vtnk_last_error()
    with pytest.raises(ValueError):
        _lib.check(rc)
    del a
