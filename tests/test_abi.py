"""C-ABI checks that need no GPU: the library loads, exports every symbol the
public header declares, and the ctypes signatures agree with the header."""

from __future__ import annotations

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "tagi_b200.h"


def _declarations():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    decls = {}
    for m in re.finditer(r"\b(?:int|size_t|uint64_t|const char\*)\s+(tagi_\w+)\s*\(([^)]*)\)\s*;",
                         text):
        args = [a.strip() for a in m.group(2).split(",") if a.strip() and a.strip() != "void"]
        decls[m.group(1)] = args
    return decls


def test_header_parses():
    d = _declarations()
    assert len(d) >= 30
    assert "tagi_fused_var_forward" in d and "tagi_param_grad" in d


def test_library_exports_every_declared_symbol():
    from triton_tagi._lib import lib

    L = lib()
    missing = [name for name in _declarations() if not hasattr(L.dll, name)]
    assert not missing, missing


def test_ctypes_signatures_match_header():
    from triton_tagi import _lib

    decls = _declarations()
    for name, codes in _lib._SIGS.items():
        assert name in decls, name
        assert len(codes) == len(decls[name]), (name, len(codes), len(decls[name]))
        for code, arg in zip(codes, decls[name]):
            if code == "p":
                assert "*" in arg, (name, arg)
            elif code == "i":
                assert arg.startswith("int64_t"), (name, arg)
            elif code == "f":
                assert arg.startswith("float") and "*" not in arg, (name, arg)
            elif code == "d":
                assert arg.startswith("double") and "*" not in arg, (name, arg)
            elif code == "n":
                assert arg.startswith("int ") or arg == "int", (name, arg)
            elif code == "z":
                assert arg.startswith("size_t"), (name, arg)
    assert set(decls) <= set(_lib._SIGS), set(decls) - set(_lib._SIGS)


def test_version_and_error_channel():
    from triton_tagi._lib import lib

    L = lib()
    assert L.fn["tagi_version"]() >= 0x100
    # An argument error is reported without touching the device.
    with pytest.raises(ValueError, match="bad sizes"):
        L("tagi_fused_var_forward", None, None, None, None, None, None, -1, 1, 1, 1, 1, 1, 1, 1,
          1, None)
    with pytest.raises(ValueError, match="cap_factor"):
        L("tagi_capped_update", 8, 8, 8, 8, 4, 0.0, None)


def test_workspace_queries_are_host_only():
    from triton_tagi._lib import lib

    L = lib()
    # A short reduction is never split; with 8 or more tiles of 256 weight rows
    # the workspace holds the optional prepared tiles of the deltas (8 K-blocks x
    # 4 tiles x 256 columns x 32 bytes); a long one over a small output is split.
    # With K a multiple of 256 the bias sums are formed apart (their one slice of
    # 2 x 256 column sums follows the weight rows' workspace).
    assert L.size("tagi_param_grad_workspace_size", 64, 784, 256, 1) == 0
    assert L.size("tagi_param_grad_workspace_size", 64, 2048, 256, 0) == 8 * 4 * 256 * 32
    assert (L.size("tagi_param_grad_workspace_size", 64, 2048, 256, 1)
            == 8 * 4 * 256 * 32 + 2 * 256 * 4)
    assert L.size("tagi_param_grad_workspace_size", 16, 30, 20, 1) == 0  # CUDA-core path
    big = L.size("tagi_param_grad_workspace_size", 128 * 1024, 576, 64, 1)
    assert big > 0 and big % 4 == 0
    # few weight rows over a long reduction (a 3x3 RGB stem): the CUDA-core slice
    # kernel, 256 slices of 512 pixels, partial sums for all 28 x 64 outputs
    assert L.size("tagi_param_grad_workspace_size", 131072, 27, 64, 1) == 2 * 256 * 28 * 64 * 4
    # 592 slices at most (4 per SM)
    assert L.size("tagi_param_grad_workspace_size", 524288, 75, 32, 1) == 2 * 586 * 76 * 32 * 4
