"""The C-ABI library loads and exports every symbol include/b200moe.h declares (no GPU)."""
import ctypes
import os
import re

from conftest import ROOT


def declared():
    src = open(os.path.join(ROOT, "include", "b200moe.h")).read()
    return sorted(set(re.findall(r"\b(b200moe_[a-z0-9_]+)\s*\(", src)))


def test_header_matches_binding():
    from b200moe import _abi
    assert sorted(_abi.EXPORTS) == declared()


def test_library_exports_every_symbol():
    from b200moe import _abi
    lib = ctypes.CDLL(_abi.LIB_PATH)
    for name in declared():
        assert hasattr(lib, name), name
    assert _abi.abi_version() == 2


def test_errors_without_device_work():
    """Argument validation answers before any CUDA call."""
    from b200moe import _abi
    L = _abi.lib()
    assert L.b200moe_q4k_dequant(None, 5, None, 0, None) == _abi.EINVAL
    assert b"NULL" in L.b200moe_last_error()
    assert L.b200moe_q4k_dequant(None, 0, None, 0, None) == _abi.OK
    assert L.b200moe_moe_decode(None, 0, 0, None, None, None, None, None, 0, None) == _abi.EINVAL
    assert L.b200moe_decode_workspace_size(0) == 0
    assert L.b200moe_decode_workspace_size(1) > 0
