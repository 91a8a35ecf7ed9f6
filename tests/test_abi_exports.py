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
    assert _abi.abi_version() == 4


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


def test_workspace_sizes_monotonic():
    """A workspace sized for T tokens serves every smaller T (the sizes never shrink as T grows,
    across the grouped path's 16-token limit too), and the stack's size is the decode size."""
    from b200moe import _abi
    L = _abi.lib()
    sizes = [L.b200moe_decode_workspace_size(T) for T in range(1, 70)]
    assert all(b >= a for a, b in zip(sizes, sizes[1:])), sizes
    assert all(L.b200moe_stack_workspace_size(T, 40) == L.b200moe_decode_workspace_size(T) for T in (1, 2, 16, 17, 64))
    # from 2 tokens the grouped path's buffers (digit planes, plan, expert outputs) are included
    assert sizes[1] - sizes[0] > 2 * 9 * 2048 * 4


def test_block_type_validation_without_device_work():
    """The layer's block types and the down stride they imply are checked before any CUDA
    call: unknown types, a Q4_K-sized stride for Q5_K rows, and a grouped-GEMM call on a layer
    that is not Q4_K throughout are refused with EINVAL. (Fake 16-byte aligned addresses: the
    refusals come before anything reads them.)"""
    import ctypes as C
    from b200moe import _abi
    lib = _abi.lib()
    a = 1 << 20  # aligned placeholder address, never dereferenced on these paths
    ws = 1 << 40

    def layer(down_type=0, sh_type=0, down_stride=2048 * 288):
        return _abi.Layer(a, a, 512 * 1152, a, down_stride, a, a, a, a, a, None, 0, None, down_type, sh_type)

    def decode(Lr):
        return lib.b200moe_moe_decode(C.c_void_p(a), _abi.BF16, 1, C.byref(Lr), C.c_void_p(a), None, None,
                                      C.c_void_p(a), ws, None)

    for Lr, why in ((layer(down_type=99), b"down_type 99"), (layer(sh_type=13), b"sh_type 13"),
                    (layer(down_type=13), b"down_expert_stride"), (layer(down_type=14, down_stride=2048 * 352),
                                                                   b"down_expert_stride")):
        assert decode(Lr) == _abi.EINVAL, why
        assert why in lib.b200moe_last_error(), (why, lib.b200moe_last_error())
    Lr = layer(down_type=13, down_stride=2048 * 352, sh_type=8)
    rc = lib.b200moe_moe_prefill(C.c_void_p(a), _abi.BF16, None, C.c_float(1e-6), 16, C.byref(Lr), C.c_void_p(a),
                                 None, C.c_void_p(a), ws, None)
    assert rc == _abi.EINVAL and b"Q4_K" in lib.b200moe_last_error()


def test_plain_c_host(tmp_path):
    """A C99 program includes the header and links the library (static CUDA runtime, no other
    CUDA dependency): version, argument refusals and the error message, no device work."""
    import shutil
    import subprocess
    from b200moe import _abi
    if not shutil.which("gcc"):
        import pytest
        pytest.skip("no C compiler")
    src = tmp_path / "host.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "b200moe.h"
int main(void) {
  b200moe_layer L;
  memset(&L, 0, sizeof L);
  if (b200moe_abi_version() != B200MOE_ABI_VERSION) return 1;
  if (b200moe_q4k_dequant(NULL, 5, NULL, B200MOE_F32, NULL) != B200MOE_EINVAL) return 2;
  if (!strstr(b200moe_last_error(), "NULL")) return 3;
  if (b200moe_moe_decode(NULL, B200MOE_BF16, 1, &L, NULL, NULL, NULL, NULL, 0, NULL) != B200MOE_EINVAL) return 4;
  if (b200moe_decode_workspace_size(1) == 0 || b200moe_decode_workspace_size(0) != 0) return 5;
  printf("ok %d\n", b200moe_abi_version());
  return 0;
}
''')
    lib_dir = os.path.dirname(_abi.LIB_PATH)
    exe = tmp_path / "host"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                    "-L", lib_dir, "-lb200moe", "-Wl,-rpath," + lib_dir, "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0 and out.stdout.strip() == "ok %d" % _abi.abi_version(), (out.returncode, out.stdout)
