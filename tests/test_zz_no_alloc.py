"""b200moe_moe_decode_noalloc: the decode entry point that allocates nothing.

Some callers cannot allocate device memory where they call the MoE block -- a plugin that
its host framework hands only input and output buffers, code that runs while a CUDA graph is
being captured, an FFI caller without a device allocator. For them the library keeps the
decode scratch in a fixed static device array (at most B200MOE_NOALLOC_MAX_T = 16 tokens).
This test drives that entry point through the C ABI and checks it against the workspace
entry point b200moe_moe_decode on two calls in a row (different tokens each time, so stale
scratch from the first call cannot pass for a result): with the decode path's own parity
tolerance on the multi-token path, and bit for bit on the single-token persistent kernel,
whose cross-CTA exchange area then lives in the static array. It checks the no-alloc status
word and that a batch above the limit is refused. It runs alone in a fresh
process or after the other tests: the per-device scratch lookup happens on the first call.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
REL_L2 = 1e-5          # the decode path's tolerance (tests/test_gpu_decode.py)


def test_noalloc_matches_workspace_entry(cuda):
    import torch
    from b200moe import _abi, moe, synth
    from b200moe.engine import DeviceLayer
    L = DeviceLayer.synthetic(0, 0, cuda)
    for call, (T, stream) in enumerate([(5, 21), (16, 22)]):
        x = torch.from_numpy(synth.tokens(0, T, stream=stream).view(np.int16)).view(torch.bfloat16).to(cuda)
        ref = torch.empty((T, 2048), dtype=torch.float32, device=cuda)
        ref_ids = torch.empty((T, 8), dtype=torch.int32, device=cuda)
        _abi.moe_decode(x, _abi.BF16, T, L.abi(), ref, ref_ids, None, moe.workspace(T, cuda))
        out = torch.full((T, 2048), float("nan"), dtype=torch.float32, device=cuda)
        ids = torch.full((T, 8), -1, dtype=torch.int32, device=cuda)
        w = torch.zeros((T, 8), dtype=torch.int16, device=cuda)
        _abi.moe_decode_noalloc(x, _abi.BF16, T, L.abi(), out, ids, w)
        torch.cuda.synchronize()
        assert torch.equal(ids, ref_ids), call
        rel = float(torch.linalg.norm(out - ref) / torch.linalg.norm(ref))
        assert rel < REL_L2, (call, rel)
        assert torch.isfinite(out).all()


def test_noalloc_single_token_persistent(cuda):
    """T = 1 runs the persistent single-token kernel with its cross-CTA exchange area carved
    from the static array, which each call clears first. Two calls in a row with different
    tokens must each equal the workspace entry point's result bit for bit (both run the same
    kernel on the same operations), report status 0, and match the f64 oracle."""
    import torch
    from conftest import host_layer
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import _abi, moe, synth
    from b200moe.engine import DeviceLayer
    L = DeviceLayer.synthetic(0, 0, cuda)
    host = host_layer(0, 0)
    for call, stream in enumerate((23, 24)):
        xb = synth.tokens(0, 1, stream=stream)
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
        ref = torch.empty((1, 2048), dtype=torch.float32, device=cuda)
        ref_ids = torch.empty((1, 8), dtype=torch.int32, device=cuda)
        _abi.moe_decode(x, _abi.BF16, 1, L.abi(), ref, ref_ids, None, moe.workspace(1, cuda))
        out = torch.full((1, 2048), float("nan"), dtype=torch.float32, device=cuda)
        ids = torch.full((1, 8), -1, dtype=torch.int32, device=cuda)
        _abi.moe_decode_noalloc(x, _abi.BF16, 1, L.abi(), out, ids, None)
        assert _abi.decode_noalloc_status(1) == 0, call
        assert torch.equal(ids, ref_ids) and torch.equal(out, ref), call
        xf = bf16_bits_to_f32(xb)
        r = OM.router(xf, host.wg)
        assert (ids.cpu().numpy() == r["ids"]).all(), call
        want = OM.moe_block_f64(xf, host, r["ids"], r["w_bf16"])["out"]
        c = OM.compare(out.cpu().numpy(), want)
        assert c["rel_l2"] < REL_L2, (call, c)


def test_noalloc_refuses_oversize(cuda):
    import torch
    from b200moe import _abi
    from b200moe.engine import DeviceLayer
    L = DeviceLayer.synthetic(0, 1, cuda)
    T = 17
    x = torch.zeros((T, 2048), dtype=torch.float32, device=cuda)
    out = torch.empty((T, 2048), dtype=torch.float32, device=cuda)
    with pytest.raises(_abi.B200MoeError) as ei:
        _abi.moe_decode_noalloc(x, _abi.F32, T, L.abi(), out, None, None)
    assert ei.value.code == _abi.ESIZE and "16" in str(ei.value)
