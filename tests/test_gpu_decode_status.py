"""Decode status read-back, and the persistent kernel's bounded waits made to run out.

The single-token persistent kernel (persist.cu) hands values between its 128 CTAs through
tagged words and waits on them with bounded polls and bounded mbarrier waits. A wait that runs
out must not hang the GPU or leave silent garbage: the kernel ends on every CTA, the call's
status word says so (b200moe_decode_status), and the next call on the same device is correct.
The failure is made on purpose without any fault: the library's test hook shortens the wait
budget to ~0.1 ms and makes one CTA withhold its first published logit pair -- a flag that
nothing then sets -- so every other CTA's gather runs out of budget (the reference's
counterpart is its loud refusal, engine/m3_forward.py:165-170).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BUDGET = 200_000      # clock cycles (~0.1 ms) for the failure-path test
WITHHELD_CTA = 5


@pytest.fixture(scope="module")
def engine4(cuda):
    from b200moe.engine import DeviceEngine
    return DeviceEngine.synthetic(4, 4, cuda)


def _x(seed, stream, T, cuda):
    import torch
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import synth
    return torch.from_numpy(bf16_bits_to_f32(synth.tokens(seed, T, stream=stream)).copy()).to(cuda)


def _decode(x, L, ws):
    import torch
    from b200moe import _abi
    T = x.shape[0]
    out = torch.full((T, 2048), float("nan"), dtype=torch.float32, device=x.device)
    ids = torch.full((T, 8), -1, dtype=torch.int32, device=x.device)
    _abi.moe_decode(x, _abi.F32, T, L.abi(), out, ids, None, ws)
    return out, ids


def test_status_zero_after_complete_calls(cuda, engine4):
    import torch
    from b200moe import _abi, moe
    L = engine4.layers[1]
    for T in (1, 3):
        ws = torch.empty(_abi.decode_workspace_size(T), dtype=torch.uint8, device=cuda)
        ws.fill_(0xFF)  # a fresh workspace's word is garbage until the first call clears it
        out, _ = _decode(_x(4, 30 + T, T, cuda), L, ws)
        assert _abi.decode_status(ws, T) == 0, T
        assert torch.isfinite(out).all()
    r = _x(4, 35, 1, cuda)
    moe.moe_stack(r, engine4, check=True)
    assert torch.isfinite(r).all()
    o, _ = moe.moe_block(_x(4, 36, 1, cuda), engine4, 2, check=True)
    assert torch.isfinite(o).all()


def test_bounded_wait_runs_out_and_is_reported(cuda, engine4):
    import torch
    from b200moe import _abi, moe
    if _abi.decode_persistent_info()[0] == 0:
        pytest.skip("this device runs the three-kernel path (no bounded waits)")
    L = engine4.layers[2]
    ws = torch.empty(_abi.decode_workspace_size(1), dtype=torch.uint8, device=cuda)
    x = _x(4, 37, 1, cuda)
    ref, ref_ids = _decode(x, L, ws)
    assert _abi.decode_status(ws, 1) == 0
    _abi.debug_decode_faults(BUDGET, WITHHELD_CTA)
    try:
        _decode(x, L, ws)
        torch.cuda.synchronize()          # every CTA ended: the call returned
        assert _abi.decode_status(ws, 1) == 1
        r = _x(4, 38, 1, cuda)
        with pytest.raises(_abi.B200MoeError, match="status word 1"):
            moe.moe_stack(r, engine4, ws=ws, check=True)
    finally:
        _abi.debug_decode_faults(0, -1)
    # the context is intact and the next call on the same workspace is complete and identical
    out, ids = _decode(x, L, ws)
    torch.cuda.synchronize()
    assert _abi.decode_status(ws, 1) == 0
    assert torch.equal(out, ref) and torch.equal(ids, ref_ids)

