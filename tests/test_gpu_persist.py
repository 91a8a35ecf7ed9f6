"""The persistent single-token decode kernel (persist.cu) against the three-kernel decode path.

At T = 1 both b200moe_moe_decode and b200moe_stack_decode run the persistent kernel; at T >= 2
they run the per-token three-kernel path, which treats every token independently. Feeding a
T = 2 call two copies of the token therefore gives the three-kernel result for it. For Q4_K
layers the persistent kernel computes the expert dots on the tensor cores with exact integer
products over a 24-bit fixed-point image of x and s, the three-kernel path in f32 on the CUDA
cores, so the two agree within the decode parity bar (rel-L2 and max-abs / max|ref| 1e-5 -- both
are within it of the f64 oracle), with the same routing ids. The oracle parity of the T = 1 path
itself is covered by test_gpu_decode.py and test_gpu_stack.py; the block-format variant (Q5_K /
Q6_K / Q8_0 layers) still matches the three-kernel path bit for bit (test_gpu_kquant_layers.py).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
PATH_REL_L2, PATH_MAX_ABS_NORM = 1e-5, 1e-5


def _close(a, b):
    import torch
    from oracle import moe as OM
    c = OM.compare(a.double().cpu().numpy(), b.double().cpu().numpy())
    print("persistent vs three-kernel path: rel-L2 %.3e, max-abs / max|ref| %.3e" % (c["rel_l2"], c["max_abs_norm"]))
    return c["rel_l2"] < PATH_REL_L2 and c["max_abs_norm"] < PATH_MAX_ABS_NORM


@pytest.fixture(scope="module")
def engine4(cuda):
    from b200moe.engine import DeviceEngine
    return DeviceEngine.synthetic(4, 4, cuda)


def _token(seed, stream, cuda):
    import torch
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import synth
    return torch.from_numpy(bf16_bits_to_f32(synth.tokens(seed, 1, stream=stream)).copy()).to(cuda)


def test_persistent_path_is_active(cuda):
    """On a B200 the single-token path must be the persistent kernel (the comparisons below
    would otherwise compare the three-kernel path with itself)."""
    from b200moe import _abi
    ctas, cluster = _abi.decode_persistent_info()
    assert ctas == 128 and cluster in (1, 2, 4, 8), (ctas, cluster)


def test_stack_persistent_equals_three_kernel_path(cuda, engine4):
    import torch
    from b200moe import moe
    x0 = _token(4, 21, cuda)
    a = x0.clone()
    ids_a = torch.empty((4, 1, 8), dtype=torch.int32, device=cuda)
    moe.moe_stack(a, engine4, ids_out=ids_a)
    b = x0.repeat(2, 1)
    ids_b = torch.empty((4, 2, 8), dtype=torch.int32, device=cuda)
    moe.moe_stack(b, engine4, ids_out=ids_b)
    torch.cuda.synchronize()
    assert torch.isfinite(a).all()
    assert torch.equal(b[0], b[1]) and _close(a[0], b[0])
    assert torch.equal(ids_a[:, 0], ids_b[:, 0])


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_layer_persistent_equals_three_kernel_path(cuda, engine4, dtype):
    import torch
    from b200moe import moe
    x = _token(4, 22, cuda)
    if dtype == "bf16":
        x = x.to(torch.bfloat16)
    o1, i1 = moe.moe_block(x.reshape(1, 1, 2048), engine4, 2)
    o2, i2 = moe.moe_block(x.repeat(2, 1).reshape(1, 2, 2048), engine4, 2)
    torch.cuda.synchronize()
    assert _close(o1[0, 0], o2[0, 0]) and torch.equal(i1["ids"][0, 0], i2["ids"][0, 0])


def test_repeated_calls_and_graph_replay(cuda, engine4):
    """The flag area is reset per call: three eager calls and two replays of a captured call
    on the same input give the same bits."""
    import torch
    from b200moe import moe
    x0 = _token(4, 23, cuda)
    ws = torch.empty(moe.stack_workspace_bytes(1), dtype=torch.uint8, device=cuda)
    outs = []
    for _ in range(3):
        r = x0.clone()
        moe.moe_stack(r, engine4, ws=ws)
        outs.append(r)
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    r = x0.clone()
    s = torch.cuda.Stream(cuda)
    s.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(s):
        moe.moe_stack(r, engine4, ws=ws)  # warm the per-device setup outside capture
    torch.cuda.current_stream(cuda).wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        moe.moe_stack(r, engine4, ws=ws)
    for _ in range(2):
        r.copy_(x0)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(r, outs[0])
    del g


def test_more_layers_than_one_launch(cuda, engine4):
    """70 layers (the persistent kernel takes at most 64 per launch) = 70 one-layer calls."""
    import torch
    from b200moe import moe
    from b200moe.engine import DeviceEngine
    layers = [engine4.layers[i % 4] for i in range(70)]
    x0 = _token(4, 24, cuda) * 0.25
    a = x0.clone()
    moe.moe_stack(a, DeviceEngine(layers))
    b = x0.clone()
    for L in layers:
        moe.moe_stack(b, DeviceEngine([L]))
    torch.cuda.synchronize()
    assert torch.isfinite(a).all() and torch.equal(a, b)
