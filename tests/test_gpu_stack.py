"""The config-4 MoE sub-stack (resid += moe(rmsnorm(resid)) per layer) on the device.

Per layer, teacher-forced: the oracle takes the device's residual entering the layer,
applies the declared-order RMSNorm and router (bit-exact ids) and the f64 block, and the
device's residual after the layer must match within rel-L2 1e-5."""
import numpy as np
import pytest

from conftest import host_layer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine4(cuda):
    from b200moe.engine import DeviceEngine
    return DeviceEngine.synthetic(4, 4, cuda)


@pytest.mark.parametrize("T", [1, 2])
def test_stack_teacher_forced(cuda, engine4, T):
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe, synth
    from b200moe.engine import DeviceEngine
    resid = torch.from_numpy(bf16_bits_to_f32(synth.tokens(4, T, stream=9)).copy()).to(cuda)
    for l in range(4):
        before = resid.cpu().numpy().copy()
        ids = torch.empty((1, T, 8), dtype=torch.int32, device=cuda)
        moe.moe_stack(resid, DeviceEngine([engine4.layers[l]]), ids_out=ids)
        after = resid.cpu().numpy()
        Lh = host_layer(4, l)
        xn = OM.rmsnorm(before)
        r = OM.router(xn, Lh.wg)
        assert (ids.cpu().numpy().reshape(T, 8) == r["ids"]).all(), l
        ref = before.astype(np.float64) + OM.moe_block_f64(xn, Lh, r["ids"], r["w_bf16"])["out"]
        c = OM.compare(after, ref)
        assert c["rel_l2"] < 1e-5, (l, c)


def test_stack_one_call_equals_layer_by_layer(cuda, engine4):
    import torch
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe, synth
    from b200moe.engine import DeviceEngine
    x0 = torch.from_numpy(bf16_bits_to_f32(synth.tokens(4, 1, stream=10)).copy()).to(cuda)
    a = x0.clone()
    moe.moe_stack(a, engine4)
    b = x0.clone()
    for L in engine4.layers:
        moe.moe_stack(b, DeviceEngine([L]))
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.isfinite(a).all()
