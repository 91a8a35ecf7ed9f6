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


def _with_norm(engine, seed):
    """The same layers with a post-attention RMSNorm weight (Form A as stored: 1 + w)."""
    import torch
    from b200moe.engine import DeviceEngine, DeviceLayer
    layers, ws = [], []
    for l, L in enumerate(engine.layers):
        w = (1.0 + np.random.default_rng(seed + l).normal(0.0, 0.05, 2048)).astype(np.float32)
        ws.append(w)
        layers.append(DeviceLayer(L.gate, L.up, L.down, L.sh_gate, L.sh_up, L.sh_down, L.router_w, L.sh_gate_w,
                                  L.logit_bias, L.gate_up_stride, norm_w=torch.from_numpy(w).to(L.gate.device)))
    return DeviceEngine(layers), ws


@pytest.mark.parametrize("T,path", [(1, "decode"), (2, "decode"), (64, "prefill")])
def test_stack_with_norm_weight_teacher_forced(cuda, engine4, T, path):
    """x = (resid * rs) * w (Form A, two roundings) inside the stack: ids bit-exact against the
    oracle's weighted declared-order RMSNorm + router, the residual within the path's bar."""
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe, synth
    from b200moe.engine import DeviceEngine
    Ew, ws = _with_norm(engine4, 77)
    resid = torch.from_numpy(bf16_bits_to_f32(synth.tokens(4, T, stream=11)).copy()).to(cuda)
    for l in range(2):
        before = resid.cpu().numpy().copy()
        ids = torch.empty((1, T, 8), dtype=torch.int32, device=cuda)
        one = DeviceEngine([Ew.layers[l]])
        if path == "decode":
            moe.moe_stack(resid, one, ids_out=ids)
        else:
            moe.moe_stack_prefill(resid, one, ids_out=ids)
            assert moe.prefill_status(T, cuda) == 0
        after = resid.cpu().numpy()
        Lh = host_layer(4, l)
        xn = OM.rmsnorm(before, w=ws[l])
        assert not np.array_equal(xn, OM.rmsnorm(before))  # the weight changes the input
        r = OM.router(xn, Lh.wg)
        assert (ids.cpu().numpy().reshape(T, 8) == r["ids"]).all(), l
        rows = np.arange(T) if T <= 8 else np.arange(0, T, 8)
        ref = before[rows].astype(np.float64) + OM.moe_block_f64(xn[rows], Lh, r["ids"][rows], r["w_bf16"][rows])["out"]
        c = OM.compare(after[rows], ref)
        assert c["rel_l2"] < (1e-5 if path == "decode" else 1e-3), (l, c)
