"""Router and shared-gate weights stored as f32 (the published file keeps ffn_gate_inp and
ffn_gate_inp_shexp in F32): every device path uses them exactly. The weights here are the
synthetic bf16 ones moved off the bf16 grid, so a path that rounded them to bf16 would change
logits. Bars as for bf16 routers: ids / R5 weights bit-exact against the declared-order oracle
fed the same f32 weights; block outputs within the decode (rel-L2 1e-5) or prefill (1e-3)
bars of the f64 restatement; the persistent single-token kernel (tensor-core expert dots) within
the decode bar of the three-kernel path (CUDA-core f32 dots), with the same ids."""
import numpy as np
import pytest

from conftest import host_layer

pytestmark = pytest.mark.gpu


def _f32_weights(seed, layer):
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import synth
    rng = np.random.default_rng(1000 + layer)
    w = bf16_bits_to_f32(synth.router_w(seed, layer)).astype(np.float32)
    g = bf16_bits_to_f32(synth.shared_gate_w(seed, layer)).astype(np.float32)
    w = (w * (1.0 + rng.uniform(-3e-3, 3e-3, w.shape))).astype(np.float32)
    g = (g * (1.0 + rng.uniform(-3e-3, 3e-3, g.shape))).astype(np.float32)
    return w, g


@pytest.fixture(scope="module")
def layer_f32(cuda):
    import torch
    from b200moe.engine import DeviceLayer
    from oracle.moe import HostLayer
    base = DeviceLayer.synthetic(2, 0, cuda)
    w, g = _f32_weights(2, 0)
    L = DeviceLayer(base.gate, base.up, base.down, base.sh_gate, base.sh_up, base.sh_down,
                    torch.from_numpy(w).to(cuda), torch.from_numpy(g).to(cuda))
    hb = host_layer(2, 0)
    Lh = HostLayer(hb._block_fn, w, g)
    return L, Lh


def _x(T, stream, cuda):
    import torch
    from b200moe import synth
    xb = synth.tokens(2, T, stream=stream)
    return xb, torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)


def test_weights_are_off_the_bf16_grid(layer_f32):
    from oracle.bf16 import round_bf16
    _, Lh = layer_f32
    assert np.mean(round_bf16(Lh.wg) != Lh.wg) > 0.9


def test_router_f32_weights_bit_exact(cuda, layer_f32):
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe
    L, Lh = layer_f32
    xb, x = _x(16, 3, cuda)
    r = moe.moe_router(x, L, 0)
    torch.cuda.synchronize()
    o = OM.router(bf16_bits_to_f32(xb), Lh.wg)
    assert (r["router_logits"].view(torch.int16).cpu().numpy().view(np.uint16) == o["logits"]).all()
    assert (r["topk_ids"].cpu().numpy() == o["ids"]).all()
    assert (r["topk_weights"].view(torch.int16).cpu().numpy().view(np.uint16) == o["w_bf16"]).all()
    # the same weights rounded to bf16 route differently somewhere: the f32 path is really exercised
    from oracle.bf16 import f32_to_bf16_bits
    o16 = OM.router(bf16_bits_to_f32(xb), f32_to_bf16_bits(Lh.wg))
    assert not (o16["logits"] == o["logits"]).all()


@pytest.mark.parametrize("T,path,rel", [(1, "decode", 1e-5), (4, "decode", 1e-5), (300, "prefill", 1e-3)])
def test_block_with_f32_router(cuda, layer_f32, T, path, rel):
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe
    L, Lh = layer_f32
    xb, x = _x(T, 4, cuda)
    out, info = moe.moe_block(x, L, 0, path=path)
    torch.cuda.synchronize()
    xf = bf16_bits_to_f32(xb)
    r = OM.router(xf, Lh.wg)
    ids = info["ids"].reshape(T, 8).cpu().numpy()
    assert (ids == r["ids"]).all()
    rows = np.arange(T) if T <= 8 else np.sort(np.random.default_rng(0).choice(T, 24, replace=False))
    ref = OM.moe_block_f64(xf[rows], Lh, ids[rows], r["w_bf16"][rows])["out"]
    c = OM.compare(out.reshape(T, 2048).cpu().numpy()[rows], ref)
    assert c["rel_l2"] < rel and np.isfinite(out.cpu().numpy()).all(), c


def test_persistent_equals_three_kernel_with_f32_router(cuda, layer_f32):
    import torch
    from b200moe import moe
    L, _ = layer_f32
    _, x = _x(1, 5, cuda)
    a, ia = moe.moe_block(x, L, 0, path="decode")
    b, ib = moe.moe_block(x.repeat(2, 1), L, 0, path="decode")
    torch.cuda.synchronize()
    from oracle import moe as OM
    c = OM.compare(a[0].double().cpu().numpy(), b[0].double().cpu().numpy())
    assert c["rel_l2"] < 1e-5 and c["max_abs_norm"] < 1e-5, c
    assert torch.equal(b[0], b[1]) and torch.equal(ia["ids"][0], ib["ids"][0])
