"""Layers in the published Q4_K_M file's block formats on the decode kernels: Q5_K / Q6_K expert
down matrices and a Q8_0 shared expert (k_gateup<true>, k_down<Q5_K|Q6_K, Q8_0|Q4_K>, and the
persistent kernel's block-format variant k_mega<2>).

Parity bar (as for the Q4_K decode path): routing ids bit-exact against the declared-order C
restatement; the f32 block output against the f64 restatement of engine/m3_forward.py:430-476
(fed the same ids, weights decoded by oracle/kquants.py, itself pinned to the reference's
decoders) within rel-L2 1e-5 and max-abs / max|ref| 1e-5. A single token goes through the
persistent kernel's format variant, several through the three-kernel path, a stack through
b200moe_stack_decode; the two decode paths agree bit for bit; the grouped GEMMs refuse the
layer."""
import numpy as np
import pytest

from conftest import host_layer

pytestmark = pytest.mark.gpu
REL_L2, MAX_ABS_NORM = 1e-5, 1e-5


def _mixed(seed, layer, down, sh, device):
    """(device layer, oracle layer): Q4_K gate / up from the synthetic generator, the down
    matrices (``down``) and, when ``sh`` is Q8_0, the shared expert as seeded random blocks."""
    import torch
    from oracle import kquants
    from oracle.moe import HostLayer
    from b200moe.engine import DeviceLayer
    from b200moe.geometry import E, H, I
    base = DeviceLayer.synthetic(seed, layer, device)
    hb = host_layer(seed, layer)
    host = {}
    if down != "Q4_K":
        host["down"] = kquants.random_blocks(down, E * H * I // kquants.BLOCK_ELTS[down], 1000 + layer)
    if sh != "Q4_K":
        for k, n, s in (("sh_gate", I * H, 1), ("sh_up", I * H, 2), ("sh_down", H * I, 3)):
            host[k] = kquants.random_blocks(sh, n // kquants.BLOCK_ELTS[sh], 2000 + 10 * layer + s)
    dev = {k: torch.from_numpy(v.reshape(-1)).to(device) for k, v in host.items()}
    L = DeviceLayer(base.gate, base.up, dev.get("down", base.down), dev.get("sh_gate", base.sh_gate),
                    dev.get("sh_up", base.sh_up), dev.get("sh_down", base.sh_down), base.router_w,
                    base.sh_gate_w, down_type=down, sh_type=sh)

    def blocks(kind, first, n):
        if kind in host:
            return host[kind].reshape(-1, host[kind].shape[-1])[first:first + n]
        return hb._block_fn(kind, first, n)

    types = {k: (down if k == "down" else sh) for k in host}
    return L, HostLayer(blocks, hb.wg, hb.wsg, types=types)


@pytest.fixture(scope="module")
def q5_q8(cuda):
    return _mixed(11, 0, "Q5_K", "Q8_0", cuda)


@pytest.fixture(scope="module")
def q6_q4(cuda):
    return _mixed(11, 1, "Q6_K", "Q4_K", cuda)


def _check_block(cuda, layers, T, stream):
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe, synth
    L, Lh = layers
    xb = synth.tokens(11, T, stream=stream)
    g = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).reshape(T, 2048).to(cuda)
    out, info = moe.moe_block(g, L)
    torch.cuda.synchronize()
    ids = info["ids"].cpu().numpy()
    x = bf16_bits_to_f32(xb)
    r = OM.router(x, Lh.wg)
    assert (ids == r["ids"]).all()
    ref = OM.moe_block_f64(x, Lh, ids, r["w_bf16"])["out"]
    c = OM.compare(out.cpu().numpy(), ref)
    assert c["rel_l2"] < REL_L2 and c["max_abs_norm"] < MAX_ABS_NORM, c
    return out


@pytest.mark.parametrize("T", [1, 4, 12])
def test_q5k_down_q80_shared(cuda, q5_q8, T):
    """T=12 is above the grouped-GEMM threshold: the auto path keeps the layer on the decode
    kernels."""
    _check_block(cuda, q5_q8, T, stream=30 + T)


@pytest.mark.parametrize("T", [1, 3])
def test_q6k_down(cuda, q6_q4, T):
    _check_block(cuda, q6_q4, T, stream=40 + T)


def test_stack_of_published_format_layers(cuda, q5_q8, q6_q4):
    """Two such layers through moe_stack (T=1: the persistent kernel's format variant) and
    moe_stack_prefill (its decode fallback for these layers), teacher-forced against the oracle
    per layer."""
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe, synth
    from b200moe.engine import DeviceEngine
    for T, run in ((1, moe.moe_stack), (3, moe.moe_stack_prefill)):
        resid = torch.from_numpy(bf16_bits_to_f32(synth.tokens(11, T, stream=50 + T)).copy()).to(cuda)
        for L, Lh in (q5_q8, q6_q4):
            before = resid.cpu().numpy().copy()
            ids = torch.empty((1, T, 8), dtype=torch.int32, device=cuda)
            run(resid, DeviceEngine([L]), ids_out=ids)
            after = resid.cpu().numpy()
            xn = OM.rmsnorm(before)
            r = OM.router(xn, Lh.wg)
            assert (ids.cpu().numpy().reshape(T, 8) == r["ids"]).all()
            ref = before.astype(np.float64) + OM.moe_block_f64(xn, Lh, r["ids"], r["w_bf16"])["out"]
            c = OM.compare(after, ref)
            assert c["rel_l2"] < REL_L2, (T, c)


def test_grouped_gemms_refuse(cuda, q5_q8):
    import torch
    from b200moe import _abi, moe
    L, _ = q5_q8
    g = torch.zeros((16, 2048), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(moe.Refused):
        moe.moe_block(g, L, path="prefill")
    out = torch.empty((16, 2048), dtype=torch.float32, device=cuda)
    with pytest.raises(_abi.B200MoeError) as ei:
        _abi.moe_prefill(g, _abi.BF16, None, 1e-6, 16, L.abi(), out, None, moe.prefill_workspace(16, cuda))
    assert ei.value.code == _abi.EINVAL and "Q4_K" in str(ei.value)


def test_device_dequant_matches_oracle_matrix(cuda, q5_q8):
    """DeviceEngine-style inspection (DeviceLayer.dequant) of the mixed types equals the
    oracle's decoded matrices bit for bit."""
    L, Lh = q5_q8
    for kind, e in (("down", 7), ("sh_gate", 0), ("sh_down", 0)):
        assert np.array_equal(L.dequant(kind, e).cpu().numpy(), Lh.matrix(kind, e)), kind


def _published(layers, cuda):
    """The same layers with what the published file also has: F32 router / shared-gate weights
    and a post-attention RMSNorm weight."""
    import torch
    from b200moe.engine import DeviceLayer
    rng = np.random.default_rng(7)
    out = []
    for L in layers:
        nw = torch.from_numpy((1.0 + rng.normal(0, 0.05, 2048)).astype(np.float32)).to(cuda)
        out.append(DeviceLayer(L.gate, L.up, L.down, L.sh_gate, L.sh_up, L.sh_down, L.router_w.float(),
                               L.sh_gate_w.float(), norm_w=nw, down_type=L.down_type, sh_type=L.sh_type))
    return out


@pytest.mark.parametrize("published", [False, True])
def test_persistent_variant_equals_three_kernel_path(cuda, q5_q8, q6_q4, published):
    """At T = 1 the persistent kernel's block-format variant runs these layers (a plain Q4_K
    layer included); at T = 2 the three-kernel path runs each token independently. Fed two
    copies of the token, the two must agree bit for bit, ids included."""
    import torch
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import _abi, moe, synth
    from b200moe.engine import DeviceEngine, DeviceLayer
    assert _abi.decode_persistent_info()[0] == 128 and _abi.decode_persistent_formats()
    layers = [q5_q8[0], DeviceLayer.synthetic(11, 2, cuda), q6_q4[0]]
    if published:
        layers = _published(layers, cuda)
    eng = DeviceEngine(layers)
    x0 = torch.from_numpy(bf16_bits_to_f32(synth.tokens(11, 1, stream=60)).copy()).to(cuda)
    a = x0.clone()
    ids_a = torch.empty((3, 1, 8), dtype=torch.int32, device=cuda)
    moe.moe_stack(a, eng, ids_out=ids_a)
    b = x0.repeat(2, 1)
    ids_b = torch.empty((3, 2, 8), dtype=torch.int32, device=cuda)
    moe.moe_stack(b, eng, ids_out=ids_b)
    torch.cuda.synchronize()
    assert torch.isfinite(a).all()
    assert torch.equal(a[0], b[0]) and torch.equal(b[0], b[1])
    assert torch.equal(ids_a[:, 0], ids_b[:, 0])
    xb = x0.to(torch.bfloat16)
    o1, i1 = moe.moe_block(xb.reshape(1, 2048), layers[0])
    o2, i2 = moe.moe_block(xb.repeat(2, 1), layers[0])
    assert torch.equal(o1[0], o2[0]) and torch.equal(i1["ids"][0], i2["ids"][0])
