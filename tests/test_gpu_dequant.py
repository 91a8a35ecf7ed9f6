"""Q4_K dequant (config 1) and the device synthetic generator vs the oracle: bit-exact."""
import numpy as np
import pytest

from conftest import golden

pytestmark = pytest.mark.gpu


def _bits_equal(a, b):
    a = np.asarray(a).view(np.uint32)
    b = np.asarray(b).view(np.uint32)
    nan = ((a & 0x7FFFFFFF) > 0x7F800000) & ((b & 0x7FFFFFFF) > 0x7F800000)
    return (a == b) | nan


def test_synth_device_equals_host_mirror(cuda):
    import torch
    from oracle import q4k
    from b200moe import _abi
    from b200moe.geometry import KIND_BLOCKS
    for seed, stream in [(0, 0), (0, 2), (1, 5), (3, 8 * 39 + 1), (2 ** 40 + 7, 12345)]:
        for first, n in [(0, 1), (0, 4096), (123457, 777)]:
            t = torch.empty(n * 144, dtype=torch.uint8, device=cuda)
            _abi.synth_q4k(seed, stream, first, n, t)
            host = q4k.synth_blocks(seed, stream, first, n)
            assert (t.cpu().numpy().reshape(n, 144) == host).all(), (seed, stream, first)
    n = KIND_BLOCKS[0]
    t = torch.empty(7 * 144, dtype=torch.uint8, device=cuda)
    _abi.synth_q4k(0, 0, n - 7, 7, t)
    assert (t.cpu().numpy().reshape(7, 144) == q4k.synth_blocks(0, 0, n - 7, 7)).all()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_dequant_golden_bit_exact(cuda, dtype):
    import torch
    from b200moe import _abi
    g = golden("q4k_dequant.npz")
    blocks = torch.from_numpy(g["blocks"].reshape(-1)).to(cuda)
    nb = g["blocks"].shape[0]
    ref = g["ref_f32_bits"].view(np.float32)
    if dtype == "f32":
        out = torch.full((nb * 256,), float("nan"), dtype=torch.float32, device=cuda)
        _abi.q4k_dequant(blocks, out, _abi.F32)
        assert _bits_equal(out.cpu().numpy(), ref).all()
    else:
        out = torch.empty((nb * 256,), dtype=torch.bfloat16, device=cuda)
        _abi.q4k_dequant(blocks, out, _abi.BF16)
        want = torch.from_numpy(ref.copy()).to(torch.bfloat16)
        got = out.cpu()
        fin = ~torch.isnan(want)
        assert torch.equal(got.view(torch.int16)[fin], want.view(torch.int16)[fin])
        assert torch.isnan(got[~fin]).all()


def test_dequant_config1_full_layer(cuda):
    """Config 1: the 3,145,728-block layer stack (gate_up [256,1024,2048] + down [256,2048,512],
    seed 1). Sampled blocks bit-exact vs the C oracle; over the full output, bf16 == RNE(f32)."""
    import torch
    from oracle import q4k
    from oracle.moe import dequant_c
    from b200moe import _abi
    from b200moe.geometry import KIND_BLOCKS, stream_id
    kinds = [0, 1, 2]
    nb = sum(KIND_BLOCKS[k] for k in kinds)
    blocks = torch.empty(nb * 144, dtype=torch.uint8, device=cuda)
    off = 0
    for k in kinds:
        n = KIND_BLOCKS[k]
        _abi.synth_q4k(1, stream_id(0, k), 0, n, blocks[off * 144:(off + n) * 144])
        off += n
    out16 = torch.empty(nb * 256, dtype=torch.bfloat16, device=cuda)
    _abi.q4k_dequant(blocks, out16, _abi.BF16)
    rng = np.random.default_rng(5)
    picks = np.unique(np.concatenate([rng.integers(0, nb, 512), [0, nb - 1, KIND_BLOCKS[0] - 1, KIND_BLOCKS[0]]]))
    starts = np.cumsum([0] + [KIND_BLOCKS[k] for k in kinds])
    for b in picks:
        kk = int(np.searchsorted(starts, b, side="right") - 1)
        host = q4k.synth_blocks(1, stream_id(0, kinds[kk]), int(b - starts[kk]), 1)
        ref = torch.from_numpy(dequant_c(host)).to(torch.bfloat16)
        assert torch.equal(out16[b * 256:(b + 1) * 256].cpu().view(torch.int16), ref.view(torch.int16)), b
    # size-independent property over the whole output, in two halves to bound memory
    half = nb // 2
    for lo, hi in [(0, half), (half, nb)]:
        o32 = torch.empty((hi - lo) * 256, dtype=torch.float32, device=cuda)
        _abi.q4k_dequant(blocks[lo * 144:hi * 144], o32, _abi.F32)
        assert torch.equal(o32.to(torch.bfloat16).view(torch.int16), out16[lo * 256:hi * 256].view(torch.int16))
        del o32


def test_dequant_edges(cuda):
    import torch
    from b200moe import _abi
    blocks = torch.zeros(144 * 4 + 16, dtype=torch.uint8, device=cuda)
    out = torch.zeros(1024, dtype=torch.float32, device=cuda)
    _abi.q4k_dequant(blocks[:0], out, _abi.F32)                      # empty: no-op
    with pytest.raises(_abi.B200MoeError):
        _abi.q4k_dequant(blocks[8:8 + 144], out, _abi.F32)           # unaligned source
    with pytest.raises(_abi.B200MoeError):
        _abi.q4k_dequant(blocks[:144], out, 7)                        # bad dtype


@pytest.mark.parametrize("tname", ["Q5_K", "Q6_K", "Q8_0"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_kquant_dequant_matches_reference_decoder(cuda, tname, dtype):
    """b200moe_dequant for the published file's other block formats against the reference's
    own decoder outputs (tests/golden/kquant_dequant.npz): bit-exact f32; bf16 = RNE of those."""
    import os
    import torch
    from oracle.bf16 import f32_to_bf16_bits
    from b200moe import _abi
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "kquant_dequant.npz"))
    blocks = g[tname + "_blocks"]
    ref = g[tname + "_ref_f32_bits"]
    dev = torch.from_numpy(blocks.reshape(-1).copy()).to(cuda)
    if dtype == "f32":
        out = torch.full((ref.size,), float("nan"), dtype=torch.float32, device=cuda)
        _abi.dequant(dev, tname, out, _abi.F32)
        torch.cuda.synchronize()
        assert _bits_equal(out.cpu().numpy(), ref).all()
    else:
        out = torch.zeros((ref.size,), dtype=torch.int16, device=cuda)
        _abi.dequant(dev, tname, out, _abi.BF16)
        torch.cuda.synchronize()
        got = out.cpu().numpy().view(np.uint16)
        want = f32_to_bf16_bits(ref.view(np.float32))
        nan = ((got & 0x7FFF) > 0x7F80) & ((want & 0x7FFF) > 0x7F80)
        assert ((got == want) | nan).all()
